/* Shape ops: reshape, transpose, slice, contiguous, detach (views when possible), index_select,
 * cat and dtype conversion.
 *
 * View rules and gradients are newch's (engine/src/ops/ops_shape.c: reshape and the ATen view
 * stride rule :47-120, transpose :126-192, slice :199-271, contiguous/detach :277-294,
 * index_select :300-361, cat :367-457, to_dtype :463-515). Copies are device kernels: a strided
 * gather for layout copies and a strided accumulate for the gradients of views.
 */
#include "nc_internal.h"

#include <stdio.h>

static nc_tensor *alias_with(nc_node *n, int ndim, const int64_t *shape, const int64_t *stride) {
    nc_tensor *t = nc__tensor_alias(n->in[0], 0);
    if (!t) return NULL;
    t->ndim = ndim;
    memcpy(t->shape, shape, sizeof(int64_t) * (size_t)ndim);
    memcpy(t->stride, stride, sizeof(int64_t) * (size_t)ndim);
    n->out = t;
    return t;
}

static nc_status same_shape_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    *dt = n->in[0]->dtype;
    *nd = n->in[0]->ndim;
    memcpy(shape, n->in[0]->shape, sizeof(int64_t) * (size_t)*nd);
    return NC_OK;
}

static nc_status copy_fwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    nck_copy_strided(nc__k(x->ctx), (int)nc__dtype_size(x->dtype), x->ndim, x->shape, x->stride, x->data,
                     n->out->data);
    return NC_OK;
}

static void flat_bwd(nc_node *n) {
    int acc;
    nc_tensor *gt = nc__grad_buf_acc(n->in[0], &acc);
    if (gt)
        (acc ? nck_axpy : nck_axpy_set)(nc__k(gt->ctx), nc_numel(gt), 1.0f, (const float *)n->out->grad->data,
                                        (float *)gt->data);
}

/* ---- reshape ------------------------------------------------------------------------------------ */

static nc_status reshape_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    int r = (int)n->p.i[NC_MAX_DIMS];
    int infer_at = -1;
    int64_t known = 1;
    for (int i = 0; i < r; i++) {
        shape[i] = n->p.i[i];
        if (shape[i] == -1 && infer_at < 0) infer_at = i;
        else if (shape[i] < 0) {
            nc__error(x->ctx, NC_ERR_SHAPE, "reshape: invalid dimension %lld", (long long)shape[i]);
            return NC_ERR_SHAPE;
        } else known *= shape[i];
    }
    int64_t total = nc_numel(x);
    if (infer_at >= 0) shape[infer_at] = known ? total / known : 0;
    if (nc__shape_numel(r, shape) != total) {
        char sa[96], sb[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "reshape: cannot view %s as %s", nc__shape_str(x->ndim, x->shape, sa, sizeof sa),
                  nc__shape_str(r, shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    *dt = x->dtype;
    *nd = r;
    return NC_OK;
}

/* Strides presenting x's elements in row-major order as `shape`, when they exist: runs of x's dims
 * that are laid out back to back must each split into whole dims of the new shape (the same rule as
 * ATen's computeStride, newch ops_shape.c:75-102). */
static int view_strides(const nc_tensor *x, int ndim, const int64_t *shape, int64_t *st) {
    if (nc_is_contiguous(x) || nc_numel(x) == 0) {
        nc__contig_strides(ndim, shape, st);
        return 1;
    }
    int vd = ndim - 1;
    int64_t run_base = x->stride[x->ndim - 1], run_n = 1, view_n = 1;
    for (int d = x->ndim - 1; d >= 0; d--) {
        run_n *= x->shape[d];
        int run_ends = d == 0 || (x->shape[d - 1] != 1 && x->stride[d - 1] != run_n * run_base);
        if (!run_ends) continue;
        while (vd >= 0 && (view_n < run_n || shape[vd] == 1)) {
            st[vd] = view_n * run_base;
            view_n *= shape[vd];
            vd--;
        }
        if (view_n != run_n) return 0;
        if (d > 0) {
            run_base = x->stride[d - 1];
            run_n = view_n = 1;
        }
    }
    return vd == -1;
}

static int reshape_view(nc_node *n, int ndim, const int64_t *shape) {
    int64_t st[NC_MAX_DIMS];
    if (!view_strides(n->in[0], ndim, shape, st)) return 0;
    return alias_with(n, ndim, shape, st) != NULL;
}

const nc_op_def nc_op_reshape = {"reshape", NC_OPF_VIEW, 0, reshape_infer, reshape_view, copy_fwd, flat_bwd};

nc_tensor *nc_reshape(nc_tensor *x, int ndim, const int64_t *shape) {
    if (x && (ndim < 0 || ndim > NC_MAX_DIMS)) {
        nc__error(x->ctx, NC_ERR_SHAPE, "reshape: ndim %d out of range", ndim);
        return NULL;
    }
    nc_op_params p;
    memset(&p, 0, sizeof p);
    for (int i = 0; i < ndim; i++) p.i[i] = shape[i];
    p.i[NC_MAX_DIMS] = ndim;
    return nc__apply(&nc_op_reshape, &x, 1, &p);
}

/* ---- transpose ---------------------------------------------------------------------------------- */

static nc_status transpose_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    int a0 = nc__norm_axis((int)n->p.i[0], x->ndim), a1 = nc__norm_axis((int)n->p.i[1], x->ndim);
    if (a0 < 0 || a1 < 0) {
        nc__error(x->ctx, NC_ERR_ARG, "transpose: axes (%d, %d) out of range for %d-d tensor", (int)n->p.i[0],
                  (int)n->p.i[1], x->ndim);
        return NC_ERR_ARG;
    }
    n->p.i[0] = a0;
    n->p.i[1] = a1;
    *dt = x->dtype;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    shape[a0] = x->shape[a1];
    shape[a1] = x->shape[a0];
    return NC_OK;
}

static void swapped_strides(const nc_node *n, int64_t *st) {
    const nc_tensor *x = n->in[0];
    memcpy(st, x->stride, sizeof(int64_t) * (size_t)x->ndim);
    int a0 = (int)n->p.i[0], a1 = (int)n->p.i[1];
    st[a0] = x->stride[a1];
    st[a1] = x->stride[a0];
}

static int transpose_view(nc_node *n, int ndim, const int64_t *shape) {
    int64_t st[NC_MAX_DIMS];
    swapped_strides(n, st);
    return alias_with(n, ndim, shape, st) != NULL;
}

static nc_status transpose_fwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    int64_t st[NC_MAX_DIMS];
    swapped_strides(n, st);
    nck_copy_strided(nc__k(x->ctx), (int)nc__dtype_size(x->dtype), n->out->ndim, n->out->shape, st, x->data,
                     n->out->data);
    return NC_OK;
}

static void transpose_bwd(nc_node *n) {
    nc_tensor *x = n->in[0], *o = n->out;
    nc_tensor *gt = nc__grad_buf(x);
    if (!gt) return;
    int64_t st[NC_MAX_DIMS];
    nc__contig_strides(x->ndim, x->shape, st);
    int a0 = (int)n->p.i[0], a1 = (int)n->p.i[1];
    int64_t t = st[a0];
    st[a0] = st[a1];
    st[a1] = t;
    nck_acc_strided(nc__k(x->ctx), o->ndim, o->shape, st, (const float *)o->grad->data, (float *)gt->data);
}

const nc_op_def nc_op_transpose = {"transpose", NC_OPF_VIEW, 0, transpose_infer, transpose_view, transpose_fwd,
                                   transpose_bwd};

nc_tensor *nc_transpose(nc_tensor *x, int axis0, int axis1) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = axis0;
    p.i[1] = axis1;
    return nc__apply(&nc_op_transpose, &x, 1, &p);
}

/* ---- slice -------------------------------------------------------------------------------------- */

static nc_status slice_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    int a = nc__norm_axis((int)n->p.i[0], x->ndim);
    int64_t start = n->p.i[1], len = n->p.i[2], step = n->p.i[3];
    if (a < 0) {
        nc__error(x->ctx, NC_ERR_ARG, "slice: axis %d out of range for %d-d tensor", (int)n->p.i[0], x->ndim);
        return NC_ERR_ARG;
    }
    if (step < 1 || len < 0 || start < 0 || start > x->shape[a] ||
        (len > 0 && start + (len - 1) * step >= x->shape[a])) {
        nc__error(x->ctx, NC_ERR_ARG, "slice: start %lld, length %lld, step %lld do not fit axis %d of size %lld",
                  (long long)start, (long long)len, (long long)step, a, (long long)x->shape[a]);
        return NC_ERR_ARG;
    }
    n->p.i[0] = a;
    *dt = x->dtype;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    shape[a] = len;
    return NC_OK;
}

static void sliced(const nc_node *n, nc_tensor *t) {
    const nc_tensor *x = n->in[0];
    int a = (int)n->p.i[0];
    *t = *x;
    t->shape[a] = n->p.i[2];
    if (t->shape[a] > 0) t->data = (char *)x->data + (size_t)(n->p.i[1] * x->stride[a]) * nc__dtype_size(x->dtype);
    t->stride[a] = x->stride[a] * n->p.i[3];
}

static int slice_view(nc_node *n, int ndim, const int64_t *shape) {
    nc_tensor t;
    sliced(n, &t);
    nc_tensor *out = alias_with(n, ndim, shape, t.stride);
    if (!out) return 0;
    out->data = t.data;
    return 1;
}

static nc_status slice_fwd(nc_node *n) {
    nc_tensor t;
    sliced(n, &t);
    nck_copy_strided(nc__k(t.ctx), (int)nc__dtype_size(t.dtype), t.ndim, t.shape, t.stride, t.data, n->out->data);
    return NC_OK;
}

static void slice_bwd(nc_node *n) {
    nc_tensor *x = n->in[0], *o = n->out;
    nc_tensor *gt = nc__grad_buf(x);
    if (!gt) return;
    int a = (int)n->p.i[0];
    if (o->shape[a] == 0 || nc_numel(o) == 0) return;
    int64_t st[NC_MAX_DIMS];
    nc__contig_strides(x->ndim, x->shape, st);
    float *base = (float *)gt->data + n->p.i[1] * st[a];
    st[a] *= n->p.i[3];
    nck_acc_strided(nc__k(x->ctx), o->ndim, o->shape, st, (const float *)o->grad->data, base);
}

const nc_op_def nc_op_slice = {"slice", NC_OPF_VIEW, 0, slice_infer, slice_view, slice_fwd, slice_bwd};

nc_tensor *nc_slice(nc_tensor *x, int axis, int64_t start, int64_t length, int64_t step) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = axis;
    p.i[1] = start;
    p.i[2] = length;
    p.i[3] = step;
    return nc__apply(&nc_op_slice, &x, 1, &p);
}

/* ---- contiguous / detach ------------------------------------------------------------------------ */

static int contiguous_view(nc_node *n, int ndim, const int64_t *shape) {
    if (!nc_is_contiguous(n->in[0])) return 0;
    return alias_with(n, ndim, shape, n->in[0]->stride) != NULL;
}

const nc_op_def nc_op_contiguous = {"contiguous", NC_OPF_VIEW, 0, same_shape_infer, contiguous_view, copy_fwd,
                                    flat_bwd};

nc_tensor *nc_contiguous(nc_tensor *x) { return nc__apply(&nc_op_contiguous, &x, 1, NULL); }

static int detach_view(nc_node *n, int ndim, const int64_t *shape) {
    return alias_with(n, ndim, shape, n->in[0]->stride) != NULL;
}

const nc_op_def nc_op_detach = {"detach", NC_OPF_VIEW | NC_OPF_NONDIFF, 0, same_shape_infer, detach_view, copy_fwd,
                                NULL};

nc_tensor *nc_detach(nc_tensor *x) { return nc__apply(&nc_op_detach, &x, 1, NULL); }

/* ---- index_select (axis 0) ---------------------------------------------------------------------- */

static nc_status index_select_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *idx = n->in[1];
    if (x->ndim < 1 || idx->ndim != 1 || idx->dtype != NC_I32) {
        char sa[96], sb[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "index_select: expected x [N, ...] and i32 indices [B], got %s and %s %s",
                  nc__shape_str(x->ndim, x->shape, sa, sizeof sa), nc__dtype_name(idx->dtype),
                  nc__shape_str(idx->ndim, idx->shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    *dt = x->dtype;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    shape[0] = idx->shape[0];
    return NC_OK;
}

/* Host-side range check when the indices' host copy is current (no device round trip); otherwise
 * the kernel checks and reports through the status word. */
static int check_indices_host(nc_ctx *ctx, nc_tensor *idx, int64_t N, const char *what, nc_status code) {
    const int32_t *h = (const int32_t *)nc__host_view(idx);
    if (!h) return 1;
    for (int64_t b = 0, B = nc_numel(idx); b < B; b++) {
        if (h[b] < 0 || h[b] >= N) {
            nc__error(ctx, code, "%s: index %d at position %lld outside [0, %lld)", what, h[b], (long long)b,
                      (long long)N);
            return 0;
        }
    }
    return 1;
}

static nc_status index_select_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *o = n->out, *it = n->in[1];
    nc_ctx *ctx = o->ctx;
    int64_t B = it->shape[0], N = x->shape[0];
    if (!check_indices_host(ctx, it, N, "index_select", NC_ERR_ARG)) return NC_ERR_ARG;
    const int32_t *idx = (const int32_t *)nc__contig(it);
    const void *src = nc__contig(x);
    if (!idx || !src) return NC_ERR_OOM;
    size_t row = (size_t)(N ? nc_numel(x) / N : 0) * nc__dtype_size(x->dtype);
    nck_index_select(nc__k(ctx), src, idx, o->data, B, N, (int64_t)row);
    n->saved = (void *)idx;
    return NC_OK;
}

static void index_select_bwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    nc_tensor *gt = nc__grad_buf(x);
    if (!gt) return;
    int64_t B = n->in[1]->shape[0], N = x->shape[0];
    int64_t row = N ? nc_numel(x) / N : 0;
    nck_index_select_bwd(nc__k(x->ctx), (const float *)n->out->grad->data, (const int32_t *)n->saved,
                         (float *)gt->data, B, N, row);
}

const nc_op_def nc_op_index_select = {"index_select", 0, 0, index_select_infer, NULL, index_select_fwd,
                                      index_select_bwd};

nc_tensor *nc_index_select(nc_tensor *x, nc_tensor *idx) {
    nc_tensor *in[2] = {x, idx};
    return nc__apply(&nc_op_index_select, in, 2, NULL);
}

/* ---- cat ------------------------------------------------------------------------------------------ */

static nc_status cat_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x0 = n->in[0];
    int axis = nc__norm_axis((int)n->p.i[0], x0->ndim);
    if (axis < 0) {
        nc__error(x0->ctx, NC_ERR_ARG, "cat: dim %d out of range for %d-d tensors", (int)n->p.i[0], x0->ndim);
        return NC_ERR_ARG;
    }
    n->p.i[0] = axis;
    memcpy(shape, x0->shape, sizeof(int64_t) * (size_t)x0->ndim);
    for (int k = 1; k < n->n_in; k++) {
        nc_tensor *x = n->in[k];
        int same = x->dtype == x0->dtype && x->ndim == x0->ndim;
        for (int i = 0; same && i < x0->ndim; i++) same = i == axis || x->shape[i] == x0->shape[i];
        if (!same) {
            char sa[96], sb[96];
            nc__error(x0->ctx, NC_ERR_SHAPE, "cat: %s %s and %s %s differ outside dim %d", nc__dtype_name(x0->dtype),
                      nc__shape_str(x0->ndim, x0->shape, sa, sizeof sa), nc__dtype_name(x->dtype),
                      nc__shape_str(x->ndim, x->shape, sb, sizeof sb), axis);
            return NC_ERR_SHAPE;
        }
        shape[axis] += x->shape[axis];
    }
    *dt = x0->dtype;
    *nd = x0->ndim;
    return NC_OK;
}

static void cat_dims(const nc_node *n, int64_t *outer, int64_t *inner) {
    const nc_tensor *x0 = n->in[0];
    int axis = (int)n->p.i[0];
    *outer = 1, *inner = 1;
    for (int i = 0; i < axis; i++) *outer *= x0->shape[i];
    for (int i = axis + 1; i < x0->ndim; i++) *inner *= x0->shape[i];
}

static nc_status cat_fwd(nc_node *n) {
    int axis = (int)n->p.i[0];
    int64_t es = (int64_t)nc__dtype_size(n->out->dtype);
    int64_t outer, inner;
    cat_dims(n, &outer, &inner);
    int64_t row_out = n->out->shape[axis] * inner, off = 0;
    for (int k = 0; k < n->n_in; k++) {
        nc_tensor *x = n->in[k];
        const void *src = nc__contig(x);
        if (!src) return NC_ERR_OOM;
        int64_t row = x->shape[axis] * inner;
        if (row * outer > 0) nck_cat_part(nc__k(x->ctx), src, n->out->data, outer, row * es, row_out * es, off * es);
        off += row;
    }
    return NC_OK;
}

static void cat_bwd(nc_node *n) {
    int axis = (int)n->p.i[0];
    int64_t outer, inner;
    cat_dims(n, &outer, &inner);
    int64_t row_out = n->out->shape[axis] * inner, off = 0;
    for (int k = 0; k < n->n_in; k++) {
        nc_tensor *x = n->in[k];
        int64_t row = x->shape[axis] * inner;
        nc_tensor *gx = nc__needs_grad(x) ? nc__grad_buf(x) : NULL;
        if (gx && row * outer > 0)
            nck_cat_part_bwd(nc__k(x->ctx), (const float *)n->out->grad->data, (float *)gx->data, outer, row, row_out,
                             off);
        off += row;
    }
}

const nc_op_def nc_op_cat = {"cat", 0, 0, cat_infer, NULL, cat_fwd, cat_bwd};

nc_tensor *nc_cat(int n, nc_tensor *const *xs, int axis) {
    if (n < 1 || n > NC_MAX_INPUTS) {
        if (n > 0 && xs[0]) nc__error(xs[0]->ctx, NC_ERR_ARG, "cat: takes 1 to %d tensors, got %d", NC_MAX_INPUTS, n);
        return NULL;
    }
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = axis;
    nc_tensor *in[NC_MAX_INPUTS];
    for (int k = 0; k < n; k++) in[k] = xs[k];
    return nc__apply(&nc_op_cat, in, n, &p);
}

/* ---- to_dtype ------------------------------------------------------------------------------------- */

static nc_status to_dtype_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_dtype to = (nc_dtype)n->p.i[0], from = n->in[0]->dtype;
    if (to == NC_F16 || from == NC_F16 || nc__dtype_size(to) == 0) {
        nc__error(n->in[0]->ctx, NC_ERR_DTYPE, "to_dtype: %s -> %s is not supported", nc__dtype_name(from),
                  nc__dtype_name(to));
        return NC_ERR_DTYPE;
    }
    *dt = to;
    return same_shape_infer(n, &from, nd, shape);
}

static nc_status to_dtype_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *o = n->out;
    const void *src = nc__contig(x);
    if (!src) return NC_ERR_OOM;
    nck_convert(nc__k(o->ctx), x->dtype, o->dtype, src, o->data, nc_numel(x));
    return NC_OK;
}

const nc_op_def nc_op_to_dtype = {"to_dtype", 0, 0, to_dtype_infer, NULL, to_dtype_fwd, flat_bwd};

nc_tensor *nc_to_dtype(nc_tensor *x, nc_dtype dt) {
    if (x && dt != NC_F32) x = nc_detach(x);
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = dt;
    return nc__apply(&nc_op_to_dtype, &x, 1, &p);
}
