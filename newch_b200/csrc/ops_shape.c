/* Layout and indexing ops: reshape, transpose, slice, contiguous, detach, index_select (axis 0), cat
 * and dtype conversion. Shapes, view rules, gradients and error messages are newch's
 * (engine/src/ops/ops_shape.c: reshape :47-120, transpose :126-192, slice :199-271,
 * contiguous / detach :277-294, index_select :300-361, cat :367-457, to_dtype :463-515).
 *
 * The layout ops share one description: a layout map turns the strides of x into the strides (and
 * element offset) under which the output's elements are read from x's storage. The same map gives
 * (1) the view, aliasing x's storage, when the op may alias; (2) the copying forward, a strided
 * gather on the device; (3) the backward, a strided accumulate of dY into x's contiguous gradient
 * (the map applied to contiguous strides). Reshape is the exception: a view only when x's layout
 * can present the new shape (view_rule), otherwise a row-major copy, and its gradient is flat.
 */
#include "nc_internal.h"

#include <stdio.h>

/* output strides `st` (and element offset `off`) over storage laid out with x-strides `xst`; 0 when
 * no such strides exist */
typedef int (*layout_map)(const nc_node *n, const int64_t *xst, int64_t *st, int64_t *off);

static int as_alias(nc_node *n, int nd, const int64_t *shape, layout_map map) {
    nc_tensor *x = n->in[0];
    int64_t st[NC_MAX_DIMS], off = 0;
    if (!map(n, x->stride, st, &off)) return 0;
    nc_tensor *t = nc__tensor_alias(x, 0);
    if (!t) return 0;
    t->ndim = nd;
    memcpy(t->shape, shape, sizeof(int64_t) * (size_t)nd);
    memcpy(t->stride, st, sizeof(int64_t) * (size_t)nd);
    if (off && nc__shape_numel(nd, shape) > 0) t->data = (char *)x->data + (size_t)off * nc__dtype_size(x->dtype);
    n->out = t;
    return 1;
}

static nc_status gather_by_map(nc_node *n, layout_map map) {
    nc_tensor *x = n->in[0], *o = n->out;
    int64_t st[NC_MAX_DIMS], off = 0;
    map(n, x->stride, st, &off);
    if (nc_numel(o) == 0) return NC_OK;
    const size_t es = nc__dtype_size(x->dtype);
    nck_copy_strided(nc__k(x->ctx), (int)es, o->ndim, o->shape, st, (const char *)x->data + (size_t)off * es, o->data);
    return NC_OK;
}

/* covers_all: the map reaches every element of x (a permutation), so a fresh gradient buffer is
 * stored whole instead of zero-filled and added to */
static void scatter_grad_by_map(nc_node *n, layout_map map, int covers_all) {
    nc_tensor *x = n->in[0], *o = n->out;
    int acc = 1;
    nc_tensor *gx = covers_all ? nc__grad_buf_acc(x, &acc) : nc__grad_buf(x);
    if (!gx || nc_numel(o) == 0) return;
    int64_t cst[NC_MAX_DIMS], st[NC_MAX_DIMS], off = 0;
    nc__contig_strides(x->ndim, x->shape, cst);
    map(n, cst, st, &off);
    nck_acc_strided(nc__k(x->ctx), o->ndim, o->shape, st, (const float *)o->grad->data, (float *)gx->data + off, acc);
}

/* gradient of an op whose output is x's elements in x's row-major order */
static void flat_grad(nc_node *n) {
    if (nc__grad_handoff(n->in[0], n->out)) return; /* x takes dY's buffer as its gradient */
    int acc;
    nc_tensor *gx = nc__grad_buf_acc(n->in[0], &acc);
    if (!gx) return;
    const float *gy = (const float *)n->out->grad->data;
    if (acc) nck_axpy(nc__k(gx->ctx), nc_numel(gx), 1.0f, gy, (float *)gx->data);
    else nck_axpy_set(nc__k(gx->ctx), nc_numel(gx), 1.0f, gy, (float *)gx->data);
}

static nc_status rowmajor_copy(nc_node *n) {
    nc_tensor *x = n->in[0];
    if (nc_numel(x) == 0) return NC_OK;
    nck_copy_strided(nc__k(x->ctx), (int)nc__dtype_size(x->dtype), x->ndim, x->shape, x->stride, x->data, n->out->data);
    return NC_OK;
}

static nc_status keep_shape(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    *dt = n->in[0]->dtype;
    *nd = n->in[0]->ndim;
    memcpy(shape, n->in[0]->shape, sizeof(int64_t) * (size_t)*nd);
    return NC_OK;
}

/* ---- reshape ------------------------------------------------------------------------------------ */

/* node parameters: i[0 .. NC_MAX_DIMS) the requested shape, i[NC_MAX_DIMS] its rank */
static nc_status reshape_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    const int rank = (int)n->p.i[NC_MAX_DIMS];
    int wild = -1; /* the first -1: inferred from the others */
    int64_t fixed = 1;
    for (int i = 0; i < rank; i++) {
        const int64_t v = n->p.i[i];
        shape[i] = v;
        if (v == -1 && wild < 0) {
            wild = i;
        } else if (v < 0) {
            nc__error(x->ctx, NC_ERR_SHAPE, "reshape: invalid dimension %lld", (long long)v);
            return NC_ERR_SHAPE;
        } else {
            fixed *= v;
        }
    }
    const int64_t total = nc_numel(x);
    if (wild >= 0) shape[wild] = fixed ? total / fixed : 0;
    if (nc__shape_numel(rank, shape) != total) {
        char sa[96], sb[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "reshape: cannot view %s as %s", nc__shape_str(x->ndim, x->shape, sa, sizeof sa),
                  nc__shape_str(rank, shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    *dt = x->dtype;
    *nd = rank;
    return NC_OK;
}

/* The strides that present x (shape xs, strides xst) in row-major order as `shape`, when they exist
 * (the rule of ATen's computeStride). x's dims fall into blocks: consecutive dims where the outer one
 * steps over exactly the elements of everything inside it (dims of extent 1 join any block). Read
 * from the innermost block outwards, the new shape must split into consecutive runs with the same
 * element counts; a run's dims take row-major strides scaled by its block's innermost stride. */
static int view_rule(int xnd, const int64_t *xs, const int64_t *xst, int nd, const int64_t *shape, int64_t *st) {
    int v = nd - 1;
    int d = xnd - 1;
    while (d >= 0) {
        /* the block ending at dim d: its innermost stride and element count */
        const int64_t unit = xst[d];
        int64_t elems = xs[d];
        while (d > 0 && (xs[d - 1] == 1 || xst[d - 1] == elems * unit)) elems *= xs[--d];
        /* the run of new dims covering the block (size-1 dims are taken along) */
        int64_t covered = 1;
        while (v >= 0 && (covered < elems || shape[v] == 1)) {
            st[v] = covered * unit;
            covered *= shape[v--];
        }
        if (covered != elems) return 0;
        d--;
    }
    return v < 0;
}

static int reshape_view(nc_node *n, int nd, const int64_t *shape) {
    nc_tensor *x = n->in[0];
    int64_t st[NC_MAX_DIMS];
    int ok = nc_is_contiguous(x) || nc_numel(x) == 0;
    if (ok) nc__contig_strides(nd, shape, st);
    else ok = view_rule(x->ndim, x->shape, x->stride, nd, shape, st);
    if (!ok) return 0;
    nc_tensor *t = nc__tensor_alias(x, 0);
    if (!t) return 0;
    t->ndim = nd;
    memcpy(t->shape, shape, sizeof(int64_t) * (size_t)nd);
    memcpy(t->stride, st, sizeof(int64_t) * (size_t)nd);
    n->out = t;
    return 1;
}

const nc_op_def nc_op_reshape = {"reshape", NC_OPF_VIEW, 0, reshape_infer, reshape_view, rowmajor_copy, flat_grad};

nc_tensor *nc_reshape(nc_tensor *x, int ndim, const int64_t *shape) {
    if (x && (ndim < 0 || ndim > NC_MAX_DIMS)) {
        nc__error(x->ctx, NC_ERR_SHAPE, "reshape: ndim %d out of range", ndim);
        return NULL;
    }
    nc_op_params p;
    memset(&p, 0, sizeof p);
    if (ndim > 0) memcpy(p.i, shape, sizeof(int64_t) * (size_t)ndim);
    p.i[NC_MAX_DIMS] = ndim;
    return nc__apply(&nc_op_reshape, &x, 1, &p);
}

/* ---- transpose ---------------------------------------------------------------------------------- */

static nc_status transpose_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    const int a0 = nc__norm_axis((int)n->p.i[0], x->ndim), a1 = nc__norm_axis((int)n->p.i[1], x->ndim);
    if (a0 < 0 || a1 < 0) {
        nc__error(x->ctx, NC_ERR_ARG, "transpose: axes (%d, %d) out of range for %d-d tensor", (int)n->p.i[0],
                  (int)n->p.i[1], x->ndim);
        return NC_ERR_ARG;
    }
    n->p.i[0] = a0, n->p.i[1] = a1;
    keep_shape(n, dt, nd, shape);
    shape[a0] = x->shape[a1];
    shape[a1] = x->shape[a0];
    return NC_OK;
}

static int transpose_map(const nc_node *n, const int64_t *xst, int64_t *st, int64_t *off) {
    const int nd = n->in[0]->ndim, a0 = (int)n->p.i[0], a1 = (int)n->p.i[1];
    memcpy(st, xst, sizeof(int64_t) * (size_t)nd);
    st[a0] = xst[a1];
    st[a1] = xst[a0];
    *off = 0;
    return 1;
}

static int transpose_view(nc_node *n, int nd, const int64_t *shape) { return as_alias(n, nd, shape, transpose_map); }
static nc_status transpose_fwd(nc_node *n) { return gather_by_map(n, transpose_map); }
static void transpose_bwd(nc_node *n) { scatter_grad_by_map(n, transpose_map, 1); }

const nc_op_def nc_op_transpose = {"transpose", NC_OPF_VIEW, 0, transpose_infer, transpose_view, transpose_fwd,
                                   transpose_bwd};

nc_tensor *nc_transpose(nc_tensor *x, int axis0, int axis1) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = axis0, p.i[1] = axis1;
    return nc__apply(&nc_op_transpose, &x, 1, &p);
}

/* ---- slice: elements start, start + step, ... (length of them) along one axis -------------------- */

static nc_status slice_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    const int a = nc__norm_axis((int)n->p.i[0], x->ndim);
    const int64_t start = n->p.i[1], len = n->p.i[2], step = n->p.i[3];
    if (a < 0) {
        nc__error(x->ctx, NC_ERR_ARG, "slice: axis %d out of range for %d-d tensor", (int)n->p.i[0], x->ndim);
        return NC_ERR_ARG;
    }
    const int64_t extent = x->shape[a];
    const int fits = step >= 1 && len >= 0 && start >= 0 && start <= extent && (len == 0 || start + (len - 1) * step < extent);
    if (!fits) {
        nc__error(x->ctx, NC_ERR_ARG, "slice: start %lld, length %lld, step %lld do not fit axis %d of size %lld",
                  (long long)start, (long long)len, (long long)step, a, (long long)extent);
        return NC_ERR_ARG;
    }
    n->p.i[0] = a;
    keep_shape(n, dt, nd, shape);
    shape[a] = len;
    return NC_OK;
}

static int slice_map(const nc_node *n, const int64_t *xst, int64_t *st, int64_t *off) {
    const int a = (int)n->p.i[0];
    memcpy(st, xst, sizeof(int64_t) * (size_t)n->in[0]->ndim);
    st[a] = xst[a] * n->p.i[3];
    *off = n->p.i[2] > 0 ? n->p.i[1] * xst[a] : 0;
    return 1;
}

static int slice_view(nc_node *n, int nd, const int64_t *shape) { return as_alias(n, nd, shape, slice_map); }
static nc_status slice_fwd(nc_node *n) { return gather_by_map(n, slice_map); }
static void slice_bwd(nc_node *n) { scatter_grad_by_map(n, slice_map, 0); }

const nc_op_def nc_op_slice = {"slice", NC_OPF_VIEW, 0, slice_infer, slice_view, slice_fwd, slice_bwd};

nc_tensor *nc_slice(nc_tensor *x, int axis, int64_t start, int64_t length, int64_t step) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = axis, p.i[1] = start, p.i[2] = length, p.i[3] = step;
    return nc__apply(&nc_op_slice, &x, 1, &p);
}

/* ---- contiguous / detach ------------------------------------------------------------------------ */

static int same_map(const nc_node *n, const int64_t *xst, int64_t *st, int64_t *off) {
    memcpy(st, xst, sizeof(int64_t) * (size_t)n->in[0]->ndim);
    *off = 0;
    return 1;
}

static int contiguous_view(nc_node *n, int nd, const int64_t *shape) {
    return nc_is_contiguous(n->in[0]) && as_alias(n, nd, shape, same_map);
}

const nc_op_def nc_op_contiguous = {"contiguous", NC_OPF_VIEW, 0, keep_shape, contiguous_view, rowmajor_copy,
                                    flat_grad};

nc_tensor *nc_contiguous(nc_tensor *x) { return nc__apply(&nc_op_contiguous, &x, 1, NULL); }

static int detach_view(nc_node *n, int nd, const int64_t *shape) { return as_alias(n, nd, shape, same_map); }

const nc_op_def nc_op_detach = {"detach", NC_OPF_VIEW | NC_OPF_NONDIFF, 0, keep_shape, detach_view, rowmajor_copy,
                                NULL};

nc_tensor *nc_detach(nc_tensor *x) { return nc__apply(&nc_op_detach, &x, 1, NULL); }

/* ---- index_select: rows of x [N, ...] picked by int32 indices [B] ---------------------------------- */

static nc_status index_select_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *idx = n->in[1];
    if (x->ndim < 1 || idx->ndim != 1 || idx->dtype != NC_I32) {
        char sa[96], sb[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "index_select: expected x [N, ...] and i32 indices [B], got %s and %s %s",
                  nc__shape_str(x->ndim, x->shape, sa, sizeof sa), nc__dtype_name(idx->dtype),
                  nc__shape_str(idx->ndim, idx->shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    keep_shape(n, dt, nd, shape);
    shape[0] = idx->shape[0];
    return NC_OK;
}

/* Indices whose host copy is current are range-checked here, before anything runs; otherwise the
 * gather checks them on the device and reports through the status word at the next sync. */
static int indices_in_range(nc_ctx *ctx, nc_tensor *idx, int64_t rows) {
    const int32_t *h = (const int32_t *)nc__host_view(idx);
    if (!h) return 1;
    const int64_t B = nc_numel(idx);
    for (int64_t b = 0; b < B; b++)
        if (h[b] < 0 || h[b] >= rows) {
            nc__error(ctx, NC_ERR_ARG, "index_select: index %d at position %lld outside [0, %lld)", h[b], (long long)b,
                      (long long)rows);
            return 0;
        }
    return 1;
}

static int64_t row_elems(const nc_tensor *x) { return x->shape[0] ? nc_numel(x) / x->shape[0] : 0; }

static nc_status index_select_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *it = n->in[1], *o = n->out;
    nc_ctx *ctx = o->ctx;
    if (!indices_in_range(ctx, it, x->shape[0])) return NC_ERR_ARG;
    const int32_t *idx = (const int32_t *)nc__contig(it);
    const void *src = nc__contig(x);
    if (!idx || !src) return NC_ERR_OOM;
    nck_index_select(nc__k(ctx), src, idx, o->data, it->shape[0], x->shape[0],
                     row_elems(x) * (int64_t)nc__dtype_size(x->dtype));
    n->saved = (void *)idx; /* the device indices, for the backward gather */
    return NC_OK;
}

static void index_select_bwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    nc_tensor *gx = nc__grad_buf(x);
    if (gx)
        nck_index_select_bwd(nc__k(x->ctx), (const float *)n->out->grad->data, (const int32_t *)n->saved,
                             (float *)gx->data, n->in[1]->shape[0], x->shape[0], row_elems(x));
}

const nc_op_def nc_op_index_select = {"index_select", 0, 0, index_select_infer, NULL, index_select_fwd,
                                      index_select_bwd};

nc_tensor *nc_index_select(nc_tensor *x, nc_tensor *idx) {
    nc_tensor *in[2] = {x, idx};
    return nc__apply(&nc_op_index_select, in, 2, NULL);
}

/* ---- cat: inputs side by side along one axis -------------------------------------------------------- */

static nc_status cat_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *first = n->in[0];
    const int axis = nc__norm_axis((int)n->p.i[0], first->ndim);
    if (axis < 0) {
        nc__error(first->ctx, NC_ERR_ARG, "cat: dim %d out of range for %d-d tensors", (int)n->p.i[0], first->ndim);
        return NC_ERR_ARG;
    }
    n->p.i[0] = axis;
    keep_shape(n, dt, nd, shape);
    for (int k = 1; k < n->n_in; k++) {
        const nc_tensor *x = n->in[k];
        int match = x->dtype == first->dtype && x->ndim == first->ndim;
        for (int i = 0; match && i < first->ndim; i++) match = i == axis || x->shape[i] == first->shape[i];
        if (!match) {
            char sa[96], sb[96];
            nc__error(first->ctx, NC_ERR_SHAPE, "cat: %s %s and %s %s differ outside dim %d",
                      nc__dtype_name(first->dtype), nc__shape_str(first->ndim, first->shape, sa, sizeof sa),
                      nc__dtype_name(x->dtype), nc__shape_str(x->ndim, x->shape, sb, sizeof sb), axis);
            return NC_ERR_SHAPE;
        }
        shape[axis] += x->shape[axis];
    }
    return NC_OK;
}

/* the output as [outer][row]: each input contributes a block of `its extent * inner` per outer index */
typedef struct {
    int64_t outer, inner, out_row;
} cat_geom;

static cat_geom cat_geometry(const nc_node *n) {
    const nc_tensor *o = n->out;
    const int axis = (int)n->p.i[0];
    cat_geom g = {1, 1, 0};
    for (int i = 0; i < axis; i++) g.outer *= o->shape[i];
    for (int i = axis + 1; i < o->ndim; i++) g.inner *= o->shape[i];
    g.out_row = o->shape[axis] * g.inner;
    return g;
}

static nc_status cat_fwd(nc_node *n) {
    const cat_geom g = cat_geometry(n);
    const int axis = (int)n->p.i[0];
    const int64_t es = (int64_t)nc__dtype_size(n->out->dtype);
    int64_t at = 0;
    for (int k = 0; k < n->n_in; k++) {
        nc_tensor *x = n->in[k];
        const int64_t row = x->shape[axis] * g.inner;
        const void *src = nc__contig(x);
        if (!src) return NC_ERR_OOM;
        if (row > 0 && g.outer > 0) nck_cat_part(nc__k(x->ctx), src, n->out->data, g.outer, row * es, g.out_row * es, at * es);
        at += row;
    }
    return NC_OK;
}

static void cat_bwd(nc_node *n) {
    const cat_geom g = cat_geometry(n);
    const int axis = (int)n->p.i[0];
    int64_t at = 0;
    for (int k = 0; k < n->n_in; k++) {
        nc_tensor *x = n->in[k];
        const int64_t row = x->shape[axis] * g.inner;
        nc_tensor *gx = nc__needs_grad(x) ? nc__grad_buf(x) : NULL;
        if (gx && row > 0 && g.outer > 0)
            nck_cat_part_bwd(nc__k(x->ctx), (const float *)n->out->grad->data, (float *)gx->data, g.outer, row,
                             g.out_row, at);
        at += row;
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
    memcpy(in, xs, sizeof(nc_tensor *) * (size_t)n);
    return nc__apply(&nc_op_cat, in, n, &p);
}

/* ---- to_dtype: elementwise conversion (saturating to the integer types) --------------------------- */

static nc_status to_dtype_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    const nc_dtype to = (nc_dtype)n->p.i[0], from = n->in[0]->dtype;
    if (to == NC_F16 || from == NC_F16 || nc__dtype_size(to) == 0) {
        nc__error(n->in[0]->ctx, NC_ERR_DTYPE, "to_dtype: %s -> %s is not supported", nc__dtype_name(from),
                  nc__dtype_name(to));
        return NC_ERR_DTYPE;
    }
    keep_shape(n, dt, nd, shape);
    *dt = to;
    return NC_OK;
}

static nc_status to_dtype_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *o = n->out;
    const void *src = nc__contig(x);
    if (!src) return NC_ERR_OOM;
    nck_convert(nc__k(o->ctx), x->dtype, o->dtype, src, o->data, nc_numel(x));
    return NC_OK;
}

const nc_op_def nc_op_to_dtype = {"to_dtype", 0, 0, to_dtype_infer, NULL, to_dtype_fwd, flat_grad};

/* only a conversion to f32 carries a gradient; any other target is taken from a detached input */
nc_tensor *nc_to_dtype(nc_tensor *x, nc_dtype dt) {
    if (x && dt != NC_F32) x = nc_detach(x);
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = dt;
    return nc__apply(&nc_op_to_dtype, &x, 1, &p);
}
