/* Reductions over one axis or over all axes: sum, mean, max, argmax (newch engine/src/ops/ops_reduce.c
 * semantics: the maximum's gradient goes to its first occurrence, argmax returns the first index,
 * an int32 sum counts in 64 bits, a mean over nothing is NaN, max / argmax of nothing is an error).
 *
 * Every reduction is one geometry, computed once in infer and kept in the node: the input read as
 * [outer, extent, inner] with the reduced extent in the middle (all axes: [1, numel, 1]). Output
 * dtype and the empty-input rule come from a per-kind table. The kernels reduce each output element
 * in a fixed order, so results do not depend on scheduling.
 */
#include "nc_internal.h"

#include <math.h>

enum { RED_SUM, RED_MEAN, RED_MAX, RED_ARGMAX };

/* what distinguishes the kinds */
static const struct {
    int empty_is_error; /* max and argmax of no elements have no value */
    int f32_result;     /* argmax gives indices; the others values */
} red_kind[4] = {{0, 1}, {0, 1}, {1, 1}, {1, 0}};

/* node parameters: i[0] axis, i[1] keepdim (the caller's); i[2..4] the geometry (from infer) */
enum { P_AXIS = 0, P_KEEP = 1, P_OUTER = 2, P_EXTENT = 3, P_INNER = 4 };

static int64_t prod(const int64_t *v, int a, int b) {
    int64_t p = 1;
    for (int i = a; i < b; i++) p *= v[i];
    return p;
}

static nc_status reduce_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    const int kind = n->op->kind, keep = (int)n->p.i[P_KEEP], axis = (int)n->p.i[P_AXIS];
    const int counting = kind == RED_SUM && x->dtype == NC_I32; /* e.g. summing a comparison */
    if (!counting && !nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    *dt = (counting || !red_kind[kind].f32_result) ? NC_I32 : NC_F32;

    if (axis == NC_ALL_AXES) {
        if (red_kind[kind].empty_is_error && nc_numel(x) == 0) {
            nc__error(x->ctx, NC_ERR_SHAPE, "%s: reduction of an empty tensor", n->op->name);
            return NC_ERR_SHAPE;
        }
        n->p.i[P_OUTER] = 1, n->p.i[P_EXTENT] = nc_numel(x), n->p.i[P_INNER] = 1;
        *nd = keep ? x->ndim : 0;
        for (int i = 0; i < *nd; i++) shape[i] = 1;
        return NC_OK;
    }
    const int a = nc__norm_axis(axis, x->ndim);
    if (a < 0) {
        nc__error(x->ctx, NC_ERR_ARG, "%s: axis %d out of range for %d-d tensor", n->op->name, axis, x->ndim);
        return NC_ERR_ARG;
    }
    if (red_kind[kind].empty_is_error && x->shape[a] == 0) {
        nc__error(x->ctx, NC_ERR_SHAPE, "%s: reduction over an empty axis", n->op->name);
        return NC_ERR_SHAPE;
    }
    n->p.i[P_OUTER] = prod(x->shape, 0, a);
    n->p.i[P_EXTENT] = x->shape[a];
    n->p.i[P_INNER] = prod(x->shape, a + 1, x->ndim);
    /* the output keeps every other axis, and the reduced one as 1 with keepdim */
    int k = 0;
    for (int i = 0; i < x->ndim; i++)
        if (i != a || keep) shape[k++] = i == a ? 1 : x->shape[i];
    *nd = k;
    return NC_OK;
}

static nc_status reduce_fwd(nc_node *n) {
    nc_ctx *ctx = n->out->ctx;
    const int64_t outer = n->p.i[P_OUTER], R = n->p.i[P_EXTENT], inner = n->p.i[P_INNER];
    const int kind = n->op->kind;
    nck_dev *k = nc__k(ctx);
    if (n->in[0]->dtype == NC_I32) {
        const int32_t *x = (const int32_t *)nc__contig(n->in[0]);
        if (!x) return NC_ERR_OOM;
        nck_reduce_sum_i32(k, x, (int32_t *)n->out->data, outer, R, inner);
        return NC_OK;
    }
    const float *x = nc__contig_f32(n->in[0]);
    if (!x) return NC_ERR_OOM;
    if (kind == RED_SUM || kind == RED_MEAN) {
        if (kind == RED_MEAN && R == 0) { /* 0 / 0 */
            nck_fill_f32(k, (float *)n->out->data, NAN, outer * inner);
            return NC_OK;
        }
        nck_reduce_sum(k, x, (float *)n->out->data, outer, R, inner, kind == RED_MEAN ? 1.0f / (float)R : 1.0f);
        return NC_OK;
    }
    /* max keeps the position of each maximum for its gradient; argmax returns it */
    int32_t *where = kind == RED_ARGMAX ? (int32_t *)n->out->data
                                        : (int32_t *)nc__arena_alloc(ctx, sizeof(int32_t) * (size_t)(outer * inner));
    if (!where) return NC_ERR_OOM;
    nck_reduce_max(k, x, kind == RED_MAX ? (float *)n->out->data : NULL, where, outer, R, inner);
    if (kind == RED_MAX) n->saved = where;
    return NC_OK;
}

static void reduce_bwd(nc_node *n) {
    int acc = 1;
    /* a sum or mean writes every element of its input's gradient: a fresh buffer is stored, not
     * zero-filled and accumulated */
    nc_tensor *gt = n->op->kind == RED_MAX ? nc__grad_buf(n->in[0]) : nc__grad_buf_acc(n->in[0], &acc);
    if (!gt) return;
    const int64_t outer = n->p.i[P_OUTER], R = n->p.i[P_EXTENT], inner = n->p.i[P_INNER];
    const float *g = (const float *)n->out->grad->data;
    nck_dev *k = nc__k(gt->ctx);
    if (n->op->kind == RED_MAX)
        nck_reduce_max_bwd(k, g, (const int32_t *)n->saved, (float *)gt->data, outer, R, inner);
    else
        nck_reduce_sum_bwd(k, g, (float *)gt->data, outer, R, inner,
                           n->op->kind == RED_MEAN ? 1.0f / (float)(R > 0 ? R : 1) : 1.0f, acc);
}

const nc_op_def nc_op_sum = {"sum", NC_OPF_REDUCTION, RED_SUM, reduce_infer, NULL, reduce_fwd, reduce_bwd};
const nc_op_def nc_op_mean = {"mean", NC_OPF_REDUCTION, RED_MEAN, reduce_infer, NULL, reduce_fwd, reduce_bwd};
const nc_op_def nc_op_max = {"max", NC_OPF_REDUCTION, RED_MAX, reduce_infer, NULL, reduce_fwd, reduce_bwd};
const nc_op_def nc_op_argmax = {"argmax", NC_OPF_REDUCTION | NC_OPF_NONDIFF, RED_ARGMAX, reduce_infer, NULL,
                                reduce_fwd, NULL};

static nc_tensor *reduce_call(const nc_op_def *op, nc_tensor *x, int axis, int keepdim) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[P_AXIS] = axis;
    p.i[P_KEEP] = keepdim != 0;
    return nc__apply(op, &x, 1, &p);
}

nc_tensor *nc_sum(nc_tensor *x, int axis, int keepdim) { return reduce_call(&nc_op_sum, x, axis, keepdim); }
nc_tensor *nc_mean(nc_tensor *x, int axis, int keepdim) { return reduce_call(&nc_op_mean, x, axis, keepdim); }
nc_tensor *nc_max(nc_tensor *x, int axis, int keepdim) { return reduce_call(&nc_op_max, x, axis, keepdim); }
nc_tensor *nc_argmax(nc_tensor *x, int axis) { return reduce_call(&nc_op_argmax, x, axis, 0); }
