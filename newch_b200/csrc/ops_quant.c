/* int8 dynamic quantization for inference (newch engine/src/ops/ops_quant.c).
 *
 * Weights: symmetric per-row int8 with an f32 scale per row (quantize_row :11-21). Activations are
 * quantized per row at run time; the int8 x int8 products accumulate exactly in int32 and one
 * rescale y = (float)acc * xs[r] * ws[o] + b[o] follows (qlinear_rows :71-80). On the device: one
 * kernel quantizes the activation rows, one int8 GEMM computes the exact accumulators and applies
 * the rescale in its epilogue.
 */
#include "nc_internal.h"

#include <stdio.h>

nc_tensor *nc_quantize_rows(nc_tensor *w, nc_tensor **scale) {
    if (!w) return NULL;
    nc_ctx *ctx = w->ctx;
    if (w->dtype != NC_F32 || w->ndim != 2) {
        nc__error(ctx, NC_ERR_SHAPE, "quantize_rows: expected a 2-D f32 tensor");
        return NULL;
    }
    const float *W = nc__contig_f32(w);
    nc_tensor *q = nc_empty(ctx, NC_I8, 2, w->shape);
    nc_tensor *s = nc_empty(ctx, NC_F32, 1, w->shape);
    if (!W || !q || !s) return NULL;
    nck_quantize_rows(nc__k(ctx), W, (int8_t *)q->data, (float *)s->data, w->shape[0], w->shape[1]);
    if (scale) *scale = s;
    return q;
}

static nc_status qlinear_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *wq = n->in[1], *ws = n->in[2], *b = n->n_in > 3 ? n->in[3] : NULL;
    if (x->dtype != NC_F32 || wq->dtype != NC_I8 || ws->dtype != NC_F32 || (b && b->dtype != NC_F32)) {
        nc__error(x->ctx, NC_ERR_DTYPE, "linear_int8: expected x f32, weight i8, scale f32, bias f32");
        return NC_ERR_DTYPE;
    }
    if (x->ndim < 1 || wq->ndim != 2 || x->shape[x->ndim - 1] != wq->shape[1] || ws->ndim != 1 ||
        ws->shape[0] != wq->shape[0] || (b && (b->ndim != 1 || b->shape[0] != wq->shape[0]))) {
        char sx[96], sw[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "linear_int8: expected x [..., in], weight [out, in], scale/bias [out]; got %s, %s",
                  nc__shape_str(x->ndim, x->shape, sx, sizeof sx), nc__shape_str(wq->ndim, wq->shape, sw, sizeof sw));
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    shape[x->ndim - 1] = wq->shape[0];
    return NC_OK;
}

static nc_status qlinear_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *wq = n->in[1];
    nc_ctx *ctx = x->ctx;
    int64_t in = wq->shape[1], out = wq->shape[0], M = in ? nc_numel(x) / in : 0;
    if (!nc_is_contiguous(wq)) {
        nc__error(ctx, NC_ERR_ARG, "linear_int8: weight must be contiguous");
        return NC_ERR_ARG;
    }
    /* a pending activation of the input (GELU between int8 layers) is applied while quantizing */
    const float *X = NULL;
    int act = -1;
    float act_s = 0.0f;
    if (!(nc__unary_recipe(x, &X, &act, &act_s) && nck_quantize_rows_act_ok(in))) act = -1, X = nc__contig_f32(x);
    const float *ws = nc__contig_f32(n->in[2]);
    const float *b = n->n_in > 3 ? nc__contig_f32(n->in[3]) : NULL;
    int8_t *xq = (int8_t *)nc__arena_alloc(ctx, (size_t)(M * in) + 16);
    float *xs = (float *)nc__arena_alloc(ctx, (size_t)(M ? M : 1) * sizeof(float));
    if (!X || !ws || (n->n_in > 3 && !b) || !xq || !xs) return NC_ERR_OOM;
    if (!M || !out) return NC_OK;
    if (act >= 0) nck_quantize_rows_act(nc__k(ctx), X, act, act_s, xq, xs, M, in);
    else nck_quantize_rows(nc__k(ctx), X, xq, xs, M, in);
    nck_qlinear(nc__k(ctx), xq, xs, (const int8_t *)nc__dev(wq), ws, b, (float *)n->out->data, M, out, in, NULL);
    return NC_OK;
}

const nc_op_def nc_op_linear_int8 = {"linear_int8", NC_OPF_NONDIFF | NC_OPF_RECIPE, 0, qlinear_infer, NULL, qlinear_fwd, NULL};

nc_tensor *nc_linear_int8(nc_tensor *x, nc_tensor *wq, nc_tensor *w_scale, nc_tensor *bias) {
    nc_tensor *in[4] = {x, wq, w_scale, bias};
    return nc__apply(&nc_op_linear_int8, in, bias ? 4 : 3, NULL);
}
