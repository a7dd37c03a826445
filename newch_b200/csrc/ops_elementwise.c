/* Elementwise ops: broadcasting binary ops, unary math and activations, comparisons.
 *
 * Shape rules, gradient formulas and the PyTorch kink conventions are newch's
 * (engine/src/ops/ops_elementwise.c: binary infer :60-84, binary backward :129-186, unary forward
 * :229-266 and backward :289-338, compare :418-488). The kernels are one fused launch per op:
 * float4 streams for same-shape operands, a stride-table kernel for broadcasts, and a
 * reduce-to-shape kernel for gradients of broadcast operands.
 */
#include "nc_internal.h"

#include <stdio.h>

enum { BIN_ADD, BIN_SUB, BIN_MUL, BIN_DIV };

static nc_status binary_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *a = n->in[0], *b = n->in[1];
    if (!nc__expect_f32(n, 0) || !nc__expect_f32(n, 1)) return NC_ERR_DTYPE;
    int r = a->ndim > b->ndim ? a->ndim : b->ndim;
    for (int i = 0; i < r; i++) {
        int ia = i - (r - a->ndim), ib = i - (r - b->ndim);
        int64_t da = ia < 0 ? 1 : a->shape[ia], db = ib < 0 ? 1 : b->shape[ib];
        if (da != db && da != 1 && db != 1) {
            char sa[96], sb[96];
            nc__error(a->ctx, NC_ERR_SHAPE, "%s: shapes %s and %s are not broadcastable", n->op->name,
                      nc__shape_str(a->ndim, a->shape, sa, sizeof sa), nc__shape_str(b->ndim, b->shape, sb, sizeof sb));
            return NC_ERR_SHAPE;
        }
        shape[i] = da == 1 ? db : da;
    }
    *dt = NC_F32;
    *nd = r;
    return NC_OK;
}

static void fill_bcast(nck_bcast *bc, const nc_tensor *a, const nc_tensor *b, const nc_tensor *o) {
    bc->ndim = o->ndim;
    memcpy(bc->shape, o->shape, sizeof(int64_t) * (size_t)o->ndim);
    nc__bcast_strides(a, o->ndim, o->shape, bc->sa);
    nc__bcast_strides(b, o->ndim, o->shape, bc->sb);
    memcpy(bc->so, o->stride, sizeof(int64_t) * (size_t)o->ndim);
}

static nc_status binary_fwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    nck_dev *k = nc__k(o->ctx);
    if (nc__same_shape(a, b) && nc_is_contiguous(a) && nc_is_contiguous(b)) {
        nck_binary_fwd_flat(k, n->op->kind, (const float *)a->data, (const float *)b->data, (float *)o->data,
                            nc_numel(o));
        return NC_OK;
    }
    nck_bcast bc;
    fill_bcast(&bc, a, b, o);
    nck_binary_fwd(k, n->op->kind, &bc, (const float *)a->data, (const float *)b->data, (float *)o->data);
    return NC_OK;
}

static void binary_bwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    nck_dev *k = nc__k(o->ctx);
    nck_bcast bc;
    fill_bcast(&bc, a, b, o);
    nc__contig_strides(o->ndim, o->shape, bc.so); /* the output grad is contiguous */
    for (int which = 0; which < 2; which++) {
        nc_tensor *x = n->in[which];
        if (!nc__needs_grad(x)) continue;
        int acc;
        nc_tensor *gx = nc__grad_buf_acc(x, &acc);
        if (!gx) return;
        int64_t sgx[NC_MAX_DIMS];
        nc__bcast_strides_shape(x->ndim, x->shape, o->ndim, o->shape, sgx);
        if ((n->op->kind == BIN_ADD || n->op->kind == BIN_SUB) && nc__same_shape(x, o)) {
            (acc ? nck_axpy : nck_axpy_set)(k, nc_numel(o), (n->op->kind == BIN_SUB && which == 1) ? -1.0f : 1.0f,
                                            (const float *)o->grad->data, (float *)gx->data);
            continue;
        }
        nck_binary_bwd(k, n->op->kind, which, &bc, (const float *)o->grad->data, (const float *)a->data,
                       (const float *)b->data, (float *)gx->data, sgx, nc_numel(x), acc);
    }
}

#define BINARY_OP(nm, KIND) \
    const nc_op_def nc_op_##nm = {#nm, NC_OPF_ELEMENTWISE, KIND, binary_infer, NULL, binary_fwd, binary_bwd};
BINARY_OP(add, BIN_ADD)
BINARY_OP(sub, BIN_SUB)
BINARY_OP(mul, BIN_MUL)
BINARY_OP(div, BIN_DIV)
#undef BINARY_OP

static nc_tensor *binary(const nc_op_def *op, nc_tensor *a, nc_tensor *b) {
    nc_tensor *in[2] = {a, b};
    return nc__apply(op, in, 2, NULL);
}

nc_tensor *nc_add(nc_tensor *a, nc_tensor *b) { return binary(&nc_op_add, a, b); }
nc_tensor *nc_sub(nc_tensor *a, nc_tensor *b) { return binary(&nc_op_sub, a, b); }
nc_tensor *nc_mul(nc_tensor *a, nc_tensor *b) { return binary(&nc_op_mul, a, b); }
nc_tensor *nc_div(nc_tensor *a, nc_tensor *b) { return binary(&nc_op_div, a, b); }

/* ---- unary -------------------------------------------------------------------------------------- */

static nc_status unary_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    if (!nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    *dt = NC_F32;
    *nd = n->in[0]->ndim;
    memcpy(shape, n->in[0]->shape, sizeof(int64_t) * (size_t)*nd);
    return NC_OK;
}

static nc_status unary_fwd(nc_node *n) {
    /* an activation of a pending BatchNorm output extends its recipe (nothing is computed yet) */
    if (n->out->ctx->fuse && n->out->ctx->fwd_on_tape && nc__defer_act(n->out, n->in[0], n->op->kind, n->p.f[0]))
        return NC_OK;
    /* a scale of pending attention scores joins the chain */
    if (n->op->kind == NCK_UN_SCALE && nc__attn_scale(n, n->p.f[0])) return NC_OK;
    /* without a tape, a GELU output waits for its reader: the int8 linear quantizes it on the fly */
    if ((n->op->kind == NCK_UN_GELU || n->op->kind == NCK_UN_GELU_TANH) && nc__defer_unary(n->out, n->in[0],
                                                                                         n->op->kind, n->p.f[0]))
        return NC_OK;
    const float *x = nc__contig_f32(n->in[0]);
    if (!x) return NC_ERR_OOM;
    nck_unary_fwd(nc__k(n->out->ctx), n->op->kind, n->p.f[0], x, (float *)n->out->data, nc_numel(n->out));
    return NC_OK;
}

static void unary_bwd(nc_node *n) {
    nc_tensor *in = n->in[0];
    const float *x = nc__contig_f32(in);
    int acc;
    nc_tensor *gt = x ? nc__grad_buf_acc(in, &acc) : NULL;
    if (!gt || !x) return;
    nck_unary_bwd(nc__k(in->ctx), n->op->kind, n->p.f[0], x, (const float *)n->out->data,
                  (const float *)n->out->grad->data, (float *)gt->data, acc, nc_numel(in));
}

int nc__unary_kind(const nc_op_def *op) { return op && op->forward == unary_fwd ? op->kind : -1; }

#define UNARY_OP(nm, KIND) \
    const nc_op_def nc_op_##nm = {#nm, NC_OPF_ELEMENTWISE | NC_OPF_RECIPE, KIND, unary_infer, NULL, unary_fwd, \
                                  unary_bwd};
UNARY_OP(neg, NCK_UN_NEG)
UNARY_OP(exp, NCK_UN_EXP)
UNARY_OP(log, NCK_UN_LOG)
UNARY_OP(sqrt, NCK_UN_SQRT)
UNARY_OP(relu, NCK_UN_RELU)
UNARY_OP(sigmoid, NCK_UN_SIGMOID)
UNARY_OP(tanh, NCK_UN_TANH)
UNARY_OP(scale, NCK_UN_SCALE)
UNARY_OP(add_scalar, NCK_UN_ADD_SCALAR)
UNARY_OP(pow_scalar, NCK_UN_POW)
UNARY_OP(leaky_relu, NCK_UN_LEAKY_RELU)
UNARY_OP(relu6, NCK_UN_RELU6)
UNARY_OP(hardsigmoid, NCK_UN_HARDSIGMOID)
UNARY_OP(hardswish, NCK_UN_HARDSWISH)
UNARY_OP(silu, NCK_UN_SILU)
UNARY_OP(gelu, NCK_UN_GELU)
UNARY_OP(gelu_tanh, NCK_UN_GELU_TANH)
#undef UNARY_OP

static nc_tensor *unary(const nc_op_def *op, nc_tensor *x, float s) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.f[0] = s;
    return nc__apply(op, &x, 1, &p);
}

nc_tensor *nc_neg(nc_tensor *x) { return unary(&nc_op_neg, x, 0); }
nc_tensor *nc_exp(nc_tensor *x) { return unary(&nc_op_exp, x, 0); }
nc_tensor *nc_log(nc_tensor *x) { return unary(&nc_op_log, x, 0); }
nc_tensor *nc_sqrt(nc_tensor *x) { return unary(&nc_op_sqrt, x, 0); }
nc_tensor *nc_relu(nc_tensor *x) { return unary(&nc_op_relu, x, 0); }
nc_tensor *nc_sigmoid(nc_tensor *x) { return unary(&nc_op_sigmoid, x, 0); }
nc_tensor *nc_tanh(nc_tensor *x) { return unary(&nc_op_tanh, x, 0); }
nc_tensor *nc_scale(nc_tensor *x, float s) { return unary(&nc_op_scale, x, s); }
nc_tensor *nc_add_scalar(nc_tensor *x, float s) { return unary(&nc_op_add_scalar, x, s); }
nc_tensor *nc_pow_scalar(nc_tensor *x, float p) { return unary(&nc_op_pow_scalar, x, p); }
nc_tensor *nc_leaky_relu(nc_tensor *x, float slope) { return unary(&nc_op_leaky_relu, x, slope); }
nc_tensor *nc_relu6(nc_tensor *x) { return unary(&nc_op_relu6, x, 0); }
nc_tensor *nc_hardsigmoid(nc_tensor *x) { return unary(&nc_op_hardsigmoid, x, 0); }
nc_tensor *nc_hardswish(nc_tensor *x) { return unary(&nc_op_hardswish, x, 0); }
nc_tensor *nc_silu(nc_tensor *x) { return unary(&nc_op_silu, x, 0); }
nc_tensor *nc_gelu(nc_tensor *x, int approximate_tanh) {
    return unary(approximate_tanh ? &nc_op_gelu_tanh : &nc_op_gelu, x, 0);
}

/* ---- compare -------------------------------------------------------------------------------------- */

static nc_status compare_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    for (int k = 0; k < 2; k++) {
        if (n->in[k]->dtype != NC_F32 && n->in[k]->dtype != NC_I32) {
            nc__error(n->in[k]->ctx, NC_ERR_DTYPE, "compare: inputs must be f32 or i32, got %s",
                      nc__dtype_name(n->in[k]->dtype));
            return NC_ERR_DTYPE;
        }
    }
    nc_tensor *a = n->in[0], *b = n->in[1];
    int r = a->ndim > b->ndim ? a->ndim : b->ndim;
    for (int i = 0; i < r; i++) {
        int ia = i - (r - a->ndim), ib = i - (r - b->ndim);
        int64_t da = ia < 0 ? 1 : a->shape[ia], db = ib < 0 ? 1 : b->shape[ib];
        if (da != db && da != 1 && db != 1) {
            char sa[96], sb[96];
            nc__error(a->ctx, NC_ERR_SHAPE, "compare: shapes %s and %s are not broadcastable",
                      nc__shape_str(a->ndim, a->shape, sa, sizeof sa), nc__shape_str(b->ndim, b->shape, sb, sizeof sb));
            return NC_ERR_SHAPE;
        }
        shape[i] = da == 1 ? db : da;
    }
    *dt = NC_I32;
    *nd = r;
    return NC_OK;
}

static nc_status compare_fwd(nc_node *n) {
    nc_tensor *a = n->in[0], *b = n->in[1], *o = n->out;
    nck_bcast bc;
    fill_bcast(&bc, a, b, o);
    nck_compare(nc__k(o->ctx), (int)n->p.i[0], &bc, a->data, a->dtype == NC_I32, b->data, b->dtype == NC_I32,
                (int32_t *)o->data);
    return NC_OK;
}

const nc_op_def nc_op_compare = {"compare", NC_OPF_NONDIFF, 0, compare_infer, NULL, compare_fwd, NULL};

nc_tensor *nc_compare(nc_tensor *a, nc_tensor *b, nc_cmp op) {
    if (a && (a->dtype == NC_U8 || a->dtype == NC_I8)) a = nc_to_dtype(a, NC_I32);
    if (b && (b->dtype == NC_U8 || b->dtype == NC_I8)) b = nc_to_dtype(b, NC_I32);
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = op;
    nc_tensor *in[2] = {a, b};
    return nc__apply(&nc_op_compare, in, 2, &p);
}
