/* Neural-network functional ops: softmax family, cross entropy, NLL, dropout, batch norm, layer
 * norm, masked_fill and the MSE composite.
 *
 * Shapes, error rules, saved state and gradient formulas follow newch engine/src/ops/ops_nn.c
 * (softmax :8-78, cross entropy :84-160, dropout :166-211, batch norm :217-361, NLL :367-426,
 * layer norm :432-534, masked_fill :540-615). Accumulations newch does in double (BN and LN
 * statistics, loss sums) are double on the device too.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>

#include <math.h>

enum { SM_LOG, SM_PLAIN };

static nc_status softmax_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    if (!nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    if (x->ndim < 1) {
        nc__error(x->ctx, NC_ERR_SHAPE, "%s: input must have at least 1 dimension", n->op->name);
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    return NC_OK;
}

static nc_status softmax_fwd(nc_node *n) {
    if (n->op->kind == SM_PLAIN && nc__attn_softmax(n)) return NC_OK; /* attention probabilities: a recipe */
    const float *x = nc__contig_f32(n->in[0]);
    if (!x) return NC_ERR_OOM;
    int64_t C = n->out->shape[n->out->ndim - 1];
    int64_t rows = C ? nc_numel(n->out) / C : 0;
    if (rows) nck_softmax_fwd(nc__k(n->out->ctx), x, (float *)n->out->data, rows, C, n->op->kind == SM_LOG);
    return NC_OK;
}

static void softmax_bwd(nc_node *n) {
    nc_tensor *gt = nc__grad_buf(n->in[0]);
    if (!gt) return;
    int64_t C = n->out->shape[n->out->ndim - 1];
    int64_t rows = C ? nc_numel(n->out) / C : 0;
    if (rows)
        nck_softmax_bwd(nc__k(gt->ctx), (const float *)n->out->data, (const float *)n->out->grad->data,
                        (float *)gt->data, rows, C, n->op->kind == SM_LOG);
}

const nc_op_def nc_op_log_softmax = {"log_softmax", 0, SM_LOG, softmax_infer, NULL, softmax_fwd, softmax_bwd};
const nc_op_def nc_op_softmax = {"softmax", NC_OPF_RECIPE, SM_PLAIN, softmax_infer, NULL, softmax_fwd, softmax_bwd};

nc_tensor *nc_log_softmax(nc_tensor *x) { return nc__apply(&nc_op_log_softmax, &x, 1, NULL); }
nc_tensor *nc_softmax(nc_tensor *x) { return nc__apply(&nc_op_softmax, &x, 1, NULL); }

/* ---- labels ------------------------------------------------------------------------------------- */

/* Checks labels against [0, C) on the host when their host copy is current (labels built from host
 * data always are); otherwise the kernel checks them and reports at the next synchronization. */
static int labels_ok(nc_ctx *ctx, nc_tensor *lab, int64_t C, const char *what) {
    const int32_t *h = (const int32_t *)nc__host_view(lab);
    if (!h) return 1;
    for (int64_t i = 0, N = nc_numel(lab); i < N; i++) {
        if (h[i] < 0 || h[i] >= C) {
            nc__error(ctx, NC_ERR_ARG, "%s: label %d at row %lld outside [0, %lld)", what, h[i], (long long)i,
                      (long long)C);
            return 0;
        }
    }
    return 1;
}

/* ---- cross entropy ------------------------------------------------------------------------------ */

static nc_status ce_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *y = n->in[1];
    (void)shape;
    if (!nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    if (y->dtype != NC_I32) {
        nc__error(x->ctx, NC_ERR_DTYPE, "cross_entropy: labels must be i32");
        return NC_ERR_DTYPE;
    }
    if (x->ndim != 2 || y->ndim != 1 || y->shape[0] != x->shape[0] || x->shape[1] < 1) {
        char sa[96], sb[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "cross_entropy: expected logits [N, C] and labels [N], got %s and %s",
                  nc__shape_str(x->ndim, x->shape, sa, sizeof sa), nc__shape_str(y->ndim, y->shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = 0;
    return NC_OK;
}

typedef struct {
    float *prob;
    const int32_t *lab;
} ce_saved;

static nc_status ce_fwd(nc_node *n) {
    nc_ctx *ctx = n->out->ctx;
    int64_t N = n->in[0]->shape[0], C = n->in[0]->shape[1];
    if (!labels_ok(ctx, n->in[1], C, "cross_entropy")) return NC_ERR_ARG;
    const float *x = nc__contig_f32(n->in[0]);
    const int32_t *lab = (const int32_t *)nc__contig(n->in[1]);
    ce_saved *sv = (ce_saved *)nc__meta_alloc(ctx, sizeof(ce_saved), 0);
    float *prob = (float *)nc__arena_alloc(ctx, (size_t)(N * C) * sizeof(float));
    if (!x || !lab || !sv || !prob) return NC_ERR_OOM;
    nck_cross_entropy_fwd(nc__k(ctx), x, lab, prob, (float *)n->out->data, N, C);
    sv->prob = prob;
    sv->lab = lab;
    n->saved = sv;
    return NC_OK;
}

static void ce_bwd(nc_node *n) {
    nc_tensor *gt = nc__grad_buf(n->in[0]);
    if (!gt) return;
    int64_t N = n->in[0]->shape[0], C = n->in[0]->shape[1];
    const ce_saved *sv = (const ce_saved *)n->saved;
    nck_cross_entropy_bwd(nc__k(gt->ctx), sv->prob, sv->lab, (const float *)n->out->grad->data, (float *)gt->data, N,
                          C);
}

const nc_op_def nc_op_cross_entropy = {"cross_entropy", 0, 0, ce_infer, NULL, ce_fwd, ce_bwd};

nc_tensor *nc_cross_entropy(nc_tensor *logits, nc_tensor *labels) {
    nc_tensor *in[2] = {logits, labels};
    return nc__apply(&nc_op_cross_entropy, in, 2, NULL);
}

nc_tensor *nc_mse_loss(nc_tensor *pred, nc_tensor *target) {
    nc_tensor *d = nc_sub(pred, target);
    return nc_mean(nc_mul(d, d), NC_ALL_AXES, 0);
}

/* ---- dropout ------------------------------------------------------------------------------------ */

static nc_status dropout_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    if (!nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    float p = n->p.f[0];
    if (!(p >= 0.0f && p <= 1.0f)) {
        nc__error(x->ctx, NC_ERR_ARG, "dropout: p must be in [0, 1], got %g", p);
        return NC_ERR_ARG;
    }
    *dt = NC_F32;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    return NC_OK;
}

/* The mask of draw i is element i's, as newch draws one value per element in order
 * (ops_nn.c:182-196). The kernel consumes draws [0, N) of the current stream; the host then skips
 * its own copy of the state past them. The mask is kept as bits (N/8 bytes) for backward. */
static nc_status dropout_fwd(nc_node *n) {
    nc_ctx *ctx = n->out->ctx;
    int64_t N = nc_numel(n->out);
    int64_t words = (N + 31) / 32 + 1;
    if (nc__attn_dropout_ok(n->in[0])) { /* attention probabilities: draw the mask only, extend the recipe */
        uint32_t *bits = NULL;
        if (N && !nc__rng_side_mask(ctx, N, n->p.f[0], &bits)) {
            bits = (uint32_t *)nc__arena_alloc(ctx, (size_t)words * sizeof(uint32_t));
            if (!bits) return NC_ERR_OOM;
            const void *polys = nc__rng_dropout_table(ctx, N);
            nck_dropout_fwd(nc__k(ctx), ctx->rng, NULL, NULL, bits, N, n->p.f[0], polys,
                            polys ? nc__rng_dropout_tabs(ctx) : NULL);
        }
        if (!bits && !(bits = (uint32_t *)nc__arena_alloc(ctx, sizeof(uint32_t)))) return NC_ERR_OOM;
        nc__rng_skip(ctx, (uint64_t)N);
        n->saved = bits;
        if (nc__attn_dropout(n, bits)) return NC_OK;
        nc__error(ctx, NC_ERR_OOM, "dropout: out of host memory");
        return NC_ERR_OOM;
    }
    const float *x = nc__contig_f32(n->in[0]);
    if (!x) return NC_ERR_OOM;
    uint32_t *bits = NULL;
    if (N && nc__rng_side_mask(ctx, N, n->p.f[0], &bits)) { /* mask drawn on the side stream */
        nck_dropout_apply(nc__k(ctx), x, bits, (float *)n->out->data, N, n->p.f[0]);
    } else {
        bits = (uint32_t *)nc__arena_alloc(ctx, (size_t)words * sizeof(uint32_t));
        if (!bits) return NC_ERR_OOM;
        if (N) {
            const void *polys = nc__rng_dropout_table(ctx, N);
            nck_dropout_fwd(nc__k(ctx), ctx->rng, x, (float *)n->out->data, bits, N, n->p.f[0], polys,
                            polys ? nc__rng_dropout_tabs(ctx) : NULL);
        }
    }
    nc__rng_skip(ctx, (uint64_t)N);
    n->saved = bits;
    return NC_OK;
}

static void dropout_bwd(nc_node *n) {
    int acc;
    nc_tensor *gt = nc__grad_buf_acc(n->in[0], &acc);
    if (!gt) return;
    int64_t N = nc_numel(n->out);
    if (N)
        nck_dropout_bwd(nc__k(gt->ctx), (const float *)n->out->grad->data, (const uint32_t *)n->saved,
                        (float *)gt->data, N, n->p.f[0], acc);
}

const nc_op_def nc_op_dropout = {"dropout", NC_OPF_ELEMENTWISE | NC_OPF_RECIPE, 0, dropout_infer, NULL, dropout_fwd,
                                  dropout_bwd};

nc_tensor *nc_dropout(nc_tensor *x, float p) {
    nc_op_params prm;
    memset(&prm, 0, sizeof prm);
    prm.f[0] = p;
    return nc__apply(&nc_op_dropout, &x, 1, &prm);
}

/* ---- batch norm --------------------------------------------------------------------------------- */

typedef struct {
    float *mean, *invstd;
} bn_saved;

static void bn_dims(const nc_tensor *x, int64_t *N, int64_t *C, int64_t *S) {
    *N = x->shape[0];
    *C = x->shape[1];
    *S = 1;
    for (int i = 2; i < x->ndim; i++) *S *= x->shape[i];
}

static nc_status bn_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    for (int i = 0; i < 5; i++)
        if (!nc__expect_f32(n, i)) return NC_ERR_DTYPE;
    if (x->ndim < 2) {
        nc__error(x->ctx, NC_ERR_SHAPE, "batch_norm: expected input [N, C, ...]");
        return NC_ERR_SHAPE;
    }
    int64_t N, C, S;
    bn_dims(x, &N, &C, &S);
    for (int i = 1; i < 5; i++) {
        nc_tensor *t = n->in[i];
        if (t->ndim != 1 || t->shape[0] != C) {
            nc__error(x->ctx, NC_ERR_SHAPE, "batch_norm: weight, bias and running stats must be [%lld]", (long long)C);
            return NC_ERR_SHAPE;
        }
    }
    if (n->p.i[0] && N * S <= 1) {
        nc__error(x->ctx, NC_ERR_SHAPE, "batch_norm: training needs more than 1 value per channel");
        return NC_ERR_SHAPE;
    }
    if (!nc_is_contiguous(n->in[3]) || !nc_is_contiguous(n->in[4])) {
        nc__error(x->ctx, NC_ERR_ARG, "batch_norm: running stats must be contiguous");
        return NC_ERR_ARG;
    }
    *dt = NC_F32;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    return NC_OK;
}

static nc_status bn_fwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    nc_ctx *ctx = x->ctx;
    int64_t N, C, S;
    bn_dims(x, &N, &C, &S);
    const float *X = nc__contig_f32(x), *w = nc__contig_f32(n->in[1]), *b = nc__contig_f32(n->in[2]);
    bn_saved *sv = (bn_saved *)nc__meta_alloc(ctx, sizeof(bn_saved), 0);
    float *stats = (float *)nc__arena_alloc(ctx, (size_t)(2 * C) * sizeof(float));
    if (!X || !w || !b || !sv || !stats) return NC_ERR_OOM;
    sv->mean = stats;
    sv->invstd = stats + C;
    nc_tensor *rm = n->in[3], *rv = n->in[4];
    if (n->p.i[0]) {
        nc__dev_write(rm);
        nc__dev_write(rv);
        float *rmd = (float *)nc__dev(rm), *rvd = (float *)nc__dev(rv);
        const int dp = ctx->dp_world > 1;
        if (dp) {
            /* data parallel: this rank's batch statistics are staged; the running statistics take all
             * ranks' updates in rank order when the step's statistics are gathered */
            float *st = nc__dp_bn_stage(ctx, rmd, rvd, C, n->p.f[0]);
            if (!st) return ctx->status;
            rmd = st, rvd = st + C;
        }
        nck_bn_stats_train(nc__k(ctx), X, sv->mean, sv->invstd, rmd, rvd, N, C, S, n->p.f[0], n->p.f[1], dp);
        if (ctx->fuse && ctx->fwd_on_tape && nc_is_contiguous(x))
            nc__defer_bn(ctx, n->out, x, X, w, b, sv->mean, sv->invstd, N, C, S); /* output left as a recipe */
        else
            nck_bn_apply(nc__k(ctx), X, w, b, sv->mean, sv->invstd, (float *)n->out->data, N, C, S, -1, 0.0f);
    } else {
        if (ctx->bn_n && !nc__dp_bn_flush(ctx, 0)) return ctx->status; /* pending updates reach rm / rv first */
        nck_bn_fwd_eval(nc__k(ctx), X, w, b, (float *)n->out->data, sv->mean, sv->invstd,
                        (const float *)nc__dev(rm), (const float *)nc__dev(rv), N, C, S, n->p.f[1]);
    }
    n->saved = sv;
    return NC_OK;
}

static void bn_bwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    int64_t N, C, S;
    bn_dims(x, &N, &C, &S);
    const bn_saved *sv = (const bn_saved *)n->saved;
    const float *X = nc__contig_f32(x), *w = nc__contig_f32(n->in[1]);
    if (!X || !w) return;
    int acc_gx = 1;
    nc_tensor *gx = nc__needs_grad(x) ? nc__grad_buf_acc(x, &acc_gx) : NULL;
    nc_tensor *gw = nc__needs_grad(n->in[1]) ? nc__grad_buf(n->in[1]) : NULL;
    nc_tensor *gb = nc__needs_grad(n->in[2]) ? nc__grad_buf(n->in[2]) : NULL;
    nck_bn_bwd(nc__k(x->ctx), X, w, (const float *)n->out->grad->data, sv->mean, sv->invstd,
               gx ? (float *)gx->data : NULL, gw ? (float *)gw->data : NULL, gb ? (float *)gb->data : NULL, N, C, S,
               (int)n->p.i[0], acc_gx);
}

const nc_op_def nc_op_batch_norm = {"batch_norm", 0, 0, bn_infer, NULL, bn_fwd, bn_bwd};

nc_tensor *nc_batch_norm(nc_tensor *x, nc_tensor *weight, nc_tensor *bias, nc_tensor *running_mean,
                         nc_tensor *running_var, int training, float momentum, float eps) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = training ? 1 : 0;
    p.f[0] = momentum;
    p.f[1] = eps;
    nc_tensor *in[5] = {x, weight, bias, running_mean, running_var};
    return nc__apply(&nc_op_batch_norm, in, 5, &p);
}

/* ---- nll loss ---------------------------------------------------------------------------------- */

static nc_status nll_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *y = n->in[1];
    (void)shape;
    if (!nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    if (y->dtype != NC_I32) {
        nc__error(x->ctx, NC_ERR_DTYPE, "nll_loss: labels must be i32");
        return NC_ERR_DTYPE;
    }
    if (x->ndim != 2 || y->ndim != 1 || y->shape[0] != x->shape[0]) {
        char sa[96], sb[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "nll_loss: expected log-probabilities [N, C] and labels [N], got %s and %s",
                  nc__shape_str(x->ndim, x->shape, sa, sizeof sa), nc__shape_str(y->ndim, y->shape, sb, sizeof sb));
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = 0;
    return NC_OK;
}

static nc_status nll_fwd(nc_node *n) {
    nc_ctx *ctx = n->out->ctx;
    int64_t N = n->in[0]->shape[0], C = n->in[0]->shape[1];
    if (!labels_ok(ctx, n->in[1], C, "nll_loss")) return NC_ERR_ARG;
    const float *x = nc__contig_f32(n->in[0]);
    const int32_t *lab = (const int32_t *)nc__contig(n->in[1]);
    if (!x || !lab) return NC_ERR_OOM;
    nck_nll_fwd(nc__k(ctx), x, lab, (float *)n->out->data, N, C, (int)n->p.i[0]);
    n->saved = (void *)lab;
    return NC_OK;
}

static void nll_bwd(nc_node *n) {
    nc_tensor *gt = nc__grad_buf(n->in[0]);
    if (!gt) return;
    int64_t N = n->in[0]->shape[0], C = n->in[0]->shape[1];
    nck_nll_bwd(nc__k(gt->ctx), (const int32_t *)n->saved, (const float *)n->out->grad->data, (float *)gt->data, N, C,
                (int)n->p.i[0]);
}

const nc_op_def nc_op_nll_loss = {"nll_loss", 0, 0, nll_infer, NULL, nll_fwd, nll_bwd};

nc_tensor *nc_nll_loss(nc_tensor *logp, nc_tensor *labels, int sum) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = sum ? 1 : 0;
    nc_tensor *in[2] = {logp, labels};
    return nc__apply(&nc_op_nll_loss, in, 2, &p);
}

/* ---- layer norm ------------------------------------------------------------------------------- */

static nc_status layer_norm_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0];
    int k = (int)n->p.i[0];
    for (int i = 0; i < n->n_in; i++)
        if (!nc__expect_f32(n, i)) return NC_ERR_DTYPE;
    if (k < 1 || k > x->ndim) {
        nc__error(x->ctx, NC_ERR_SHAPE, "layer_norm: normalized_shape has %d dims, input only %d", k, x->ndim);
        return NC_ERR_SHAPE;
    }
    int64_t D = nc__shape_numel(k, x->shape + x->ndim - k);
    for (int i = 1; i < n->n_in; i++) {
        if (nc_numel(n->in[i]) != D) {
            nc__error(x->ctx, NC_ERR_SHAPE, "layer_norm: weight/bias need %lld elements, got %lld", (long long)D,
                      (long long)nc_numel(n->in[i]));
            return NC_ERR_SHAPE;
        }
    }
    *dt = NC_F32;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    return NC_OK;
}

static int64_t ln_dim(const nc_node *n) {
    const nc_tensor *x = n->in[0];
    int k = (int)n->p.i[0];
    return nc__shape_numel(k, x->shape + x->ndim - k);
}

static nc_status layer_norm_fwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    int has_w = (int)n->p.i[1], has_b = (int)n->p.i[2];
    const float *w = has_w ? nc__contig_f32(n->in[1]) : NULL;
    const float *b = has_b ? nc__contig_f32(n->in[1 + has_w]) : NULL;
    const float *X = nc__contig_f32(x);
    int64_t D = ln_dim(n), R = D ? nc_numel(x) / D : 0;
    float *stats = (float *)nc__arena_alloc(x->ctx, (size_t)(2 * R + 1) * sizeof(float));
    if (!X || !stats || (has_w && !w) || (has_b && !b)) return NC_ERR_OOM;
    if (R) nck_ln_fwd(nc__k(x->ctx), X, w, b, (float *)n->out->data, stats, R, D, n->p.f[0]);
    n->saved = stats;
    return NC_OK;
}

static void layer_norm_bwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    int has_w = (int)n->p.i[1], has_b = (int)n->p.i[2];
    nc_tensor *wt = has_w ? n->in[1] : NULL, *bt = has_b ? n->in[1 + has_w] : NULL;
    const float *X = nc__contig_f32(x), *w = wt ? nc__contig_f32(wt) : NULL;
    int64_t D = ln_dim(n), R = D ? nc_numel(x) / D : 0;
    if (!X || (wt && !w)) return;
    int acc = 1;  /* the input gradient is written whole: a fresh buffer is stored */
    nc_tensor *gx = nc__needs_grad(x) ? nc__grad_buf_acc(x, &acc) : NULL;
    nc_tensor *gw = wt && nc__needs_grad(wt) ? nc__grad_buf(wt) : NULL;
    nc_tensor *gb = bt && nc__needs_grad(bt) ? nc__grad_buf(bt) : NULL;
    if (R)
        nck_ln_bwd(nc__k(x->ctx), X, w, (const float *)n->out->grad->data, (const float *)n->saved,
                   gx ? (float *)gx->data : NULL, gw ? (float *)gw->data : NULL, gb ? (float *)gb->data : NULL, R, D,
                   acc);
}

const nc_op_def nc_op_layer_norm = {"layer_norm", 0, 0, layer_norm_infer, NULL, layer_norm_fwd, layer_norm_bwd};

nc_tensor *nc_layer_norm(nc_tensor *x, int normalized_ndim, nc_tensor *weight, nc_tensor *bias, float eps) {
    nc_tensor *in[3] = {x, NULL, NULL};
    int k = 1;
    if (weight) in[k++] = weight;
    if (bias) in[k++] = bias;
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = normalized_ndim;
    p.i[1] = weight != NULL;
    p.i[2] = bias != NULL;
    p.f[0] = eps;
    return nc__apply(&nc_op_layer_norm, in, k, &p);
}

/* ---- masked_fill ------------------------------------------------------------------------------- */

static nc_status masked_fill_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *m = n->in[1];
    if (!nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    int ok = m->dtype == NC_I32 && m->ndim <= x->ndim;
    for (int i = 0; ok && i < m->ndim; i++) {
        int64_t dm = m->shape[i], dx = x->shape[x->ndim - m->ndim + i];
        ok = dm == dx || dm == 1;
    }
    if (!ok) {
        char sx[96], sm[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "masked_fill: mask %s %s does not broadcast to input %s",
                  nc__dtype_name(m->dtype), nc__shape_str(m->ndim, m->shape, sm, sizeof sm),
                  nc__shape_str(x->ndim, x->shape, sx, sizeof sx));
        return NC_ERR_SHAPE;
    }
    *dt = NC_F32;
    *nd = x->ndim;
    memcpy(shape, x->shape, sizeof(int64_t) * (size_t)x->ndim);
    return NC_OK;
}

static void mf_bcast(const nc_node *n, nck_bcast *bc, int grad) {
    nc_tensor *x = n->in[0], *m = n->in[1], *o = n->out;
    bc->ndim = o->ndim;
    memcpy(bc->shape, o->shape, sizeof(int64_t) * (size_t)o->ndim);
    if (grad) nc__contig_strides(o->ndim, o->shape, bc->sa);
    else memcpy(bc->sa, x->stride, sizeof(int64_t) * (size_t)o->ndim);
    nc__bcast_strides(m, o->ndim, o->shape, bc->sb);
    nc__contig_strides(o->ndim, o->shape, bc->so);
}

/* Elements of the mask's repeating block when the mask is contiguous over the output's last dims and
 * broadcast over the leading ones (an attention mask), else 0. */
static int64_t mask_tail(const nc_node *n) {
    const nc_tensor *m = n->in[1], *o = n->out;
    if (!nc_is_contiguous(m)) return 0;
    int64_t sb[NC_MAX_DIMS];
    nc__bcast_strides(m, o->ndim, o->shape, sb);
    for (int k = 0; k <= o->ndim; k++) { /* the block is dims k.. of the output */
        int ok = 1;
        for (int i = 0; i < k && ok; i++) ok = sb[i] == 0 || o->shape[i] == 1;
        int64_t step = 1;
        for (int i = o->ndim - 1; i >= k && ok; i--) {
            ok = o->shape[i] == 1 || sb[i] == step;
            step *= o->shape[i];
        }
        if (ok) return step == nc_numel(m) ? step : 0;
    }
    return 0;
}

static nc_status masked_fill_fwd(nc_node *n) {
    if (nc__attn_mask(n)) return NC_OK; /* masked attention scores: a recipe */
    nc_tensor *x = n->in[0];
    nc__dev(x);
    const int64_t tail = nc_is_contiguous(x) ? mask_tail(n) : 0;
    if (tail && nck_masked_fill_tail(nc__k(n->out->ctx), 0, (const float *)x->data, (const int32_t *)n->in[1]->data,
                                     n->p.f[0], (float *)n->out->data, nc_numel(n->out), tail, 0))
        return NC_OK;
    nck_bcast bc;
    mf_bcast(n, &bc, 0);
    nck_masked_fill_fwd(nc__k(n->out->ctx), &bc, (const float *)n->in[0]->data, (const int32_t *)n->in[1]->data,
                        n->p.f[0], (float *)n->out->data);
    return NC_OK;
}

static void masked_fill_bwd(nc_node *n) {
    const int64_t tail = mask_tail(n);
    if (tail) {
        int acc;
        nc_tensor *g = nc__grad_buf_acc(n->in[0], &acc);
        if (g && nck_masked_fill_tail(nc__k(g->ctx), 1, (const float *)n->out->grad->data,
                                      (const int32_t *)n->in[1]->data, 0.0f, (float *)g->data, nc_numel(n->out), tail,
                                      acc))
            return;
        if (g && !acc) nc__cuda_ok(g->ctx, cudaMemsetAsync(g->data, 0, g->bytes, (cudaStream_t)g->ctx->dev.stream),
                                   "memset");
    }
    nc_tensor *gx = nc__grad_buf(n->in[0]);
    if (!gx) return;
    nck_bcast bc;
    mf_bcast(n, &bc, 1);
    nck_masked_fill_bwd(nc__k(gx->ctx), &bc, (const float *)n->out->grad->data, (const int32_t *)n->in[1]->data,
                        (float *)gx->data);
}

const nc_op_def nc_op_masked_fill = {"masked_fill", NC_OPF_RECIPE, 0, masked_fill_infer, NULL, masked_fill_fwd,
                                      masked_fill_bwd};

nc_tensor *nc_masked_fill(nc_tensor *x, nc_tensor *mask, float value) {
    if (mask && mask->dtype != NC_I32) mask = nc_to_dtype(mask, NC_I32);
    nc_tensor *in[2] = {x, mask};
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.f[0] = value;
    return nc__apply(&nc_op_masked_fill, in, 2, &p);
}
