/* 2-D convolution and pooling on NCHW tensors.
 *
 * Geometry, validation and gradients follow newch engine/src/ops/ops_conv.c (geometry :11-40,
 * window checks :42-63, conv infer :146-172, depthwise selection :174, forward :290-316, backward
 * :318-357, pooling :375-509). The schedule is the B200 one:
 *   - depthwise (groups == C == OC) and few-input-channel convolutions run direct kernels;
 *   - 1x1 stride-1 convolutions are plain strided-batch GEMMs on the activations themselves;
 *   - other stride-1 convolutions (groups 1) pack x (and, for the backward, dY) once into a
 *     zero-padded position-major matrix and run Y, dX and dW as tap-shifted tcgen05 GEMMs over it
 *     (nck_convtap: every filter tap is a row shift of the packed matrix, no unfolded copy);
 *   - the rest unfold a chunk of samples at once (im2col over the whole chunk, bounded to 256 MiB)
 *     and run one strided-batch GEMM per group for Y, dX and dW; dW sums over the samples inside
 *     the GEMM, so no atomics and a fixed summation order.
 */
#include "nc_internal.h"

#include <cuda_runtime_api.h>

#include <math.h>
#include <stdio.h>

static int64_t out_size(int64_t in, int64_t k, int s, int p, int d) { return (in + 2 * p - d * (k - 1) - 1) / s + 1; }

static nck_conv geom(const nc_node *n, int64_t kh, int64_t kw, int64_t oc) {
    const nc_tensor *x = n->in[0];
    nck_conv g;
    memset(&g, 0, sizeof g);
    g.N = x->shape[0], g.C = x->shape[1], g.H = x->shape[2], g.W = x->shape[3];
    g.sh = (int)n->p.i[0], g.sw = (int)n->p.i[1], g.ph = (int)n->p.i[2], g.pw = (int)n->p.i[3];
    g.dh = g.dw = 1;
    g.G = 1;
    g.KH = kh, g.KW = kw, g.OC = oc;
    g.OH = out_size(g.H, kh, g.sh, g.ph, 1);
    g.OW = out_size(g.W, kw, g.sw, g.pw, 1);
    return g;
}

static nck_conv conv_geom_of(const nc_node *n) {
    const nc_tensor *w = n->in[1];
    nck_conv g = geom(n, w->shape[2], w->shape[3], w->shape[0]);
    g.dh = (int)n->p.i[4], g.dw = (int)n->p.i[5];
    g.G = n->p.i[6];
    g.OH = out_size(g.H, g.KH, g.sh, g.ph, g.dh);
    g.OW = out_size(g.W, g.KW, g.sw, g.pw, g.dw);
    return g;
}

static nc_status check_window(nc_node *n, int64_t kh, int64_t kw) {
    nc_tensor *x = n->in[0];
    if (n->p.i[0] < 1 || n->p.i[1] < 1 || n->p.i[2] < 0 || n->p.i[3] < 0 || kh < 1 || kw < 1) {
        nc__error(x->ctx, NC_ERR_ARG, "%s: stride must be >= 1, padding >= 0, kernel >= 1", n->op->name);
        return NC_ERR_ARG;
    }
    if (x->ndim != 4) {
        char sx[96];
        nc__error(x->ctx, NC_ERR_SHAPE, "%s: expected input [N, C, H, W], got %s", n->op->name,
                  nc__shape_str(x->ndim, x->shape, sx, sizeof sx));
        return NC_ERR_SHAPE;
    }
    nck_conv g = geom(n, kh, kw, 0);
    if (g.OH < 1 || g.OW < 1) {
        nc__error(x->ctx, NC_ERR_SHAPE, "%s: kernel %lldx%lld does not fit input %lldx%lld with padding %d,%d",
                  n->op->name, (long long)kh, (long long)kw, (long long)g.H, (long long)g.W, g.ph, g.pw);
        return NC_ERR_SHAPE;
    }
    return NC_OK;
}

static nc_status conv_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    for (int i = 0; i < n->n_in; i++)
        if (!nc__expect_f32(n, i)) return NC_ERR_DTYPE;
    int64_t G = n->p.i[6];
    if (G < 1 || n->p.i[4] < 1 || n->p.i[5] < 1) {
        nc__error(x->ctx, NC_ERR_ARG, "conv2d: dilation and groups must be >= 1");
        return NC_ERR_ARG;
    }
    if (w->ndim != 4 || x->ndim != 4 || x->shape[1] != w->shape[1] * G || w->shape[0] % G != 0 ||
        (b && (b->ndim != 1 || b->shape[0] != w->shape[0]))) {
        char sx[96], sw[96];
        nc__error(x->ctx, NC_ERR_SHAPE,
                  "conv2d: expected x [N, C, H, W], weight [OC, C/groups, KH, KW] with OC divisible by groups (%lld), "
                  "bias [OC]; got %s and %s",
                  (long long)G, nc__shape_str(x->ndim, x->shape, sx, sizeof sx),
                  nc__shape_str(w->ndim, w->shape, sw, sizeof sw));
        return NC_ERR_SHAPE;
    }
    nc_status st = check_window(n, n->p.i[4] * (w->shape[2] - 1) + 1, n->p.i[5] * (w->shape[3] - 1) + 1);
    if (st != NC_OK) return st;
    nck_conv g = conv_geom_of(n);
    *dt = NC_F32;
    *nd = 4;
    shape[0] = g.N, shape[1] = g.OC, shape[2] = g.OH, shape[3] = g.OW;
    return NC_OK;
}

/* depthwise layers the shared-memory plane kernels take (others go through the grouped paths) */
static int is_depthwise(const nck_conv *g) { return g->G == g->C && g->OC == g->C && nck_dw_ok(g); }
static int is_pointwise(const nck_conv *g) {
    return g->KH == 1 && g->KW == 1 && g->sh == 1 && g->sw == 1 && g->ph == 0 && g->pw == 0;
}
/* few taps per group: the direct kernels (a 1x1 convolution over 16 or more channels is a GEMM of
 * real depth and goes to the tensor cores instead) */
static int use_direct(const nck_conv *g) {
    return (g->C / g->G) * g->KH * g->KW <= 32 && g->OC / g->G <= 64 && !(is_pointwise(g) && g->C / g->G >= 16);
}

/* samples per im2col chunk: the unfolded buffer stays under 256 MiB */
static int64_t chunk_samples(const nck_conv *g) {
    int64_t per = g->C * g->KH * g->KW * g->OH * g->OW * (int64_t)sizeof(float);
    int64_t nb = per ? ((int64_t)256 << 20) / per : g->N;
    if (nb < 1) nb = 1;
    return nb > g->N ? g->N : nb;
}

/* Y[n, g] = W_g @ X[n, g] (+ bias rows) for samples [n0, n0 + nb); B operand of sample n at B + n * sB */
static void gemm_fwd(nc_ctx *ctx, const nck_conv *g, const float *W, const float *B, int64_t sB, int64_t ldb,
                     const float *bias, float *Y, int64_t nb) {
    int64_t Cg = g->C / g->G, OCg = g->OC / g->G, CKK = Cg * g->KH * g->KW, L = g->OH * g->OW;
    for (int64_t gi = 0; gi < g->G; gi++) {
        nck_gemm_args a;
        memset(&a, 0, sizeof a);
        a.M = OCg, a.N = L, a.K = CKK, a.alpha = 1.0f, a.beta = 0.0f;
        a.A = W + gi * OCg * CKK, a.lda = CKK, a.sA = 0;
        a.B = B + gi * CKK * ldb, a.ldb = ldb, a.sB = sB;
        a.C = Y + gi * OCg * L, a.ldc = L, a.sC = g->OC * L;
        a.batch = nb;
        a.bias = bias ? bias + gi * OCg : NULL;
        a.bias_per_row = 1;
        nck_gemm(nc__k(ctx), &a);
    }
}

/* what the forward left for the backward: x unfolded (whole batch in one chunk) or x packed for the
 * tap-shifted path */
enum { SAVED_COL = 1, SAVED_TAP = 2 };

/* Off the tape nothing keeps the packed input for a backward, so the packed copy (channels padded
 * to 32, two planes for 3xTF32) need not hold the whole batch: samples per pack, keeping the
 * workspace at most half the output's size (4 MiB at least). On the tape the whole batch. */
static int64_t tap_chunk(const nc_ctx *ctx, const nck_conv *g, const nck_tapgeom *tg) {
    if (ctx->fwd_on_tape) return g->N;
    const int64_t per = tg->Hp * tg->Wp * tg->Cp * tg->planes * (int64_t)sizeof(float);
    int64_t budget = g->N * g->OC * g->OH * g->OW * (int64_t)sizeof(float) / 2;
    if (budget < ((int64_t)4 << 20)) budget = (int64_t)4 << 20;
    const int64_t nb = budget / per;
    return nb < 1 ? 1 : nb > g->N ? g->N : nb;
}

/* the tap convolution a chunk of samples at a time through one packed buffer (stream order makes
 * each pack wait for the previous chunk's GEMM); 0 if the tap kernel turned a chunk down, in which
 * case the caller's next path rewrites the whole output */
static int tap_fwd_chunked(nc_ctx *ctx, const nck_conv *g, const nck_tapgeom *tg, const float *X, const float *Wt,
                           const float *B, float *Y) {
    const int64_t nb = tap_chunk(ctx, g, tg);
    float *wp = (float *)nc__arena_alloc(ctx, (size_t)(g->OC * tg->T * tg->Cp * tg->planes) * sizeof(float));
    float *xp = (float *)nc__arena_alloc(ctx, (size_t)(nb * tg->Hp * tg->Wp * tg->Cp * tg->planes) * sizeof(float));
    if (!wp || !xp) return 0;
    nck_tap_pack_w(nc__k(ctx), g, tg, Wt, wp, 0);
    const int64_t xs = g->C * g->H * g->W, ys = g->OC * g->OH * g->OW;
    for (int64_t n0 = 0; n0 < g->N; n0 += nb) {
        nck_conv gc = *g;
        gc.N = g->N - n0 < nb ? g->N - n0 : nb;
        nck_tapgeom tc;
        if (!nck_convtap_plan(nc__k(ctx), &gc, &tc)) return 0;
        nck_tap_pack(nc__k(ctx), X + n0 * xs, gc.N, g->C, g->H, g->W, &tc, g->ph, g->pw, tc.Cp, xp, NULL);
        if (!nck_convtap(nc__k(ctx), 0, &gc, &tc, xp, wp, Y + n0 * ys, B, 0)) return 0;
    }
    return 1;
}
typedef struct {
    int kind;
    float *buf;
} conv_saved;

static nc_status conv_fwd(nc_node *n) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    nc_ctx *ctx = x->ctx;
    nck_conv g = conv_geom_of(n);
    const float *X = nc__contig_f32(x), *Wt = nc__contig_f32(w), *B = b ? nc__contig_f32(b) : NULL;
    if (!X || !Wt || (b && !B)) return NC_ERR_OOM;
    float *Y = (float *)n->out->data;
    if (!g.N) return NC_OK;
    if (is_depthwise(&g)) {
        nck_dw_fwd(nc__k(ctx), &g, X, Wt, B, Y);
        return NC_OK;
    }
    if (use_direct(&g)) {
        nck_conv_direct_fwd(nc__k(ctx), &g, X, Wt, B, Y);
        return NC_OK;
    }
    int64_t L = g.OH * g.OW, HW = g.H * g.W;
    if (is_pointwise(&g)) {
        gemm_fwd(ctx, &g, Wt, X, g.C * HW, HW, B, Y, g.N);
        return NC_OK;
    }
    nck_tapgeom tg;
    if (nck_convtap_plan(nc__k(ctx), &g, &tg) && tap_chunk(ctx, &g, &tg) < g.N) {
        if (tap_fwd_chunked(ctx, &g, &tg, X, Wt, B, Y)) return NC_OK;
    } else if (nck_convtap_plan(nc__k(ctx), &g, &tg)) {
        /* x packed once; the backward's weight gradient reads the same packed copy */
        conv_saved *sv = (conv_saved *)nc__meta_alloc(ctx, sizeof(conv_saved), 0);
        float *xp = (float *)nc__arena_alloc(ctx, (size_t)(tg.Nv * tg.Cp * tg.planes) * sizeof(float));
        float *wp = (float *)nc__arena_alloc(ctx, (size_t)(g.OC * tg.T * tg.Cp * tg.planes) * sizeof(float));
        if (!sv || !xp || !wp) return NC_ERR_OOM;
        nck_tap_pack(nc__k(ctx), X, g.N, g.C, g.H, g.W, &tg, g.ph, g.pw, tg.Cp, xp, NULL);
        nck_tap_pack_w(nc__k(ctx), &g, &tg, Wt, wp, 0);
        if (nck_convtap(nc__k(ctx), 0, &g, &tg, xp, wp, Y, B, 0)) {
            sv->kind = SAVED_TAP, sv->buf = xp;
            n->saved = sv;
            return NC_OK;
        }
    }
    if (nck_conv_implicit(nc__k(ctx), 0, &g, X, Wt, Y, B)) return NC_OK; /* tensor cores, no unfolded copy */
    int64_t CKKL = g.C * g.KH * g.KW * L, nbmax = chunk_samples(&g);
    float *col = (float *)nc__arena_alloc(ctx, (size_t)(nbmax * CKKL) * sizeof(float));
    if (!col) return NC_ERR_OOM;
    for (int64_t n0 = 0; n0 < g.N; n0 += nbmax) {
        int64_t nb = g.N - n0 < nbmax ? g.N - n0 : nbmax;
        nck_im2col(nc__k(ctx), &g, X, col, n0, nb);
        gemm_fwd(ctx, &g, Wt, col, CKKL, L, B, Y + n0 * g.OC * L, nb);
    }
    /* one chunk held the whole batch: the unfolded input stays valid in the step arena until step end
     * and the weight gradient reads it instead of unfolding x again */
    if (nbmax >= g.N) {
        conv_saved *sv = (conv_saved *)nc__meta_alloc(ctx, sizeof(conv_saved), 0);
        if (sv) sv->kind = SAVED_COL, sv->buf = col, n->saved = sv;
    }
    return NC_OK;
}

/* dW_g += sum_n dY[n, g] @ Xcol[n, g]^T over samples of the chunk */
static void gemm_dw(nc_ctx *ctx, const nck_conv *g, const float *G, const float *col, int64_t sB, int64_t ldb,
                    float *gw, int64_t nb) {
    int64_t Cg = g->C / g->G, OCg = g->OC / g->G, CKK = Cg * g->KH * g->KW, L = g->OH * g->OW;
    for (int64_t gi = 0; gi < g->G; gi++) {
        nck_gemm_args a;
        memset(&a, 0, sizeof a);
        a.ta = 0, a.tb = 1, a.M = OCg, a.N = CKK, a.K = L, a.alpha = 1.0f, a.beta = 1.0f;
        a.A = G + gi * OCg * L, a.lda = L, a.sA = g->OC * L;
        a.B = col + gi * CKK * ldb, a.ldb = ldb, a.sB = sB;
        a.C = gw + gi * OCg * CKK, a.ldc = CKK, a.sC = 0;
        a.batch = nb;
        a.reduce_batch = 1;
        nck_gemm(nc__k(ctx), &a);
    }
}

/* dcol[n, g] (or dX directly for 1x1) = W_g^T @ dY[n, g] */
static void gemm_dx(nc_ctx *ctx, const nck_conv *g, const float *W, const float *G, float *dst, int64_t sC,
                    int64_t ldc, float beta, int64_t nb) {
    int64_t Cg = g->C / g->G, OCg = g->OC / g->G, CKK = Cg * g->KH * g->KW, L = g->OH * g->OW;
    for (int64_t gi = 0; gi < g->G; gi++) {
        nck_gemm_args a;
        memset(&a, 0, sizeof a);
        a.ta = 1, a.tb = 0, a.M = CKK, a.N = L, a.K = OCg, a.alpha = 1.0f, a.beta = beta;
        a.A = W + gi * OCg * CKK, a.lda = CKK, a.sA = 0;
        a.B = G + gi * OCg * L, a.ldb = L, a.sB = g->OC * L;
        a.C = dst + gi * CKK * ldc, a.ldc = ldc, a.sC = sC;
        a.batch = nb;
        nck_gemm(nc__k(ctx), &a);
    }
}

/* a fresh (not zero-filled) gradient buffer about to be added into: zero it first */
static void zero_if_fresh(nc_ctx *ctx, nc_tensor *gt, int *acc) {
    if (*acc) return;
    nc__cuda_ok(ctx, cudaMemsetAsync(gt->data, 0, gt->bytes, (cudaStream_t)ctx->dev.stream), "memset");
    *acc = 1;
}

static void conv_bwd(nc_node *n) {
    nc_tensor *x = n->in[0], *w = n->in[1], *b = n->n_in > 2 ? n->in[2] : NULL;
    nc_ctx *ctx = x->ctx;
    nck_conv g = conv_geom_of(n);
    const float *G = (const float *)n->out->grad->data;
    const float *X = nc__contig_f32(x), *Wt = nc__contig_f32(w);
    if (!X || !Wt) return;
    int acc_gx = 1; /* 0: gx is a fresh buffer, not zero-filled, that the path below must store whole */
    nc_tensor *gx = nc__needs_grad(x) ? nc__grad_buf_acc(x, &acc_gx) : NULL;
    nc_tensor *gw = nc__needs_grad(w) ? nc__grad_buf(w) : NULL;
    nc_tensor *gb = b && nc__needs_grad(b) ? nc__grad_buf(b) : NULL;
    int64_t L = g.OH * g.OW, HW = g.H * g.W;
    if (!g.N) return;
    /* the bias gradient (channel sums of dY) rides along with a pass that reads all of dY anyway: the
     * direct 3x3 weight gradient, or the packing of dY for the tap-shifted path; else its own pass */
    nck_tapgeom tg;
    const int direct_dw = gw && use_direct(&g) && !is_depthwise(&g);
    const int tap = !is_depthwise(&g) && !is_pointwise(&g) && ((gw && !direct_dw) || gx) &&
                    nck_convtap_plan(nc__k(ctx), &g, &tg);
    float *gb_direct = gb && direct_dw && nck_conv_direct_dw_bias_ok(&g) ? (float *)gb->data : NULL;
    float *gb_tap = gb && !gb_direct && tap && nck_tap_pack_colsum_ok(nc__k(ctx), &tg, tg.OCp) ? (float *)gb->data : NULL;
    /* depthwise: the weight-gradient pass also sums the bias gradient */
    float *gb_dw = gb && gw && is_depthwise(&g) ? (float *)gb->data : NULL;
    if (gb && !gb_direct && !gb_tap && !gb_dw) nck_conv_bias_grad(nc__k(ctx), G, (float *)gb->data, g.N, g.OC, L);
    if (is_depthwise(&g)) {
        if (gx) nck_dw_dx(nc__k(ctx), &g, G, Wt, (float *)gx->data, acc_gx);
        if (gw) nck_dw_dw(nc__k(ctx), &g, X, G, (float *)gw->data, gb_dw);
        return;
    }
    if (gw && use_direct(&g)) {
        /* few taps per group: dW straight from x and dY, no unfolded copy */
        nck_conv_direct_dw(nc__k(ctx), &g, X, G, (float *)gw->data, gb_direct);
        gw = NULL;
        if (!gx) return;
    }
    const conv_saved *sv = (const conv_saved *)n->saved;
    if (tap) {
        /* dY packed once on the padded grid of x; dW against the packed x the forward left, dX from
         * the shifted dY rows */
        float *gp = (float *)nc__arena_alloc(ctx, (size_t)(tg.Nv * tg.OCp * tg.planes) * sizeof(float));
        if (!gp) return;
        nck_tap_pack(nc__k(ctx), G, g.N, g.OC, g.OH, g.OW, &tg, 0, 0, tg.OCp, gp, gb_tap);
        if (gw) {
            float *xp = sv && sv->kind == SAVED_TAP ? sv->buf : NULL;
            if (!xp) {
                xp = (float *)nc__arena_alloc(ctx, (size_t)(tg.Nv * tg.Cp * tg.planes) * sizeof(float));
                if (!xp) return;
                nck_tap_pack(nc__k(ctx), X, g.N, g.C, g.H, g.W, &tg, g.ph, g.pw, tg.Cp, xp, NULL);
            }
            if (nck_convtap(nc__k(ctx), 2, &g, &tg, xp, gp, (float *)gw->data, NULL, 1)) gw = NULL;
        }
        if (gx) {
            float *wp = (float *)nc__arena_alloc(ctx, (size_t)(g.C * tg.T * tg.OCp * tg.planes) * sizeof(float));
            if (!wp) return;
            nck_tap_pack_w(nc__k(ctx), &g, &tg, Wt, wp, 1);
            if (nck_convtap(nc__k(ctx), 1, &g, &tg, gp, wp, (float *)gx->data, NULL, acc_gx)) gx = NULL;
        }
        if (!gw && !gx) return;
    }
    if (!is_pointwise(&g)) {
        /* tensor cores straight from x and dY (dX for unit strides); what is not handled here takes
         * the unfolded path below */
        if (gw && nck_conv_implicit(nc__k(ctx), 2, &g, X, G, (float *)gw->data, NULL)) gw = NULL;
        if (gx && !acc_gx && nck_conv_implicit_supported(nc__k(ctx), 1, &g)) zero_if_fresh(ctx, gx, &acc_gx);
        if (gx && nck_conv_implicit(nc__k(ctx), 1, &g, G, Wt, (float *)gx->data, NULL)) gx = NULL;
        if (!gw && !gx) return;
    }
    if (is_pointwise(&g)) {
        if (gw) gemm_dw(ctx, &g, G, X, g.C * HW, HW, (float *)gw->data, g.N);
        if (gx) gemm_dx(ctx, &g, Wt, G, (float *)gx->data, g.C * HW, HW, acc_gx ? 1.0f : 0.0f, g.N);
        return;
    }
    int64_t CKKL = g.C * g.KH * g.KW * L, nbmax = chunk_samples(&g);
    const float *fwd_col = nbmax >= g.N && sv && sv->kind == SAVED_COL ? sv->buf : NULL; /* x unfolded by the forward */
    if (gw && fwd_col) {
        gemm_dw(ctx, &g, G, fwd_col, CKKL, L, (float *)gw->data, g.N);
        gw = NULL;
        if (!gx) return;
    }
    float *col = (float *)nc__arena_alloc(ctx, (size_t)(nbmax * CKKL) * sizeof(float));
    if (!col) return;
    for (int64_t n0 = 0; n0 < g.N; n0 += nbmax) {
        int64_t nb = g.N - n0 < nbmax ? g.N - n0 : nbmax;
        if (gw) {
            nck_im2col(nc__k(ctx), &g, X, col, n0, nb);
            gemm_dw(ctx, &g, G + n0 * g.OC * L, col, CKKL, L, (float *)gw->data, nb);
        }
        if (gx) {
            gemm_dx(ctx, &g, Wt, G + n0 * g.OC * L, col, CKKL, L, 0.0f, nb);
            nck_col2im(nc__k(ctx), &g, col, (float *)gx->data, n0, nb, acc_gx);
        }
    }
}

const nc_op_def nc_op_conv2d = {"conv2d", 0, 0, conv_infer, NULL, conv_fwd, conv_bwd};

nc_tensor *nc_conv2d_ex(nc_tensor *x, nc_tensor *weight, nc_tensor *bias, int stride_h, int stride_w, int pad_h,
                        int pad_w, int dilation_h, int dilation_w, int groups) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = stride_h, p.i[1] = stride_w, p.i[2] = pad_h, p.i[3] = pad_w;
    p.i[4] = dilation_h, p.i[5] = dilation_w, p.i[6] = groups;
    nc_tensor *in[3] = {x, weight, bias};
    return nc__apply(&nc_op_conv2d, in, bias ? 3 : 2, &p);
}

nc_tensor *nc_conv2d(nc_tensor *x, nc_tensor *weight, nc_tensor *bias, int stride_h, int stride_w, int pad_h,
                     int pad_w) {
    return nc_conv2d_ex(x, weight, bias, stride_h, stride_w, pad_h, pad_w, 1, 1, 1);
}

/* ---- pooling ------------------------------------------------------------------------------------- */

enum { POOL_MAX, POOL_AVG };

static nc_status pool_infer(nc_node *n, nc_dtype *dt, int *nd, int64_t *shape) {
    if (!nc__expect_f32(n, 0)) return NC_ERR_DTYPE;
    int64_t kh = n->p.i[4], kw = n->p.i[5];
    nc_status st = check_window(n, kh, kw);
    if (st != NC_OK) return st;
    if (n->p.i[2] * 2 > kh || n->p.i[3] * 2 > kw) {
        nc__error(n->in[0]->ctx, NC_ERR_ARG, "%s: padding must be at most half the kernel size", n->op->name);
        return NC_ERR_ARG;
    }
    nck_conv g = geom(n, kh, kw, 0);
    *dt = NC_F32;
    *nd = 4;
    shape[0] = g.N, shape[1] = g.C, shape[2] = g.OH, shape[3] = g.OW;
    return NC_OK;
}

/* 2 x 2 / stride 2 max pooling straight from the pending recipe of its input (BatchNorm and maybe
 * an activation, fusion.c): returns 1 when it did the pooling */
/* 2 x 2 / stride 2 max pooling of a pending BatchNorm (+ activation) output, straight from its input:
 * the saved buffer holds the argmax and, after it, the input value there (for the fused backward) */
static int pool_from_recipe(nc_node *n) {
    nc_tensor *x = n->in[0];
    const nc_deferred *d = nc__deferred_of(x);
    const int64_t *p = n->p.i;
    if (!d || d->kind != NC_DEF_BN || x->ndim != 4 || p[0] != 2 || p[1] != 2 || p[2] != 0 || p[3] != 0 || p[4] != 2 ||
        p[5] != 2)
        return 0;
    if (!nck_bn_pool2x2_ok(x->shape[0], x->shape[1], x->shape[2], x->shape[3])) return 0;
    const int64_t L = nc_numel(n->out);
    int32_t *arg = (int32_t *)nc__arena_alloc(x->ctx, (size_t)L * (sizeof(int32_t) + sizeof(float)));
    if (!arg) return 0;
    n->saved = arg;
    nck_bn_act_pool2x2(nc__k(x->ctx), d->x, d->w, d->b, d->mean, d->invstd, d->act, d->act_s, (float *)n->out->data,
                       arg, (float *)(arg + L), x->shape[0], x->shape[1], x->shape[2], x->shape[3]);
    return 1;
}

const float *nc__pool_xarg(const nc_node *n) {
    return n->op == &nc_op_max_pool2d && n->saved && n->p.i[6] == 1 ? (const float *)((const int32_t *)n->saved +
                                                                                       nc_numel(n->out))
                                                                    : NULL;
}

static nc_status pool_fwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    nck_conv g = geom(n, n->p.i[4], n->p.i[5], 0);
    int is_max = n->op->kind == POOL_MAX;
    int32_t *arg = NULL;
    if (is_max) {
        if (nc_numel(n->out) && pool_from_recipe(n)) {
            n->p.i[6] = 1; /* saved: argmax, then x there */
            return NC_OK;
        }
        arg = (int32_t *)nc__arena_alloc(x->ctx, (size_t)nc_numel(n->out) * sizeof(int32_t));
        if (!arg) return NC_ERR_OOM;
        n->saved = arg;
    }
    const float *X = nc__contig_f32(x);
    if (!X) return NC_ERR_OOM;
    if (nc_numel(n->out)) nck_pool_fwd(nc__k(x->ctx), &g, X, (float *)n->out->data, arg, is_max);
    return NC_OK;
}

static void pool_bwd(nc_node *n) {
    nc_tensor *x = n->in[0];
    int acc;
    nc_tensor *gt = nc__grad_buf_acc(x, &acc);
    if (!gt) return;
    nck_conv g = geom(n, n->p.i[4], n->p.i[5], 0);
    if (nc_numel(n->out))
        nck_pool_bwd(nc__k(x->ctx), &g, (const float *)n->out->grad->data, (const int32_t *)n->saved,
                     (float *)gt->data, n->op->kind == POOL_MAX, acc);
    else if (!acc)
        zero_if_fresh(x->ctx, gt, &acc);
}

const nc_op_def nc_op_max_pool2d = {"max_pool2d", NC_OPF_RECIPE, POOL_MAX, pool_infer, NULL, pool_fwd, pool_bwd};
const nc_op_def nc_op_avg_pool2d = {"avg_pool2d", 0, POOL_AVG, pool_infer, NULL, pool_fwd, pool_bwd};

static nc_tensor *pool(const nc_op_def *op, nc_tensor *x, int kh, int kw, int sh, int sw, int ph, int pw) {
    nc_op_params p;
    memset(&p, 0, sizeof p);
    p.i[0] = sh, p.i[1] = sw, p.i[2] = ph, p.i[3] = pw, p.i[4] = kh, p.i[5] = kw;
    return nc__apply(op, &x, 1, &p);
}

nc_tensor *nc_max_pool2d(nc_tensor *x, int k_h, int k_w, int stride_h, int stride_w, int pad_h, int pad_w) {
    return pool(&nc_op_max_pool2d, x, k_h, k_w, stride_h, stride_w, pad_h, pad_w);
}

nc_tensor *nc_avg_pool2d(nc_tensor *x, int k_h, int k_w, int stride_h, int stride_w, int pad_h, int pad_w) {
    return pool(&nc_op_avg_pool2d, x, k_h, k_w, stride_h, stride_w, pad_h, pad_w);
}
