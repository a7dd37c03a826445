/* Launch interface between the C11 host engine and the sm_100a kernels.
 *
 * Plain C: every launcher takes the device context (stream, status word, SM count) and raw device
 * pointers with sizes. Nothing here knows about tensors, autograd or the arena. Each launcher
 * enqueues its kernels on d->stream and adds the number of kernels it launched to d->launches.
 * Sizes are int64 element counts unless noted. Launchers never synchronize.
 */
#ifndef NCK_H
#define NCK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nck_timer nck_timer;

typedef struct nck_dev {
    void *stream;      /* cudaStream_t */
    int *status;       /* device word: first kernel-detected error code (0 = ok) */
    int *status_host;  /* pinned mirror read at sync points */
    int device;
    int sm_count;
    int64_t launches;  /* kernels enqueued so far */
    int gemm_mode;     /* NCK_GEMM_* */
    int conv_implicit; /* 1: convolutions try the implicit-GEMM kernels before unfolding (NC_CONV=implicit) */
    int conv_tap;      /* 1: stride-1 convolutions run as tap-shifted GEMMs (default; NC_CONV=unfolded|implicit: 0) */
    int gemm_small;    /* 1: small products take the one-thread / one-warp-per-output kernels (NC_GEMM_SMALL=0: off) */
    int qgemm_tc;      /* 1: int8 GEMMs on tcgen05 kind::i8 where TMA allows (NC_QGEMM=dp4a: CUDA cores) */
    int bn_bulk_stage; /* bulk-fed BatchNorm reductions: stage bytes; < 0: statistics of planes >= 4 KiB only
                        * (the default); 0: none (NC_BN_BULK=0) */
    int math_mode;     /* NCK_MATH_*: how exp / sigmoid / tanh / erf are evaluated */
    nck_timer *timer;  /* per-kernel CUDA-event timing, NULL when off */
    void *scratch;     /* device scratch for split reductions (owned by the context) */
    unsigned *counters; /* device counters for last-block-finishes reductions; each user leaves it at 0 */
    size_t scratch_bytes;
} nck_dev;

/* kernel-detected error codes written to *status (first one wins) */
enum { NCK_OK = 0, NCK_ERR_INDEX = 1, NCK_ERR_LABEL = 2, NCK_ERR_PIPELINE = 3, NCK_ERR_LAUNCH = 4 };

enum { NCK_GEMM_FFMA = 0, NCK_GEMM_TF32 = 1, NCK_GEMM_3XTF32 = 2 };

/* NCK_MATH_POLY: newch's AVX2-tier polynomials (bit-identical to that tier; the default);
 * NCK_MATH_LIBM: CUDA's libm functions, as newch's reference tier calls the C library
 * (force_reference, or NC_MATH=libm). The values equal nck::MATH_POLY / MATH_LIBM (k_math.cuh). */
enum { NCK_MATH_POLY = 0, NCK_MATH_LIBM = 1 };

/* ---- timing (bench instrumentation) ------------------------------------------------------ */
void nck_timer_enable(nck_dev *d, int on);
/* flops / bytes: the algorithmic work of the launches in this scope (0 when not accounted) */
void nck_timer_begin(nck_dev *d, const char *name, double flops, double bytes);
void nck_timer_end(nck_dev *d);
/* total milliseconds and launch count for kernels whose name starts with `prefix` ("" = all) */
int nck_timer_query(nck_dev *d, const char *prefix, double *ms, int64_t *count);
/* algorithmic work recorded for those kernels */
int nck_timer_work(nck_dev *d, const char *prefix, double *flops, double *bytes);
/* name, total ms, launches, flops, bytes of timed kernel class i (0 .. n-1); returns 0 past the end */
int nck_timer_entry(nck_dev *d, int i, const char **name, double *ms, int64_t *count, double *flops,
                    double *bytes);
void nck_timer_reset(nck_dev *d);

/* ---- memory helpers ---------------------------------------------------------------------- */
void nck_fill_f32(nck_dev *d, float *y, float v, int64_t n);
void nck_fill_i32(nck_dev *d, int32_t *y, int32_t v, int64_t n);
void nck_add_scalar_inplace(nck_dev *d, float *y, float v); /* y[0] += v */
/* y[i] += a * x[i] */
void nck_axpy(nck_dev *d, int64_t n, float a, const float *x, float *y);
/* y = a * x (the first writer of a fresh gradient buffer) */
void nck_axpy_set(nck_dev *d, int64_t n, float a, const float *x, float *y);
/* dst (contiguous, element size es) = src viewed through shape/stride (elements) */
void nck_copy_strided(nck_dev *d, int es, int ndim, const int64_t *shape, const int64_t *stride, const void *src,
                      void *dst);
/* dst viewed through shape/dst_stride += src (contiguous): backward of a strided view */
void nck_acc_strided(nck_dev *d, int ndim, const int64_t *shape, const int64_t *dst_stride, const float *src,
                     float *dst, int acc); /* acc 0: every strided element is stored, not added */
/* dtype conversion (reference dtype codes: 0 f32, 1 i32, 3 i8, 4 u8); saturating, NaN -> 0 */
void nck_convert(nck_dev *d, int from, int to, const void *src, void *dst, int64_t n);

/* Gradient launchers with an `acc` argument: acc = 1 adds into the gradient buffer; acc = 0 means the
 * buffer was handed over without zero-filling (a fresh gradient) and the launcher stores every
 * element (or zero-fills first when its kernel only touches some). */

/* ---- elementwise --------------------------------------------------------------------------- */
enum {
    NCK_UN_NEG, NCK_UN_EXP, NCK_UN_LOG, NCK_UN_SQRT, NCK_UN_RELU, NCK_UN_SIGMOID, NCK_UN_TANH, NCK_UN_SCALE,
    NCK_UN_ADD_SCALAR, NCK_UN_POW, NCK_UN_LEAKY_RELU, NCK_UN_RELU6, NCK_UN_HARDSIGMOID, NCK_UN_HARDSWISH,
    NCK_UN_SILU, NCK_UN_GELU, NCK_UN_GELU_TANH
};
void nck_unary_fwd(nck_dev *d, int kind, float s, const float *x, float *y, int64_t n);
/* gi += g * d/dx f(x) (y = f(x) for kinds that use it) */
void nck_unary_bwd(nck_dev *d, int kind, float s, const float *x, const float *y, const float *g, float *gi, int acc,
                   int64_t n);

enum { NCK_BIN_ADD, NCK_BIN_SUB, NCK_BIN_MUL, NCK_BIN_DIV };
#define NCK_MAXD 6
typedef struct {
    int ndim;
    int64_t shape[NCK_MAXD];
    int64_t sa[NCK_MAXD], sb[NCK_MAXD], so[NCK_MAXD]; /* element strides, 0 = broadcast */
} nck_bcast;
void nck_binary_fwd(nck_dev *d, int kind, const nck_bcast *bc, const float *a, const float *b, float *o);
/* same-shape contiguous fast path */
void nck_binary_fwd_flat(nck_dev *d, int kind, const float *a, const float *b, float *o, int64_t n);
/* gradient of input `which` (0 = a, 1 = b) accumulated into gx whose shape broadcasts to bc->shape;
 * gx_stride gives gx's strides over the output dims (0 on broadcast dims). g is contiguous. */
void nck_binary_bwd(nck_dev *d, int kind, int which, const nck_bcast *bc, const float *g, const float *a,
                    const float *b, float *gx, const int64_t *gx_stride, int64_t gx_numel, int acc);
/* compare: a, b f32 or i32 (type flags), result i32 */
void nck_compare(nck_dev *d, int op, const nck_bcast *bc, const void *a, int a_i32, const void *b, int b_i32,
                 int32_t *o);
/* out = mask ? v : x with mask i32 broadcast (strides in bc->sb), x strides in bc->sa, out contiguous */
/* masked_fill when x and the output are contiguous and the mask covers the last dims (Mn elements)
 * repeated over the leading ones: bwd 0: o = mask ? v : x; bwd 1: o (+ when acc)= mask ? 0 : x.
 * Returns 0 (nothing launched) when the sizes do not fit it. */
int nck_masked_fill_tail(nck_dev *d, int bwd, const float *x, const int32_t *m, float v, float *o, int64_t n,
                         int64_t Mn, int acc);
void nck_masked_fill_fwd(nck_dev *d, const nck_bcast *bc, const float *x, const int32_t *m, float v, float *o);
void nck_masked_fill_bwd(nck_dev *d, const nck_bcast *bc, const float *g, const int32_t *m, float *gx);

/* ---- reductions ---------------------------------------------------------------------------- */
/* y[n] (n < n1) or y2[n - n1] (n >= n1) += sum over r < splits of part[r * ldp + n], in a fixed order
 * (the combine step of split column reductions) */
void nck_combine_cols(nck_dev *d, const float *part, int64_t ldp, int splits, int64_t N, float *y, int64_t n1,
                      float *y2);
/* x viewed as [outer, R, inner], contiguous. mean: scale = 1/R. */
void nck_reduce_sum(nck_dev *d, const float *x, float *y, int64_t outer, int64_t R, int64_t inner, float scale);
void nck_reduce_sum_i32(nck_dev *d, const int32_t *x, int32_t *y, int64_t outer, int64_t R, int64_t inner);
/* max value (may be NULL) and first argmax index */
void nck_reduce_max(nck_dev *d, const float *x, float *y, int32_t *arg, int64_t outer, int64_t R, int64_t inner);
/* gy[n] += sum_m x[m, n] for a contiguous [M, N] matrix (bias gradients) */
void nck_colsum_acc(nck_dev *d, const float *x, float *gy, int64_t M, int64_t N);
/* gy[n] += sum over m of x[m * ld + n], one launch (for matrices of a few million elements at most) */
void nck_colsum_ld(nck_dev *d, const float *x, int64_t ld, float *gy, int64_t M, int64_t N);
void nck_reduce_sum_bwd(nck_dev *d, const float *g, float *gi, int64_t outer, int64_t R, int64_t inner,
                        float scale, int acc); /* acc == 0: gi is fresh and is stored */
void nck_reduce_max_bwd(nck_dev *d, const float *g, const int32_t *arg, float *gi, int64_t outer, int64_t R,
                        int64_t inner);
/* fills *out (double, device) with sum of squares of n floats; accumulates when `accumulate` */
void nck_sumsq(nck_dev *d, const float *x, int64_t n, double *out, int accumulate);

/* ---- nn ------------------------------------------------------------------------------------- */
/* rows x C, contiguous. log_form: log-softmax. */
void nck_softmax_fwd(nck_dev *d, const float *x, float *y, int64_t rows, int64_t C, int log_form);
void nck_softmax_bwd(nck_dev *d, const float *y, const float *g, float *gi, int64_t rows, int64_t C, int log_form);
/* cross entropy: prob = softmax rows (saved), loss = mean -log p[label] (double accumulation) */
void nck_cross_entropy_fwd(nck_dev *d, const float *x, const int32_t *lab, float *prob, float *loss, int64_t N,
                           int64_t C);
void nck_cross_entropy_bwd(nck_dev *d, const float *prob, const int32_t *lab, const float *gloss, float *gi,
                           int64_t N, int64_t C);
void nck_nll_fwd(nck_dev *d, const float *x, const int32_t *lab, float *loss, int64_t N, int64_t C, int sum);
void nck_nll_bwd(nck_dev *d, const int32_t *lab, const float *gloss, float *gi, int64_t N, int64_t C, int sum);
/* inverted dropout with the engine's xoshiro256** stream: draw i (0-based from `state`) decides element i;
 * x = y = NULL draws the keep mask only */
/* polys: the device table of run polynomials (nck_rng_polys) or NULL to jump by matrices; tabs: the
 * launch's Horner window tables built by the host (NULL: a one-block kernel builds them first) */
void nck_dropout_fwd(nck_dev *d, const uint64_t state[4], const float *x, float *y, uint32_t *bits, int64_t n,
                     float p, const void *polys, const void *tabs);
/* device copy of x^(64 k) mod P for k < count from the host table (uploaded once, grown on demand) */
const void *nck_rng_polys(nck_dev *d, const uint64_t *host, int64_t count);
void nck_dropout_bwd(nck_dev *d, const float *g, const uint32_t *bits, float *gi, int64_t n, float p, int acc);
/* y = x * (keep ? 1 / (1 - p) : 0) from a keep mask drawn by nck_dropout_fwd (x = y = NULL) */
void nck_dropout_apply(nck_dev *d, const float *x, const uint32_t *bits, float *y, int64_t n, float p);

/* Attention over B independent heads: scores S = Q K^T (FFMA, d in order), masked_fill where the mask is
 * nonzero, row softmax, inverted dropout, and the product with V. Operands are strided views, element
 * (b, r, c) at p[b * s[0] + r * s[1] + c * s[2]]; the mask is broadcast by zero strides. stage says how
 * far along the chain the probabilities are: a materialisation writes that tensor, and the products
 * use it as their left operand. */
enum { NCK_ATT_SCORES = 0, NCK_ATT_MASKED = 1, NCK_ATT_SOFTMAX = 2, NCK_ATT_DROPOUT = 3 };
typedef struct {
    const float *q, *k, *v;   /* q (b, i, d), k (b, j, d), v (b, j, e) */
    int64_t qs[3], ks[3], vs[3];
    const int32_t *mask;      /* (b, i, j): nonzero -> fill; NULL = no mask */
    int64_t ms[3];
    float fill;
    const uint32_t *bits;     /* dropout keep bits of element (b * L + i) * S + j */
    float p;
    float scale;              /* scaled: the scores are multiplied by scale before the mask */
    int scaled;
    int64_t B, L, S, D, Dv;
    int stage;
} nck_attn;
/* shapes the fused kernels take: L, S <= 128, D, Dv <= 32 */
int nck_attn_ok(int64_t L, int64_t S, int64_t D, int64_t Dv);
/* o [B, L, Dv] = probs(stage) @ V */
void nck_attn_fwd(nck_dev *d, const nck_attn *a, float *o);
/* out [B, L, S] = the chain's tensor at a->stage */
void nck_attn_probs(nck_dev *d, const nck_attn *a, float *out);
/* Gradients of o = probs @ V given dO [B, L, Dv] (contiguous): dq [B, L, D], dkt [B, D, S] (K^T's
 * layout), dv [B, S, Dv], each contiguous, NULL when not wanted, added to when its acc flag is set.
 * The probabilities are recomputed, so they equal the forward's. */
void nck_attn_bwd(nck_dev *d, const nck_attn *a, const float *dout, float *dq, int acc_q, float *dkt, int acc_k,
                  float *dv, int acc_v);
/* one-time upload of the xoshiro256** jump tables (host-computed) */
int nck_rng_tables_upload(nck_dev *d, const uint64_t *tables, size_t bytes);

/* batch norm over x [N, C, S] */
/* activations a BatchNorm epilogue applies (piecewise: ReLU, ReLU6, leaky ReLU, hardsigmoid,
 * hardswish); -1 = none */
static inline int nck_epi_supported(int kind) {
    return kind < 0 || kind == NCK_UN_RELU || kind == NCK_UN_RELU6 || kind == NCK_UN_LEAKY_RELU ||
           kind == NCK_UN_HARDSIGMOID || kind == NCK_UN_HARDSWISH;
}
/* BatchNorm statistics only (training): mean, invstd and running statistics (see stage) */
void nck_bn_stats_train(nck_dev *d, const float *x, float *mean, float *invstd, float *rm, float *rv, int64_t N,
                        int64_t C, int64_t S, float mom, float eps, int stage);
/* y = act(x * w * invstd + (b - mean * w * invstd)) per channel; act = NCK_UN_* kind or -1 (none) */
void nck_bn_apply(nck_dev *d, const float *x, const float *w, const float *b, const float *mean, const float *invstd,
                  float *y, int64_t N, int64_t C, int64_t S, int act, float act_s);
/* BatchNorm (given statistics) + activation + 2 x 2 / stride 2 max pooling in one pass (even H, W);
 * xarg (may be NULL) receives x at each window's argmax, for the fused backward's sums */
int nck_bn_pool2x2_ok(int64_t N, int64_t C, int64_t H, int64_t W);
void nck_bn_act_pool2x2(nck_dev *d, const float *x, const float *w, const float *b, const float *mean,
                        const float *invstd, int act, float act_s, float *y, int32_t *arg, float *xarg, int64_t N,
                        int64_t C, int64_t H, int64_t W);
/* backward of act(BatchNorm(x)) given the activation output's gradient g (act < 0: plain BatchNorm) */
void nck_bn_bwd_ex(nck_dev *d, const float *x, const float *w, const float *b, const float *g, const float *mean,
                   const float *invstd, float *gx, float *gw, float *gb, int64_t N, int64_t C, int64_t S, int training,
                   int acc_gx, int act, float act_s);
/* backward of max_pool2x2(act(BatchNorm(x))) given the pooled gradient and argmax (training); xarg:
 * the forward's x at the argmax (NULL: gathered from x) */
void nck_bn_pool_bwd(nck_dev *d, const float *x, const float *w, const float *b, const float *gpool,
                     const int32_t *arg, const float *xarg, const float *mean, const float *invstd, float *gx,
                     float *gw, float *gb, int64_t N, int64_t C, int64_t H, int64_t W, int acc_gx, int act,
                     float act_s);
void nck_bn_fwd_train(nck_dev *d, const float *x, const float *w, const float *b, float *y, float *mean,
                      float *invstd, float *rm, float *rv, int64_t N, int64_t C, int64_t S, float mom, float eps,
                      int stage);
/* data-parallel BatchNorm: a forward's staged statistics at off (means, then C unbiased variances) */
typedef struct {
    int64_t off;
    float mom;
    int32_t pad;
} nck_bn_staged;
/* one running-statistics pair and its staged forwards [e0, e1) */
typedef struct {
    float *rm, *rv;
    int64_t C;
    int32_t e0, e1;
} nck_bn_group;
void nck_bn_running_apply(nck_dev *d, const nck_bn_group *groups, int ngroups, const nck_bn_staged *staged,
                          const float *gathered, int64_t rank_stride, int ranks);
void nck_bn_fwd_eval(nck_dev *d, const float *x, const float *w, const float *b, float *y, float *mean,
                     float *invstd, const float *rm, const float *rv, int64_t N, int64_t C, int64_t S, float eps);
void nck_bn_bwd(nck_dev *d, const float *x, const float *w, const float *g, const float *mean, const float *invstd,
                float *gx, float *gw, float *gb, int64_t N, int64_t C, int64_t S, int training, int acc_gx);
/* layer norm over rows of D */
void nck_ln_fwd(nck_dev *d, const float *x, const float *w, const float *b, float *y, float *stats, int64_t R,
                int64_t D, float eps);
void nck_ln_bwd(nck_dev *d, const float *x, const float *w, const float *g, const float *stats, float *gx,
                float *gw, float *gb, int64_t R, int64_t D, int acc_gx); /* acc_gx == 0: gx is fresh, stored */

/* ---- gather / scatter ------------------------------------------------------------------------ */
void nck_index_select(nck_dev *d, const void *x, const int32_t *idx, void *y, int64_t B, int64_t N,
                      int64_t row_bytes);
void nck_index_select_bwd(nck_dev *d, const float *g, const int32_t *idx, float *gx, int64_t B, int64_t N,
                          int64_t row);
/* cat / split along a [outer, len*inner] view */
void nck_cat_part(nck_dev *d, const void *x, void *y, int64_t outer, int64_t row_bytes, int64_t out_row_bytes,
                  int64_t off_bytes);
void nck_cat_part_bwd(nck_dev *d, const float *g, float *gx, int64_t outer, int64_t row, int64_t out_row,
                      int64_t off);

/* ---- convolution / pooling (NCHW) ---------------------------------------------------------- */
typedef struct {
    int64_t N, C, H, W, OC, KH, KW, OH, OW;
    int sh, sw, ph, pw, dh, dw;
    int64_t G;
} nck_conv;
/* col [n][g][Cg*KH*KW][OH*OW] for samples [n0, n0+nb) */
void nck_im2col(nck_dev *d, const nck_conv *g, const float *x, float *col, int64_t n0, int64_t nb);
/* dx[n] += fold(col[n]) */
void nck_col2im(nck_dev *d, const nck_conv *g, const float *col, float *dx, int64_t n0, int64_t nb, int acc);
/* gb[oc] += sum over n, l of g[n, oc, l] */
void nck_conv_bias_grad(nck_dev *d, const float *g, float *gb, int64_t N, int64_t OC, int64_t L);
/* direct convolution for few input channels per group (Cg*KH*KW <= 64) */
void nck_conv_direct_fwd(nck_dev *d, const nck_conv *g, const float *x, const float *w, const float *b, float *y);
/* implicit-GEMM convolution on tcgen05 (groups 1): mode 0 y = conv(x) + bias (in = x, q = w),
 * 1 gx += conv-transpose(gy) for unit strides (in = gy, q = w), 2 gw += dY x taps (in = x, q = gy).
 * Returns 0, launching nothing, for a convolution it does not handle. */
int nck_conv_implicit(nck_dev *d, int mode, const nck_conv *g, const float *in, const float *q, float *out,
                      const float *bias);
/* whether nck_conv_implicit would take this convolution (nothing is launched) */
int nck_conv_implicit_supported(const nck_dev *d, int mode, const nck_conv *g);
/* Stride-1 convolutions (groups 1) as tap-shifted GEMMs on tcgen05. An activation or output gradient
 * is packed into a zero-padded, position-major matrix: row v = n*Hp*Wp + h'*Wp + w' of the padded grid
 * (Hp = H + 2ph, Wp = W + 2pw), channels padded to a multiple of 32 along the row. Filter tap (ki, kj)
 * is then the row shift ki*dh*Wp + kj*dw of that matrix, so every tap is a plain TMA tile load. In
 * 3xTF32 mode every packed buffer is followed by its TF32 remainders (planes = 2, same shape). */
typedef struct {
    int64_t Hp, Wp, Nv, Cp, OCp, T;
    int planes;
} nck_tapgeom;
/* 1 when the convolution takes the tap-shifted path; fills *t */
int nck_convtap_plan(const nck_dev *d, const nck_conv *g, nck_tapgeom *t);
/* dst[v][k] (Kp columns) from src [N][C][Hs][Ws] placed at padded offset (eh, ew), zero elsewhere;
 * colsum (optional): colsum[c] += the sum of channel c of src, computed from the same pass */
void nck_tap_pack(nck_dev *d, const float *src, int64_t N, int64_t C, int64_t Hs, int64_t Ws, const nck_tapgeom *t,
                  int eh, int ew, int64_t Kp, float *dst, float *colsum);
/* whether nck_tap_pack can add the channel sums (its per-block sums fit the scratch) */
int nck_tap_pack_colsum_ok(const nck_dev *d, const nck_tapgeom *t, int64_t Kp);
/* weights for the forward, [OC][T][Cp] (tr 0), or for dX, [C][T][OCp] (tr 1) */
void nck_tap_pack_w(nck_dev *d, const nck_conv *g, const nck_tapgeom *t, const float *w, float *dst, int tr);
/* mode 0: y = conv(x) + bias (P = packed x, Q = forward weights); 1: gx (+)= conv-transpose(gy)
 * (P = packed gy, Q = dX weights); 2: gw += sum over positions (P = packed x, Q = packed gy).
 * acc: add into out (modes 1, 2) instead of storing. Returns 0 when nothing was launched. */
int nck_convtap(nck_dev *d, int mode, const nck_conv *g, const nck_tapgeom *t, const float *P, const float *Q,
                float *out, const float *bias, int acc);
/* gw[oc, k] += sum over n, l of gy[n, oc, l] * x-tap k at l (same eligibility as the direct forward) */
/* gb (optional): when the 3x3 one-channel kernel runs, gb[oc] += sum of gy[:, oc] from the same pass
 * and 1 is returned; otherwise gb is left alone and 0 is returned */
int nck_conv_direct_dw(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw, float *gb);
/* whether nck_conv_direct_dw takes the 3x3 one-channel kernel (and can add the bias gradient) */
int nck_conv_direct3_ok(const nck_conv *g);
/* nck_conv_direct_dw also sums the bias gradient for this geometry (when given gb) */
int nck_conv_direct_dw_bias_ok(const nck_conv *g);
/* depthwise (groups == C == OC): shared-memory plane tiles; nck_dw_ok says whether a geometry fits
 * them (at most NCK_DW_MAX_TAPS taps, tiles within shared memory) */
#define NCK_DW_MAX_TAPS 25
int nck_dw_ok(const nck_conv *g);
void nck_dw_fwd(nck_dev *d, const nck_conv *g, const float *x, const float *w, const float *b, float *y);
/* gx = (acc ? gx : 0) + input gradient */
void nck_dw_dx(nck_dev *d, const nck_conv *g, const float *gy, const float *w, float *gx, int acc);
/* gw += weight gradient; gb (may be NULL) += bias gradient */
void nck_dw_dw(nck_dev *d, const nck_conv *g, const float *x, const float *gy, float *gw, float *gb);
void nck_pool_fwd(nck_dev *d, const nck_conv *g, const float *x, float *y, int32_t *arg, int is_max);
void nck_pool_bwd(nck_dev *d, const nck_conv *g, const float *gy, const int32_t *arg, float *gx, int is_max, int acc);

/* ---- GEMM -------------------------------------------------------------------------------------- */
/* C_b = alpha * op(A_b) op(B_b) + beta * C_b for b in [0, batch); row-major; ta/tb as the newch kernel
 * table (ta: A stored K x M). With reduce_batch, C = alpha * sum_b op(A_b) op(B_b) + beta * C. */
typedef struct {
    int ta, tb;
    int64_t M, N, K;
    float alpha, beta;
    const float *A;
    int64_t lda, sA;
    const float *B;
    int64_t ldb, sB;
    float *C;
    int64_t ldc, sC;
    int64_t batch;
    int reduce_batch;
    const float *bias; /* optional: C[m, n] = alpha * acc + bias[n] (or bias[m] with bias_per_row) + beta * C */
    int bias_per_row;
} nck_gemm_args;
void nck_gemm(nck_dev *d, const nck_gemm_args *a);
/* tensor-core path (tcgen05 kind::tf32 via TMA); returns 0 when the operands do not meet its
 * alignment rules, leaving the GEMM to the caller */
int nck_gemm_tc(nck_dev *d, const nck_gemm_args *a);
/* one kernel whose pipeline wait never completes: it gives up after its bound and sets
 * NCK_ERR_PIPELINE (tests the failure reporting of the tcgen05 kernels' bounded waits) */
void nck_pipeline_wait_probe(nck_dev *d);

/* ---- optimizers -------------------------------------------------------------------------------- */
typedef struct {
    float *w;
    const float *g;
    float *m, *v;
    int64_t n;
    int32_t param; /* index into the presence bytes */
    int32_t pad;
} nck_param_seg;
/* one block's work: elements [off, off + len) of segment seg (off a multiple of 4) */
typedef struct {
    int32_t seg;
    int32_t len;
    int64_t off;
} nck_opt_chunk;
enum { NCK_OPT_SGD, NCK_OPT_ADAM, NCK_OPT_ADAMW, NCK_OPT_RMSPROP };
typedef struct {
    int kind;
    float lr, momentum, weight_decay, beta1, beta2, eps, gs, bc1, bc2;
    int eps_inside_sqrt;
} nck_opt_hyper;
#define NCK_OPT_CHUNK 1024 /* elements per block: one float4 per thread (a 422k-parameter model: ~400 blocks) */
/* fills chunks (when not NULL) for the segments; returns how many there are */
int nck_optim_chunks(const nck_param_seg *segs, int nseg, nck_opt_chunk *chunks);
/* One launch over device-resident tables: dsegs[nseg], dchunks[nchunk]; total = elements in all
 * segments (for the timer's byte count). present (device, may be NULL): a segment whose
 * present[param] is 0 is left as it is. */
void nck_optim_step(nck_dev *d, const nck_opt_hyper *h, const nck_param_seg *dsegs, const nck_opt_chunk *dchunks,
                    int nchunk, int64_t total, const unsigned char *present);

/* ---- int8 quantization -------------------------------------------------------------------------- */
/* rows of act(x) quantized as nck_quantize_rows does (act: a NCK_UN_* kind applied on the fly, -1 none);
 * act >= 0 needs nck_quantize_rows_act_ok(cols) and 16-byte aligned x and q */
int nck_quantize_rows_act_ok(int64_t cols);
void nck_quantize_rows_act(nck_dev *d, const float *x, int act, float act_s, int8_t *q, float *scale, int64_t rows,
                           int64_t cols);
void nck_quantize_rows(nck_dev *d, const float *x, int8_t *q, float *scale, int64_t rows, int64_t cols);
/* y[r, o] = (float)acc * xs[r] * ws[o] + b[o], acc = sum_k xq[r,k] * wq[o,k] (exact int32) */
void nck_qlinear(nck_dev *d, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, const float *b,
                 float *y, int64_t M, int64_t N, int64_t K, int32_t *acc_out);

#ifdef __cplusplus
}
#endif

#endif /* NCK_H */
