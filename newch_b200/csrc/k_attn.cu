// Fused attention over B independent heads: o = dropout(softmax(masked_fill(Q K^T))) V, and its
// backward, each head in one CTA with every operand tile in shared memory, so the [L, S] score,
// probability and gradient matrices never reach HBM.
//
// The chain is the one newch's nn.MultiheadAttention builds from separate ops (newch/net/__init__.py
// :811-820: q @ k^T, _apply_mask, softmax(-1), dropout, @ v); engine semantics per op:
//   masked_fill    x where the mask is 0, the fill value where it is nonzero (ops_nn.c masked_fill)
//   softmax        m = row max, e = exp(x - m), y = e * (1 / sum e)           (ops_nn.c :22-35)
//   dropout        y * (keep ? 1 / (1 - p) : 0), keep drawn from the context stream (ops_nn.c :182-204)
//   backward       dropout g * m; softmax y (g - <g, y>); masked_fill zero where masked
// The softmax, dropout and their backward use exactly the arithmetic of the unfused kernels (same
// per-lane column walk, same warp trees, same exp), so fused and unfused probabilities agree bit for
// bit given the same scores. The products are fp32 FFMA chains over the contraction index in order.
//
// Geometry: 256 threads, warp w owns rows 16 w .. 16 w + 15 of a [128 x 128] score tile and lane l its
// columns l, l + 32, l + 64, l + 96 (the unfused softmax's column walk); L, S <= 128 and D, Dv <= 32,
// zero-padded in shared memory. Tiles of Q / K / V / dO have a row pitch of 36 floats (float4 rows,
// conflict-free float4 reads across a quarter warp); the probability tiles 132.
#include <math.h>

#include "k_common.cuh"
#include "k_math.cuh"

using namespace nck;

namespace {

constexpr int kAT = 256;       // threads per head
constexpr int kR = 128;        // max rows L and columns S
constexpr int kDm = 32;        // max D and Dv
constexpr int kLd = kDm + 4;   // pitch of the [128 x 32] operand tiles
constexpr int kLp = kR + 4;    // pitch of the [128 x 128] probability tiles
constexpr int kLt = kR + 1;    // pitch of the transposed dK staging tile
constexpr int kTile = kR * kLd;   // floats per operand tile
constexpr int kPTile = kR * kLp;  // floats per probability tile

__device__ __forceinline__ float wmax(float v) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float wsum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// rows x cols of the strided view at p + b * s[0] into a zero-padded [128 x 32] tile: float4 loads
// (every one issued before the stores) when the rows are unit-stride and 16-byte aligned
__device__ __forceinline__ void load_tile(float *__restrict__ dst, const float *__restrict__ p, const int64_t *s,
                                          int64_t b, int rows, int cols) {
    const float *base = p + b * s[0];
    const bool vec = s[2] == 1 && (cols & 3) == 0 && (s[1] & 3) == 0 && ((uintptr_t)base & 15) == 0;
    if (vec) {
        constexpr int kPer = kR * (kDm / 4) / kAT;  // float4 items per thread
        float4 v[kPer];
#pragma unroll
        for (int u = 0; u < kPer; u++) {
            const int idx = threadIdx.x + u * kAT, r = idx >> 3, c4 = (idx & 7) * 4;
            v[u] = r < rows && c4 < cols ? __ldg(reinterpret_cast<const float4 *>(base + r * s[1] + c4))
                                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < kPer; u++) {
            const int idx = threadIdx.x + u * kAT, r = idx >> 3, c4 = (idx & 7) * 4;
            *reinterpret_cast<float4 *>(dst + r * kLd + c4) = v[u];
        }
        return;
    }
    for (int idx = threadIdx.x; idx < kR * kDm; idx += kAT) {
        const int r = idx >> 5, c = idx & 31;
        float v = 0.0f;
        if (r < rows && c < cols) v = __ldg(base + r * s[1] + c * s[2]);
        dst[r * kLd + c] = v;
    }
}

// acc[r][c] = sum_d A[16 w + r][d] * Bt[lane + 32 c][d], d ascending (FFMA chains); D4 = D rounded up to 4
__device__ __forceinline__ void rows_by_cols(const float *__restrict__ A, const float *__restrict__ Bt, int D4,
                                             float (&acc)[16][4]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < 16; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[r][c] = 0.0f;
    for (int d = 0; d < D4; d += 4) {
        float4 bv[4];
#pragma unroll
        for (int c = 0; c < 4; c++) bv[c] = *reinterpret_cast<const float4 *>(Bt + (lane + 32 * c) * kLd + d);
#pragma unroll
        for (int r = 0; r < 16; r++) {
            const float4 av = *reinterpret_cast<const float4 *>(A + (16 * w + r) * kLd + d);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                acc[r][c] = fmaf(av.x, bv[c].x, acc[r][c]);
                acc[r][c] = fmaf(av.y, bv[c].y, acc[r][c]);
                acc[r][c] = fmaf(av.z, bv[c].z, acc[r][c]);
                acc[r][c] = fmaf(av.w, bv[c].w, acc[r][c]);
            }
        }
    }
}

// scores -> (scale) -> masked -> softmax -> dropout, in place, up to `stage`; columns >= S hold 0
// after the softmax (and are skipped by its reductions), rows >= L are left as they are
template <int M>
__device__ __forceinline__ void chain_forward(const nck_attn &a, int64_t b, int stage, float (&v)[16][4]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int L = (int)a.L, S = (int)a.S;
    if (stage >= NCK_ATT_MASKED && a.mask) {
        const int32_t *mb = a.mask + b * a.ms[0];
#pragma unroll
        for (int r = 0; r < 16; r++) {
            const int i = 16 * w + r;
            if (i >= L) continue;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int j = lane + 32 * c;
                if (j < S && __ldg(mb + i * a.ms[1] + j * a.ms[2]) != 0) v[r][c] = a.fill;
            }
        }
    }
    if (stage < NCK_ATT_SOFTMAX) return;
    const float keepv = a.p < 1.0f ? 1.0f / (1.0f - a.p) : 0.0f;
#pragma unroll
    for (int r = 0; r < 16; r++) {
        float m = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; c++)
            if (lane + 32 * c < S) m = fmaxf(m, v[r][c]);
        m = wmax(m);
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; c++)
            if (lane + 32 * c < S) {
                v[r][c] = m_exp<M>(v[r][c] - m);
                s += v[r][c];
            }
        s = wsum(s);
        const float inv = 1.0f / s;
#pragma unroll
        for (int c = 0; c < 4; c++) v[r][c] = lane + 32 * c < S ? inv * v[r][c] : 0.0f;
    }
    if (stage < NCK_ATT_DROPOUT || !a.bits) return;
#pragma unroll
    for (int r = 0; r < 16; r++) {
        const int i = 16 * w + r;
        if (i >= L) continue;
        const int64_t row = (b * a.L + i) * a.S;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int j = lane + 32 * c;
            if (j < S) {
                const int64_t e = row + j;
                v[r][c] *= (__ldg(a.bits + (e >> 5)) >> (e & 31)) & 1u ? keepv : 0.0f;
            }
        }
    }
}

// the scores of head b (scaled when the chain scales them) into v; Q and K already staged
__device__ __forceinline__ void scores(const nck_attn &a, const float *Qs, const float *Ks, float (&v)[16][4]) {
    rows_by_cols(Qs, Ks, ((int)a.D + 3) & ~3, v);
    if (a.scaled)
#pragma unroll
        for (int r = 0; r < 16; r++)
#pragma unroll
            for (int c = 0; c < 4; c++) v[r][c] = a.scale * v[r][c];
}

// out[16 w + r][lane] = sum_j P[16 w + r][j] X[j][lane], j ascending (P pitch kLp, X pitch kLd)
__device__ __forceinline__ void rows_times_tile(const float *__restrict__ P, const float *__restrict__ X, int S4,
                                                float (&acc)[16]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < 16; r++) acc[r] = 0.0f;
    for (int j = 0; j < S4; j += 4) {
        const float x0 = X[(j + 0) * kLd + lane], x1 = X[(j + 1) * kLd + lane];
        const float x2 = X[(j + 2) * kLd + lane], x3 = X[(j + 3) * kLd + lane];
#pragma unroll
        for (int r = 0; r < 16; r++) {
            const float4 pv = *reinterpret_cast<const float4 *>(P + (16 * w + r) * kLp + j);
            acc[r] = fmaf(pv.x, x0, acc[r]);
            acc[r] = fmaf(pv.y, x1, acc[r]);
            acc[r] = fmaf(pv.z, x2, acc[r]);
            acc[r] = fmaf(pv.w, x3, acc[r]);
        }
    }
}

// out[16 w + r][lane] = sum_i P[i][16 w + r] X[i][lane], i ascending: the transposed product
__device__ __forceinline__ void cols_times_tile(const float *__restrict__ P, const float *__restrict__ X, int L,
                                                float (&acc)[16]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < 16; r++) acc[r] = 0.0f;
    for (int i = 0; i < L; i++) {
        const float x = X[i * kLd + lane];
        const float4 *pr = reinterpret_cast<const float4 *>(P + i * kLp + 16 * w);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 pv = pr[q];
            acc[4 * q + 0] = fmaf(pv.x, x, acc[4 * q + 0]);
            acc[4 * q + 1] = fmaf(pv.y, x, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(pv.z, x, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(pv.w, x, acc[4 * q + 3]);
        }
    }
}

// the rows of v into a [128 x 128] tile (columns >= S as 0)
__device__ __forceinline__ void store_rows(float *__restrict__ P, const float (&v)[16][4], int S) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < 16; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int j = lane + 32 * c;
            P[(16 * w + r) * kLp + j] = j < S ? v[r][c] : 0.0f;
        }
}

template <int M>
__global__ void __launch_bounds__(kAT, 1) k_attn_fwd(const nck_attn a, float *__restrict__ o) {
    extern __shared__ float4 smem4[];
    float *Qs = reinterpret_cast<float *>(smem4), *Ks = Qs + kTile, *Vs = Ks + kTile, *Ps = Vs + kTile;
    const int64_t b = blockIdx.x;
    const int L = (int)a.L, S = (int)a.S;
    load_tile(Qs, a.q, a.qs, b, L, (int)a.D);
    load_tile(Ks, a.k, a.ks, b, S, (int)a.D);
    load_tile(Vs, a.v, a.vs, b, S, (int)a.Dv);
    __syncthreads();
    float v[16][4];
    scores(a, Qs, Ks, v);
    chain_forward<M>(a, b, a.stage, v);
    store_rows(Ps, v, S);
    __syncthreads();
    float acc[16];
    rows_times_tile(Ps, Vs, (S + 3) & ~3, acc);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane < a.Dv)
#pragma unroll
        for (int r = 0; r < 16; r++) {
            const int i = 16 * w + r;
            if (i < L) o[(b * a.L + i) * a.Dv + lane] = acc[r];
        }
}

template <int M>
__global__ void __launch_bounds__(kAT, 1) k_attn_probs(const nck_attn a, float *__restrict__ out) {
    extern __shared__ float4 smem4[];
    float *Qs = reinterpret_cast<float *>(smem4), *Ks = Qs + kTile;
    const int64_t b = blockIdx.x;
    const int L = (int)a.L, S = (int)a.S;
    load_tile(Qs, a.q, a.qs, b, L, (int)a.D);
    load_tile(Ks, a.k, a.ks, b, S, (int)a.D);
    __syncthreads();
    float v[16][4];
    scores(a, Qs, Ks, v);
    chain_forward<M>(a, b, a.stage, v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < 16; r++) {
        const int i = 16 * w + r;
        if (i >= L) continue;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int j = lane + 32 * c;
            if (j < S) out[(b * a.L + i) * a.S + j] = v[r][c];
        }
    }
}

// Backward of one head. Shared memory: Q, K, V, dO tiles, the dropped probabilities (for dV) and the
// score gradient (for dQ and dK); the dK staging tile reuses the probability tile.
template <int M>
__global__ void __launch_bounds__(kAT, 1) k_attn_bwd(const nck_attn a, const float *__restrict__ dout,
                                                     float *__restrict__ dq, int acc_q, float *__restrict__ dkt,
                                                     int acc_k, float *__restrict__ dv, int acc_v) {
    extern __shared__ float4 smem4[];
    float *Qs = reinterpret_cast<float *>(smem4), *Ks = Qs + kTile, *Vs = Ks + kTile, *Gs = Vs + kTile;
    float *Ps = Gs + kTile, *Ds = Ps + kPTile;
    const int64_t b = blockIdx.x;
    const int L = (int)a.L, S = (int)a.S, D = (int)a.D, Dv = (int)a.Dv;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t gs[3] = {a.L * a.Dv, a.Dv, 1};
    load_tile(Qs, a.q, a.qs, b, L, D);
    load_tile(Ks, a.k, a.ks, b, S, D);
    load_tile(Vs, a.v, a.vs, b, S, Dv);
    load_tile(Gs, dout, gs, b, L, Dv);
    __syncthreads();

    // probabilities y (after the softmax) and the gradient reaching them through the dropout
    float y[16][4], g[16][4];
    scores(a, Qs, Ks, y);
    chain_forward<M>(a, b, NCK_ATT_SOFTMAX, y);
    rows_by_cols(Gs, Vs, (Dv + 3) & ~3, g);  // dO V^T: the gradient of the dropped probabilities
    const bool drop = a.stage >= NCK_ATT_DROPOUT && a.bits;
    const float keepv = a.p < 1.0f ? 1.0f / (1.0f - a.p) : 0.0f;
#pragma unroll
    for (int r = 0; r < 16; r++) {
        const int i = 16 * w + r;
        const int64_t row = (b * a.L + i) * a.S;
        float dot = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int j = lane + 32 * c;
            float pd = y[r][c];
            if (drop && i < L && j < S) {
                const int64_t e = row + j;
                const float mk = (__ldg(a.bits + (e >> 5)) >> (e & 31)) & 1u ? keepv : 0.0f;
                pd = y[r][c] * mk;
                g[r][c] = 0.0f + g[r][c] * mk;  // dropout backward into a fresh gradient
            }
            Ps[i * kLp + j] = j < S && i < L ? pd : 0.0f;
            if (j < S) dot += g[r][c] * y[r][c];
        }
        dot = wsum(dot);
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int j = lane + 32 * c;
            float ds = j < S && i < L ? 0.0f + y[r][c] * (g[r][c] - dot) : 0.0f;
            if (a.mask && i < L && j < S && __ldg(a.mask + b * a.ms[0] + i * a.ms[1] + j * a.ms[2]) != 0) ds = 0.0f;
            Ds[i * kLp + j] = a.scaled ? a.scale * ds : ds;  // through the scale's backward
        }
    }
    __syncthreads();

    float acc[16];
    if (dv) {  // dV = P_drop^T dO
        cols_times_tile(Ps, Gs, L, acc);
        if (lane < Dv)
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const int j = 16 * w + r;
                if (j < S) {
                    float *p = dv + (b * a.S + j) * a.Dv + lane;
                    *p = acc_v ? *p + acc[r] : acc[r];
                }
            }
    }
    if (dq) {  // dQ = dS K
        rows_times_tile(Ds, Ks, (S + 3) & ~3, acc);
        if (lane < D)
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const int i = 16 * w + r;
                if (i < L) {
                    float *p = dq + (b * a.L + i) * a.D + lane;
                    *p = acc_q ? *p + acc[r] : acc[r];
                }
            }
    }
    if (dkt) {  // dK = dS^T Q, written as K^T [D, S] through a transposed staging tile
        cols_times_tile(Ds, Qs, L, acc);
        __syncthreads();  // every warp is done with Ps (dV) before it is reused
        float *T = Ps;
#pragma unroll
        for (int r = 0; r < 16; r++) T[lane * kLt + 16 * w + r] = acc[r];
        __syncthreads();
        for (int idx = threadIdx.x; idx < D * S; idx += kAT) {
            const int dd = idx / S, j = idx - dd * S;
            float *p = dkt + (b * a.D + dd) * a.S + j;
            const float val = T[dd * kLt + j];
            *p = acc_k ? *p + val : val;
        }
    }
}

constexpr size_t kFwdSmem = (size_t)(3 * kTile + kPTile) * sizeof(float);
constexpr size_t kProbSmem = (size_t)(2 * kTile) * sizeof(float);
constexpr size_t kBwdSmem = (size_t)(4 * kTile + 2 * kPTile) * sizeof(float);

template <typename K>
void set_smem(K kernel, size_t bytes) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

struct AttrOnce {
    AttrOnce() {
        set_smem(k_attn_fwd<MATH_POLY>, kFwdSmem);
        set_smem(k_attn_fwd<MATH_LIBM>, kFwdSmem);
        set_smem(k_attn_probs<MATH_POLY>, kProbSmem);
        set_smem(k_attn_probs<MATH_LIBM>, kProbSmem);
        set_smem(k_attn_bwd<MATH_POLY>, kBwdSmem);
        set_smem(k_attn_bwd<MATH_LIBM>, kBwdSmem);
    }
};

void attrs() { static AttrOnce once; }

}  // namespace

extern "C" int nck_attn_ok(int64_t L, int64_t S, int64_t D, int64_t Dv) {
    return L >= 1 && L <= kR && S >= 1 && S <= kR && D >= 1 && D <= kDm && Dv >= 1 && Dv <= kDm;
}

extern "C" void nck_attn_fwd(nck_dev *d, const nck_attn *a, float *o) {
    if (a->B <= 0) return;
    attrs();
    Scope sc(d, "attn_fwd", 2.0 * a->B * a->L * a->S * (a->D + a->Dv),
             4.0 * a->B * (a->L * a->D + a->S * (a->D + a->Dv) + a->L * a->Dv));
    auto k = d->math_mode == MATH_LIBM ? k_attn_fwd<MATH_LIBM> : k_attn_fwd<MATH_POLY>;
    k<<<(unsigned)a->B, kAT, kFwdSmem, NCK_STREAM(d)>>>(*a, o);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_attn_probs(nck_dev *d, const nck_attn *a, float *out) {
    if (a->B <= 0) return;
    attrs();
    Scope sc(d, "attn_probs", 2.0 * a->B * a->L * a->S * a->D, 4.0 * a->B * a->L * a->S);
    auto k = d->math_mode == MATH_LIBM ? k_attn_probs<MATH_LIBM> : k_attn_probs<MATH_POLY>;
    k<<<(unsigned)a->B, kAT, kProbSmem, NCK_STREAM(d)>>>(*a, out);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_attn_bwd(nck_dev *d, const nck_attn *a, const float *dout, float *dq, int acc_q, float *dkt,
                             int acc_k, float *dv, int acc_v) {
    if (a->B <= 0 || (!dq && !dkt && !dv)) return;
    attrs();
    Scope sc(d, "attn_bwd", 2.0 * a->B * a->L * a->S * (2.0 * a->D + 3.0 * a->Dv),
             4.0 * a->B * (2.0 * (a->L * a->D + a->S * a->D + a->S * a->Dv) + a->L * a->Dv));
    auto k = d->math_mode == MATH_LIBM ? k_attn_bwd<MATH_LIBM> : k_attn_bwd<MATH_POLY>;
    k<<<(unsigned)a->B, kAT, kBwdSmem, NCK_STREAM(d)>>>(*a, dout, dq, acc_q, dkt, acc_k, dv, acc_v);
    NCK_LAUNCHED(d, 1);
}
