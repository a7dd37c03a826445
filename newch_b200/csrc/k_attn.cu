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
// Geometry: 512 threads (16 warps, four per scheduler), warp w owns rows 8 w .. 8 w + 7 of a
// [128 x 128] score tile and lane l its columns l, l + 32, l + 64, l + 96 (the unfused softmax's
// column walk); L, S <= 128 and D, Dv <= 32, zero-padded in shared memory. Tiles of Q / K / V / dO
// have a row pitch of 36 floats (float4 rows, conflict-free float4 reads across a quarter warp); the
// probability tiles 132. The transposed products of the backward (dV, dK) give each of 8 warps 16
// output rows, the two products running side by side on the two halves of the block.
#include <math.h>

#include "k_common.cuh"
#include "k_math.cuh"

using namespace nck;

namespace {

constexpr int kAT = 512;       // threads per head
constexpr int kRW = 8;         // score rows per warp
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

// acc[r][c] = sum_d A[row0 + r][d] * Bt[lane + 32 c][d], d ascending (FFMA chains); D4 = D rounded up to 4
template <int NR>
__device__ __forceinline__ void rows_by_cols(const float *__restrict__ A, const float *__restrict__ Bt, int D4,
                                             int row0, float (&acc)[NR][4]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[r][c] = 0.0f;
    for (int d = 0; d < D4; d += 4) {
        float4 bv[4];
#pragma unroll
        for (int c = 0; c < 4; c++) bv[c] = *reinterpret_cast<const float4 *>(Bt + (lane + 32 * c) * kLd + d);
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const float4 av = *reinterpret_cast<const float4 *>(A + (row0 + r) * kLd + d);
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

// the dropout keep bits of columns lane + 32 c of row i (bit c of the result)
__device__ __forceinline__ uint32_t keep_bits(const nck_attn &a, int64_t b, int i) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (b * a.L + i) * a.S;
    uint32_t k = 0;
    if ((a.S & 127) == 0 && ((uintptr_t)a.bits & 15) == 0) {  // the row's first four words, one load
        const uint4 w4 = __ldg(reinterpret_cast<const uint4 *>(a.bits + (row >> 5)));
        k = ((w4.x >> lane) & 1u) | (((w4.y >> lane) & 1u) << 1) | (((w4.z >> lane) & 1u) << 2) |
            (((w4.w >> lane) & 1u) << 3);
        return k;
    }
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int64_t e = row + lane + 32 * c;
        if (lane + 32 * c < a.S) k |= ((__ldg(a.bits + (e >> 5)) >> (e & 31)) & 1u) << c;
    }
    return k;
}

// the mask of columns lane + 32 c of row i (bit c set: masked)
__device__ __forceinline__ uint32_t mask_bits(const nck_attn &a, int64_t b, int i) {
    const int lane = threadIdx.x & 31;
    const int32_t *mr = a.mask + b * a.ms[0] + i * a.ms[1];
    uint32_t m = 0;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int j = lane + 32 * c;
        if (j < a.S && __ldg(mr + j * a.ms[2]) != 0) m |= 1u << c;
    }
    return m;
}

// scores -> (scale) -> masked -> softmax -> dropout, in place, up to `stage`, for rows row0 ..
// row0 + NR - 1; columns >= S hold 0 after the softmax (and are skipped by its reductions), rows >= L
// are left as they are
template <int M, int NR>
__device__ __forceinline__ void chain_forward(const nck_attn &a, int64_t b, int stage, int row0, float (&v)[NR][4]) {
    const int lane = threadIdx.x & 31;
    const int L = (int)a.L, S = (int)a.S;
    if (stage >= NCK_ATT_MASKED && a.mask) {
#pragma unroll
        for (int r = 0; r < NR; r++) {
            if (row0 + r >= L) continue;
            const uint32_t m = mask_bits(a, b, row0 + r);
#pragma unroll
            for (int c = 0; c < 4; c++)
                if ((m >> c) & 1u) v[r][c] = a.fill;
        }
    }
    if (stage < NCK_ATT_SOFTMAX) return;
#pragma unroll
    for (int r = 0; r < NR; r++) {
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
    const float keepv = a.p < 1.0f ? 1.0f / (1.0f - a.p) : 0.0f;
#pragma unroll
    for (int r = 0; r < NR; r++) {
        if (row0 + r >= L) continue;
        const uint32_t k = keep_bits(a, b, row0 + r);
#pragma unroll
        for (int c = 0; c < 4; c++)
            if (lane + 32 * c < S) v[r][c] *= (k >> c) & 1u ? keepv : 0.0f;
    }
}

// the scores of rows row0 .. into v (scaled when the chain scales them); Q and K already staged
template <int NR>
__device__ __forceinline__ void scores(const nck_attn &a, const float *Qs, const float *Ks, int row0,
                                       float (&v)[NR][4]) {
    rows_by_cols<NR>(Qs, Ks, ((int)a.D + 3) & ~3, row0, v);
    if (a.scaled)
#pragma unroll
        for (int r = 0; r < NR; r++)
#pragma unroll
            for (int c = 0; c < 4; c++) v[r][c] = a.scale * v[r][c];
}

// acc[r] = sum_j P[row0 + r][j] X[j][lane], j ascending (P pitch kLp, X pitch kLd)
template <int NR>
__device__ __forceinline__ void rows_times_tile(const float *__restrict__ P, const float *__restrict__ X, int S4,
                                                int row0, float (&acc)[NR]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r] = 0.0f;
    for (int j = 0; j < S4; j += 4) {
        const float x0 = X[(j + 0) * kLd + lane], x1 = X[(j + 1) * kLd + lane];
        const float x2 = X[(j + 2) * kLd + lane], x3 = X[(j + 3) * kLd + lane];
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const float4 pv = *reinterpret_cast<const float4 *>(P + (row0 + r) * kLp + j);
            acc[r] = fmaf(pv.x, x0, acc[r]);
            acc[r] = fmaf(pv.y, x1, acc[r]);
            acc[r] = fmaf(pv.z, x2, acc[r]);
            acc[r] = fmaf(pv.w, x3, acc[r]);
        }
    }
}

// acc[r] = sum_i P[i][col0 + r] X[i][lane], i ascending: the transposed product
template <int NR>
__device__ __forceinline__ void cols_times_tile(const float *__restrict__ P, const float *__restrict__ X, int L,
                                                int col0, float (&acc)[NR]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r] = 0.0f;
    for (int i = 0; i < L; i++) {
        const float x = X[i * kLd + lane];
        const float4 *pr = reinterpret_cast<const float4 *>(P + i * kLp + col0);
#pragma unroll
        for (int q = 0; q < NR / 4; q++) {
            const float4 pv = pr[q];
            acc[4 * q + 0] = fmaf(pv.x, x, acc[4 * q + 0]);
            acc[4 * q + 1] = fmaf(pv.y, x, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(pv.z, x, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(pv.w, x, acc[4 * q + 3]);
        }
    }
}

template <int M>
__global__ void __launch_bounds__(kAT, 1) k_attn_fwd(const nck_attn a, float *__restrict__ o) {
    extern __shared__ float4 smem4[];
    float *Qs = reinterpret_cast<float *>(smem4), *Ks = Qs + kTile, *Vs = Ks + kTile, *Ps = Vs + kTile;
    const int64_t b = blockIdx.x;
    const int L = (int)a.L, S = (int)a.S;
    const int lane = threadIdx.x & 31, row0 = kRW * (threadIdx.x >> 5);
    load_tile(Qs, a.q, a.qs, b, L, (int)a.D);
    load_tile(Ks, a.k, a.ks, b, S, (int)a.D);
    load_tile(Vs, a.v, a.vs, b, S, (int)a.Dv);
    __syncthreads();
    float v[kRW][4];
    scores<kRW>(a, Qs, Ks, row0, v);
    chain_forward<M, kRW>(a, b, a.stage, row0, v);
#pragma unroll
    for (int r = 0; r < kRW; r++)  // the warp's own rows: only it reads them back
#pragma unroll
        for (int c = 0; c < 4; c++) Ps[(row0 + r) * kLp + lane + 32 * c] = lane + 32 * c < S ? v[r][c] : 0.0f;
    __syncwarp();
    float acc[kRW];
    rows_times_tile<kRW>(Ps, Vs, (S + 3) & ~3, row0, acc);
    if (lane < a.Dv)
#pragma unroll
        for (int r = 0; r < kRW; r++)
            if (row0 + r < L) o[(b * a.L + row0 + r) * a.Dv + lane] = acc[r];
}

template <int M>
__global__ void __launch_bounds__(kAT, 1) k_attn_probs(const nck_attn a, float *__restrict__ out) {
    extern __shared__ float4 smem4[];
    float *Qs = reinterpret_cast<float *>(smem4), *Ks = Qs + kTile;
    const int64_t b = blockIdx.x;
    const int L = (int)a.L, S = (int)a.S;
    const int lane = threadIdx.x & 31, row0 = kRW * (threadIdx.x >> 5);
    load_tile(Qs, a.q, a.qs, b, L, (int)a.D);
    load_tile(Ks, a.k, a.ks, b, S, (int)a.D);
    __syncthreads();
    float v[kRW][4];
    scores<kRW>(a, Qs, Ks, row0, v);
    chain_forward<M, kRW>(a, b, a.stage, row0, v);
#pragma unroll
    for (int r = 0; r < kRW; r++) {
        if (row0 + r >= L) continue;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int j = lane + 32 * c;
            if (j < S) out[(b * a.L + row0 + r) * a.S + j] = v[r][c];
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
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, row0 = kRW * w;
    const int64_t gs[3] = {a.L * a.Dv, a.Dv, 1};
    load_tile(Qs, a.q, a.qs, b, L, D);
    load_tile(Ks, a.k, a.ks, b, S, D);
    load_tile(Vs, a.v, a.vs, b, S, Dv);
    load_tile(Gs, dout, gs, b, L, Dv);
    __syncthreads();

    {  // probabilities y (after the softmax), the gradient reaching them through the dropout, dS
        float y[kRW][4], g[kRW][4];
        scores<kRW>(a, Qs, Ks, row0, y);
        chain_forward<M, kRW>(a, b, NCK_ATT_SOFTMAX, row0, y);
        rows_by_cols<kRW>(Gs, Vs, (Dv + 3) & ~3, row0, g);  // dO V^T: the gradient of the dropped probabilities
        const bool drop = a.stage >= NCK_ATT_DROPOUT && a.bits;
        const float keepv = a.p < 1.0f ? 1.0f / (1.0f - a.p) : 0.0f;
#pragma unroll
        for (int r = 0; r < kRW; r++) {
            const int i = row0 + r;
            const uint32_t kb = drop && i < L ? keep_bits(a, b, i) : 0xFu;
            const uint32_t mb = a.mask && i < L ? mask_bits(a, b, i) : 0u;
            float dot = 0.0f;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int j = lane + 32 * c;
                float pd = y[r][c];
                if (drop) {
                    const float mk = (kb >> c) & 1u ? keepv : 0.0f;
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
                float ds = j < S && i < L && !((mb >> c) & 1u) ? 0.0f + y[r][c] * (g[r][c] - dot) : 0.0f;
                Ds[i * kLp + j] = a.scaled ? a.scale * ds : ds;  // through the scale's backward
            }
        }
    }
    __syncthreads();

    // dV = P_drop^T dO on warps 0-7 and dK = dS^T Q on warps 8-15, 16 output rows per warp
    const int half = w >> 3, col0 = 16 * (w & 7);
    float acc[16];
    if (half == 0 && dv) {
        cols_times_tile<16>(Ps, Gs, L, col0, acc);
        if (lane < Dv)
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const int j = col0 + r;
                if (j < S) {
                    float *p = dv + (b * a.S + j) * a.Dv + lane;
                    *p = acc_v ? *p + acc[r] : acc[r];
                }
            }
    }
    if (half == 1 && dkt) cols_times_tile<16>(Ds, Qs, L, col0, acc);
    if (dq) {  // dQ = dS K
        float aq[kRW];
        rows_times_tile<kRW>(Ds, Ks, (S + 3) & ~3, row0, aq);
        if (lane < D)
#pragma unroll
            for (int r = 0; r < kRW; r++) {
                const int i = row0 + r;
                if (i < L) {
                    float *p = dq + (b * a.L + i) * a.D + lane;
                    *p = acc_q ? *p + aq[r] : aq[r];
                }
            }
    }
    if (dkt) {  // dK written as K^T [D, S] through a transposed staging tile
        __syncthreads();  // every warp is done with Ps (dV) before it is reused
        float *T = Ps;
        if (half == 1)
#pragma unroll
            for (int r = 0; r < 16; r++) T[lane * kLt + col0 + r] = acc[r];
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
