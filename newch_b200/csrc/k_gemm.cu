// FP32 GEMM on the CUDA cores (FFMA): C_b = alpha op(A_b) op(B_b) + beta C_b (+ bias), row-major
// operands with newch's transpose convention (engine/src/kernels/kernels.h:34-41), strided batches,
// an optional sum over the batch (conv dW over samples) and split-K for narrow outputs.
//
// Tiles of 128 x 128 x 8 per 256-thread block, 8 x 8 outputs per thread, register-prefetched
// double-buffered shared memory. When the output tiles alone cannot fill the GPU, the reduction
// range (K, or the batch when it is summed) is split into slices whose partial tiles go to scratch
// and are combined in slice order by a second kernel: deterministic, no atomics.
#include "k_common.cuh"

using namespace nck;

namespace {

constexpr int BM = 128, BN = 128, BK = 8, PAD = 4;

struct GemmP {
    int ta, tb;
    int64_t M, N, K;
    float alpha, beta;
    const float *A;
    int64_t lda, sA;
    const float *B;
    int64_t ldb, sB;
    float *C;
    int64_t ldc, sC;
    const float *bias;
    int bias_row;
    int64_t batch;    // batches in the problem
    int reduce;       // sum over the batch into one output
    int splits;       // slices per output batch
    int64_t bper;     // reduce: batches per slice
    int64_t kper;     // split-K: K per slice (multiple of BK)
    float *part;      // partial tiles [z][M][N] when splits > 1
    int vecA, vecB, vecC;
};

__device__ __forceinline__ float epi(const GemmP &p, float acc, int64_t m, int64_t n, const float *cold) {
    float v = p.alpha * acc;
    if (p.bias) v = v + (p.bias_row ? p.bias[m] : p.bias[n]);
    if (p.beta != 0.0f) v = fmaf(p.beta, *cold, v);
    return v;
}

__global__ void __launch_bounds__(256) k_sgemm(GemmP p) {
    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
    const int64_t z = blockIdx.z;

    // iteration space of this block: batches [b0, b1) x K range [k0, k1)
    int64_t b0, b1, k0 = 0, k1 = p.K, ob;
    if (p.reduce) {
        b0 = z * p.bper;
        b1 = b0 + p.bper < p.batch ? b0 + p.bper : p.batch;
        ob = 0;
    } else {
        ob = z / p.splits;
        int64_t s = z % p.splits;
        b0 = ob, b1 = ob + 1;
        k0 = s * p.kper;
        k1 = k0 + p.kper < p.K ? k0 + p.kper : p.K;
    }
    int64_t kt = (k1 - k0 + BK - 1) / BK;
    int64_t T = (b1 > b0 ? (b1 - b0) : 0) * kt;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

    float ra[4], rb[4];
    // fetch tile t of the iteration space into registers
    auto fetch = [&](int64_t t) {
        int64_t b = b0 + t / kt, kk = k0 + (t % kt) * BK;
        const float *A = p.A + b * p.sA, *B = p.B + b * p.sB;
        if (!p.ta) {
            int64_t m = m0 + (tid >> 1), k = kk + (tid & 1) * 4;
            if (p.vecA) {
                float4 v = make_float4(0, 0, 0, 0);
                if (m < p.M && k < k1) v = *(const float4 *)(A + m * p.lda + k);
                ra[0] = v.x, ra[1] = v.y, ra[2] = v.z, ra[3] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) ra[j] = (m < p.M && k + j < k1) ? A[m * p.lda + k + j] : 0.0f;
            }
        } else {
            int64_t k = kk + (tid >> 5), m = m0 + (tid & 31) * 4;
            if (p.vecA) {
                float4 v = make_float4(0, 0, 0, 0);
                if (k < k1 && m < p.M) v = *(const float4 *)(A + k * p.lda + m);
                ra[0] = v.x, ra[1] = v.y, ra[2] = v.z, ra[3] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) ra[j] = (k < k1 && m + j < p.M) ? A[k * p.lda + m + j] : 0.0f;
            }
        }
        if (!p.tb) {
            int64_t k = kk + (tid >> 5), n = n0 + (tid & 31) * 4;
            if (p.vecB) {
                float4 v = make_float4(0, 0, 0, 0);
                if (k < k1 && n < p.N) v = *(const float4 *)(B + k * p.ldb + n);
                rb[0] = v.x, rb[1] = v.y, rb[2] = v.z, rb[3] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) rb[j] = (k < k1 && n + j < p.N) ? B[k * p.ldb + n + j] : 0.0f;
            }
        } else {
            int64_t n = n0 + (tid >> 1), k = kk + (tid & 1) * 4;
            if (p.vecB) {
                float4 v = make_float4(0, 0, 0, 0);
                if (n < p.N && k < k1) v = *(const float4 *)(B + n * p.ldb + k);
                rb[0] = v.x, rb[1] = v.y, rb[2] = v.z, rb[3] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) rb[j] = (n < p.N && k + j < k1) ? B[n * p.ldb + k + j] : 0.0f;
            }
        }
    };
    auto stash = [&](int buf) {
        if (!p.ta) {
            int r = tid >> 1, kc = (tid & 1) * 4;
#pragma unroll
            for (int j = 0; j < 4; j++) As[buf][kc + j][r] = ra[j];
        } else {
            int kr = tid >> 5, mc = (tid & 31) * 4;
            *(float4 *)&As[buf][kr][mc] = make_float4(ra[0], ra[1], ra[2], ra[3]);
        }
        if (!p.tb) {
            int kr = tid >> 5, nc = (tid & 31) * 4;
            *(float4 *)&Bs[buf][kr][nc] = make_float4(rb[0], rb[1], rb[2], rb[3]);
        } else {
            int r = tid >> 1, kc = (tid & 1) * 4;
#pragma unroll
            for (int j = 0; j < 4; j++) Bs[buf][kc + j][r] = rb[j];
        }
    };

    if (T > 0) {
        fetch(0);
        stash(0);
        __syncthreads();
    }
    for (int64_t t = 0; t < T; t++) {
        int cur = t & 1;
        if (t + 1 < T) fetch(t + 1);
#pragma unroll
        for (int k = 0; k < BK; k++) {
            float4 a0 = *(const float4 *)&As[cur][k][ty * 4], a1 = *(const float4 *)&As[cur][k][64 + ty * 4];
            float4 c0 = *(const float4 *)&Bs[cur][k][tx * 4], c1 = *(const float4 *)&Bs[cur][k][64 + tx * 4];
            float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float b[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (t + 1 < T) {
            stash(cur ^ 1);
            __syncthreads();
        }
    }

    // epilogue: final values, or raw partial sums for the combine kernel
    const bool partial = p.splits > 1;
    float *out = partial ? p.part + z * p.M * p.N : p.C + ob * p.sC;
    int64_t ldo = partial ? p.N : p.ldc;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= p.M) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            int64_t n = n0 + h * 64 + tx * 4;
            float *row = out + m * ldo;
            if (partial) {
                if (p.vecC && n + 3 < p.N) {
                    *(float4 *)(row + n) = make_float4(acc[i][h * 4], acc[i][h * 4 + 1], acc[i][h * 4 + 2],
                                                       acc[i][h * 4 + 3]);
                } else {
                    for (int j = 0; j < 4; j++)
                        if (n + j < p.N) row[n + j] = acc[i][h * 4 + j];
                }
            } else {
                for (int j = 0; j < 4; j++)
                    if (n + j < p.N) row[n + j] = epi(p, acc[i][h * 4 + j], m, n + j, row + n + j);
            }
        }
    }
}

// C[ob] = epilogue(sum over the slices of partial tiles), slices added in order
__global__ void k_sgemm_combine(GemmP p, int64_t nout) {
    int64_t MN = p.M * p.N, total = nout * MN;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t ob = t / MN, r = t - ob * MN, m = r / p.N, n = r - m * p.N;
        const float *src = p.part + ob * p.splits * MN + r;
        float s = 0.0f;
        for (int k = 0; k < p.splits; k++) s += src[k * MN];
        float *c = p.C + ob * p.sC + m * p.ldc + n;
        *c = epi(p, s, m, n, c);
    }
}

// ---- small problems ---------------------------------------------------------------------------------
//
// Products with few outputs (at most 64k) and little work (at most 4M multiply-adds), where 128 x 128
// tiles would leave most SMs idle: one thread per output when the reduction (K, times the batch when
// it is summed) is short, a block per 32 columns of one row when A is transposed and the reduction
// long, else one warp per output with the lanes taking strided runs of it and a fixed shuffle tree
// (a block per output for very long reductions). Exact fp32 in every GEMM mode.

__device__ __forceinline__ float op_a(const GemmP &p, int64_t b, int64_t m, int64_t k) {
    return __ldg(p.A + b * p.sA + (p.ta ? k * p.lda + m : m * p.lda + k));
}
__device__ __forceinline__ float op_b(const GemmP &p, int64_t b, int64_t k, int64_t n) {
    return __ldg(p.B + b * p.sB + (p.tb ? n * p.ldb + k : k * p.ldb + n));
}

// acc + the r-th product of output (ob, m, n), r over (batch when summed) x K, one fused multiply-add
__device__ __forceinline__ float small_fma(const GemmP &p, int64_t ob, int64_t m, int64_t n, int64_t r, float acc) {
    const int64_t b = p.reduce ? r / p.K : ob, k = p.reduce ? r - (r / p.K) * p.K : r;
    return fmaf(op_a(p, p.sA ? b : 0, m, k), op_b(p, p.sB ? b : 0, k, n), acc);
}

__global__ void __launch_bounds__(256) k_sgemm_small_thread(GemmP p, int64_t nout) {
    const int64_t MN = p.M * p.N, total = nout * MN, R = p.reduce ? p.batch * p.K : p.K;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t ob = t / MN, rm = t - ob * MN, m = rm / p.N, n = rm - m * p.N;
        float acc = 0.0f;
        int64_t r = 0;
        if (!p.reduce) {
            // four terms' operands loaded before their multiply-adds (added in order: r ascending)
            const int64_t ba = p.sA ? ob : 0, bb = p.sB ? ob : 0;
            for (; r + 4 <= R; r += 4) {
                float a[4], b[4];
#pragma unroll
                for (int u = 0; u < 4; u++) a[u] = op_a(p, ba, m, r + u), b[u] = op_b(p, bb, r + u, n);
#pragma unroll
                for (int u = 0; u < 4; u++) acc = fmaf(a[u], b[u], acc);
            }
        }
        for (; r < R; r++) acc = small_fma(p, ob, m, n, r, acc);
        float *c = p.C + ob * p.sC + m * p.ldc + n;
        *c = epi(p, acc, m, n, c);
    }
}

__global__ void __launch_bounds__(256) k_sgemm_small_warp(GemmP p, int64_t nout) {
    const int lane = threadIdx.x & 31;
    const int64_t MN = p.M * p.N, total = nout * MN, R = p.reduce ? p.batch * p.K : p.K;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; t < total; t += warps) {
        const int64_t ob = t / MN, rm = t - ob * MN, m = rm / p.N, n = rm - m * p.N;
        // four independent chains per lane, so the loads of several terms are in flight together
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        int64_t r = lane;
        for (; r + 96 < R; r += 128) {
            a0 = small_fma(p, ob, m, n, r, a0);
            a1 = small_fma(p, ob, m, n, r + 32, a1);
            a2 = small_fma(p, ob, m, n, r + 64, a2);
            a3 = small_fma(p, ob, m, n, r + 96, a3);
        }
        for (; r < R; r += 32) a0 = small_fma(p, ob, m, n, r, a0);
        float acc = (a0 + a1) + (a2 + a3);
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            float *c = p.C + ob * p.sC + m * p.ldc + n;
            *c = epi(p, acc, m, n, c);
        }
    }
}

// Transposed-A products with a long reduction (a weight gradient dY^T X, one batch entry): both
// operands are rows of the reduction index, so the lanes take 32 consecutive columns n (one coalesced
// row segment of B, one broadcast element of A per row) and the block's eight warps interleaved rows
// r = w, w + 8, ... over eight running sums; the sums are added in a fixed tree, the warps' in order.
__global__ void __launch_bounds__(256) k_sgemm_small_rows(GemmP p) {
    __shared__ float red[8][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t ngrp = (p.N + 31) / 32, m = blockIdx.x / ngrp, n = (blockIdx.x - m * ngrp) * 32 + lane;
    const bool live = n < p.N;
    const float *a = p.A + m, *b = p.B + (live ? n : 0);
    const int64_t R = p.K, lda = p.lda, ldb = p.ldb;
    float s[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    int64_t r = warp;
    for (; r + 56 < R; r += 64) {
        float av[8], bv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) av[u] = __ldg(a + (r + 8 * u) * lda), bv[u] = __ldg(b + (r + 8 * u) * ldb);
#pragma unroll
        for (int u = 0; u < 8; u++) s[u] = fmaf(av[u], bv[u], s[u]);
    }
    for (; r < R; r += 8) s[0] = fmaf(__ldg(a + r * lda), __ldg(b + r * ldb), s[0]);
    red[warp][lane] = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
    __syncthreads();
    if (warp == 0 && live) {
        float t = red[0][lane];
        for (int w = 1; w < 8; w++) t += red[w][lane];
        float *c = p.C + m * p.ldc + n;
        *c = epi(p, t, m, n, c);
    }
}

// long reductions (R >= 2048): a block of 256 threads per output, thread t taking terms t, t + 256, ...
// over four running sums; the lanes' sums go through a fixed shuffle tree and the eight warps' are
// added in order
__global__ void __launch_bounds__(256) k_sgemm_small_block(GemmP p, int64_t nout) {
    __shared__ float red[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t MN = p.M * p.N, total = nout * MN, R = p.reduce ? p.batch * p.K : p.K;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        const int64_t ob = t / MN, rm = t - ob * MN, m = rm / p.N, n = rm - m * p.N;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        int64_t r = threadIdx.x;
        for (; r + 768 < R; r += 1024) {
            a0 = small_fma(p, ob, m, n, r, a0);
            a1 = small_fma(p, ob, m, n, r + 256, a1);
            a2 = small_fma(p, ob, m, n, r + 512, a2);
            a3 = small_fma(p, ob, m, n, r + 768, a3);
        }
        for (; r < R; r += 256) a0 = small_fma(p, ob, m, n, r, a0);
        float acc = (a0 + a1) + (a2 + a3);
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            float s = red[0];
            for (int k = 1; k < 8; k++) s += red[k];
            float *c = p.C + ob * p.sC + m * p.ldc + n;
            *c = epi(p, s, m, n, c);
        }
        __syncthreads();
    }
}

}  // namespace

extern "C" void nck_gemm(nck_dev *d, const nck_gemm_args *a) {
    if (a->M <= 0 || a->N <= 0 || a->batch <= 0) return;
    const int64_t nout_s = a->reduce_batch && a->batch > 1 ? 1 : a->batch;
    const bool small = d->gemm_small && a->M * a->N * nout_s <= ((int64_t)1 << 16) &&
                       a->M * a->N * a->K * a->batch <= ((int64_t)1 << 22);
    if (!small && d->gemm_mode != NCK_GEMM_FFMA && nck_gemm_tc(d, a)) return;
    double nA = a->sA ? (double)a->batch : 1.0, nB = a->sB ? (double)a->batch : 1.0;
    double nC = (a->reduce_batch ? 1.0 : (double)a->batch) * (a->beta != 0.0f ? 2.0 : 1.0);
    Scope sc(d, "gemm_f32", 2.0 * a->M * a->N * a->K * a->batch,
             4.0 * (nA * a->M * a->K + nB * a->K * a->N + nC * a->M * a->N));
    GemmP p;
    p.ta = a->ta, p.tb = a->tb, p.M = a->M, p.N = a->N, p.K = a->K, p.alpha = a->alpha, p.beta = a->beta;
    p.A = a->A, p.lda = a->lda, p.sA = a->sA, p.B = a->B, p.ldb = a->ldb, p.sB = a->sB;
    p.C = a->C, p.ldc = a->ldc, p.sC = a->sC, p.bias = a->bias, p.bias_row = a->bias_per_row;
    p.batch = a->batch, p.reduce = a->reduce_batch && a->batch > 1;
    int64_t contA = a->ta ? a->M : a->K, contB = a->tb ? a->K : a->N;
    int64_t bstepA = a->batch > 1 ? a->sA : 0, bstepB = a->batch > 1 ? a->sB : 0;
    p.vecA = (a->lda % 4 == 0) && (contA % 4 == 0) && (bstepA % 4 == 0) && (((uintptr_t)a->A & 15) == 0);
    p.vecB = (a->ldb % 4 == 0) && (contB % 4 == 0) && (bstepB % 4 == 0) && (((uintptr_t)a->B & 15) == 0);
    p.vecC = a->N % 4 == 0;

    if (small) {
        const int64_t R = p.reduce ? a->batch * a->K : a->K, outs = nout_s * a->M * a->N;
        if (R <= 64) k_sgemm_small_thread<<<grid_for(d, outs), 256, 0, NCK_STREAM(d)>>>(p, nout_s);
        else if (a->ta && !a->tb && a->batch == 1 && a->N >= 32 && R >= 256)
            k_sgemm_small_rows<<<(unsigned)(a->M * ((a->N + 31) / 32)), 256, 0, NCK_STREAM(d)>>>(p);
        else if (R >= 2048 && outs <= 4 * (int64_t)d->sm_count * 8)
            k_sgemm_small_block<<<(unsigned)outs, 256, 0, NCK_STREAM(d)>>>(p, nout_s);
        else k_sgemm_small_warp<<<grid_for(d, outs * 32), 256, 0, NCK_STREAM(d)>>>(p, nout_s);
        NCK_LAUNCHED(d, 1);
        return;
    }
    int64_t tiles = ((a->M + BM - 1) / BM) * ((a->N + BN - 1) / BN);
    int64_t nout = p.reduce ? 1 : a->batch;
    int64_t target = (int64_t)d->sm_count * 2;
    int64_t maxpart = (int64_t)(d->scratch_bytes / sizeof(float)) / (a->M * a->N * nout);
    int64_t splits = 1;
    if (tiles * nout < target) {
        splits = (target + tiles * nout - 1) / (tiles * nout);
        int64_t cap = p.reduce ? a->batch : (a->K + 8 * BK - 1) / (8 * BK); /* split-K slices of >= 64 */
        if (splits > cap) splits = cap;
        if (splits > maxpart) splits = maxpart;
        if (splits < 1) splits = 1;
    }
    if (p.reduce) {
        p.bper = (a->batch + splits - 1) / splits;
        splits = (a->batch + p.bper - 1) / p.bper;
        p.kper = a->K;
    } else {
        p.bper = 1;
        p.kper = ((a->K + splits - 1) / splits + BK - 1) / BK * BK;
        if (p.kper < BK) p.kper = BK;
        splits = a->K > 0 ? (a->K + p.kper - 1) / p.kper : 1;
    }
    p.splits = (int)splits;
    p.part = (float *)d->scratch;
    dim3 grid((unsigned)((a->N + BN - 1) / BN), (unsigned)((a->M + BM - 1) / BM), (unsigned)(nout * splits));
    k_sgemm<<<grid, 256, 0, NCK_STREAM(d)>>>(p);
    int launched = 1;
    if (splits > 1) {
        k_sgemm_combine<<<grid_for(d, nout * a->M * a->N), kThreads, 0, NCK_STREAM(d)>>>(p, nout);
        launched++;
    }
    NCK_LAUNCHED(d, launched);
}
