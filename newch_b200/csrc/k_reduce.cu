// Reductions: axis sums / means / max / argmax and their gradients, column sums for bias
// gradients, sums of squares for gradient clipping. Every output is produced by one thread, one
// warp or a fixed split followed by an in-order combine: results do not depend on scheduling.
#include <math.h>

#include "k_common.cuh"

using namespace nck;

// ---- per-output sums ---------------------------------------------------------------------------------

// inner == 1: one warp per output row, lanes stride the row, a fixed shuffle tree combines them
__global__ void k_rowsum(const float *__restrict__ x, float *__restrict__ y, int64_t rows, int64_t R, float scale) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < rows; r += nwarps) {
        const float *p = x + r * R;
        float s = 0.0f;
        for (int64_t i = lane; i < R; i += 32) s += p[i];
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) y[r] = scale * s;
    }
}

// short rows (R a multiple of 4, at most 128, 16-byte aligned): LPR lanes per row (R / 4 rounded up
// to a power of two), one float4 each, a tree over the row's lanes; a warp takes 32 / LPR rows per pass
// and four passes' loads are issued before their sums
template <int LPR>
__global__ void k_rowsum_short(const float *__restrict__ x, float *__restrict__ y, int64_t rows, int R, float scale) {
    constexpr int RPW = 32 / LPR;  // rows per warp pass
    const int lane = threadIdx.x & 31, sub = lane % LPR, rw = lane / LPR;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const bool col = 4 * sub < R;
    for (int64_t r0 = warp * RPW; r0 < rows; r0 += 4 * nwarps * RPW) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t r = r0 + (int64_t)u * nwarps * RPW + rw;
            v[u] = (r < rows && col) ? __ldg(reinterpret_cast<const float4 *>(x + r * R) + sub)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t r = r0 + (int64_t)u * nwarps * RPW + rw;
            float s = (v[u].x + v[u].y) + (v[u].z + v[u].w);
#pragma unroll
            for (int o = LPR / 2; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (sub == 0 && r < rows) y[r] = scale * s;
        }
    }
}

// inner > 1: one thread per (outer, inner) column, rows added in order with the scale fused
__global__ void k_colsum_strided(const float *__restrict__ x, float *__restrict__ y, int64_t outer, int64_t R,
                                 int64_t inner, float scale) {
    int64_t n = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = t / inner, i = t - o * inner;
        const float *p = x + o * R * inner + i;
        float acc = 0.0f;
        for (int64_t r = 0; r < R; r++) acc = fmaf(scale, p[r * inner], acc);
        y[t] = acc;
    }
}

// few long rows (a full-tensor sum): block (slice, row) sums a contiguous slice with four
// accumulators and a fixed tree; k_rowsum_combine adds the slices of a row in order
__global__ void __launch_bounds__(256) k_rowsum_split(const float *__restrict__ x, float *__restrict__ part, int64_t R,
                                                      int64_t per, int vec) {
    __shared__ float sm[8];
    const int64_t r = blockIdx.y, s0 = blockIdx.x * per, s1 = s0 + per < R ? s0 + per : R;
    const float *p = x + r * R;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    if (vec) {  // per and the row base are multiples of 4 floats
        const float4 *q = reinterpret_cast<const float4 *>(p + s0);
        const int64_t n4 = (s1 - s0) / 4;
        for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
            float4 v = __ldg(q + i);
            a0 += v.x, a1 += v.y, a2 += v.z, a3 += v.w;
        }
        for (int64_t i = s0 + n4 * 4 + threadIdx.x; i < s1; i += blockDim.x) a0 += __ldg(p + i);
    } else {
        for (int64_t i = s0 + threadIdx.x; i < s1; i += blockDim.x) a0 += __ldg(p + i);
    }
    float acc = (a0 + a1) + (a2 + a3);
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) t += sm[k];
        part[r * gridDim.x + blockIdx.x] = t;
    }
}

__global__ void k_rowsum_combine(const float *__restrict__ part, int splits, int64_t rows, float *__restrict__ y,
                                 float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        float s = 0.0f;
        for (int k = lane; k < splits; k += 32) s += part[r * splits + k];
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) y[r] = scale * s;
    }
}

extern "C" void nck_reduce_sum(nck_dev *d, const float *x, float *y, int64_t outer, int64_t R, int64_t inner,
                               float scale) {
    int64_t n = outer * inner;
    if (n <= 0) return;
    Scope sc(d, "reduce_sum", 0.0, 4.0 * (n * R + n));
    if (R == 0) {
        cudaMemsetAsync(y, 0, (size_t)n * sizeof(float), NCK_STREAM(d));
        return;
    }
    const int64_t sms = d->sm_count > 0 ? d->sm_count : 148;
    if (inner == 1 && n < sms * 4 && R >= 65536) {
        int64_t splits = (sms * 8 + n - 1) / n;
        int64_t per = ((R + splits - 1) / splits + 3) / 4 * 4;
        splits = (R + per - 1) / per;
        if (n * splits * (int64_t)sizeof(float) <= (int64_t)d->scratch_bytes && splits <= 65535) {
            float *part = (float *)d->scratch;
            const int vec = (R % 4 == 0) && (((uintptr_t)x & 15) == 0);
            dim3 grid((unsigned)splits, (unsigned)n);
            k_rowsum_split<<<grid, 256, 0, NCK_STREAM(d)>>>(x, part, R, per, vec);
            k_rowsum_combine<<<grid_for(d, n * 32), kThreads, 0, NCK_STREAM(d)>>>(part, (int)splits, n, y, scale);
            NCK_LAUNCHED(d, 2);
            return;
        }
    }
    if (inner == 1 && R % 4 == 0 && R <= 128 && ((uintptr_t)x & 15) == 0) {
        const int lpr = R <= 4 ? 1 : R <= 8 ? 2 : R <= 16 ? 4 : R <= 32 ? 8 : R <= 64 ? 16 : 32;
        const int64_t warps = (n * lpr + 31) / 32, items = (warps + 3) / 4 * 32;
#define NCK_RS(L) k_rowsum_short<L><<<grid_for(d, items), kThreads, 0, NCK_STREAM(d)>>>(x, y, n, (int)R, scale)
        if (lpr == 1) NCK_RS(1);
        else if (lpr == 2) NCK_RS(2);
        else if (lpr == 4) NCK_RS(4);
        else if (lpr == 8) NCK_RS(8);
        else if (lpr == 16) NCK_RS(16);
        else NCK_RS(32);
#undef NCK_RS
    } else if (inner == 1) {
        k_rowsum<<<grid_for(d, n * 32), kThreads, 0, NCK_STREAM(d)>>>(x, y, n, R, scale);
    } else {
        k_colsum_strided<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(x, y, outer, R, inner, scale);
    }
    NCK_LAUNCHED(d, 1);
}

__global__ void k_reduce_sum_i32(const int32_t *__restrict__ x, int32_t *__restrict__ y, int64_t outer, int64_t R,
                                 int64_t inner) {
    int64_t n = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = t / inner, i = t - o * inner;
        int64_t s = 0;
        for (int64_t r = 0; r < R; r++) s += x[(o * R + r) * inner + i];
        y[t] = (int32_t)s;
    }
}

extern "C" void nck_reduce_sum_i32(nck_dev *d, const int32_t *x, int32_t *y, int64_t outer, int64_t R,
                                   int64_t inner) {
    int64_t n = outer * inner;
    if (n <= 0) return;
    Scope sc(d, "reduce_sum_i32");
    k_reduce_sum_i32<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(x, y, outer, R, inner);
    NCK_LAUNCHED(d, 1);
}

// first maximum wins (strictly greater replaces), as newch's reduce (ops_reduce.c:101-108)
__global__ void k_reduce_max(const float *__restrict__ x, float *__restrict__ y, int32_t *__restrict__ arg,
                             int64_t outer, int64_t R, int64_t inner) {
    int64_t n = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = t / inner, i = t - o * inner;
        const float *p = x + o * R * inner + i;
        float bv = p[0];
        int32_t best = 0;
        for (int64_t r = 1; r < R; r++) {
            float v = p[r * inner];
            if (v > bv) bv = v, best = (int32_t)r;
        }
        arg[t] = best;
        if (y) y[t] = bv;
    }
}

extern "C" void nck_reduce_max(nck_dev *d, const float *x, float *y, int32_t *arg, int64_t outer, int64_t R,
                               int64_t inner) {
    int64_t n = outer * inner;
    if (n <= 0) return;
    Scope sc(d, y ? "reduce_max" : "argmax");
    k_reduce_max<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(x, y, arg, outer, R, inner);
    NCK_LAUNCHED(d, 1);
}

// ---- gradients --------------------------------------------------------------------------------------

// gi (+)= scale * g broadcast over the reduced extent R. acc == 0: gi is a fresh buffer and is
// stored (scale * g, what accumulating into zeros gives). R a multiple of 4 with inner == 1: float4
// items, each inside one broadcast run, with 32-bit fast division.
template <bool ACC>
__global__ void k_reduce_sum_bwd(const float *__restrict__ g, float *__restrict__ gi, int64_t outer, int64_t R,
                                 int64_t inner, float scale, int vec, FastDiv dR) {
    const int64_t n = outer * R * inner, stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {
        float4 *g4 = reinterpret_cast<float4 *>(gi);
        for (int64_t t4 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t4 < n / 4; t4 += stride) {
            const float v = scale * __ldg(g + dR.div((uint32_t)(4 * t4)));
            float4 o;
            if (ACC) {
                o = g4[t4];
                o.x = o.x + v, o.y = o.y + v, o.z = o.z + v, o.w = o.w + v;
            } else {
                o = make_float4(v, v, v, v);
            }
            g4[t4] = o;
        }
        return;
    }
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += stride) {
        int64_t i = t % inner, o = t / (R * inner);
        float gv = g[o * inner + i];
        if (ACC) gi[t] = inner == 1 ? gi[t] + scale * gv : fmaf(scale, gv, gi[t]);
        else gi[t] = scale * gv;
    }
}

extern "C" void nck_reduce_sum_bwd(nck_dev *d, const float *g, float *gi, int64_t outer, int64_t R, int64_t inner,
                                   float scale, int acc) {
    int64_t n = outer * R * inner;
    if (n <= 0) return;
    Scope sc(d, "reduce_sum_bwd", 0.0, 4.0 * (outer * inner + (acc ? 2.0 : 1.0) * n));
    const int vec = inner == 1 && R % 4 == 0 && ((uintptr_t)gi & 15) == 0 && n < ((int64_t)1 << 32);
    const FastDiv dR = make_fastdiv((uint32_t)(vec ? R : 1));
    const int64_t items = vec ? n / 4 : n;
    if (acc) k_reduce_sum_bwd<true><<<grid_for(d, items), kThreads, 0, NCK_STREAM(d)>>>(g, gi, outer, R, inner, scale, vec, dR);
    else k_reduce_sum_bwd<false><<<grid_for(d, items), kThreads, 0, NCK_STREAM(d)>>>(g, gi, outer, R, inner, scale, vec, dR);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_reduce_max_bwd(const float *__restrict__ g, const int32_t *__restrict__ arg, float *__restrict__ gi,
                                 int64_t outer, int64_t R, int64_t inner) {
    int64_t n = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = t / inner, i = t - o * inner;
        gi[(o * R + arg[t]) * inner + i] += g[t];
    }
}

extern "C" void nck_reduce_max_bwd(nck_dev *d, const float *g, const int32_t *arg, float *gi, int64_t outer, int64_t R,
                                   int64_t inner) {
    int64_t n = outer * inner;
    if (n <= 0) return;
    Scope sc(d, "reduce_max_bwd");
    k_reduce_max_bwd<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(g, arg, gi, outer, R, inner);
    NCK_LAUNCHED(d, 1);
}

// ---- column sums of a [M, N] matrix (bias gradients): split M, combine the partials in order ----------

constexpr int kColRows = 8;  // threadIdx.y extent

__global__ void k_colsum_partial(const float *__restrict__ x, float *__restrict__ part, int64_t M, int64_t N,
                                 int64_t rows_per_split) {
    __shared__ float sm[kColRows][33];
    int64_t n = blockIdx.x * 32 + threadIdx.x;
    int64_t m0 = blockIdx.y * rows_per_split, m1 = m0 + rows_per_split < M ? m0 + rows_per_split : M;
    float acc = 0.0f;
    if (n < N) {
        // four rows' loads in flight, added in row order
        int64_t m = m0 + threadIdx.y;
        for (; m + 3 * kColRows < m1; m += 4 * kColRows) {
            const float v0 = __ldg(x + m * N + n), v1 = __ldg(x + (m + kColRows) * N + n);
            const float v2 = __ldg(x + (m + 2 * kColRows) * N + n), v3 = __ldg(x + (m + 3 * kColRows) * N + n);
            acc += v0, acc += v1, acc += v2, acc += v3;
        }
        for (; m < m1; m += kColRows) acc += __ldg(x + m * N + n);
    }
    sm[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && n < N) {
        float s = sm[0][threadIdx.x];
        for (int k = 1; k < kColRows; k++) s += sm[k][threadIdx.x];
        part[blockIdx.y * N + n] = s;
    }
}

// float4 columns: a block of (32, kColRows) threads takes 128 columns; thread (x, y) adds rows
// y, y + kColRows, ... of columns 4x .. 4x + 3 with four rows' loads in flight, in row order; the
// kColRows partial sums are added in order
__global__ void k_colsum_partial4(const float *__restrict__ x, float *__restrict__ part, int64_t M, int64_t N,
                                  int64_t rows_per_split) {
    __shared__ float4 sm[kColRows][32];
    const int64_t n = blockIdx.x * 128 + 4 * threadIdx.x;
    const int64_t m0 = blockIdx.y * rows_per_split, m1 = m0 + rows_per_split < M ? m0 + rows_per_split : M;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n < N) {
        int64_t m = m0 + threadIdx.y;
        for (; m + 3 * kColRows < m1; m += 4 * kColRows) {
            const float4 v0 = __ldg(reinterpret_cast<const float4 *>(x + m * N + n));
            const float4 v1 = __ldg(reinterpret_cast<const float4 *>(x + (m + kColRows) * N + n));
            const float4 v2 = __ldg(reinterpret_cast<const float4 *>(x + (m + 2 * kColRows) * N + n));
            const float4 v3 = __ldg(reinterpret_cast<const float4 *>(x + (m + 3 * kColRows) * N + n));
            acc.x += v0.x, acc.y += v0.y, acc.z += v0.z, acc.w += v0.w;
            acc.x += v1.x, acc.y += v1.y, acc.z += v1.z, acc.w += v1.w;
            acc.x += v2.x, acc.y += v2.y, acc.z += v2.z, acc.w += v2.w;
            acc.x += v3.x, acc.y += v3.y, acc.z += v3.z, acc.w += v3.w;
        }
        for (; m < m1; m += kColRows) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(x + m * N + n));
            acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
        }
    }
    sm[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && n < N) {
        float4 t = sm[0][threadIdx.x];
        for (int k = 1; k < kColRows; k++) {
            const float4 u = sm[k][threadIdx.x];
            t.x += u.x, t.y += u.y, t.z += u.z, t.w += u.w;
        }
        *reinterpret_cast<float4 *>(part + blockIdx.y * N + n) = t;
    }
}

__global__ void k_colsum_combine(const float *__restrict__ part, float *__restrict__ gy, int64_t N, int splits) {
    for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N; n += (int64_t)gridDim.x * blockDim.x) {
        float s = gy[n];
        for (int k = 0; k < splits; k++) s += part[k * N + n];
        gy[n] = s;
    }
}

// small matrices in one launch: a block of 32 warps takes 32 columns; warp w adds rows w, w + 32, ...
// of each column (two running sums), and the 32 warp sums are added in order; rows are ld apart
__global__ void __launch_bounds__(1024) k_colsum_small(const float *__restrict__ x, int64_t ld, float *__restrict__ gy,
                                                        int64_t M, int64_t N) {
    __shared__ float sm[32][33];
    const int64_t n = blockIdx.x * 32 + threadIdx.x;
    float a0 = 0.0f, a1 = 0.0f;
    if (n < N) {
        int64_t m = threadIdx.y;
        for (; m + 32 < M; m += 64) a0 += __ldcg(x + m * ld + n), a1 += __ldcg(x + (m + 32) * ld + n);
        if (m < M) a0 += __ldcg(x + m * ld + n);
    }
    sm[threadIdx.y][threadIdx.x] = a0 + a1;
    __syncthreads();
    if (threadIdx.y == 0 && n < N) {
        float s = gy[n];
        for (int k = 0; k < 32; k++) s += sm[k][threadIdx.x];
        gy[n] = s;
    }
}

// Sums of `splits` partial rows (row r at part + r * ldp) per column, added to y[n] (n < n1) or
// y2[n - n1] (n >= n1): a block of 32 warps takes 32 columns, warp w adds rows w, w + 32, ... in
// order (loads four rows ahead), and the 32 warp sums are added in warp order. A fixed order for a
// given split count, with a few loads in flight per warp instead of one thread walking every row.
__global__ void __launch_bounds__(1024) k_combine_cols(const float *__restrict__ part, int64_t ldp, int splits,
                                                       int64_t N, float *__restrict__ y, int64_t n1,
                                                       float *__restrict__ y2) {
    __shared__ float sm[32][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t n = blockIdx.x * 32 + lane;
    float a = 0.0f;
    if (n < N) {
        int r = w;
        for (; r + 96 < splits; r += 128) {
            const float v0 = __ldcg(part + (int64_t)r * ldp + n), v1 = __ldcg(part + (int64_t)(r + 32) * ldp + n);
            const float v2 = __ldcg(part + (int64_t)(r + 64) * ldp + n), v3 = __ldcg(part + (int64_t)(r + 96) * ldp + n);
            a += v0, a += v1, a += v2, a += v3;
        }
        for (; r < splits; r += 32) a += __ldcg(part + (int64_t)r * ldp + n);
    }
    sm[w][lane] = a;
    __syncthreads();
    if (w == 0 && n < N) {
        float s = 0.0f;
        for (int k = 0; k < 32; k++) s += sm[k][lane];
        if (n < n1) y[n] += s;
        else y2[n - n1] += s;
    }
}

extern "C" void nck_combine_cols(nck_dev *d, const float *part, int64_t ldp, int splits, int64_t N, float *y,
                                 int64_t n1, float *y2) {
    if (N <= 0 || splits <= 0) return;
    k_combine_cols<<<(unsigned)((N + 31) / 32), 1024, 0, NCK_STREAM(d)>>>(part, ldp, splits, N, y, n1, y2);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_colsum_acc(nck_dev *d, const float *x, float *gy, int64_t M, int64_t N) {
    if (M <= 0 || N <= 0) return;
    Scope sc(d, "colsum");
    // one block per 32 columns only when that fills the GPU or the columns are short
    if (M * N <= ((int64_t)1 << 20) && (M <= 1024 || (N + 31) / 32 >= d->sm_count)) {
        k_colsum_small<<<(unsigned)((N + 31) / 32), dim3(32, 32), 0, NCK_STREAM(d)>>>(x, N, gy, M, N);
        NCK_LAUNCHED(d, 1);
        return;
    }
    // float4 columns (N a multiple of 4, 16-byte rows) and about eight blocks per SM: enough loads in
    // flight for HBM; otherwise one float per thread
    const bool v4 = N % 4 == 0 && ((uintptr_t)x & 15) == 0;
    int64_t col_blocks = v4 ? (N + 127) / 128 : (N + 31) / 32;
    int64_t want = (int64_t)d->sm_count * (v4 ? 8 : 4);
    int64_t splits = want / col_blocks;
    if (splits < 1) splits = 1;
    if (splits > M / 64 + 1) splits = M / 64 + 1;
    if (splits * N * (int64_t)sizeof(float) > (int64_t)d->scratch_bytes) splits = (int64_t)d->scratch_bytes / (N * 4);
    if (splits < 1) splits = 1;
    int64_t rows_per = (M + splits - 1) / splits;
    splits = (M + rows_per - 1) / rows_per;
    float *part = (float *)d->scratch;
    dim3 grid((unsigned)col_blocks, (unsigned)splits), block(32, kColRows);
    if (v4) k_colsum_partial4<<<grid, block, 0, NCK_STREAM(d)>>>(x, part, M, N, rows_per);
    else k_colsum_partial<<<grid, block, 0, NCK_STREAM(d)>>>(x, part, M, N, rows_per);
    NCK_LAUNCHED(d, 1);
    nck_combine_cols(d, part, N, (int)splits, N, gy, N, nullptr);
}

// ---- sum of squares (double) ---------------------------------------------------------------------------

__global__ void k_sumsq_partial(const float *__restrict__ x, int64_t n, double *__restrict__ part) {
    __shared__ double sm[kThreads / 32];
    double acc = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        acc += (double)x[i] * (double)x[i];
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int k = 0; k < kThreads / 32; k++) s += sm[k];
        part[blockIdx.x] = s;
    }
}

__global__ void k_sumsq_combine(const double *__restrict__ part, int nb, double *out, int accumulate) {
    double s = accumulate ? *out : 0.0;
    for (int k = 0; k < nb; k++) s += part[k];
    *out = s;
}

extern "C" void nck_sumsq(nck_dev *d, const float *x, int64_t n, double *out, int accumulate) {
    Scope sc(d, "sumsq");
    int nb = n > 0 ? grid_for(d, n, kThreads, 4) : 1;
    double *part = (double *)d->scratch;
    if (n > 0) k_sumsq_partial<<<nb, kThreads, 0, NCK_STREAM(d)>>>(x, n, part);
    else cudaMemsetAsync(part, 0, sizeof(double), NCK_STREAM(d));
    k_sumsq_combine<<<1, 1, 0, NCK_STREAM(d)>>>(part, nb, out, accumulate);
    NCK_LAUNCHED(d, 2);
}

extern "C" void nck_colsum_ld(nck_dev *d, const float *x, int64_t ld, float *gy, int64_t M, int64_t N) {
    if (M <= 0 || N <= 0) return;
    k_colsum_small<<<(unsigned)((N + 31) / 32), dim3(32, 32), 0, NCK_STREAM(d)>>>(x, ld, gy, M, N);
    NCK_LAUNCHED(d, 1);
}
