// int8 dynamic quantization: per-row symmetric quantization (one warp per row) and the int8 GEMM
// with exact int32 accumulation and the fused rescale y = (float)acc * xs[r] * ws[o] + b[o].
//
// Rounding and clamping follow newch's quantize_row (engine/src/ops/ops_quant.c:11-21: scale
// amax / 127, reciprocal, round half to even, clamp to +-127) and its rescale (:77-78). The file is
// compiled without FMA contraction, so the rescale rounds as newch's.
#include <math.h>

#include <string.h>

#include "k_common.cuh"
#include "k_tcgen05.cuh"
#include "k_unary.cuh"

using namespace nck;

__global__ void k_quantize_rows(const float *__restrict__ x, int8_t *__restrict__ q, float *__restrict__ scale,
                                int64_t rows, int64_t cols) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5, nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < rows; r += nw) {
        const float *p = x + r * cols;
        float amax = 0.0f;
        for (int64_t i = lane; i < cols; i += 32) amax = fmaxf(amax, fabsf(p[i]));
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        float inv = 1.0f / s;
        int8_t *qr = q + r * cols;
        for (int64_t i = lane; i < cols; i += 32) {
            float v = rintf(p[i] * inv);
            qr[i] = (int8_t)(v > 127.0f ? 127.0f : v < -127.0f ? -127.0f : v);
        }
        if (lane == 0) scale[r] = s;
    }
}

// One block per row of 1024 NV columns, the row in registers (NV float4 per thread): one read of x,
// the activation (act >= 0: a NCK_UN_* kind applied to x first, as the unary kernel computes it)
// evaluated once per element, the row's amax by a warp tree and a block tree (a maximum: any order
// gives the same value), then the same scale, reciprocal, rounding and clamp as k_quantize_rows.
template <int M, int NV>
__global__ void __launch_bounds__(256) k_quantize_rows_reg(const float *__restrict__ x, int act, float act_s,
                                                           int8_t *__restrict__ q, float *__restrict__ scale,
                                                           int64_t cols) {
    __shared__ float red[8];
    const int64_t r = blockIdx.x;
    const float4 *p = reinterpret_cast<const float4 *>(x + r * cols);
    float4 v[NV];
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; k++) {
        v[k] = __ldcs(p + threadIdx.x + 256 * k);
        if (act >= 0) {
            v[k].x = unary_f<M>(act, act_s, v[k].x), v[k].y = unary_f<M>(act, act_s, v[k].y);
            v[k].z = unary_f<M>(act, act_s, v[k].z), v[k].w = unary_f<M>(act, act_s, v[k].w);
        }
        amax = fmaxf(amax, fabsf(v[k].x)), amax = fmaxf(amax, fabsf(v[k].y));
        amax = fmaxf(amax, fabsf(v[k].z)), amax = fmaxf(amax, fabsf(v[k].w));
    }
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < 8; w++) amax = fmaxf(amax, red[w]);
    const float sc = amax > 0.0f ? amax / 127.0f : 1.0f;
    const float inv = 1.0f / sc;
    char4 *qr = reinterpret_cast<char4 *>(q + r * cols);
#pragma unroll
    for (int k = 0; k < NV; k++) {
        const float e[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        signed char o[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float t = rintf(e[i] * inv);
            o[i] = (signed char)(t > 127.0f ? 127.0f : t < -127.0f ? -127.0f : t);
        }
        qr[threadIdx.x + 256 * k] = make_char4(o[0], o[1], o[2], o[3]);
    }
    if (threadIdx.x == 0) scale[r] = sc;
}

extern "C" int nck_quantize_rows_act_ok(int64_t cols) {
    return cols == 1024 || cols == 2048 || cols == 4096 || cols == 8192;
}

extern "C" void nck_quantize_rows_act(nck_dev *d, const float *x, int act, float act_s, int8_t *q, float *scale,
                                      int64_t rows, int64_t cols) {
    if (rows <= 0) return;
    Scope sc(d, act >= 0 ? "act_quantize_rows" : "quantize_rows", 0.0, 5.0 * rows * cols + 4.0 * rows);
    const bool aligned = (((uintptr_t)x | (uintptr_t)q) & 15) == 0;
    if (!aligned || !nck_quantize_rows_act_ok(cols)) {
        /* the general kernel has no activation: this form is only used for act < 0 */
        k_quantize_rows<<<grid_for(d, rows * 32), kThreads, 0, NCK_STREAM(d)>>>(x, q, scale, rows, cols);
        NCK_LAUNCHED(d, 1);
        return;
    }
    const bool libm = d->math_mode == MATH_LIBM;
#define NCK_QR(NV)                                                                                          \
    (libm ? k_quantize_rows_reg<MATH_LIBM, NV> : k_quantize_rows_reg<MATH_POLY, NV>)<<<(unsigned)rows, 256, 0, \
                                                                                    NCK_STREAM(d)>>>(           \
        x, act, act_s, q, scale, cols)
    if (cols == 1024) NCK_QR(1);
    else if (cols == 2048) NCK_QR(2);
    else if (cols == 4096) NCK_QR(4);
    else NCK_QR(8);
#undef NCK_QR
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_quantize_rows(nck_dev *d, const float *x, int8_t *q, float *scale, int64_t rows, int64_t cols) {
    if (rows <= 0) return;
    if ((((uintptr_t)x | (uintptr_t)q) & 15) == 0 && nck_quantize_rows_act_ok(cols)) {
        nck_quantize_rows_act(d, x, -1, 0.0f, q, scale, rows, cols);
        return;
    }
    Scope sc(d, "quantize_rows", 0.0, 5.0 * rows * cols + 4.0 * rows);
    k_quantize_rows<<<grid_for(d, rows * 32), kThreads, 0, NCK_STREAM(d)>>>(x, q, scale, rows, cols);
    NCK_LAUNCHED(d, 1);
}

// ---- int8 GEMM (dp4a): acc[m, n] = sum_k xq[m, k] * wq[n, k], both K-contiguous -------------------------

namespace {
constexpr int QBM = 128, QBN = 128, QBK = 32;  // QBK bytes of K per tile (8 packed words)

__global__ void __launch_bounds__(256) k_qgemm(const int8_t *__restrict__ A, const int8_t *__restrict__ B,
                                               const float *__restrict__ xs, const float *__restrict__ ws,
                                               const float *__restrict__ bias, float *__restrict__ Y,
                                               int32_t *__restrict__ acc_out, int64_t M, int64_t N, int64_t K,
                                               int vec) {
    __shared__ int32_t As[QBK / 4][QBM + 4];
    __shared__ int32_t Bs[QBK / 4][QBN + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * QBM, n0 = (int64_t)blockIdx.x * QBN;
    int32_t acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0;
    const int r = tid >> 1, part = (tid & 1) * 16;  // 16 bytes of one row per thread
    for (int64_t k0 = 0; k0 < K; k0 += QBK) {
        int32_t wa[4], wb[4];
        int64_t m = m0 + r, n = n0 + r, k = k0 + part;
        if (vec) {
            int4 va = make_int4(0, 0, 0, 0), vb = make_int4(0, 0, 0, 0);
            if (m < M && k < K) va = *(const int4 *)(A + m * K + k);
            if (n < N && k < K) vb = *(const int4 *)(B + n * K + k);
            wa[0] = va.x, wa[1] = va.y, wa[2] = va.z, wa[3] = va.w;
            wb[0] = vb.x, wb[1] = vb.y, wb[2] = vb.z, wb[3] = vb.w;
        } else {
            for (int w = 0; w < 4; w++) {
                uint32_t pa = 0, pb = 0;
                for (int b = 0; b < 4; b++) {
                    int64_t kk = k + w * 4 + b;
                    uint32_t ea = (m < M && kk < K) ? (uint8_t)A[m * K + kk] : 0u;
                    uint32_t eb = (n < N && kk < K) ? (uint8_t)B[n * K + kk] : 0u;
                    pa |= ea << (8 * b), pb |= eb << (8 * b);
                }
                wa[w] = (int32_t)pa, wb[w] = (int32_t)pb;
            }
        }
        __syncthreads();
#pragma unroll
        for (int w = 0; w < 4; w++) {
            As[part / 4 + w][r] = wa[w];
            Bs[part / 4 + w][r] = wb[w];
        }
        __syncthreads();
#pragma unroll
        for (int kw = 0; kw < QBK / 4; kw++) {
            int4 a0 = *(const int4 *)&As[kw][ty * 4], a1 = *(const int4 *)&As[kw][64 + ty * 4];
            int4 b0 = *(const int4 *)&Bs[kw][tx * 4], b1 = *(const int4 *)&Bs[kw][64 + tx * 4];
            int a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            int b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = __dp4a(a[i], b[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= M) continue;
        float xsm = xs[m];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int64_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (n >= N) continue;
            if (acc_out) acc_out[m * N + n] = acc[i][j];
            Y[m * N + n] = (float)acc[i][j] * xsm * ws[n] + (bias ? bias[n] : 0.0f);
        }
    }
}
}  // namespace

// ---- int8 GEMM on the tensor cores (tcgen05.mma kind::i8) ------------------------------------------------
//
// acc[m, n] = sum_k xq[m, k] * wq[n, k] exactly in int32 (the tensor core adds integer products without
// rounding), then y[m, n] = (float)acc * xs[m] * ws[n] + b[n] as above. Weight rows n run on the 128
// TMEM lanes and activation rows m along the accumulator's BN columns, so each epilogue warp store
// writes 32 consecutive outputs of one row. Persistent CTAs, one per SM: warps 0-3 epilogue, warp 4
// TMA loader (K in steps of 128 bytes, 128-byte swizzle, no multicast), warp 5 MMA issuer (4 MMAs of
// K = 32 per stage); two TMEM accumulators. Every mbarrier wait is bounded and a timeout is reported
// through the status word, after which the CTA drains its copies and MMAs and frees its TMEM.
namespace {
using namespace tc;

constexpr int kQStageP = TM * 128, kQThreads = 6 * 32;  // stage bytes of the weight tile

struct QtcParams {
    int64_t M, N, K;
    int64_t tiles_p, tiles_q, units;
    int stages;
    const float *xs, *ws, *bias;
    float *y;
    int32_t *acc_out;
    int *status;
};

struct QBars {
    uint64_t full[kMaxStages], empty[kMaxStages];
    uint64_t tfull[2], tempty[2], mma_done;
    uint32_t tmem;
};

template <int kQBN>
__global__ void __launch_bounds__(kQThreads, 1) k_qgemm_tc(const __grid_constant__ CUtensorMap tmW,
                                                           const __grid_constant__ CUtensorMap tmX, QtcParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~(uintptr_t)1023);
    QBars &s = *reinterpret_cast<QBars *>(base);
    const int S = p.stages;
    unsigned char *const ring_p = base + 1024;
    unsigned char *const ring_q = ring_p + S * kQStageP;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tcols = tmem_cols(kQBN), stage_bytes = (uint32_t)(TM + kQBN) * 128;
    const int64_t ksteps = (p.K + 127) / 128;

    if (tid == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s.tfull[i], 1);
            mbar_init(&s.tempty[i], 4);
        }
        mbar_init(&s.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem)),
                     "r"(tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = s.tmem;

    if (warp == 4) {
        if (lane == 0) {
            int64_t it = 0;
            int st = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
                // the activation tiles of one weight tile are neighbours: the weight tile stays in L2
                const int p0 = (int)((u / p.tiles_q) * TM), q0 = (int)((u % p.tiles_q) * kQBN);
                for (int64_t t = 0; t < ksteps; t++, it++) {
                    if (it >= S && !(ok = mbar_wait(&s.empty[st], ph ^ 1, p.status))) break;
                    mbar_expect_tx(&s.full[st], stage_bytes);
                    tma_2d(ring_p + st * kQStageP, &tmW, (int)(t * 128), p0, &s.full[st]);
                    tma_2d(ring_q + st * (kQBN * 128), &tmX, (int)(t * 128), q0, &s.full[st]);
                    if (++st == S) st = 0, ph ^= 1;
                }
            }
            int64_t first = it > S ? it - S : 0;
            for (int64_t j = first; j < it; j++)
                if (!mbar_wait(&s.full[j % S], (uint32_t)((j / S) & 1), p.status)) break;
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = idesc_s8(kQBN);
            const uint64_t dA = stage_desc(smem_u32(ring_p), 0, 0), dB = stage_desc(smem_u32(ring_q), 0, 0);
            const uint32_t stA = (uint32_t)kQStageP >> 4, stB = (uint32_t)(kQBN * 128) >> 4;
            int64_t local = 0;
            int st = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, local++) {
                const int acc = (int)(local & 1);
                if (local >= 2 && !(ok = mbar_wait(&s.tempty[acc], (uint32_t)(((local >> 1) & 1) ^ 1), p.status)))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t d = tmem + (uint32_t)acc * (tcols / 2);
                for (int64_t t = 0; t < ksteps; t++) {
                    if (!(ok = mbar_wait(&s.full[st], ph, p.status))) break;
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint64_t a0 = dA + (uint64_t)(st * stA), b0 = dB + (uint64_t)(st * stB);
#pragma unroll
                    for (int k = 0; k < 4; k++)  // K = 32 bytes per MMA: 2 descriptor units
                        mma_s8(d, a0 + (uint64_t)(k * 2), b0 + (uint64_t)(k * 2), idesc, (t > 0 || k > 0) ? 1u : 0u);
                    mma_commit(&s.empty[st]);
                    if (++st == S) st = 0, ph ^= 1;
                }
                if (ok) mma_commit(&s.tfull[acc]);
            }
            mma_commit(&s.mma_done);
            mbar_wait(&s.mma_done, 0, p.status);
        }
    } else if (warp < 4) {
        int64_t local = 0;
        for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x, local++) {
            const int64_t p0 = (u / p.tiles_q) * TM, q0 = (u % p.tiles_q) * kQBN;
            const int acc = (int)(local & 1);
            if (!mbar_wait(&s.tfull[acc], (uint32_t)((local >> 1) & 1), p.status)) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int64_t n = p0 + warp * 32 + lane;
            const bool live = n < p.N;
            const float wsn = live ? p.ws[n] : 0.0f, bn = (live && p.bias) ? p.bias[n] : 0.0f;
            for (int c0 = 0; c0 < kQBN; c0 += 16) {
                // the chunk's 16 row scales are read before the accumulator and the stores (a store to y
                // could alias xs for the compiler, which would otherwise re-read xs after every store)
                float xv[16];
#pragma unroll
                for (int jj = 0; jj < 16; jj++) {
                    const int64_t m = q0 + c0 + jj;
                    xv[jj] = m < p.M ? __ldg(p.xs + m) : 0.0f;
                }
                uint32_t r[16];
                tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)acc * (tcols / 2) + (uint32_t)c0, r);
                if (!live) continue;
                float *yo = p.y + (q0 + c0) * p.N + n;
                int32_t *ao = p.acc_out ? p.acc_out + (q0 + c0) * p.N + n : nullptr;
                const int nj = p.M - (q0 + c0) < 16 ? (int)(p.M - (q0 + c0)) : 16;
#pragma unroll
                for (int jj = 0; jj < 16; jj++) {
                    if (jj < nj) {
                        const int32_t a = (int32_t)r[jj];
                        if (ao) ao[jj * p.N] = a;
                        yo[jj * p.N] = (float)a * xv[jj] * wsn + bn;
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.tempty[acc]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
}

template <int kQBN>
int qgemm_tc_launch(nck_dev *d, const int8_t *wq, const int8_t *xq, const float *xs, const float *ws, const float *b,
                    float *y, int64_t M, int64_t N, int64_t K, int32_t *acc_out);

// 1 when launched on the tensor cores; 0 when the operands do not fit TMA (K not a multiple of 16
// bytes, unaligned bases) or the product is tiny, and the dp4a kernel is used
int qgemm_tc(nck_dev *d, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, const float *b,
             float *y, int64_t M, int64_t N, int64_t K, int32_t *acc_out) {
    if (!d->qgemm_tc || K % 16 || (((uintptr_t)xq | (uintptr_t)wq) & 15) || M * N < 4096 || M >= ((int64_t)1 << 31) ||
        N >= ((int64_t)1 << 31) || K >= ((int64_t)1 << 31))
        return 0;
    // activation rows per tile: 256 for tall products (each weight panel staged from L2 once per 256
    // rows instead of 128, halving the panel traffic per MMA), 128 otherwise
    if (M >= 2048) return qgemm_tc_launch<256>(d, wq, xq, xs, ws, b, y, M, N, K, acc_out);
    return qgemm_tc_launch<128>(d, wq, xq, xs, ws, b, y, M, N, K, acc_out);
}

template <int kQBN>
int qgemm_tc_launch(nck_dev *d, const int8_t *wq, const int8_t *xq, const float *xs, const float *ws, const float *b,
                    float *y, int64_t M, int64_t N, int64_t K, int32_t *acc_out) {
    CUtensorMap mw, mx;
    if (!make_map_u8(&mw, wq, K, N, K, 128, TM) || !make_map_u8(&mx, xq, K, M, K, 128, kQBN)) return 0;
    static int attr = 0;
    if (!attr) {
        if (cudaFuncSetAttribute(k_qgemm_tc<kQBN>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) !=
            cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        attr = 1;
    }
    QtcParams p;
    memset(&p, 0, sizeof p);
    p.M = M, p.N = N, p.K = K, p.xs = xs, p.ws = ws, p.bias = b, p.y = y, p.acc_out = acc_out, p.status = d->status;
    p.tiles_p = (N + TM - 1) / TM, p.tiles_q = (M + kQBN - 1) / kQBN, p.units = p.tiles_p * p.tiles_q;
    const size_t per = (size_t)(TM + kQBN) * 128;
    size_t nst = (kSmemLimit - 2048) / per;
    p.stages = (int)(nst > (size_t)kMaxStages ? kMaxStages : nst);
    const size_t smem = 2048 + (size_t)p.stages * per;
    const int64_t sms = d->sm_count > 0 ? d->sm_count : 148;
    const unsigned grid = (unsigned)(p.units < sms ? p.units : sms);
    k_qgemm_tc<kQBN><<<grid, kQThreads, smem, NCK_STREAM(d)>>>(mw, mx, p);
    if (cudaGetLastError() != cudaSuccess) *(volatile int *)d->status_host = NCK_ERR_LAUNCH;
    NCK_LAUNCHED(d, 1);
    return 1;
}
}  // namespace

extern "C" void nck_qlinear(nck_dev *d, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                            const float *b, float *y, int64_t M, int64_t N, int64_t K, int32_t *acc_out) {
    if (M <= 0 || N <= 0) return;
    Scope sc(d, "qgemm_i8", 2.0 * M * N * K, (double)M * K + (double)N * K + 4.0 * M * N);
    if (qgemm_tc(d, xq, xs, wq, ws, b, y, M, N, K, acc_out)) return;
    int vec = K % 16 == 0 && (((uintptr_t)xq | (uintptr_t)wq) & 15) == 0;
    dim3 grid((unsigned)((N + QBN - 1) / QBN), (unsigned)((M + QBM - 1) / QBM));
    k_qgemm<<<grid, 256, 0, NCK_STREAM(d)>>>(xq, wq, xs, ws, b, y, acc_out, M, N, K, vec);
    NCK_LAUNCHED(d, 1);
}
