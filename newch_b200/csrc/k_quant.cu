// int8 dynamic quantization: per-row symmetric quantization (one warp per row) and the int8 GEMM
// with exact int32 accumulation and the fused rescale y = (float)acc * xs[r] * ws[o] + b[o].
//
// Rounding and clamping follow newch's quantize_row (engine/src/ops/ops_quant.c:11-21: scale
// amax / 127, reciprocal, round half to even, clamp to +-127) and its rescale (:77-78). The file is
// compiled without FMA contraction, so the rescale rounds as newch's.
#include <math.h>

#include "k_common.cuh"

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

extern "C" void nck_quantize_rows(nck_dev *d, const float *x, int8_t *q, float *scale, int64_t rows, int64_t cols) {
    if (rows <= 0) return;
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

extern "C" void nck_qlinear(nck_dev *d, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                            const float *b, float *y, int64_t M, int64_t N, int64_t K, int32_t *acc_out) {
    if (M <= 0 || N <= 0) return;
    Scope sc(d, "qgemm_i8", 2.0 * M * N * K, (double)M * K + (double)N * K + 4.0 * M * N);
    int vec = K % 16 == 0 && (((uintptr_t)xq | (uintptr_t)wq) & 15) == 0;
    dim3 grid((unsigned)((N + QBN - 1) / QBN), (unsigned)((M + QBM - 1) / QBM));
    k_qgemm<<<grid, 256, 0, NCK_STREAM(d)>>>(xq, wq, xs, ws, b, y, acc_out, M, N, K, vec);
    NCK_LAUNCHED(d, 1);
}
