// NN kernels: softmax / log-softmax rows, cross entropy, NLL, dropout on the engine's xoshiro256**
// stream, batch norm, layer norm.
//
// Arithmetic follows newch engine/src/ops/ops_nn.c (softmax_row :22-35, cross entropy :107-149,
// dropout :182-204, batch norm :262-349, NLL :387-416, layer norm :463-522), including its double
// accumulators; this file is compiled without FMA contraction so the float expressions round as
// newch's C loops do. Reductions run as fixed-shape trees and splits combined in a fixed order.
#include <math.h>

#include "k_act.cuh"
#include "k_common.cuh"
#include "k_tcgen05.cuh"
#include "k_math.cuh"

#include <mutex>
#include <type_traits>

#include "../../include/nc_ext.h"

using namespace nck;

__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- softmax rows: one warp per row --------------------------------------------------------------------

// row maximum the way newch scans it (first element, then strictly greater): NaN rows stay NaN-free
// only if newch's are; for finite rows every order gives the same maximum
__device__ __forceinline__ float row_max(const float *p, int64_t C, int lane) {
    float m = -INFINITY;
    for (int64_t c = lane; c < C; c += 32) m = fmaxf(m, p[c]);
    return warp_max(m);
}

template <int M>
__global__ void k_softmax_fwd(const float *__restrict__ x, float *__restrict__ y, int64_t rows, int64_t C, int logf_) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5, nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < rows; r += nw) {
        const float *p = x + r * C;
        float *q = y + r * C;
        float m = row_max(p, C, lane);
        float s = 0.0f;
        for (int64_t c = lane; c < C; c += 32) s += m_exp<M>(p[c] - m);
        s = warp_sum(s);
        if (logf_) {
            float ls = logf(s);
            for (int64_t c = lane; c < C; c += 32) q[c] = p[c] - m - ls;
        } else {
            float inv = 1.0f / s;
            for (int64_t c = lane; c < C; c += 32) q[c] = inv * m_exp<M>(p[c] - m);
        }
    }
}

extern "C" void nck_softmax_fwd(nck_dev *d, const float *x, float *y, int64_t rows, int64_t C, int log_form) {
    Scope sc(d, log_form ? "log_softmax" : "softmax", 0.0, 8.0 * rows * C);
    auto k = d->math_mode == MATH_LIBM ? k_softmax_fwd<MATH_LIBM> : k_softmax_fwd<MATH_POLY>;
    k<<<grid_for(d, rows * 32), kThreads, 0, NCK_STREAM(d)>>>(x, y, rows, C, log_form);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_softmax_bwd(const float *__restrict__ y, const float *__restrict__ g, float *__restrict__ gi,
                              int64_t rows, int64_t C, int logf_) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5, nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < rows; r += nw) {
        const float *yr = y + r * C, *gr = g + r * C;
        float *o = gi + r * C;
        float acc = 0.0f;
        if (logf_) {
            for (int64_t c = lane; c < C; c += 32) acc += gr[c];
            acc = warp_sum(acc);
            for (int64_t c = lane; c < C; c += 32) o[c] += gr[c] - expf(yr[c]) * acc;
        } else {
            for (int64_t c = lane; c < C; c += 32) acc += gr[c] * yr[c];
            acc = warp_sum(acc);
            for (int64_t c = lane; c < C; c += 32) o[c] += yr[c] * (gr[c] - acc);
        }
    }
}

extern "C" void nck_softmax_bwd(nck_dev *d, const float *y, const float *g, float *gi, int64_t rows, int64_t C,
                                int log_form) {
    Scope sc(d, log_form ? "log_softmax_bwd" : "softmax_bwd", 0.0, 16.0 * rows * C);
    k_softmax_bwd<<<grid_for(d, rows * 32), kThreads, 0, NCK_STREAM(d)>>>(y, g, gi, rows, C, log_form);
    NCK_LAUNCHED(d, 1);
}

// ---- losses ----------------------------------------------------------------------------------------------

// sum of n per-row terms in double (fixed tree), negated and divided: out = -sum / div (div 0 = NaN mean)
__global__ void k_loss_combine(const float *__restrict__ terms, int64_t n, float *out, int mean) {
    __shared__ double sm[kThreads / 32];
    double acc = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) acc += (double)terms[i];
    acc = warp_sum_d(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int k = 0; k < kThreads / 32; k++) s += sm[k];
        double loss = -s;
        *out = mean ? (n ? (float)(loss / (double)n) : NAN) : (float)loss;
    }
}

__device__ __forceinline__ int32_t checked_label(const int32_t *lab, int64_t i, int64_t C, int *status) {
    int32_t l = lab[i];
    if (l < 0 || l >= C) {
        report(status, NCK_ERR_LABEL);
        return 0;
    }
    return l;
}

// the loss from the rows' terms, summed by the block that finishes last in k_loss_combine's order
__device__ void loss_combine_block(const float *terms, int64_t n, float *out, int mean) {
    __shared__ double sm[kThreads / 32];
    double acc = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) acc += (double)__ldcg(terms + i);
    acc = warp_sum_d(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int k = 0; k < kThreads / 32; k++) s += sm[k];
        double loss = -s;
        *out = mean ? (n ? (float)(loss / (double)n) : NAN) : (float)loss;
    }
}

template <int M>
__global__ void k_ce_rows(const float *__restrict__ x, const int32_t *__restrict__ lab, float *__restrict__ prob,
                          float *__restrict__ terms, int64_t N, int64_t C, int *status, float *loss,
                          unsigned *counter) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5, nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < N; r += nw) {
        const float *p = x + r * C;
        float *q = prob + r * C;
        float m = row_max(p, C, lane);
        float s = 0.0f;
        for (int64_t c = lane; c < C; c += 32) s += m_exp<M>(p[c] - m);
        float ls = logf(warp_sum(s));
        int32_t l = checked_label(lab, r, C, status);
        for (int64_t c = lane; c < C; c += 32) {
            float lp = p[c] - m - ls;
            if (c == l) terms[r] = lp;
            q[c] = m_exp<M>(lp);
        }
    }
    // loss (optional): the mean over rows, by the last block (one launch for the whole forward)
    if (loss && last_block_done(counter)) loss_combine_block(terms, N, loss, 1);
}

extern "C" void nck_cross_entropy_fwd(nck_dev *d, const float *x, const int32_t *lab, float *prob, float *loss,
                                      int64_t N, int64_t C) {
    Scope sc(d, "cross_entropy", 0.0, 8.0 * N * C + 4.0 * N);
    float *terms = (float *)d->scratch;
    if (N > 0) {
        auto k = d->math_mode == MATH_LIBM ? k_ce_rows<MATH_LIBM> : k_ce_rows<MATH_POLY>;
        k<<<grid_for(d, N * 32), kThreads, 0, NCK_STREAM(d)>>>(x, lab, prob, terms, N, C, d->status, loss, d->counters);
        NCK_LAUNCHED(d, 1);
        return;
    }
    k_loss_combine<<<1, kThreads, 0, NCK_STREAM(d)>>>(terms, N, loss, 1);
    NCK_LAUNCHED(d, 1);
}

// ---- cross entropy on caller-owned buffers, with no allocation ------------------------------------------
//
// Some callers cannot let a library allocate device memory while they run: a runtime that owns the
// whole device pool and accounts for every byte itself, a latency-critical loop in which an
// allocator call (and the device synchronisation it may imply) would stall the stream, or a process
// at its memory limit, where a failed allocation half-way through a step would leave it half done.
// nc_ext_cross_entropy_fwd_noalloc serves them. It runs the same two kernels as the engine's cross
// entropy (per-row log-probabilities, then the fixed-order double sum of the label terms) but keeps
// the per-row terms in the fixed static array below instead of the context's scratch buffer, so it
// needs no nc_ctx and allocates nothing.
//
// - Size limit: rows <= NC_EXT_CE_NOALLOC_MAX_ROWS (1 MiB of float terms); larger calls are rejected
//   with NC_ERR_ARG before anything is launched.
// - Set-up: the first call on each device (with that device current) looks up the array's device
//   address with cudaGetSymbolAddress and caches it with the SM count and the CUDA context it was
//   taken in; a call under another context (after cudaDeviceReset, say) looks it up again. Make the
//   first call on a device, and the first after such a change, before any stream capture begins.
// - Nothing in the array has to start at zero: each call writes terms[0, rows) before reading them.
//   The caller's status word must start at zero; a label outside [0, classes) sets it to 2.
// - The array is shared by every call on a device: two calls whose kernels can overlap (different
//   streams with no ordering between them) race on it and may return wrong losses. Calls ordered on
//   one stream are safe.
static __device__ __align__(256) float g_ce_terms_static[NC_EXT_CE_NOALLOC_MAX_ROWS];

namespace {
constexpr int kMaxDevices = 64;
struct NoAllocDevice {
    float *terms;
    int sm_count;
    void *cu_ctx;  // the CUDA context the address belongs to
    bool ready;
};
NoAllocDevice g_noalloc_dev[kMaxDevices];
std::mutex g_noalloc_mu;

// The calling thread's current CUDA context (driver cuCtxGetCurrent, reached through the runtime's
// entry-point table so the library needs no link against the driver library).
void *current_cu_context() {
    typedef int (*GetCurrent)(void **);
    static GetCurrent fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (GetCurrent)f;
    });
    void *c = nullptr;
    if (!fn || fn(&c) != 0) return nullptr;
    return c;
}

// Address of the static terms array and the SM count of the current device. Looked up on the first
// call on a device and again whenever the current context differs from the one the address was
// taken in (after cudaDeviceReset the module is loaded anew, at another address).
bool noalloc_device(NoAllocDevice *out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    void *cu = current_cu_context();
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocDevice &e = g_noalloc_dev[dev];
    if (!e.ready || e.cu_ctx != cu) {
        void *p = nullptr;
        int sms = 0;
        if (cudaGetSymbolAddress(&p, g_ce_terms_static) != cudaSuccess || !p) return false;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return false;
        // the symbol lookup may have created the context: take its handle after the lookup
        e.cu_ctx = current_cu_context();
        e.terms = (float *)p;
        e.sm_count = sms;
        e.ready = true;
    }
    *out = e;
    return true;
}
}  // namespace

extern "C" NC_API int nc_ext_cross_entropy_fwd_noalloc(const float *logits, const int32_t *labels, int64_t rows,
                                                       int64_t classes, float *prob, float *loss, int *status,
                                                       void *stream) {
    if (rows < 0 || rows > NC_EXT_CE_NOALLOC_MAX_ROWS || classes <= 0) return NC_ERR_ARG;
    if (!loss || !status || (rows > 0 && (!logits || !labels || !prob))) return NC_ERR_ARG;
    NoAllocDevice dev;
    if (!noalloc_device(&dev)) {
        cudaGetLastError();  // the failed lookup's error is this call's, not the caller's
        return NC_ERR_STATE;
    }
    cudaStream_t st = (cudaStream_t)stream;
    // each launch's own status: an error the caller left pending is neither reported here nor cleared
    float *terms = dev.terms;
    if (rows > 0) {
        int64_t want = (rows * 32 + kThreads - 1) / kThreads, cap = (int64_t)dev.sm_count * 8;
        int grid = (int)(want < cap ? want : cap);
        unsigned *no_counter = nullptr;
        float *no_loss = nullptr;
        void *a[] = {(void *)&logits, (void *)&labels, (void *)&prob, (void *)&terms, (void *)&rows,
                     (void *)&classes, (void *)&status, (void *)&no_loss, (void *)&no_counter};
        if (cudaLaunchKernel((const void *)k_ce_rows<MATH_POLY>, dim3(grid), dim3(kThreads), a, 0, st) != cudaSuccess) {
            cudaGetLastError();
            return NC_ERR_STATE;
        }
    }
    const float *cterms = terms;
    int mean = 1;
    void *b[] = {(void *)&cterms, (void *)&rows, (void *)&loss, (void *)&mean};
    if (cudaLaunchKernel((const void *)k_loss_combine, dim3(1), dim3(kThreads), b, 0, st) != cudaSuccess) {
        cudaGetLastError();
        return NC_ERR_STATE;
    }
    return NC_OK;
}

__global__ void k_ce_bwd(const float *__restrict__ prob, const int32_t *__restrict__ lab,
                         const float *__restrict__ gloss, float *__restrict__ gi, int64_t N, int64_t C) {
    float s = gloss[0] / (float)(N ? N : 1);
    int64_t n = N * C;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = t / C, c = t - i * C;
        float v = gi[t] + s * prob[t];
        int32_t l = lab[i];
        if (c == l) v -= s;
        gi[t] = v;
    }
}

extern "C" void nck_cross_entropy_bwd(nck_dev *d, const float *prob, const int32_t *lab, const float *gloss, float *gi,
                                      int64_t N, int64_t C) {
    if (N * C <= 0) return;
    Scope sc(d, "cross_entropy_bwd");
    k_ce_bwd<<<grid_for(d, N * C), kThreads, 0, NCK_STREAM(d)>>>(prob, lab, gloss, gi, N, C);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_nll_terms(const float *__restrict__ x, const int32_t *__restrict__ lab, float *__restrict__ terms,
                            int64_t N, int64_t C, int *status) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x)
        terms[i] = x[i * C + checked_label(lab, i, C, status)];
}

extern "C" void nck_nll_fwd(nck_dev *d, const float *x, const int32_t *lab, float *loss, int64_t N, int64_t C,
                            int sum) {
    Scope sc(d, "nll_loss");
    float *terms = (float *)d->scratch;
    if (N > 0) k_nll_terms<<<grid_for(d, N), kThreads, 0, NCK_STREAM(d)>>>(x, lab, terms, N, C, d->status);
    k_loss_combine<<<1, kThreads, 0, NCK_STREAM(d)>>>(terms, N, loss, !sum);
    NCK_LAUNCHED(d, 2);
}

__global__ void k_nll_bwd(const int32_t *__restrict__ lab, const float *__restrict__ gloss, float *__restrict__ gi,
                          int64_t N, int64_t C, int sum) {
    float g = gloss[0];
    float s = sum ? g : g / (float)(N ? N : 1);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x)
        gi[i * C + lab[i]] -= s;
}

extern "C" void nck_nll_bwd(nck_dev *d, const int32_t *lab, const float *gloss, float *gi, int64_t N, int64_t C,
                            int sum) {
    if (N <= 0) return;
    Scope sc(d, "nll_loss_bwd");
    k_nll_bwd<<<grid_for(d, N), kThreads, 0, NCK_STREAM(d)>>>(lab, gloss, gi, N, C, sum);
    NCK_LAUNCHED(d, 1);
}

// ---- dropout on the xoshiro256** stream ------------------------------------------------------------------
//
// Block b owns draws [b * 8192, (b + 1) * 8192); its thread t owns the 64 draws starting at t * 64
// inside that. Jump tables (uploaded once): tab[k] = T^(2^(6 + k)) for k < 36, T the 256x256 GF(2)
// transition matrix of xoshiro256**, stored by column (image of each state bit).
//   block base  = prod over set bits k of b   of T^(8192 * 2^k) = tab[7 + k]
//   thread start = doubling prefix over the block: state[t] = T^(64 * 2^r) state[t - 2^r] = tab[r]
// The seven prefix matrices (56 KiB) are staged in shared memory: the block applies them 127 times.

constexpr int kDropDraws = 64;                         // draws per thread
constexpr int kDropLog = 7;                            // log2 threads per block
constexpr int kDropThreads = 1 << kDropLog;            // 128 threads per block
constexpr int kDropBlock = kDropDraws * kDropThreads;  // 8192 draws per block
constexpr int kRngTables = 36;
constexpr size_t kDropSmem = (size_t)kDropLog * 256 * sizeof(ulonglong4);

__device__ ulonglong4 *g_rng_tab;  // device copy of the jump matrices (kRngTables x 256 columns)

// once per device and process: the tables never change
extern "C" int nck_rng_tables_upload(nck_dev *d, const uint64_t *tables, size_t bytes) {
    static int done[128];
    if (bytes != (size_t)kRngTables * 256 * 32 || d->device < 0 || d->device >= 128) return 1;
    if (done[d->device]) return 0;
    void *dev = nullptr;
    if (cudaMalloc(&dev, bytes) != cudaSuccess) return 1;
    if (cudaMemcpy(dev, tables, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return 1;
    if (cudaMemcpyToSymbol(g_rng_tab, &dev, sizeof dev) != cudaSuccess) return 1;
    done[d->device] = 1;
    return 0;
}

// out = M v for a 256x256 bit matrix by columns: each lane XORs 8 columns, the warp XOR-reduces.
// Every lane returns the full product.
__device__ __forceinline__ ulonglong4 warp_matvec(const ulonglong4 *__restrict__ M, const ulonglong4 &v, int lane) {
    // lane owns columns c = 32 i + lane (i < 8): consecutive lanes read consecutive columns
    const unsigned long long words[4] = {v.x, v.y, v.z, v.w};
    ulonglong4 acc = make_ulonglong4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        ulonglong4 c = M[i * 32 + lane];
        unsigned long long m = 0ull - ((words[i >> 1] >> ((i & 1) * 32 + lane)) & 1ull);
        acc.x ^= c.x & m, acc.y ^= c.y & m, acc.z ^= c.z & m, acc.w ^= c.w & m;
    }
    for (int o = 16; o; o >>= 1) {
        acc.x ^= __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y ^= __shfl_xor_sync(0xffffffffu, acc.y, o);
        acc.z ^= __shfl_xor_sync(0xffffffffu, acc.z, o);
        acc.w ^= __shfl_xor_sync(0xffffffffu, acc.w, o);
    }
    return acc;
}

__device__ __forceinline__ unsigned long long rotl64(unsigned long long x, int k) { return (x << k) | (x >> (64 - k)); }

// one xoshiro256** state transition
__device__ __forceinline__ void xo_step(unsigned long long (&s)[4]) {
    const unsigned long long t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
}

// y = x * mask * 1/(1-p) and the mask words for the block's 8192 draws (mask bits in shared memory):
// float4 items, all of a thread's loads issued before its stores; a scalar tail when n is not a
// multiple of 4 or the pointers are not 16-byte aligned. y == NULL: the mask words only.
__device__ __forceinline__ void drop_block_write(const float *__restrict__ x, float *__restrict__ y,
                                                 uint32_t *__restrict__ bits, int64_t n, float p, const uint32_t *mb) {
    const float keepv = p < 1.0f ? 1.0f / (1.0f - p) : 0.0f;
    const int64_t base = (int64_t)blockIdx.x * kDropBlock;
    const bool vec = (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
    constexpr int kItems = kDropBlock / 4;
    if (!y) {
        // the mask only (a fused consumer applies it)
    } else if (vec && base + kDropBlock <= n) {
        for (int i0 = threadIdx.x; i0 < kItems; i0 += 4 * blockDim.x) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * blockDim.x;
                if (i < kItems) v[u] = __ldcs(reinterpret_cast<const float4 *>(x + base) + i);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * blockDim.x;
                if (i < kItems) {
                    const uint32_t m4 = (mb[i >> 3] >> ((i & 7) * 4)) & 15u;
                    v[u].x *= (m4 & 1u) ? keepv : 0.0f;
                    v[u].y *= (m4 & 2u) ? keepv : 0.0f;
                    v[u].z *= (m4 & 4u) ? keepv : 0.0f;
                    v[u].w *= (m4 & 8u) ? keepv : 0.0f;
                    __stcs(reinterpret_cast<float4 *>(y + base) + i, v[u]);
                }
            }
        }
    } else {
        for (int jj = threadIdx.x; jj < kDropBlock; jj += blockDim.x) {
            const int64_t e = base + jj;
            if (e < n) {
                const float m = (mb[jj >> 5] >> (jj & 31)) & 1u ? keepv : 0.0f;
                y[e] = x[e] * m;
            }
        }
    }
    const int64_t words = (n + 31) / 32;
    for (int w = threadIdx.x; w < kDropBlock / 32; w += blockDim.x) {
        const int64_t gw = (int64_t)blockIdx.x * (kDropBlock / 32) + w;
        if (gw < words) bits[gw] = mb[w];
    }
}

// The thread's 64 draws from state s0 (uniform u = (r >> 40) * 2^-24, exact; kept when u >= p) into
// its two mask words in shared memory, then the block's 8192 outputs and mask words, coalesced.
__device__ __forceinline__ void drop_block_out(const unsigned long long (&s0)[4], const float *__restrict__ x,
                                               float *__restrict__ y, uint32_t *__restrict__ bits, int64_t n, float p,
                                               uint32_t *mb) {
    const int tid = threadIdx.x;
    unsigned long long s[4] = {s0[0], s0[1], s0[2], s0[3]};
    uint32_t w0 = 0, w1 = 0;
#pragma unroll 8
    for (int i = 0; i < kDropDraws; i++) {
        const unsigned long long r = rotl64(s[1] * 5ull, 7) * 9ull;
        xo_step(s);
        const float u = (float)(r >> 40) * (1.0f / 16777216.0f);
        const uint32_t keep = u >= p ? 1u : 0u;
        if (i < 32) w0 |= keep << i;
        else w1 |= keep << (i - 32);
    }
    mb[2 * tid] = w0;
    mb[2 * tid + 1] = w1;
    __syncthreads();
    drop_block_write(x, y, bits, n, p, mb);
}

// Run k of the grid (draws [64 k, 64 k + 64), the same runs as the matrix-jump kernel below) is taken
// by four consecutive lanes. Its start state is q_k(T) s0 with q_k = x^(64 k) mod P (P the
// characteristic polynomial of the transition T, q_k from the host's table). Splitting q_k into its
// four 64-bit words r_j gives q_k(T) s0 = sum_j r_j(T) (T^(64 j) s0): lane j evaluates its word by
// Horner's rule from the base state T^(64 j) s0 (the host passes the four bases), 64 transitions with a
// conditional XOR, and the four partial states are XORed across the lanes. Lane j then moves 16 j
// further and makes draws [16 j, 16 j + 16) of the run; the 64 mask bits are gathered by shuffles.
// The Horner sums depend on the launch's bases only, so each block tabulates them in 4-bit windows:
// tab[j][n][v] = XOR over the set bits t of v of T^(4 n + t) b_j, and a lane's word costs 16 table
// reads instead of 64 transitions.
constexpr int kDropGroup = 4;                              // lanes per run
constexpr int kDropPolyThreads = kDropThreads * kDropGroup;  // one run per lane group: 512 threads

// The launch's Horner tables (they depend on the four base states only), built once per launch by one
// block and read by every block of the main kernel.
__global__ void __launch_bounds__(256) k_dropout_tables(ulonglong4 b0, ulonglong4 b1, ulonglong4 b2, ulonglong4 b3,
                                                        ulonglong4 *__restrict__ gtab) {
    __shared__ ulonglong4 vtab[4][64];  // T^i b_j
    if (threadIdx.x < 4) {
        const int jj = threadIdx.x;
        const ulonglong4 bj = jj == 0 ? b0 : jj == 1 ? b1 : jj == 2 ? b2 : b3;
        unsigned long long st[4] = {bj.x, bj.y, bj.z, bj.w};
        for (int i = 0; i < 64; i++) {
            vtab[jj][i] = make_ulonglong4(st[0], st[1], st[2], st[3]);
            xo_step(st);
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 4 * 16 * 16; e += blockDim.x) {
        const int jj = e >> 8, nn = (e >> 4) & 15, v = e & 15;
        ulonglong4 acc = make_ulonglong4(0, 0, 0, 0);
#pragma unroll
        for (int t = 0; t < 4; t++)
            if ((v >> t) & 1) {
                const ulonglong4 q = vtab[jj][4 * nn + t];
                acc.x ^= q.x, acc.y ^= q.y, acc.z ^= q.z, acc.w ^= q.w;
            }
        gtab[e] = acc;
    }
}

__global__ void __launch_bounds__(kDropPolyThreads) k_dropout_fwd_poly(const ulonglong4 *__restrict__ gtab,
                                                                   const ulonglong4 *__restrict__ polys,
                                                                   const float *__restrict__ x, float *__restrict__ y,
                                                                   uint32_t *__restrict__ bits, int64_t n, float p) {
    __shared__ uint32_t mb[kDropBlock / 32];
    __shared__ ulonglong4 tab[4][16][16];   // 4-bit windows of the Horner sums
    const int j = threadIdx.x & (kDropGroup - 1);
    for (int e = threadIdx.x; e < 4 * 16 * 16; e += blockDim.x) (&tab[0][0][0])[e] = gtab[e];
    __syncthreads();
    const int64_t base_run = (int64_t)blockIdx.x * kDropThreads;  // runs of this block: kDropThreads of them
    {
        const int rr = threadIdx.x / kDropGroup;  // the block's run rr, of kDropThreads
        const int64_t k = base_run + rr;
        const bool live = k * kDropDraws < n;
        unsigned long long a[4] = {0, 0, 0, 0};
        if (live) {
            const ulonglong4 q = polys[k];
            const unsigned long long w = j == 0 ? q.x : j == 1 ? q.y : j == 2 ? q.z : q.w;
#pragma unroll
            for (int nn = 0; nn < 16; nn++) {
                const ulonglong4 t = tab[j][nn][(w >> (4 * nn)) & 15];
                a[0] ^= t.x, a[1] ^= t.y, a[2] ^= t.z, a[3] ^= t.w;
            }
        }
        // XOR of the four partial states: every lane of the group gets the run's start state
#pragma unroll
        for (int o = 1; o < kDropGroup; o <<= 1)
#pragma unroll
            for (int e = 0; e < 4; e++) a[e] ^= __shfl_xor_sync(0xffffffffu, a[e], o);
        // lane j: draws [16 j, 16 j + 16) of the run
        for (int t = 0; t < 16 * j; t++) xo_step(a);
        uint32_t bits16 = 0;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const unsigned long long r = rotl64(a[1] * 5ull, 7) * 9ull;
            xo_step(a);
            const float u = (float)(r >> 40) * (1.0f / 16777216.0f);
            bits16 |= (u >= p ? 1u : 0u) << i;
        }
        const uint32_t lo = __shfl_sync(0xffffffffu, bits16, (threadIdx.x & 31 & ~3) + 0) |
                            (__shfl_sync(0xffffffffu, bits16, (threadIdx.x & 31 & ~3) + 1) << 16);
        const uint32_t hi = __shfl_sync(0xffffffffu, bits16, (threadIdx.x & 31 & ~3) + 2) |
                            (__shfl_sync(0xffffffffu, bits16, (threadIdx.x & 31 & ~3) + 3) << 16);
        if (j == 0) mb[2 * rr] = lo, mb[2 * rr + 1] = hi;
    }
    __syncthreads();
    drop_block_write(x, y, bits, n, p, mb);
}

// One thread per run: thread t of block b evaluates the whole polynomial of run k = 128 b + t (its
// four words, 64 window lookups) into the run's start state and makes the run's 64 draws itself, so no
// lane steps the generator past draws another lane makes. Same runs, mask words and outputs as the
// kernels above.
__global__ void __launch_bounds__(kDropThreads) k_dropout_fwd_run(const ulonglong4 *__restrict__ gtab,
                                                                  const ulonglong4 *__restrict__ polys,
                                                                  const float *__restrict__ x, float *__restrict__ y,
                                                                  uint32_t *__restrict__ bits, int64_t n, float p) {
    __shared__ uint32_t mb[kDropBlock / 32];
    __shared__ ulonglong4 tab[4][16][16];
    for (int e = threadIdx.x; e < 4 * 16 * 16; e += blockDim.x) (&tab[0][0][0])[e] = gtab[e];
    __syncthreads();
    const int64_t k = (int64_t)blockIdx.x * kDropThreads + threadIdx.x;
    uint32_t w0 = 0, w1 = 0;
    if (k * kDropDraws < n) {
        const ulonglong4 q = polys[k];
        const unsigned long long words[4] = {q.x, q.y, q.z, q.w};
        unsigned long long a[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int nn = 0; nn < 16; nn++) {
                const ulonglong4 t = tab[j][nn][(words[j] >> (4 * nn)) & 15];
                a[0] ^= t.x, a[1] ^= t.y, a[2] ^= t.z, a[3] ^= t.w;
            }
#pragma unroll 8
        for (int i = 0; i < kDropDraws; i++) {
            const unsigned long long r = rotl64(a[1] * 5ull, 7) * 9ull;
            xo_step(a);
            const float u = (float)(r >> 40) * (1.0f / 16777216.0f);
            const uint32_t keep = u >= p ? 1u : 0u;
            if (i < 32) w0 |= keep << i;
            else w1 |= keep << (i - 32);
        }
    }
    mb[2 * threadIdx.x] = w0;
    mb[2 * threadIdx.x + 1] = w1;
    __syncthreads();
    drop_block_write(x, y, bits, n, p, mb);
}

// Mask only, two runs per thread: thread t jumps to run 2 t by the window tables (the polynomial of
// run 2 t) and makes the 128 draws of runs 2 t and 2 t + 1 in sequence, so the jump (64 table reads)
// is paid once per 128 draws; the four mask words go straight to global memory. The same draws and
// mask words as the kernels above.
__global__ void __launch_bounds__(kDropThreads) k_dropout_mask_run2(const ulonglong4 *__restrict__ gtab,
                                                                    const ulonglong4 *__restrict__ polys,
                                                                    uint32_t *__restrict__ bits, int64_t n, float p) {
    __shared__ ulonglong4 tab[4][16][16];
    for (int e = threadIdx.x; e < 4 * 16 * 16; e += blockDim.x) (&tab[0][0][0])[e] = gtab[e];
    __syncthreads();
    const int64_t t = (int64_t)blockIdx.x * kDropThreads + threadIdx.x, k = 2 * t;
    if (k * kDropDraws >= n) return;
    const ulonglong4 q = polys[k];
    const unsigned long long words[4] = {q.x, q.y, q.z, q.w};
    unsigned long long a[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int nn = 0; nn < 16; nn++) {
            const ulonglong4 e = tab[j][nn][(words[j] >> (4 * nn)) & 15];
            a[0] ^= e.x, a[1] ^= e.y, a[2] ^= e.z, a[3] ^= e.w;
        }
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll 8
    for (int i = 0; i < 2 * kDropDraws; i++) {
        const unsigned long long r = rotl64(a[1] * 5ull, 7) * 9ull;
        xo_step(a);
        const float u = (float)(r >> 40) * (1.0f / 16777216.0f);
        w[i >> 5] |= (u >= p ? 1u : 0u) << (i & 31);
    }
    const int64_t nw = (n + 31) / 32, w0 = 4 * t;
    if (w0 + 4 <= nw) {
        *reinterpret_cast<uint4 *>(bits + w0) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        for (int j = 0; j < 4; j++)
            if (w0 + j < nw) bits[w0 + j] = w[j];
    }
}

__global__ void __launch_bounds__(kDropThreads) k_dropout_fwd(ulonglong4 s0, const float *__restrict__ x,
                                                              float *__restrict__ y, uint32_t *__restrict__ bits,
                                                              int64_t n, float p) {
    extern __shared__ ulonglong4 ptab[];  // kDropLog prefix matrices
    __shared__ ulonglong4 st[kDropThreads];
    __shared__ uint32_t mb[kDropBlock / 32];
    const ulonglong4 *tab = g_rng_tab;
    int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < kDropLog * 256; i += kDropThreads) ptab[i] = tab[i];
    if (warp == 0) {
        ulonglong4 v = s0;
        unsigned long long b = blockIdx.x;
        for (int k = 0; b; k++, b >>= 1)
            if (b & 1) v = warp_matvec(tab + (size_t)(kDropLog + k) * 256, v, lane);
        if (lane == 0) st[0] = v;
    }
    __syncthreads();
    for (int r = 0; r < kDropLog; r++) {
        int cnt = 1 << r;
        for (int t = cnt + warp; t < 2 * cnt; t += kDropThreads / 32) {
            ulonglong4 v = warp_matvec(ptab + r * 256, st[t - cnt], lane);
            if (lane == 0) st[t] = v;
        }
        __syncthreads();
    }
    const unsigned long long s[4] = {st[tid].x, st[tid].y, st[tid].z, st[tid].w};
    drop_block_out(s, x, y, bits, n, p, mb);
}

// the device copy of the run polynomials x^(64 k) mod P: grown on demand, never shrunk
struct PolyTable {
    void *dev;
    int64_t n;
};
static PolyTable g_polys[128];

extern "C" const void *nck_rng_polys(nck_dev *d, const uint64_t *host, int64_t count) {
    if (d->device < 0 || d->device >= 128) return nullptr;
    PolyTable &t = g_polys[d->device];
    if (t.n >= count) return t.dev;
    void *dev = nullptr;
    if (cudaMalloc(&dev, (size_t)count * 32) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (cudaMemcpy(dev, host, (size_t)count * 32, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(dev);
        return nullptr;
    }
    if (t.dev) {
        // kernels in flight may still read the shorter table
        cudaDeviceSynchronize();
        cudaFree(t.dev);
    }
    t.dev = dev, t.n = count;
    return dev;
}

extern "C" void nck_dropout_fwd(nck_dev *d, const uint64_t state[4], const float *x, float *y, uint32_t *bits,
                                int64_t n, float p, const void *polys, const void *host_tabs) {
    if (n <= 0) return;
    Scope sc(d, y ? "dropout" : "dropout_mask", 0.0, (y ? 8.0 * n : 0.0) + n / 8.0);
    ulonglong4 s0 = make_ulonglong4(state[0], state[1], state[2], state[3]);
    int64_t blocks = (n + kDropBlock - 1) / kDropBlock;
    if (polys && host_tabs && !y && n >= ((int64_t)1 << 21) && ((uintptr_t)bits & 15) == 0) {
        /* a large mask on its own: two runs per thread */
        const int64_t threads = (n + 2 * kDropDraws - 1) / (2 * kDropDraws);
        k_dropout_mask_run2<<<(unsigned)((threads + kDropThreads - 1) / kDropThreads), kDropThreads, 0, NCK_STREAM(d)>>>(
            reinterpret_cast<const ulonglong4 *>(host_tabs), reinterpret_cast<const ulonglong4 *>(polys), bits, n, p);
        NCK_LAUNCHED(d, 1);
        return;
    }
    if (polys && host_tabs) {
        k_dropout_fwd_run<<<(unsigned)blocks, kDropThreads, 0, NCK_STREAM(d)>>>(
            reinterpret_cast<const ulonglong4 *>(host_tabs), reinterpret_cast<const ulonglong4 *>(polys), x, y, bits,
            n, p);
        NCK_LAUNCHED(d, 1);
        return;
    }
    if (polys) {
        // base states T^(64 j) s0, j < 4: 64, 128 and 192 transitions of the host's copy
        uint64_t st[4] = {state[0], state[1], state[2], state[3]};
        ulonglong4 bj[4];
        for (int j = 0; j < 4; j++) {
            bj[j] = make_ulonglong4(st[0], st[1], st[2], st[3]);
            for (int t = 0; t < 64; t++) {
                const uint64_t tt = st[1] << 17;
                st[2] ^= st[0], st[3] ^= st[1], st[1] ^= st[2], st[0] ^= st[3], st[2] ^= tt;
                st[3] = (st[3] << 45) | (st[3] >> 19);
            }
        }
        /* the tables live past the split-reduction area of the scratch buffer */
        ulonglong4 *tabs = reinterpret_cast<ulonglong4 *>((char *)d->scratch + d->scratch_bytes - 4 * 16 * 16 * 32);
        k_dropout_tables<<<1, 256, 0, NCK_STREAM(d)>>>(bj[0], bj[1], bj[2], bj[3], tabs);
        k_dropout_fwd_poly<<<(unsigned)blocks, kDropPolyThreads, 0, NCK_STREAM(d)>>>(
            tabs, reinterpret_cast<const ulonglong4 *>(polys), x, y, bits, n, p);
        NCK_LAUNCHED(d, 2);
        return;
    }
    static int attr_done = 0;
    if (!attr_done) {
        cudaFuncSetAttribute(k_dropout_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDropSmem);
        attr_done = 1;
    }
    k_dropout_fwd<<<(unsigned)blocks, kDropThreads, kDropSmem, NCK_STREAM(d)>>>(s0, x, y, bits, n, p);
    NCK_LAUNCHED(d, 1);
}

// y = x * (keep ? 1 / (1 - p) : 0) from a drawn keep mask: float4 items with all of a thread's loads
// in flight before its stores, the same product as the drawing kernels' output pass
__global__ void __launch_bounds__(256) k_dropout_apply(const float *__restrict__ x, const uint32_t *__restrict__ bits,
                                                       float *__restrict__ y, int64_t n, float p, int vec) {
    const float keepv = p < 1.0f ? 1.0f / (1.0f - p) : 0.0f;
    const int64_t n4 = vec ? n / 4 : 0, stride = (int64_t)gridDim.x * blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 *y4 = reinterpret_cast<float4 *>(y);
    for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < n4; i0 += 4 * stride) {
        float4 v[4];
        uint32_t m[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t i = i0 + u * stride;
            if (i < n4) v[u] = __ldcs(x4 + i), m[u] = (__ldg(bits + (i >> 3)) >> ((i & 7) * 4)) & 15u;
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t i = i0 + u * stride;
            if (i >= n4) break;
            v[u].x *= (m[u] & 1u) ? keepv : 0.0f;
            v[u].y *= (m[u] & 2u) ? keepv : 0.0f;
            v[u].z *= (m[u] & 4u) ? keepv : 0.0f;
            v[u].w *= (m[u] & 8u) ? keepv : 0.0f;
            __stcs(y4 + i, v[u]);
        }
    }
    for (int64_t e = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += stride)
        y[e] = x[e] * ((__ldg(bits + (e >> 5)) >> (e & 31)) & 1u ? keepv : 0.0f);
}

extern "C" void nck_dropout_apply(nck_dev *d, const float *x, const uint32_t *bits, float *y, int64_t n, float p) {
    if (n <= 0) return;
    Scope sc(d, "dropout", 0.0, 8.0 * n + n / 8.0);
    const int vec = (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
    k_dropout_apply<<<grid_for(d, vec ? n / 16 + 1 : n), 256, 0, NCK_STREAM(d)>>>(x, bits, y, n, p, vec);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_dropout_bwd(const float *__restrict__ g, const uint32_t *__restrict__ bits, float *__restrict__ gi,
                              int64_t n, float p, int acc) {
    float keepv = p < 1.0f ? 1.0f / (1.0f - p) : 0.0f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float m = (bits[i >> 5] >> (i & 31)) & 1u ? keepv : 0.0f;
        gi[i] = (acc ? gi[i] : 0.0f) + g[i] * m;
    }
}

extern "C" void nck_dropout_bwd(nck_dev *d, const float *g, const uint32_t *bits, float *gi, int64_t n, float p,
                                int acc) {
    if (n <= 0) return;
    Scope sc(d, "dropout_bwd", 0.0, (acc ? 12.0 : 8.0) * n + n / 8.0);
    k_dropout_bwd<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(g, bits, gi, n, p, acc);
    NCK_LAUNCHED(d, 1);
}

// ---- batch norm over x [N, C, S] -----------------------------------------------------------------------
//
// Per-channel statistics: grid (C, splits); each block sums its samples' planes in double, a
// finalize kernel combines the splits in order. Variance from the double sums of x and x^2.

__device__ __forceinline__ void block_sum2(double &a, double &b, double *sm) {
    a = warp_sum_d(a);
    b = warp_sum_d(b);
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) sm[w] = a, sm[32 + w] = b;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0, t = 0;
        for (int k = 0; k < nw; k++) s += sm[k], t += sm[32 + k];
        a = s, b = t;
    }
}

// One block per (channel, run of samples). The block's elements are walked as a flat list of float4
// (planes of a multiple of 4 floats) or floats, two independent double accumulator pairs per thread
// and loads unrolled so that enough bytes are in flight to keep HBM busy.
template <int V>
__device__ __forceinline__ void bn_load(const float *p, int64_t i, float (&v)[V]) {
    if constexpr (V == 4) {
        float4 q = __ldg(reinterpret_cast<const float4 *>(p) + i);
        v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
    } else {
        v[0] = __ldg(p + i);
    }
}

// per-channel statistics -> mean, invstd and running statistics (unbiased variance), splits in order.
// stage != 0 (data-parallel runs): rm / rv receive this batch's mean and unbiased variance instead,
// for the running-statistic updates applied later in rank order (nck_bn_running_apply).
struct BnFwdFin {
    float *mean, *invstd, *rm, *rv;
    float mom, eps;
    int splits;
    int stage;
};

// Finalize work of the last block: eight lanes per channel add strided runs of the splits and a
// three-step shuffle tree (within the eight) combines them; the order is fixed.
__device__ __forceinline__ unsigned group8_mask() { return 0xFFu << (threadIdx.x & 24); }

__device__ __forceinline__ void sum_splits8(const double *part, int splits, int64_t C, int64_t c, double &s,
                                            double &t) {
    s = 0.0, t = 0.0;
    for (int k = threadIdx.x & 7; k < splits; k += 8) s += __ldcg(part + (k * C + c) * 2), t += __ldcg(part + (k * C + c) * 2 + 1);
    const unsigned m = group8_mask();
    for (int o = 4; o; o >>= 1) s += __shfl_xor_sync(m, s, o, 8), t += __shfl_xor_sync(m, t, o, 8);
}

__device__ void bn_fwd_finalize(const double *part, int64_t C, int64_t M, const BnFwdFin &f) {
    for (int64_t c = threadIdx.x >> 3; c < C; c += blockDim.x >> 3) {
        double s, ss;
        sum_splits8(part, f.splits, C, c, s, ss);
        if ((threadIdx.x & 7) == 0) {
            double mu = s / (double)M;
            double dev = ss - s * mu; /* sum of squared deviations */
            if (dev < 0.0) dev = 0.0;
            f.mean[c] = (float)mu;
            f.invstd[c] = (float)(1.0 / sqrt(dev / (double)M + (double)f.eps));
            if (f.stage) {
                f.rm[c] = (float)mu;
                f.rv[c] = (float)(dev / (double)(M - 1));
            } else {
                f.rm[c] = (1.0f - f.mom) * f.rm[c] + f.mom * (float)mu;
                f.rv[c] = (1.0f - f.mom) * f.rv[c] + f.mom * (float)(dev / (double)(M - 1));
            }
        }
    }
}

template <int V>
__global__ void __launch_bounds__(256) k_bn_stats(const float *__restrict__ x, double *__restrict__ part, int64_t N,
                                                  int64_t C, int64_t S, int64_t per_split, BnFwdFin fin,
                                                  unsigned *counter) {
    __shared__ double sm[64];
    const int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    // four items in flight per thread, then their double sums (two chains)
    const int64_t pstride = C * S;
    const float *xc = x + (n0 * C + c) * S;
    ChanWalk w;
    w.init((int)(S / V), n1 > n0 ? n1 - n0 : 0);
    double s0 = 0.0, q0 = 0.0, s1 = 0.0, q1 = 0.0;
    while (w.live()) {
        float v[4][V];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (w.live()) bn_load<V>(xc + w.na * pstride, w.ia, v[j]);
            else
#pragma unroll
                for (int k = 0; k < V; k++) v[j][k] = 0.0f;
            w.next();
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int k = 0; k < V; k++) {
                const double a = (double)v[j][k];
                if (j & 1) s1 += a, q1 += a * a;
                else s0 += a, q0 += a * a;
            }
    }
    double s = s0 + s1, ss = q0 + q1;
    block_sum2(s, ss, sm);
    if (threadIdx.x == 0) {
        part[(blockIdx.y * C + c) * 2] = s;
        part[(blockIdx.y * C + c) * 2 + 1] = ss;
    }
    if (last_block_done(counter)) bn_fwd_finalize(part, C, N * S, fin);
}

__global__ void k_bn_eval_stats(const float *__restrict__ rm, const float *__restrict__ rv, float *mean, float *invstd,
                                int64_t C, float eps) {
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < C; c += (int64_t)gridDim.x * blockDim.x) {
        mean[c] = rm[c];
        invstd[c] = 1.0f / sqrtf(rv[c] + eps);
    }
}

// y = act(x * a + d) per channel, a = w * invstd, d = b - mean * a (act < 0: none); flat over all
// elements (V = 4: float4 items, planes of a multiple of 4 floats)
template <int V>
__global__ void __launch_bounds__(256) k_bn_norm(const float *__restrict__ x, const float *__restrict__ w,
                                                 const float *__restrict__ b, const float *__restrict__ mean,
                                                 const float *__restrict__ invstd, float *__restrict__ y, int64_t NC,
                                                 int64_t C, int64_t S, FastDiv dsv, FastDiv dc, int act = -1,
                                                 float act_s = 0.0f) {
    const int64_t SV = S / V, total = NC * SV;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c;
        if (total <= 0x7fffffff) {
            const uint32_t q = dsv.div((uint32_t)i);
            c = (int64_t)(q - dc.div(q) * (uint32_t)C);
        } else {
            c = (i / SV) % C;
        }
        float a = __ldg(w + c) * __ldg(invstd + c), dd = __ldg(b + c) - __ldg(mean + c) * a;
        if constexpr (V == 4) {
            float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
            v.x = epi_fwd(act, act_s, v.x * a + dd), v.y = epi_fwd(act, act_s, v.y * a + dd);
            v.z = epi_fwd(act, act_s, v.z * a + dd), v.w = epi_fwd(act, act_s, v.w * a + dd);
            reinterpret_cast<float4 *>(y)[i] = v;
        } else {
            y[i] = epi_fwd(act, act_s, __ldg(x + i) * a + dd);
        }
    }
}

// divisors of the flat element walk: by S / V (float4 items per plane) and by C
#define BN_DIVS(S, V) make_fastdiv((uint32_t)((S) / (V)))

static bool bn_vec4(int64_t S, const void *p, const void *q, const void *r) {
    return (S & 3) == 0 && (((uintptr_t)p | (uintptr_t)q | (uintptr_t)r) & 15) == 0;
}

static int flat_grid(const nck_dev *d, int64_t items) {
    int64_t want = (items + 255) / 256, cap = (int64_t)(d->sm_count > 0 ? d->sm_count : 148) * 16;
    if (want > cap) want = cap;
    return want < 1 ? 1 : (int)want;
}

// runs of samples per channel: as many blocks as fit on the GPU at once (`resident`, one full wave),
// and at most 2^30 elements per block (the statistics kernels index a block's elements with 32-bit
// integers)
static int64_t bn_splits(int64_t resident, int64_t N, int64_t C, int64_t S) {
    int64_t want = resident / C;
    int64_t need = (N * S + ((int64_t)1 << 30) - 1) >> 30;
    if (want < need) want = need;
    if (want < 1) want = 1;
    return want > N ? N : want;
}


// backward sums -> weight / bias gradients and the two means the input gradient needs
struct BnBwdFin {
    float *gw, *gb, *coef;
    int splits;
};

__device__ void bn_bwd_finalize(const double *part, int64_t C, int64_t M, const BnBwdFin &f) {
    for (int64_t c = threadIdx.x >> 3; c < C; c += blockDim.x >> 3) {
        double sg, sgx;
        sum_splits8(part, f.splits, C, c, sg, sgx);
        if ((threadIdx.x & 7) == 0) {
            if (f.gw) f.gw[c] += (float)sgx;
            if (f.gb) f.gb[c] += (float)sg;
            f.coef[2 * c] = (float)(sg / (double)M);
            f.coef[2 * c + 1] = (float)(sgx / (double)M);
        }
    }
}

// ---- channel reductions fed by bulk copies --------------------------------------------------------------
//
// The statistics and backward-sum passes read whole planes of one channel (S contiguous floats per
// sample and channel). In these kernels one thread streams the block's planes into a ring of
// shared-memory stages with cp.async.bulk (no multicast; one mbarrier per stage counts the bytes),
// kBnRing stages ahead of the block's threads, which reduce each stage from shared memory. A block
// keeps up to kBnRing * 16 KiB of loads in flight without holding registers for them (the register-fed
// kernels above keep 64 bytes per thread in flight, short of what HBM needs under their occupancy).
// Used when a plane is a multiple of 16 bytes and fits a stage. The waits are bounded like the
// tensor-core pipelines': a block that gives up reports NCK_ERR_PIPELINE, lets its copies land (again
// bounded) and stops.
constexpr int kBnRing = 4, kBnStageMax = 16384;

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

// planes [n0, n1) of channel c of NT tensors [N][C][S], PP planes of each per stage, each plane in a
// slot of SP floats. al: every plane starts on a 16-byte boundary and S is a multiple of 4 (SP = S,
// the stage is one contiguous run of floats). Otherwise each plane's copy starts at the 16-byte
// boundary at or below it and ends at the one at or above its end (SP = S + 3 rounded up to 4; the
// plane then sits lead(t, s, j) floats into its slot): device blocks are 256-byte aligned and sized
// in whole 256-byte units, so these few bytes around a plane lie inside its tensor's allocation.
template <int NT>
struct PlaneRing {
    const float *src[NT];
    int64_t C, S, n0, n1, c;
    int PP, SP, al;
    float *buf;  // kBnRing stages of NT * PP * SP floats
    uint64_t *full;
    __device__ int64_t stages() const { return n1 > n0 ? (n1 - n0 + PP - 1) / PP : 0; }
    __device__ const float *stage(int slot, int t) const { return buf + ((int64_t)slot * NT + t) * PP * SP; }
    __device__ int planes(int64_t s) const {
        const int64_t left = n1 - (n0 + s * PP);
        return (int)(left < PP ? left : PP);
    }
    __device__ const float *plane_src(int t, int64_t s, int j) const { return src[t] + ((n0 + s * PP + j) * C + c) * S; }
    // floats between the slot's start and the plane's first element
    __device__ int lead(int t, int64_t s, int j) const { return al ? 0 : (int)(((uintptr_t)plane_src(t, s, j) >> 2) & 3); }
    // one thread: stage s of the walk into its ring slot
    __device__ void issue(int64_t s) const {
        const int slot = (int)(s % kBnRing), np = planes(s);
        uint32_t total = 0;
        for (int t = 0; t < NT; t++)
            for (int j = 0; j < np; j++) {
                const uintptr_t p = (uintptr_t)plane_src(t, s, j), a = p & ~(uintptr_t)15;
                total += al ? (uint32_t)(S * 4) : (uint32_t)(((p + S * 4 + 15) & ~(uintptr_t)15) - a);
            }
        tc::mbar_expect_tx(&full[slot], total);
        for (int t = 0; t < NT; t++)
            for (int j = 0; j < np; j++) {
                const uintptr_t p = (uintptr_t)plane_src(t, s, j), a = p & ~(uintptr_t)15;
                const uint32_t bytes = al ? (uint32_t)(S * 4) : (uint32_t)(((p + S * 4 + 15) & ~(uintptr_t)15) - a);
                bulk_g2s(buf + ((int64_t)slot * NT + t) * PP * SP + (int64_t)j * SP, (const void *)a, bytes, &full[slot]);
            }
    }
    // every thread: the ring's barriers, then the first stages in flight
    __device__ void start() const {
        if (threadIdx.x == 0) {
            for (int i = 0; i < kBnRing; i++) tc::mbar_init(&full[i], 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int64_t s = 0; s < kBnRing && s < stages(); s++) issue(s);
    }
    // after a failed wait at stage s: the copies issued past it land (bounded) before the block exits
    __device__ void drain(int64_t s, int *status) const {
        if (threadIdx.x != 0) return;
        const int64_t end = s + kBnRing < stages() ? s + kBnRing : stages();
        for (int64_t j = s; j < end; j++)
            if (!tc::mbar_wait(&full[j % kBnRing], (uint32_t)((j / kBnRing) & 1), status)) break;
    }
};

// per-channel statistics from bulk-copied planes (the same partials and finalize as k_bn_stats)
__global__ void __launch_bounds__(256) k_bn_stats_bulk(const float *__restrict__ x, double *__restrict__ part,
                                                       int64_t N, int64_t C, int64_t S, int64_t per_split, int PP,
                                                       int SP, int al, FastDiv dS, BnFwdFin fin, unsigned *counter,
                                                       int *status) {
    extern __shared__ __align__(128) float bn_ring[];
    __shared__ __align__(8) uint64_t full[kBnRing];
    __shared__ double sm[64];
    const int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    PlaneRing<1> r{{x}, C, S, n0, n1, c, PP, SP, al, bn_ring, full};
    r.start();
    double s0 = 0.0, q0 = 0.0, s1 = 0.0, q1 = 0.0;
    const int64_t ns = r.stages();
    for (int64_t st = 0; st < ns; st++) {
        const int slot = (int)(st % kBnRing);
        const bool got = tc::mbar_wait(&full[slot], (uint32_t)((st / kBnRing) & 1), status);
        if (got && al) {
            const float4 *p = reinterpret_cast<const float4 *>(r.stage(slot, 0));
            const int n4 = r.planes(st) * (int)(S / 4);
            for (int i = threadIdx.x; i < n4; i += 2 * blockDim.x) {
                const float4 a = p[i];
                s0 += (double)a.x, q0 += (double)a.x * a.x, s0 += (double)a.y, q0 += (double)a.y * a.y;
                s0 += (double)a.z, q0 += (double)a.z * a.z, s0 += (double)a.w, q0 += (double)a.w * a.w;
                if (i + (int)blockDim.x < n4) {
                    const float4 b = p[i + blockDim.x];
                    s1 += (double)b.x, q1 += (double)b.x * b.x, s1 += (double)b.y, q1 += (double)b.y * b.y;
                    s1 += (double)b.z, q1 += (double)b.z * b.z, s1 += (double)b.w, q1 += (double)b.w * b.w;
                }
            }
        } else if (got) {
            const float *p = r.stage(slot, 0);
            const int n = r.planes(st) * (int)S;
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int j = (int)dS.div((uint32_t)i);
                const double a = (double)p[j * SP + r.lead(0, st, j) + (i - j * (int)S)];
                if (i & 256) s1 += a, q1 += a * a;
                else s0 += a, q0 += a * a;
            }
        }
        if (!__syncthreads_and(got)) {
            r.drain(st, status);
            return;
        }
        if (threadIdx.x == 0 && st + kBnRing < ns) r.issue(st + kBnRing);
    }
    double s = s0 + s1, ss = q0 + q1;
    block_sum2(s, ss, sm);
    if (threadIdx.x == 0) {
        part[(blockIdx.y * C + c) * 2] = s;
        part[(blockIdx.y * C + c) * 2 + 1] = ss;
    }
    if (last_block_done(counter)) bn_fwd_finalize(part, C, N * S, fin);
}

// backward sums from bulk-copied planes of x (or, after a pool, x at the argmax) and of the gradient:
// the same per-element terms, partials and finalize as k_bn_bwd_sums / k_bn_pool_bwd_sums_x; M is the
// element count of the statistics
__global__ void __launch_bounds__(256) k_bn_sums_bulk(const float *__restrict__ x, const float *__restrict__ g,
                                                      const float *__restrict__ mean, const float *__restrict__ invstd,
                                                      double *__restrict__ part, int64_t N, int64_t C, int64_t S,
                                                      int64_t per_split, int PP, int SP, int al, FastDiv dS,
                                                      int64_t M, BnBwdFin fin, unsigned *counter, int *status,
                                                      const float *__restrict__ wt, const float *__restrict__ bs,
                                                      int act, float act_s) {
    extern __shared__ __align__(128) float bn_ring[];
    __shared__ __align__(8) uint64_t full[kBnRing];
    __shared__ double sm[64];
    const int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    const float mu = mean[c], is = invstd[c];
    const float ea = act >= 0 ? wt[c] * is : 0.0f, ed = act >= 0 ? bs[c] - mu * ea : 0.0f;
    PlaneRing<2> r{{x, g}, C, S, n0, n1, c, PP, SP, al, bn_ring, full};
    r.start();
    double g0 = 0.0, h0 = 0.0, g1 = 0.0, h1 = 0.0;
    const int64_t ns = r.stages();
    for (int64_t st = 0; st < ns; st++) {
        const int slot = (int)(st % kBnRing);
        const bool got = tc::mbar_wait(&full[slot], (uint32_t)((st / kBnRing) & 1), status);
        if (got && !al) {
            const float *px = r.stage(slot, 0), *pg = r.stage(slot, 1);
            const int n = r.planes(st) * (int)S;
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int j = (int)dS.div((uint32_t)i), e = i - j * (int)S;
                const float xv = px[j * SP + r.lead(0, st, j) + e];
                float gv = pg[j * SP + r.lead(1, st, j) + e];
                if (act >= 0) gv = epi_grad(act, act_s, xv * ea + ed, gv);
                if (i & 256) g1 += gv, h1 += gv * (xv - mu) * is;
                else g0 += gv, h0 += gv * (xv - mu) * is;
            }
        } else if (got) {
            const float *px = r.stage(slot, 0), *pg = r.stage(slot, 1);
            const int n = r.planes(st) * (int)S;
            for (int i = 4 * threadIdx.x; i < n; i += 4 * blockDim.x) {
                const float4 xv = *reinterpret_cast<const float4 *>(px + i);
                float4 gv = *reinterpret_cast<const float4 *>(pg + i);
                if (act >= 0) {
                    gv.x = epi_grad(act, act_s, xv.x * ea + ed, gv.x), gv.y = epi_grad(act, act_s, xv.y * ea + ed, gv.y);
                    gv.z = epi_grad(act, act_s, xv.z * ea + ed, gv.z), gv.w = epi_grad(act, act_s, xv.w * ea + ed, gv.w);
                }
                g0 += gv.x, h0 += gv.x * (xv.x - mu) * is, g1 += gv.y, h1 += gv.y * (xv.y - mu) * is;
                g0 += gv.z, h0 += gv.z * (xv.z - mu) * is, g1 += gv.w, h1 += gv.w * (xv.w - mu) * is;
            }
        }
        if (!__syncthreads_and(got)) {
            r.drain(st, status);
            return;
        }
        if (threadIdx.x == 0 && st + kBnRing < ns) r.issue(st + kBnRing);
    }
    double sg = g0 + g1, sgx = h0 + h1;
    block_sum2(sg, sgx, sm);
    if (threadIdx.x == 0) {
        part[(blockIdx.y * C + c) * 2] = sg;
        part[(blockIdx.y * C + c) * 2 + 1] = sgx;
    }
    if (last_block_done(counter)) bn_bwd_finalize(part, C, M, fin);
}

// the ring layout of the bulk-fed kernels for NT tensors with S floats per plane: planes per stage
// (0: not eligible: planes shorter than 4 floats or longer than a stage), slot floats, aligned case
struct BnBulk {
    int PP, SP, al;
    FastDiv dS;
};

static BnBulk bn_bulk_plan(const nck_dev *d, int64_t S, int NT, const void *p, const void *q) {
    BnBulk b = {0, 0, 0, make_fastdiv(1)};
    // default policy (stage < 0): the statistics pass (NT = 1) over planes of at least 4 KiB, where the
    // bulk feed measured faster (cfg3's 32 x 32 planes); the backward sums stay register-fed
    const int auto_ = d->bn_bulk_stage < 0;
    if (d->bn_bulk_stage == 0 || S < 4 || S >= ((int64_t)1 << 20) || (auto_ && (NT != 1 || S < 1024))) return b;
    b.al = (S & 3) == 0 && (((uintptr_t)p | (uintptr_t)q) & 15) == 0;
    b.SP = (int)(b.al ? S : (S + 3 + 3) / 4 * 4);
    const int stage = d->bn_bulk_stage < 0 ? -d->bn_bulk_stage : d->bn_bulk_stage;
    int64_t pp = (stage < kBnStageMax ? stage : kBnStageMax) / NT / ((int64_t)b.SP * 4);
    if (pp > 64) pp = 64;
    b.PP = (int)pp;
    b.dS = make_fastdiv((uint32_t)S);
    return b;
}

static size_t bn_bulk_smem(const BnBulk &b, int NT) { return (size_t)kBnRing * NT * b.PP * b.SP * sizeof(float); }

// one wave of (channel, run of samples) blocks for a bulk-fed kernel
template <typename K>
static void bn_bulk_grid(nck_dev *d, K kernel, size_t smem, int64_t N, int64_t C, int64_t S, int64_t &splits,
                         int64_t &per) {
    static int attr = 0;
    static size_t seen_smem[4];
    static int seen_res[4], nseen = 0;
    if (!attr) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBnRing * kBnStageMax);
        attr = 1;
    }
    int res = 0;  // resident blocks, cached per ring size (the occupancy query is a host call)
    for (int i = 0; i < nseen && !res; i++)
        if (seen_smem[i] == smem) res = seen_res[i];
    if (!res) {
        res = resident_blocks(d, kernel, 256, smem);
        const int slot = nseen < 4 ? nseen++ : 3;
        seen_smem[slot] = smem, seen_res[slot] = res;
    }
    splits = bn_splits(res, N, C, S);
    per = (N + splits - 1) / splits;
    splits = (N + per - 1) / per;
}

extern "C" void nck_bn_stats_train(nck_dev *d, const float *x, float *mean, float *invstd, float *rm, float *rv,
                                   int64_t N, int64_t C, int64_t S, float mom, float eps, int stage) {
    Scope sc(d, "bn_fwd", 0.0, 4.0 * N * C * S);
    const BnBulk bb = bn_bulk_plan(d, S, 1, x, x);
    if (bb.PP) {
        const size_t smem = bn_bulk_smem(bb, 1);
        int64_t splits, per;
        bn_bulk_grid(d, k_bn_stats_bulk, smem, N, C, S, splits, per);
        const BnFwdFin fin = {mean, invstd, rm, rv, mom, eps, (int)splits, stage};
        k_bn_stats_bulk<<<dim3((unsigned)C, (unsigned)splits), 256, smem, NCK_STREAM(d)>>>(
            x, (double *)d->scratch, N, C, S, per, bb.PP, bb.SP, bb.al, bb.dS, fin, d->counters, d->status);
        NCK_LAUNCHED(d, 1);
        return;
    }
    const bool v4 = bn_vec4(S, x, x, x);
    static int res4 = 0, res1 = 0;
    if (v4 && !res4) res4 = resident_blocks(d, k_bn_stats<4>, kThreads);
    if (!v4 && !res1) res1 = resident_blocks(d, k_bn_stats<1>, kThreads);
    int64_t splits = bn_splits(v4 ? res4 : res1, N, C, S), per = (N + splits - 1) / splits;
    splits = (N + per - 1) / per;
    double *part = (double *)d->scratch;
    dim3 g1((unsigned)C, (unsigned)splits);
    const BnFwdFin fin = {mean, invstd, rm, rv, mom, eps, (int)splits, stage};
    if (v4) k_bn_stats<4><<<g1, kThreads, 0, NCK_STREAM(d)>>>(x, part, N, C, S, per, fin, d->counters);
    else k_bn_stats<1><<<g1, kThreads, 0, NCK_STREAM(d)>>>(x, part, N, C, S, per, fin, d->counters);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_bn_apply(nck_dev *d, const float *x, const float *w, const float *b, const float *mean,
                             const float *invstd, float *y, int64_t N, int64_t C, int64_t S, int act, float act_s) {
    const int64_t planes = N * C;
    if (planes * S <= 0) return;
    Scope sc(d, act < 0 ? "bn_fwd" : "bn_act_fwd", 0.0, 8.0 * planes * S);
    if (bn_vec4(S, x, y, x))
        k_bn_norm<4><<<flat_grid(d, planes * S / 4), 256, 0, NCK_STREAM(d)>>>(x, w, b, mean, invstd, y, planes, C, S,
                                                                         BN_DIVS(S, 4), make_fastdiv((uint32_t)C), act,
                                                                         act_s);
    else
        k_bn_norm<1><<<flat_grid(d, planes * S), 256, 0, NCK_STREAM(d)>>>(x, w, b, mean, invstd, y, planes, C, S,
                                                                         BN_DIVS(S, 1), make_fastdiv((uint32_t)C), act,
                                                                         act_s);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_bn_fwd_train(nck_dev *d, const float *x, const float *w, const float *b, float *y, float *mean,
                                 float *invstd, float *rm, float *rv, int64_t N, int64_t C, int64_t S, float mom,
                                 float eps, int stage) {
    nck_bn_stats_train(d, x, mean, invstd, rm, rv, N, C, S, mom, eps, stage);
    nck_bn_apply(d, x, w, b, mean, invstd, y, N, C, S, -1, 0.0f);
}

// ---- BatchNorm + activation + 2 x 2 / stride 2 max pooling, fused ---------------------------------------
//
// The pooled output and its first-max argmax (index in the input plane, as the pooling kernels
// store it) straight from the BatchNorm input: each element of a window is normalised and activated
// in registers (the same arithmetic as k_bn_norm), so the full-size normalised and activated tensors
// are never written. Even H and W (every window whole).
__global__ void __launch_bounds__(256) k_bn_act_pool2x2(const float *__restrict__ x, const float *__restrict__ w,
                                                        const float *__restrict__ b, const float *__restrict__ mean,
                                                        const float *__restrict__ invstd, int act, float act_s,
                                                        float *__restrict__ y, int32_t *__restrict__ arg,
                                                        float *__restrict__ xarg, uint32_t planes, uint32_t C,
                                                        uint32_t W, uint32_t OH, uint32_t OW, FastDiv dow,
                                                        FastDiv doh, FastDiv dc) {
    const uint32_t total = planes * OH * OW;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = dow.div(t), ox = t - r * OW, pl = doh.div(r), oy = r - pl * OH;
        const uint32_t c = pl - dc.div(pl) * C;
        const float a = __ldg(w + c) * __ldg(invstd + c), dd = __ldg(b + c) - __ldg(mean + c) * a;
        const uint32_t H = 2 * OH;
        const float *r0 = x + (size_t)pl * H * W + (size_t)(2 * oy) * W + 2 * ox;
        const float2 p = __ldg(reinterpret_cast<const float2 *>(r0));
        const float2 q = __ldg(reinterpret_cast<const float2 *>(r0 + W));
        const float v0 = epi_fwd(act, act_s, p.x * a + dd), v1 = epi_fwd(act, act_s, p.y * a + dd);
        const float v2 = epi_fwd(act, act_s, q.x * a + dd), v3 = epi_fwd(act, act_s, q.y * a + dd);
        const int32_t i0 = (int32_t)(2 * oy * W + 2 * ox);
        float best = v0, bx = p.x;
        int32_t bi = i0;
        if (v1 > best) best = v1, bi = i0 + 1, bx = p.y;
        if (v2 > best) best = v2, bi = i0 + (int32_t)W, bx = q.x;
        if (v3 > best) best = v3, bi = i0 + (int32_t)W + 1, bx = q.y;
        y[t] = best;
        arg[t] = bi;
        if (xarg) xarg[t] = bx;
    }
}

extern "C" int nck_bn_pool2x2_ok(int64_t N, int64_t C, int64_t H, int64_t W) {
    return H % 2 == 0 && W % 2 == 0 && N * C * H * W < ((int64_t)1 << 31) && H > 0 && W > 0;
}

extern "C" void nck_bn_act_pool2x2(nck_dev *d, const float *x, const float *w, const float *b, const float *mean,
                                   const float *invstd, int act, float act_s, float *y, int32_t *arg, float *xarg,
                                   int64_t N, int64_t C, int64_t H, int64_t W) {
    const int64_t planes = N * C, OH = H / 2, OW = W / 2, total = planes * OH * OW;
    if (total <= 0) return;
    Scope sc(d, "bn_act_pool", 0.0, 4.0 * planes * H * W + (xarg ? 12.0 : 8.0) * total);
    k_bn_act_pool2x2<<<grid_for(d, total), 256, 0, NCK_STREAM(d)>>>(
        x, w, b, mean, invstd, act, act_s, y, arg, xarg, (uint32_t)planes, (uint32_t)C, (uint32_t)W, (uint32_t)OH,
        (uint32_t)OW, make_fastdiv((uint32_t)OW), make_fastdiv((uint32_t)OH), make_fastdiv((uint32_t)C));
    NCK_LAUNCHED(d, 1);
}

// Running statistics of data-parallel BatchNorm: group g (one running_mean / running_var pair) takes
// the momentum updates of its staged forwards, rank by rank and, within a rank, in recording order,
// which is the order newch applies them when it runs the ranks' batches one after another
// (engine/src/ops/ops_nn.c:291-292, the same two-product update as bn_fwd_finalize).
__global__ void k_bn_running(const nck_bn_group *__restrict__ groups, const nck_bn_staged *__restrict__ staged,
                             const float *__restrict__ gathered, int64_t rank_stride, int ranks) {
    const nck_bn_group gr = groups[blockIdx.x];
    for (int64_t c = threadIdx.x; c < gr.C; c += blockDim.x) {
        float m = gr.rm[c], v = gr.rv[c];
        for (int r = 0; r < ranks; r++)
            for (int e = gr.e0; e < gr.e1; e++) {
                const float *g = gathered + r * rank_stride + staged[e].off;
                const float mom = staged[e].mom;
                m = (1.0f - mom) * m + mom * g[c];
                v = (1.0f - mom) * v + mom * g[gr.C + c];
            }
        gr.rm[c] = m;
        gr.rv[c] = v;
    }
}

extern "C" void nck_bn_running_apply(nck_dev *d, const nck_bn_group *groups, int ngroups, const nck_bn_staged *staged,
                                     const float *gathered, int64_t rank_stride, int ranks) {
    if (ngroups <= 0) return;
    Scope sc(d, "bn_running");
    k_bn_running<<<ngroups, 256, 0, NCK_STREAM(d)>>>(groups, staged, gathered, rank_stride, ranks);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_bn_fwd_eval(nck_dev *d, const float *x, const float *w, const float *b, float *y, float *mean,
                                float *invstd, const float *rm, const float *rv, int64_t N, int64_t C, int64_t S,
                                float eps) {
    Scope sc(d, "bn_fwd");
    k_bn_eval_stats<<<grid_for(d, C), kThreads, 0, NCK_STREAM(d)>>>(rm, rv, mean, invstd, C, eps);
    int64_t planes = N * C;
    if (planes * S > 0) {
        if (bn_vec4(S, x, y, x))
            k_bn_norm<4><<<flat_grid(d, planes * S / 4), 256, 0, NCK_STREAM(d)>>>(x, w, b, mean, invstd, y, planes, C, S,
                                                                             BN_DIVS(S, 4), make_fastdiv((uint32_t)C));
        else
            k_bn_norm<1><<<flat_grid(d, planes * S), 256, 0, NCK_STREAM(d)>>>(x, w, b, mean, invstd, y, planes, C, S,
                                                                             BN_DIVS(S, 1), make_fastdiv((uint32_t)C));
    }
    NCK_LAUNCHED(d, 2);
}

// backward sums per channel: sg = sum g, sgx = sum g * xhat (float products, double sums); same
// walk as the statistics kernel
// act >= 0: g is the gradient of act(BatchNorm output); the BatchNorm output's own gradient is formed
// on the fly from x (the activation's backward fused in)
template <int V>
__global__ void __launch_bounds__(256) k_bn_bwd_sums(const float *__restrict__ x, const float *__restrict__ g,
                                                     const float *__restrict__ mean, const float *__restrict__ invstd,
                                                     double *__restrict__ part, int64_t N, int64_t C, int64_t S,
                                                     int64_t per_split, BnBwdFin fin, unsigned *counter,
                                                     const float *__restrict__ wt = nullptr,
                                                     const float *__restrict__ bs = nullptr, int act = -1,
                                                     float act_s = 0.0f) {
    __shared__ double sm[64];
    const int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    const float mu = mean[c], is = invstd[c];
    const float ea = act >= 0 ? wt[c] * is : 0.0f, ed = act >= 0 ? bs[c] - mu * ea : 0.0f;
    // four items of x and g in flight per thread, then float products into double sums (two chains)
    const int64_t pstride = C * S, cbase = (n0 * C + c) * S;
    ChanWalk w;
    w.init((int)(S / V), n1 > n0 ? n1 - n0 : 0);
    double g0 = 0.0, h0 = 0.0, g1 = 0.0, h1 = 0.0;
    while (w.live()) {
        float xv[4][V], gv[4][V];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (w.live()) {
                const int64_t o = cbase + w.na * pstride;
                bn_load<V>(x + o, w.ia, xv[j]);
                bn_load<V>(g + o, w.ia, gv[j]);
            } else {
#pragma unroll
                for (int k = 0; k < V; k++) xv[j][k] = mu, gv[j][k] = 0.0f;
            }
            w.next();
        }
        if (act >= 0)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int k = 0; k < V; k++) gv[j][k] = epi_grad(act, act_s, xv[j][k] * ea + ed, gv[j][k]);
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int k = 0; k < V; k++) {
                if (j & 1) g1 += gv[j][k], h1 += gv[j][k] * (xv[j][k] - mu) * is;
                else g0 += gv[j][k], h0 += gv[j][k] * (xv[j][k] - mu) * is;
            }
    }
    double sg = g0 + g1, sgx = h0 + h1;
    block_sum2(sg, sgx, sm);
    if (threadIdx.x == 0) {
        part[(blockIdx.y * C + c) * 2] = sg;
        part[(blockIdx.y * C + c) * 2 + 1] = sgx;
    }
    if (last_block_done(counter)) bn_bwd_finalize(part, C, N * S, fin);
}

// gx += k * (g - mean(g) - xhat * mean(g * xhat)) in training, gx += k * g in eval; flat walk
template <int V>
__global__ void __launch_bounds__(256) k_bn_bwd_dx(const float *__restrict__ x, const float *__restrict__ w,
                                                   const float *__restrict__ g, const float *__restrict__ mean,
                                                   const float *__restrict__ invstd, const float *__restrict__ coef,
                                                   float *__restrict__ gx, int64_t NC, int64_t C, int64_t S,
                                                   int training, int acc, FastDiv dsv, FastDiv dc,
                                                   const float *__restrict__ b = nullptr, int act = -1,
                                                   float act_s = 0.0f) {
    const int64_t SV = S / V, total = NC * SV;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c;
        if (total <= 0x7fffffff) {
            const uint32_t q = dsv.div((uint32_t)i);
            c = (int64_t)(q - dc.div(q) * (uint32_t)C);
        } else {
            c = (i / SV) % C;
        }
        float mu = __ldg(mean + c), is = __ldg(invstd + c), k = __ldg(w + c) * is;
        float mg = __ldg(coef + 2 * c), mgx = __ldg(coef + 2 * c + 1);
        float xv[V], gv[V], ov[V];
        bn_load<V>(x, i, xv);
        bn_load<V>(g, i, gv);
        if (act >= 0) {
            const float ea = __ldg(w + c) * is, ed = __ldg(b + c) - mu * ea;
#pragma unroll
            for (int e = 0; e < V; e++) gv[e] = epi_grad(act, act_s, xv[e] * ea + ed, gv[e]);
        }
        if (!acc) {
#pragma unroll
            for (int e = 0; e < V; e++) ov[e] = 0.0f;
        } else if constexpr (V == 4) {
            float4 o = reinterpret_cast<float4 *>(gx)[i];
            ov[0] = o.x, ov[1] = o.y, ov[2] = o.z, ov[3] = o.w;
        } else {
            ov[0] = gx[i];
        }
#pragma unroll
        for (int e = 0; e < V; e++)
            ov[e] += training ? k * (gv[e] - mg - (xv[e] - mu) * is * mgx) : k * gv[e];
        if constexpr (V == 4) reinterpret_cast<float4 *>(gx)[i] = make_float4(ov[0], ov[1], ov[2], ov[3]);
        else gx[i] = ov[0];
    }
}

extern "C" void nck_bn_bwd_ex(nck_dev *d, const float *x, const float *w, const float *b, const float *g,
                              const float *mean, const float *invstd, float *gx, float *gw, float *gb, int64_t N,
                              int64_t C, int64_t S, int training, int acc_gx, int act, float act_s) {
    Scope sc(d, act < 0 ? "bn_bwd" : "bn_act_bwd", 0.0, (gx ? (acc_gx ? 16.0 : 12.0) : 8.0) * N * C * S);
    const bool v4 = bn_vec4(S, x, g, gx ? (const void *)gx : (const void *)x);
    const BnBulk bb = bn_bulk_plan(d, S, 2, x, g);
    static int res4 = 0, res1 = 0;
    int64_t splits, per;
    if (bb.PP) {
        bn_bulk_grid(d, k_bn_sums_bulk, bn_bulk_smem(bb, 2), N, C, S, splits, per);
    } else {
        if (v4 && !res4) res4 = resident_blocks(d, k_bn_bwd_sums<4>, kThreads);
        if (!v4 && !res1) res1 = resident_blocks(d, k_bn_bwd_sums<1>, kThreads);
        splits = bn_splits(v4 ? res4 : res1, N, C, S), per = (N + splits - 1) / splits;
        splits = (N + per - 1) / per;
    }
    double *part = (double *)d->scratch;
    float *coef = (float *)((char *)d->scratch + (size_t)splits * C * 2 * sizeof(double));
    dim3 g1((unsigned)C, (unsigned)splits);
    const BnBwdFin fin = {gw, gb, coef, (int)splits};
    if (bb.PP)
        k_bn_sums_bulk<<<g1, 256, bn_bulk_smem(bb, 2), NCK_STREAM(d)>>>(x, g, mean, invstd, part, N, C, S, per, bb.PP,
                                                                       bb.SP, bb.al, bb.dS, N * S, fin, d->counters,
                                                                       d->status, w, b, act, act_s);
    else if (v4) k_bn_bwd_sums<4><<<g1, kThreads, 0, NCK_STREAM(d)>>>(x, g, mean, invstd, part, N, C, S, per, fin, d->counters, w, b, act, act_s);
    else k_bn_bwd_sums<1><<<g1, kThreads, 0, NCK_STREAM(d)>>>(x, g, mean, invstd, part, N, C, S, per, fin, d->counters, w,
                                                               b, act, act_s);
    int launched = 1;
    if (gx) {
        int64_t planes = N * C;
        if (v4)
            k_bn_bwd_dx<4><<<flat_grid(d, planes * S / 4), 256, 0, NCK_STREAM(d)>>>(
                x, w, g, mean, invstd, coef, gx, planes, C, S, training, acc_gx, BN_DIVS(S, 4), make_fastdiv((uint32_t)C), b, act,
                act_s);
        else
            k_bn_bwd_dx<1><<<flat_grid(d, planes * S), 256, 0, NCK_STREAM(d)>>>(
                x, w, g, mean, invstd, coef, gx, planes, C, S, training, acc_gx, BN_DIVS(S, 1), make_fastdiv((uint32_t)C), b, act,
                act_s);
        launched++;
    }
    NCK_LAUNCHED(d, launched);
}

extern "C" void nck_bn_bwd(nck_dev *d, const float *x, const float *w, const float *g, const float *mean,
                           const float *invstd, float *gx, float *gw, float *gb, int64_t N, int64_t C, int64_t S,
                           int training, int acc_gx) {
    nck_bn_bwd_ex(d, x, w, nullptr, g, mean, invstd, gx, gw, gb, N, C, S, training, acc_gx, -1, 0.0f);
}

// ---- backward of BatchNorm + activation + 2 x 2 max pooling, fused -----------------------------------
//
// The BatchNorm output's gradient is nonzero only at each window's argmax, where it is the pooled
// gradient through the activation (evaluated at the recomputed BatchNorm output): the sums walk the
// pooled elements only; the input gradient is written window by window, with the dense formula at
// every element (the same arithmetic as k_bn_bwd_dx given that sparse gradient).
__global__ void __launch_bounds__(256) k_bn_pool_bwd_sums(const float *__restrict__ x, const float *__restrict__ gp,
                                                          const int32_t *__restrict__ arg,
                                                          const float *__restrict__ w, const float *__restrict__ b,
                                                          const float *__restrict__ mean,
                                                          const float *__restrict__ invstd, int act, float act_s,
                                                          double *__restrict__ part, int64_t N, int64_t C, int64_t HW,
                                                          int64_t L, int64_t per_split, BnBwdFin fin,
                                                          unsigned *counter) {
    __shared__ double sm[64];
    const int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    const float mu = mean[c], is = invstd[c], ea = w[c] * is, ed = b[c] - mu * ea;
    // the channel's pooled elements plane by plane (a plane's L elements are contiguous): four items
    // in flight per thread, the argmax gathers from x issued together, two double chains
    double g0 = 0.0, h0 = 0.0, g1 = 0.0, h1 = 0.0;
    ChanWalk wk;
    wk.init((int)L, n1 > n0 ? n1 - n0 : 0);
    const int64_t pbase = n0 * C + c;
    while (wk.live()) {
        float gv[4], xv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            gv[j] = 0.0f, xv[j] = mu;
            if (wk.live()) {
                const int64_t pl = pbase + (int64_t)wk.na * C;
                const int32_t a = __ldg(arg + pl * L + wk.ia);
                gv[j] = __ldg(gp + pl * L + wk.ia);
                xv[j] = __ldg(x + pl * HW + a);
            }
            wk.next();
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float g = epi_grad(act, act_s, xv[j] * ea + ed, gv[j]);
            if (j & 1) g1 += g, h1 += g * (xv[j] - mu) * is;
            else g0 += g, h0 += g * (xv[j] - mu) * is;
        }
    }
    double sg = g0 + g1, sgx = h0 + h1;
    block_sum2(sg, sgx, sm);
    if (threadIdx.x == 0) {
        part[(blockIdx.y * C + c) * 2] = sg;
        part[(blockIdx.y * C + c) * 2 + 1] = sgx;
    }
    if (last_block_done(counter)) bn_bwd_finalize(part, C, N * HW, fin);
}

// The sums from the forward's x at the argmax (xarg, pooled layout): two contiguous streams per plane,
// V-wide loads, the same per-element terms as the gathering kernel above.
template <int V>
__global__ void __launch_bounds__(256) k_bn_pool_bwd_sums_x(const float *__restrict__ xarg,
                                                            const float *__restrict__ gp,
                                                            const float *__restrict__ w, const float *__restrict__ b,
                                                            const float *__restrict__ mean,
                                                            const float *__restrict__ invstd, int act, float act_s,
                                                            double *__restrict__ part, int64_t N, int64_t C,
                                                            int64_t L, int64_t per_split, BnBwdFin fin,
                                                            unsigned *counter) {
    using VT = typename std::conditional<V == 4, float4, float>::type;
    __shared__ double sm[64];
    const int64_t c = blockIdx.x, n0 = blockIdx.y * per_split, n1 = n0 + per_split < N ? n0 + per_split : N;
    const float mu = mean[c], is = invstd[c], ea = w[c] * is, ed = b[c] - mu * ea;
    double g0 = 0.0, h0 = 0.0, g1 = 0.0, h1 = 0.0;
    ChanWalk wk;
    const int SV = (int)(L / V);
    wk.init(SV, n1 > n0 ? n1 - n0 : 0);
    const int64_t pbase = n0 * C + c;
    // items in flight per thread: two float4, or eight floats for planes that are not float4 multiples
    constexpr int U = V == 4 ? 2 : 8;
    while (wk.live()) {
        VT gv[U], xv[U];
        bool on[U];
#pragma unroll
        for (int j = 0; j < U; j++) {
            on[j] = wk.live();
            if (on[j]) {
                const int64_t off = (pbase + (int64_t)wk.na * C) * SV + wk.ia;
                gv[j] = __ldg(reinterpret_cast<const VT *>(gp) + off);
                xv[j] = __ldg(reinterpret_cast<const VT *>(xarg) + off);
            }
            wk.next();
        }
#pragma unroll
        for (int j = 0; j < U; j++) {
            if (!on[j]) continue;
            const float *ge = reinterpret_cast<const float *>(&gv[j]), *xe = reinterpret_cast<const float *>(&xv[j]);
#pragma unroll
            for (int e = 0; e < V; e++) {
                const float g = epi_grad(act, act_s, xe[e] * ea + ed, ge[e]);
                if (e & 1) g1 += g, h1 += g * (xe[e] - mu) * is;
                else g0 += g, h0 += g * (xe[e] - mu) * is;
            }
        }
    }
    double sg = g0 + g1, sgx = h0 + h1;
    block_sum2(sg, sgx, sm);
    if (threadIdx.x == 0) {
        part[(blockIdx.y * C + c) * 2] = sg;
        part[(blockIdx.y * C + c) * 2 + 1] = sgx;
    }
    if (last_block_done(counter)) bn_bwd_finalize(part, C, N * L * 4, fin);
}

__global__ void __launch_bounds__(256) k_bn_pool_bwd_dx(const float *__restrict__ x, const float *__restrict__ gp,
                                                        const int32_t *__restrict__ arg, const float *__restrict__ w,
                                                        const float *__restrict__ b, const float *__restrict__ mean,
                                                        const float *__restrict__ invstd,
                                                        const float *__restrict__ coef, int act, float act_s,
                                                        float *__restrict__ gx, int acc, uint32_t planes, uint32_t C,
                                                        uint32_t W, uint32_t OH, uint32_t OW, FastDiv dow,
                                                        FastDiv doh, FastDiv dc) {
    const uint32_t total = planes * OH * OW;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const uint32_t r = dow.div(t), ox = t - r * OW, pl = doh.div(r), oy = r - pl * OH;
        const uint32_t c = pl - dc.div(pl) * C;
        const float mu = __ldg(mean + c), is = __ldg(invstd + c), k = __ldg(w + c) * is;
        const float ea = k, ed = __ldg(b + c) - mu * ea;
        const float mg = __ldg(coef + 2 * c), mgx = __ldg(coef + 2 * c + 1);
        const size_t base = (size_t)pl * (2 * OH) * W + (size_t)(2 * oy) * W + 2 * ox;
        const float2 p = __ldg(reinterpret_cast<const float2 *>(x + base));
        const float2 q = __ldg(reinterpret_cast<const float2 *>(x + base + W));
        const int32_t a = __ldg(arg + t) - (int32_t)(2 * oy * W + 2 * ox); // 0, 1, W or W + 1
        const float xs[4] = {p.x, p.y, q.x, q.y};
        const int32_t at[4] = {0, 1, (int32_t)W, (int32_t)W + 1};
        const float gval = __ldg(gp + t);
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float ge = at[e] == a ? epi_grad(act, act_s, xs[e] * ea + ed, gval) : 0.0f;
            o[e] = k * (ge - mg - (xs[e] - mu) * is * mgx);
        }
        float2 *d0 = reinterpret_cast<float2 *>(gx + base), *d1 = reinterpret_cast<float2 *>(gx + base + W);
        if (acc) {
            const float2 u = *d0, v = *d1;
            o[0] = u.x + o[0], o[1] = u.y + o[1], o[2] = v.x + o[2], o[3] = v.y + o[3];
        } else {
            o[0] = 0.0f + o[0], o[1] = 0.0f + o[1], o[2] = 0.0f + o[2], o[3] = 0.0f + o[3];
        }
        *d0 = make_float2(o[0], o[1]);
        *d1 = make_float2(o[2], o[3]);
    }
}

extern "C" void nck_bn_pool_bwd(nck_dev *d, const float *x, const float *w, const float *b, const float *gpool,
                                const int32_t *arg, const float *xarg, const float *mean, const float *invstd,
                                float *gx, float *gw, float *gb, int64_t N, int64_t C, int64_t H, int64_t W,
                                int acc_gx, int act, float act_s) {
    const int64_t HW = H * W, OH = H / 2, OW = W / 2, L = OH * OW;
    Scope sc(d, "bn_pool_bwd", 0.0, 4.0 * N * C * (HW + 2 * L) + (gx ? (acc_gx ? 8.0 : 4.0) * N * C * HW : 0.0));
    static int res = 0, res4 = 0, res1 = 0;
    if (!res) res = resident_blocks(d, k_bn_pool_bwd_sums, kThreads);
    if (!res4) res4 = resident_blocks(d, k_bn_pool_bwd_sums_x<4>, kThreads);
    if (!res1) res1 = resident_blocks(d, k_bn_pool_bwd_sums_x<1>, kThreads);
    const bool v4 = xarg && L % 4 == 0 && (((uintptr_t)xarg | (uintptr_t)gpool) & 15) == 0;
    const BnBulk bb = xarg ? bn_bulk_plan(d, L, 2, xarg, gpool) : BnBulk{0, 0, 0, make_fastdiv(1)};
    int64_t splits, per;
    if (bb.PP) {
        bn_bulk_grid(d, k_bn_sums_bulk, bn_bulk_smem(bb, 2), N, C, L, splits, per);
    } else {
        splits = bn_splits(xarg ? (v4 ? res4 : res1) : res, N, C, L), per = (N + splits - 1) / splits;
        splits = (N + per - 1) / per;
    }
    double *part = (double *)d->scratch;
    float *coef = (float *)((char *)d->scratch + (size_t)splits * C * 2 * sizeof(double));
    const BnBwdFin fin = {gw, gb, coef, (int)splits};
    dim3 g1((unsigned)C, (unsigned)splits);
    if (bb.PP)
        k_bn_sums_bulk<<<g1, 256, bn_bulk_smem(bb, 2), NCK_STREAM(d)>>>(xarg, gpool, mean, invstd, part, N, C, L, per,
                                                                       bb.PP, bb.SP, bb.al, bb.dS, N * L * 4, fin,
                                                                       d->counters, d->status, w, b, act, act_s);
    else if (v4)
        k_bn_pool_bwd_sums_x<4><<<g1, kThreads, 0, NCK_STREAM(d)>>>(xarg, gpool, w, b, mean, invstd, act, act_s, part, N,
                                                                   C, L, per, fin, d->counters);
    else if (xarg)
        k_bn_pool_bwd_sums_x<1><<<g1, kThreads, 0, NCK_STREAM(d)>>>(xarg, gpool, w, b, mean, invstd, act, act_s, part, N,
                                                                   C, L, per, fin, d->counters);
    else
        k_bn_pool_bwd_sums<<<g1, kThreads, 0, NCK_STREAM(d)>>>(x, gpool, arg, w, b, mean, invstd, act, act_s, part, N, C,
                                                              HW, L, per, fin, d->counters);
    int launched = 1;
    if (gx) {
        const int64_t total = N * C * L;
        k_bn_pool_bwd_dx<<<grid_for(d, total), 256, 0, NCK_STREAM(d)>>>(
            x, gpool, arg, w, b, mean, invstd, coef, act, act_s, gx, acc_gx, (uint32_t)(N * C), (uint32_t)C,
            (uint32_t)W, (uint32_t)OH, (uint32_t)OW, make_fastdiv((uint32_t)OW), make_fastdiv((uint32_t)OH),
            make_fastdiv((uint32_t)C));
        launched++;
    }
    NCK_LAUNCHED(d, launched);
}

// ---- layer norm over rows of D: one warp per row -------------------------------------------------------

__global__ void k_ln_fwd(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
                         float *__restrict__ y, float *__restrict__ stats, int64_t R, int64_t D, float eps) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5, nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < R; r += nw) {
        const float *p = x + r * D;
        double s = 0.0;
        for (int64_t i = lane; i < D; i += 32) s += (double)p[i];
        s = warp_sum_d(s);
        double mean = s / (double)D;
        double ss = 0.0;
        for (int64_t i = lane; i < D; i += 32) {
            double dv = (double)p[i] - mean;
            ss += dv * dv;
        }
        ss = warp_sum_d(ss);
        float rstd = (float)(1.0 / sqrt(ss / (double)D + (double)eps));
        float fm = (float)mean;
        if (lane == 0) stats[2 * r] = fm, stats[2 * r + 1] = rstd;
        float *q = y + r * D;
        for (int64_t i = lane; i < D; i += 32) {
            float v = (p[i] - fm) * rstd;
            q[i] = (w ? v * w[i] : v) + (b ? b[i] : 0.0f);
        }
    }
}

// Rows of D = 128 NV floats kept in registers (one warp per row, NV float4 per lane): one read of x
// for the statistics and the output; the same arithmetic as k_ln_fwd.
template <int NV>
__global__ void __launch_bounds__(256) k_ln_fwd_reg(const float *__restrict__ x, const float *__restrict__ w,
                                                    const float *__restrict__ b, float *__restrict__ y,
                                                    float *__restrict__ stats, int64_t R, float eps) {
    constexpr int D = 128 * NV;
    const int lane = threadIdx.x & 31;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < R; r += nw) {
        const float4 *p = reinterpret_cast<const float4 *>(x + r * D);
        float4 v[NV];
        double s = 0.0;
#pragma unroll
        for (int k = 0; k < NV; k++) {
            v[k] = __ldg(p + lane + 32 * k);
            s += (double)v[k].x, s += (double)v[k].y, s += (double)v[k].z, s += (double)v[k].w;
        }
        s = warp_sum_d(s);
        const double mean = s / (double)D;
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const double a = (double)v[k].x - mean, bb = (double)v[k].y - mean, c = (double)v[k].z - mean,
                         e = (double)v[k].w - mean;
            ss += a * a, ss += bb * bb, ss += c * c, ss += e * e;
        }
        ss = warp_sum_d(ss);
        const float rstd = (float)(1.0 / sqrt(ss / (double)D + (double)eps));
        const float fm = (float)mean;
        if (lane == 0) stats[2 * r] = fm, stats[2 * r + 1] = rstd;
        float4 *q = reinterpret_cast<float4 *>(y + r * D);
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const int i = lane + 32 * k;
            const float4 wv = w ? __ldg(reinterpret_cast<const float4 *>(w) + i) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float4 bv = b ? __ldg(reinterpret_cast<const float4 *>(b) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 o;
            o.x = (w ? ((v[k].x - fm) * rstd) * wv.x : (v[k].x - fm) * rstd) + bv.x;
            o.y = (w ? ((v[k].y - fm) * rstd) * wv.y : (v[k].y - fm) * rstd) + bv.y;
            o.z = (w ? ((v[k].z - fm) * rstd) * wv.z : (v[k].z - fm) * rstd) + bv.z;
            o.w = (w ? ((v[k].w - fm) * rstd) * wv.w : (v[k].w - fm) * rstd) + bv.w;
            q[i] = o;
        }
    }
}

// Backward with the row in registers: dx in one read of x and g, and the weight / bias column sums
// of the block's rows (lane-private running sums, then a fixed tree over the block's warps) as one
// partial per block, combined in a fixed order by nck_combine_cols.
template <int NV>
__global__ void __launch_bounds__(256) k_ln_bwd_reg(const float *__restrict__ x, const float *__restrict__ w,
                                                    const float *__restrict__ g, const float *__restrict__ stats,
                                                    float *__restrict__ gx, float *__restrict__ part, int64_t R,
                                                    int want_wb, int acc_gx) {
    constexpr int D = 128 * NV;
    __shared__ float red[8][128];  // one 128-column slice at a time
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    float4 aw[NV], ab[NV];
#pragma unroll
    for (int k = 0; k < NV; k++) aw[k] = ab[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < R; r += nw) {
        const float4 *p = reinterpret_cast<const float4 *>(x + r * D), *q = reinterpret_cast<const float4 *>(g + r * D);
        const float mean = __ldg(stats + 2 * r), rstd = __ldg(stats + 2 * r + 1);
        float4 xh[NV], gi[NV], gr[NV];
        double sg = 0.0, sgx = 0.0;
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const int i = lane + 32 * k;
            const float4 xv = __ldg(p + i);
            gr[k] = __ldg(q + i);
            const float4 wv = w ? __ldg(reinterpret_cast<const float4 *>(w) + i) : make_float4(1.f, 1.f, 1.f, 1.f);
            xh[k] = make_float4((xv.x - mean) * rstd, (xv.y - mean) * rstd, (xv.z - mean) * rstd, (xv.w - mean) * rstd);
            gi[k] = w ? make_float4(gr[k].x * wv.x, gr[k].y * wv.y, gr[k].z * wv.z, gr[k].w * wv.w) : gr[k];
            sg += gi[k].x, sg += gi[k].y, sg += gi[k].z, sg += gi[k].w;
            sgx += gi[k].x * xh[k].x, sgx += gi[k].y * xh[k].y, sgx += gi[k].z * xh[k].z, sgx += gi[k].w * xh[k].w;
            if (want_wb) {
                aw[k].x += gr[k].x * xh[k].x, aw[k].y += gr[k].y * xh[k].y;
                aw[k].z += gr[k].z * xh[k].z, aw[k].w += gr[k].w * xh[k].w;
                ab[k].x += gr[k].x, ab[k].y += gr[k].y, ab[k].z += gr[k].z, ab[k].w += gr[k].w;
            }
        }
        sg = warp_sum_d(sg);
        sgx = warp_sum_d(sgx);
        if (gx) {
            const float mg = (float)(sg / (double)D), mgx = (float)(sgx / (double)D);
            float4 *o = reinterpret_cast<float4 *>(gx + r * D);
#pragma unroll
            for (int k = 0; k < NV; k++) {
                const int i = lane + 32 * k;
                float4 a = acc_gx ? o[i] : make_float4(0.f, 0.f, 0.f, 0.f);  // a fresh buffer is stored
                a.x += rstd * (gi[k].x - mg - xh[k].x * mgx), a.y += rstd * (gi[k].y - mg - xh[k].y * mgx);
                a.z += rstd * (gi[k].z - mg - xh[k].z * mgx), a.w += rstd * (gi[k].w - mg - xh[k].w * mgx);
                o[i] = a;
            }
        }
    }
    if (!want_wb) return;
    // block partials: column c of the weight sums (then the bias sums at D + c), warps added in order
#pragma unroll
    for (int k = 0; k < NV; k++) {
        __syncthreads();
        const int c = 4 * lane; // columns of float4 slice k: 4 * (lane + 32 k) .. + 3, staged as 4 * lane
        red[warp][c] = aw[k].x, red[warp][c + 1] = aw[k].y, red[warp][c + 2] = aw[k].z, red[warp][c + 3] = aw[k].w;
        __syncthreads();
        if (threadIdx.x < 128) {
            float t = 0.0f;
            for (int q = 0; q < (int)(blockDim.x >> 5); q++) t += red[q][threadIdx.x];
            part[(int64_t)blockIdx.x * 2 * D + 128 * k + threadIdx.x] = t;
        }
        __syncthreads();
        red[warp][c] = ab[k].x, red[warp][c + 1] = ab[k].y, red[warp][c + 2] = ab[k].z, red[warp][c + 3] = ab[k].w;
        __syncthreads();
        if (threadIdx.x < 128) {
            float t = 0.0f;
            for (int q = 0; q < (int)(blockDim.x >> 5); q++) t += red[q][threadIdx.x];
            part[(int64_t)blockIdx.x * 2 * D + D + 128 * k + threadIdx.x] = t;
        }
    }
}

extern "C" void nck_ln_fwd(nck_dev *d, const float *x, const float *w, const float *b, float *y, float *stats,
                           int64_t R, int64_t D, float eps) {
    Scope sc(d, "ln_fwd", 0.0, 8.0 * R * D);
    const bool vec = D % 128 == 0 && D <= 1024 && (((uintptr_t)x | (uintptr_t)y | (uintptr_t)w | (uintptr_t)b) & 15) == 0;
    const int g = grid_for(d, R * 32);
    if (vec && D == 128) k_ln_fwd_reg<1><<<g, 256, 0, NCK_STREAM(d)>>>(x, w, b, y, stats, R, eps);
    else if (vec && D == 256) k_ln_fwd_reg<2><<<g, 256, 0, NCK_STREAM(d)>>>(x, w, b, y, stats, R, eps);
    else if (vec && D == 512) k_ln_fwd_reg<4><<<g, 256, 0, NCK_STREAM(d)>>>(x, w, b, y, stats, R, eps);
    else if (vec && D == 1024) k_ln_fwd_reg<8><<<g, 256, 0, NCK_STREAM(d)>>>(x, w, b, y, stats, R, eps);
    else k_ln_fwd<<<g, kThreads, 0, NCK_STREAM(d)>>>(x, w, b, y, stats, R, D, eps);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_ln_bwd_dx(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ g,
                            const float *__restrict__ stats, float *__restrict__ gx, int64_t R, int64_t D,
                            int acc_gx) {
    int lane = threadIdx.x & 31;
    int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5, nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < R; r += nw) {
        const float *p = x + r * D, *q = g + r * D;
        float mean = stats[2 * r], rstd = stats[2 * r + 1];
        double sg = 0.0, sgx = 0.0;
        for (int64_t i = lane; i < D; i += 32) {
            float xhat = (p[i] - mean) * rstd, gi = w ? q[i] * w[i] : q[i];
            sg += gi;
            sgx += gi * xhat;
        }
        sg = warp_sum_d(sg);
        sgx = warp_sum_d(sgx);
        float mg = (float)(sg / (double)D), mgx = (float)(sgx / (double)D);
        float *o = gx + r * D;
        for (int64_t i = lane; i < D; i += 32) {
            float xhat = (p[i] - mean) * rstd, gi = w ? q[i] * w[i] : q[i];
            o[i] = (acc_gx ? o[i] : 0.0f) + rstd * (gi - mg - xhat * mgx);
        }
    }
}

// weight / bias grads: column sums over rows of g * xhat and g, split over row ranges
__global__ void k_ln_bwd_wb(const float *__restrict__ x, const float *__restrict__ g, const float *__restrict__ stats,
                            float *__restrict__ part, int64_t R, int64_t D, int64_t rows_per) {
    __shared__ float sw[8][33], sb[8][33];
    int64_t i = blockIdx.x * 32 + threadIdx.x;
    int64_t r0 = blockIdx.y * rows_per, r1 = r0 + rows_per < R ? r0 + rows_per : R;
    float aw = 0.0f, ab = 0.0f;
    if (i < D)
        for (int64_t r = r0 + threadIdx.y; r < r1; r += 8) {
            float gv = g[r * D + i];
            aw += gv * ((x[r * D + i] - stats[2 * r]) * stats[2 * r + 1]);
            ab += gv;
        }
    sw[threadIdx.y][threadIdx.x] = aw;
    sb[threadIdx.y][threadIdx.x] = ab;
    __syncthreads();
    if (threadIdx.y == 0 && i < D) {
        float a = 0.0f, b = 0.0f;
        for (int k = 0; k < 8; k++) a += sw[k][threadIdx.x], b += sb[k][threadIdx.x];
        part[(blockIdx.y * 2) * D + i] = a;
        part[(blockIdx.y * 2 + 1) * D + i] = b;
    }
}

__global__ void k_ln_bwd_wb_combine(const float *__restrict__ part, int splits, int64_t D, float *gw, float *gb) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < D; i += (int64_t)gridDim.x * blockDim.x) {
        float a = 0.0f, b = 0.0f;
        for (int k = 0; k < splits; k++) a += part[(2 * k) * D + i], b += part[(2 * k + 1) * D + i];
        if (gw) gw[i] += a;
        if (gb) gb[i] += b;
    }
}

// the weight / bias sums from the per-split partials (split k: D weight sums, then D bias sums); a
// missing output is skipped by summing only the half that exists
static void ln_wb_combine(nck_dev *d, const float *part, int splits, int64_t D, float *gw, float *gb) {
    if (gw && gb) nck_combine_cols(d, part, 2 * D, splits, 2 * D, gw, D, gb);
    else if (gw) nck_combine_cols(d, part, 2 * D, splits, D, gw, D, nullptr);
    else if (gb) nck_combine_cols(d, part + D, 2 * D, splits, D, gb, D, nullptr);
}

extern "C" void nck_ln_bwd(nck_dev *d, const float *x, const float *w, const float *g, const float *stats, float *gx,
                           float *gw, float *gb, int64_t R, int64_t D, int acc_gx) {
    Scope sc(d, "ln_bwd", 0.0, (gx ? (acc_gx ? 16.0 : 12.0) : 8.0) * R * D);
    int launched = 0;
    const bool vec = (D == 128 || D == 256 || D == 512 || D == 1024) &&
                     (((uintptr_t)x | (uintptr_t)g | (uintptr_t)gx | (uintptr_t)w) & 15) == 0;
    if (vec) {
        static int resident = 0;
        if (!resident) resident = resident_blocks(d, k_ln_bwd_reg<2>, 256);
        int64_t blocks = (R + 7) / 8;
        if (blocks > resident) blocks = resident;
        if ((gw || gb) && blocks * 2 * D * (int64_t)sizeof(float) > (int64_t)d->scratch_bytes)
            blocks = (int64_t)d->scratch_bytes / (2 * D * (int64_t)sizeof(float));
        if (blocks < 1) blocks = 1;
        float *part = (float *)d->scratch;
        const int want = gw || gb;
        if (D == 128) k_ln_bwd_reg<1><<<(unsigned)blocks, 256, 0, NCK_STREAM(d)>>>(x, w, g, stats, gx, part, R, want, acc_gx);
        else if (D == 256) k_ln_bwd_reg<2><<<(unsigned)blocks, 256, 0, NCK_STREAM(d)>>>(x, w, g, stats, gx, part, R, want, acc_gx);
        else if (D == 512) k_ln_bwd_reg<4><<<(unsigned)blocks, 256, 0, NCK_STREAM(d)>>>(x, w, g, stats, gx, part, R, want, acc_gx);
        else k_ln_bwd_reg<8><<<(unsigned)blocks, 256, 0, NCK_STREAM(d)>>>(x, w, g, stats, gx, part, R, want, acc_gx);
        launched = 1;
        NCK_LAUNCHED(d, launched);
        if (want) ln_wb_combine(d, part, (int)blocks, D, gw, gb);
        return;
    }
    if (gx) {
        k_ln_bwd_dx<<<grid_for(d, R * 32), kThreads, 0, NCK_STREAM(d)>>>(x, w, g, stats, gx, R, D, acc_gx);
        launched++;
    }
    if (gw || gb) {
        int64_t col_blocks = (D + 31) / 32;
        int64_t splits = ((int64_t)d->sm_count * 4 + col_blocks - 1) / col_blocks;
        if (splits > R / 16 + 1) splits = R / 16 + 1;
        int64_t maxs = (int64_t)d->scratch_bytes / (2 * D * (int64_t)sizeof(float));
        if (splits > maxs) splits = maxs;
        if (splits < 1) splits = 1;
        int64_t per = (R + splits - 1) / splits;
        splits = (R + per - 1) / per;
        float *part = (float *)d->scratch;
        dim3 grid((unsigned)col_blocks, (unsigned)splits), block(32, 8);
        k_ln_bwd_wb<<<grid, block, 0, NCK_STREAM(d)>>>(x, g, stats, part, R, D, per);
        launched++;
        NCK_LAUNCHED(d, launched);
        ln_wb_combine(d, part, (int)splits, D, gw, gb);
        return;
    }
    NCK_LAUNCHED(d, launched);
}
