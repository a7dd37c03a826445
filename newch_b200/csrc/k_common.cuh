// Shared helpers for the sm_100a kernels: launch geometry, the kernel status word, timing hooks.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "nck.h"

#define NCK_STREAM(d) ((cudaStream_t)(d)->stream)

namespace nck {

constexpr int kThreads = 256;

// Grid for a grid-stride loop over n items: enough blocks to fill every SM several times over,
// never more than the work needs.
inline int grid_for(const nck_dev *d, int64_t n, int threads = kThreads, int per_sm = 8) {
    int64_t want = (n + threads - 1) / threads;
    int64_t cap = (int64_t)(d->sm_count > 0 ? d->sm_count : 148) * per_sm;
    if (want > cap) want = cap;
    return want < 1 ? 1 : (int)want;
}

// n / d for 32-bit n < 2^31 by multiply-high with a precomputed magic number (Granlund-Montgomery):
// l = ceil(log2 d), mul = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, mul) + n) >> l
struct FastDiv {
    uint32_t d, mul, shift;
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        return d == 1 ? n : (uint32_t)((__umulhi(n, mul) + n) >> shift);
    }
};

inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f;
    f.d = d;
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) l++;
    f.shift = l;
    f.mul = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    if (d <= 1) f.mul = 0, f.shift = 0, f.d = 1;
    return f;
}

// Blocks of `kernel` that fit on the whole GPU at once (its occupancy per SM times the SMs): grids of
// split reductions are sized to one full wave, so no block runs in a second, mostly idle wave. The
// occupancy query runs once per call site (cache it in a static).
template <typename K>
inline int resident_blocks(const nck_dev *d, K kernel, int threads, size_t smem = 0) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess) {
        cudaGetLastError();
        per_sm = 1;
    }
    if (per_sm < 1) per_sm = 1;
    return per_sm * (d->sm_count > 0 ? d->sm_count : 148);
}

// A block's walk over the items of one channel in an [N][C][S] tensor: planes [n0, n1) of channel c,
// SV vector items per plane. Thread t takes items t, t + B, t + 2B, ... (B = blockDim.x) and advances
// its (plane, item) pair by a carry instead of a division per item.
struct ChanWalk {
    int na, ia, dn, dr, SV;
    int64_t cnt;
    __device__ __forceinline__ void init(int sv, int64_t planes) {
        SV = sv, cnt = planes;
        na = (int)(threadIdx.x / (unsigned)sv), ia = (int)threadIdx.x - na * sv;
        dn = (int)(blockDim.x / (unsigned)sv), dr = (int)blockDim.x - dn * sv;
    }
    __device__ __forceinline__ bool live() const { return na < cnt; }
    __device__ __forceinline__ void next() {
        ia += dr, na += dn;
        if (ia >= SV) ia -= SV, na++;
    }
};

// Records a kernel-detected error (first one wins). The host reads it at its next synchronization.
__device__ __forceinline__ void report(int *status, int code) { atomicCAS(status, 0, code); }

// True in the one block of the grid that finishes last: every block's thread 0 publishes its
// partial result, fences and counts itself in; the block that makes the count complete sees all the
// partials (read them with ld.global.cg) and re-arms the counter to 0 for the next launch.
__device__ __forceinline__ bool last_block_done(unsigned *counter) {
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned total = gridDim.x * gridDim.y * gridDim.z;
        last = atomicAdd(counter, 1u) == total - 1;
        if (last) atomicExch(counter, 0u);
    }
    __syncthreads();
    if (last) __threadfence();
    return last;
}

// RAII timing scope: when the device has a timer, brackets the launches inside with CUDA events.
struct Scope {
    nck_dev *d;
    Scope(nck_dev *dev, const char *name, double flops = 0.0, double bytes = 0.0) : d(dev) {
        if (d->timer) nck_timer_begin(d, name, flops, bytes);
    }
    ~Scope() {
        if (d->timer) nck_timer_end(d);
    }
};

}  // namespace nck

#define NCK_LAUNCHED(d, k) ((d)->launches += (k))
