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

// Records a kernel-detected error (first one wins). The host reads it at its next synchronization.
__device__ __forceinline__ void report(int *status, int code) { atomicCAS(status, 0, code); }

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
