// Memory kernels: fills, axpy, strided gather / accumulate, dtype conversion, and the per-kernel
// CUDA-event timer used by the benchmark.
#include <math.h>
#include <string.h>

#include <string>
#include <vector>

#include "k_common.cuh"

using namespace nck;

// ---- timer -------------------------------------------------------------------------------------

struct nck_timer {
    struct Rec {
        int name;
        cudaEvent_t a, b;
    };
    std::vector<std::string> names;
    std::vector<Rec> recs;
    std::vector<cudaEvent_t> pool;
    int open = -1;
    std::vector<double> ms_by_name, flops_by_name, bytes_by_name;
    std::vector<int64_t> n_by_name;
};

static cudaEvent_t take_event(nck_timer *t) {
    if (!t->pool.empty()) {
        cudaEvent_t e = t->pool.back();
        t->pool.pop_back();
        return e;
    }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
}

extern "C" void nck_timer_enable(nck_dev *d, int on) {
    if (on && !d->timer) {
        d->timer = new nck_timer();
    } else if (!on && d->timer) {
        nck_timer *t = d->timer;
        for (auto &r : t->recs) {
            cudaEventDestroy(r.a);
            cudaEventDestroy(r.b);
        }
        for (auto e : t->pool) cudaEventDestroy(e);
        delete t;
        d->timer = nullptr;
    }
}

extern "C" void nck_timer_begin(nck_dev *d, const char *name, double flops, double bytes) {
    nck_timer *t = d->timer;
    if (!t || t->open >= 0) return;  // nested scopes: the outer one times them all
    int id = -1;
    for (size_t i = 0; i < t->names.size(); i++)
        if (t->names[i] == name) id = (int)i;
    if (id < 0) {
        t->names.push_back(name);
        t->ms_by_name.push_back(0);
        t->flops_by_name.push_back(0);
        t->bytes_by_name.push_back(0);
        t->n_by_name.push_back(0);
        id = (int)t->names.size() - 1;
    }
    t->flops_by_name[id] += flops;
    t->bytes_by_name[id] += bytes;
    nck_timer::Rec r{id, take_event(t), take_event(t)};
    cudaEventRecord(r.a, NCK_STREAM(d));
    t->recs.push_back(r);
    t->open = (int)t->recs.size() - 1;
}

extern "C" void nck_timer_end(nck_dev *d) {
    nck_timer *t = d->timer;
    if (!t || t->open < 0) return;
    cudaEventRecord(t->recs[t->open].b, NCK_STREAM(d));
    t->open = -1;
}

static void settle(nck_timer *t) {
    for (auto &r : t->recs) {
        float ms = 0;
        cudaEventSynchronize(r.b);
        cudaEventElapsedTime(&ms, r.a, r.b);
        t->ms_by_name[r.name] += ms;
        t->n_by_name[r.name] += 1;
        t->pool.push_back(r.a);
        t->pool.push_back(r.b);
    }
    t->recs.clear();
}

extern "C" int nck_timer_query(nck_dev *d, const char *prefix, double *ms, int64_t *count) {
    nck_timer *t = d->timer;
    *ms = 0;
    *count = 0;
    if (!t) return 5;
    settle(t);
    size_t lp = strlen(prefix);
    for (size_t i = 0; i < t->names.size(); i++) {
        if (strncmp(t->names[i].c_str(), prefix, lp) != 0) continue;
        *ms += t->ms_by_name[i];
        *count += t->n_by_name[i];
    }
    return 0;
}

extern "C" int nck_timer_work(nck_dev *d, const char *prefix, double *flops, double *bytes) {
    nck_timer *t = d->timer;
    *flops = 0;
    *bytes = 0;
    if (!t) return 5;
    size_t lp = strlen(prefix);
    for (size_t i = 0; i < t->names.size(); i++) {
        if (strncmp(t->names[i].c_str(), prefix, lp) != 0) continue;
        *flops += t->flops_by_name[i];
        *bytes += t->bytes_by_name[i];
    }
    return 0;
}

extern "C" int nck_timer_entry(nck_dev *d, int i, const char **name, double *ms, int64_t *count, double *flops,
                               double *bytes) {
    nck_timer *t = d->timer;
    if (!t) return 0;
    settle(t);
    if (i < 0 || i >= (int)t->names.size()) return 0;
    *name = t->names[i].c_str();
    *ms = t->ms_by_name[i];
    *count = t->n_by_name[i];
    *flops = t->flops_by_name[i];
    *bytes = t->bytes_by_name[i];
    return 1;
}

extern "C" void nck_timer_reset(nck_dev *d) {
    nck_timer *t = d->timer;
    if (!t) return;
    settle(t);
    for (auto &v : t->ms_by_name) v = 0;
    for (auto &v : t->flops_by_name) v = 0;
    for (auto &v : t->bytes_by_name) v = 0;
    for (auto &v : t->n_by_name) v = 0;
}

// ---- fills -------------------------------------------------------------------------------------

template <typename T>
__global__ void k_fill(T *__restrict__ y, T v, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = v;
}

extern "C" void nck_fill_f32(nck_dev *d, float *y, float v, int64_t n) {
    if (n <= 0) return;
    Scope s(d, "fill");
    k_fill<float><<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(y, v, n);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_fill_i32(nck_dev *d, int32_t *y, int32_t v, int64_t n) {
    if (n <= 0) return;
    Scope s(d, "fill");
    k_fill<int32_t><<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(y, v, n);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_add_scalar_inplace(float *y, float v) { y[0] += v; }

extern "C" void nck_add_scalar_inplace(nck_dev *d, float *y, float v) {
    k_add_scalar_inplace<<<1, 1, 0, NCK_STREAM(d)>>>(y, v);
    NCK_LAUNCHED(d, 1);
}

// y += a * x, float4 body when both pointers are 16-byte aligned
__global__ void k_axpy(int64_t n, float a, const float *__restrict__ x, float *__restrict__ y, int vec) {
    int64_t stride = (int64_t)gridDim.x * blockDim.x, t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (vec) {
        int64_t n4 = n >> 2;
        const float4 *x4 = (const float4 *)x;
        float4 *y4 = (float4 *)y;
        for (int64_t i = t; i < n4; i += stride) {
            float4 xv = x4[i], yv = y4[i];
            yv.x += a * xv.x, yv.y += a * xv.y, yv.z += a * xv.z, yv.w += a * xv.w;
            y4[i] = yv;
        }
        for (int64_t i = (n4 << 2) + t; i < n; i += stride) y[i] += a * x[i];
    } else {
        for (int64_t i = t; i < n; i += stride) y[i] += a * x[i];
    }
}

__global__ void k_axpy_set(int64_t n, float a, const float *__restrict__ x, float *__restrict__ y, int vec) {
    int64_t stride = (int64_t)gridDim.x * blockDim.x, t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (vec) {
        const int64_t n4 = n >> 2;
        for (int64_t i = t; i < n4; i += stride) {
            float4 xv = __ldg((const float4 *)x + i);
            ((float4 *)y)[i] = make_float4(0.0f + a * xv.x, 0.0f + a * xv.y, 0.0f + a * xv.z, 0.0f + a * xv.w);
        }
        done = n4 << 2;
    }
    for (int64_t i = done + t; i < n; i += stride) y[i] = 0.0f + a * x[i];
}

extern "C" void nck_axpy_set(nck_dev *d, int64_t n, float a, const float *x, float *y) {
    if (n <= 0) return;
    Scope s(d, "axpy", 0.0, 8.0 * n);
    int vec = (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
    k_axpy_set<<<grid_for(d, vec ? (n + 3) / 4 : n), kThreads, 0, NCK_STREAM(d)>>>(n, a, x, y, vec);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_axpy(nck_dev *d, int64_t n, float a, const float *x, float *y) {
    if (n <= 0) return;
    Scope s(d, "axpy");
    int vec = (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
    k_axpy<<<grid_for(d, vec ? (n + 3) / 4 : n), kThreads, 0, NCK_STREAM(d)>>>(n, a, x, y, vec);
    NCK_LAUNCHED(d, 1);
}

// ---- strided copies ------------------------------------------------------------------------------
//
// A strided view is walked in row-major order of its shape: element i of the contiguous side maps to
// offset(i) on the strided side. Dims laid out back to back are merged first. When the innermost
// merged dim is contiguous on both sides with a length and outer strides that keep 16-byte
// alignment, each thread moves a float4 and divides only for the outer dims; index arithmetic is
// 32-bit with precomputed multiply-shift divisors whenever the view's offsets fit.

struct Strided {
    int nd;
    int64_t shape[NCK_MAXD];
    int64_t stride[NCK_MAXD];
};

struct Strided32 {
    int nd;
    uint32_t shape[NCK_MAXD];
    uint32_t stride[NCK_MAXD];
    FastDiv div[NCK_MAXD];
};

// element offset of linear (row-major) index i in a strided view
__device__ __forceinline__ int64_t strided_offset(const Strided &v, int64_t i) {
    int64_t off = 0;
    for (int k = v.nd - 1; k >= 0; k--) {
        int64_t q = i / v.shape[k];
        off += (i - q * v.shape[k]) * v.stride[k];
        i = q;
    }
    return off;
}

__device__ __forceinline__ uint32_t strided_offset32(const Strided32 &v, uint32_t i) {
    uint32_t off = 0;
#pragma unroll
    for (int k = NCK_MAXD - 1; k >= 0; k--) {
        if (k >= v.nd) continue;
        const uint32_t q = v.div[k].div(i);
        off += (i - q * v.shape[k]) * v.stride[k];
        i = q;
    }
    return off;
}

// MODE 0: dst[i] = src[off(i)] (gather); 1: dst[off(i)] += src[i]; 2: dst[off(i)] = src[i]
template <typename T, int MODE>
__global__ void k_strided64(Strided v, const T *__restrict__ src, T *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = strided_offset(v, i);
        if (MODE == 0) dst[i] = src[o];
        else if (MODE == 1) dst[o] += src[i];
        else dst[o] = src[i];
    }
}

// four items per thread per pass, all their loads issued before the first store
template <typename T, int MODE>
__global__ void k_strided32(Strided32 v, const T *__restrict__ src, T *__restrict__ dst, uint32_t n) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < n; i0 += 4 * stride) {
        uint32_t o[4];
        T a[4], b[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t i = i0 + u * stride;
            if (i < n) {
                o[u] = strided_offset32(v, i);
                if (MODE == 0) a[u] = src[o[u]];
                else a[u] = src[i];
                if (MODE == 1) b[u] = dst[o[u]];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t i = i0 + u * stride;
            if (i < n) {
                if (MODE == 0) dst[i] = a[u];
                else if (MODE == 1) dst[o[u]] = b[u] + a[u];
                else dst[o[u]] = a[u];
            }
        }
    }
}

// float4 items: v describes the view in items of 4 floats (the innermost dim divided by 4); four
// items per thread per pass, all their loads issued before the first store
template <int MODE>
__global__ void k_strided32_v4(Strided32 v, const float4 *__restrict__ src, float4 *__restrict__ dst, uint32_t n4) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < n4; i0 += 4 * stride) {
        uint32_t o[4];
        float4 a[4], b[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t i = i0 + u * stride;
            if (i < n4) {
                o[u] = strided_offset32(v, i);
                a[u] = MODE == 0 ? __ldg(src + o[u]) : __ldg(src + i);
                if (MODE == 1) b[u] = dst[o[u]];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t i = i0 + u * stride;
            if (i < n4) {
                if (MODE == 0) {
                    dst[i] = a[u];
                } else if (MODE == 1) {
                    float4 c = b[u];
                    c.x += a[u].x, c.y += a[u].y, c.z += a[u].z, c.w += a[u].w;
                    dst[o[u]] = c;
                } else {
                    dst[o[u]] = a[u];
                }
            }
        }
    }
}

// merges dims that are laid out back to back (fewer divisions per element)
static Strided simplify(int ndim, const int64_t *shape, const int64_t *stride) {
    Strided v;
    v.nd = 0;
    for (int k = 0; k < ndim; k++) {
        if (shape[k] == 1) continue;
        if (v.nd > 0 && v.stride[v.nd - 1] == stride[k] * shape[k]) {
            v.shape[v.nd - 1] *= shape[k];
            v.stride[v.nd - 1] = stride[k];
            continue;
        }
        v.shape[v.nd] = shape[k];
        v.stride[v.nd] = stride[k];
        v.nd++;
    }
    if (v.nd == 0) {
        v.nd = 1;
        v.shape[0] = 1;
        v.stride[0] = 1;
    }
    return v;
}

// the 32-bit form of v when every index and offset fits (strides >= 0); `unit` elements per item
static bool to32(const Strided &v, int64_t n, int unit, Strided32 *o) {
    if (n >= ((int64_t)1 << 31)) return false;
    int64_t span = 0;
    o->nd = v.nd;
    for (int k = 0; k < v.nd; k++) {
        int64_t sh = v.shape[k], st = v.stride[k];
        if (k == v.nd - 1 && unit > 1) sh /= unit, st = 1;
        else if (unit > 1) st /= unit;
        if (st < 0) return false;
        span += (sh - 1) * st;
        o->shape[k] = (uint32_t)sh;
        o->stride[k] = (uint32_t)st;
        o->div[k] = make_fastdiv((uint32_t)sh);
    }
    return span < ((int64_t)1 << 31);
}

// float4 items possible: contiguous innermost dim of a multiple of 4, outer strides multiples of 4,
// both base pointers 16-byte aligned
static bool vec4_ok(const Strided &v, const void *a, const void *b) {
    if (v.stride[v.nd - 1] != 1 || (v.shape[v.nd - 1] & 3) || (((uintptr_t)a | (uintptr_t)b) & 15)) return false;
    for (int k = 0; k < v.nd - 1; k++)
        if (v.stride[k] & 3) return false;
    return true;
}

template <int MODE>
static void strided_launch(nck_dev *d, int es, const Strided &v, int64_t n, const void *src, void *dst) {
    cudaStream_t st = NCK_STREAM(d);
    Strided32 v32;
    if (es == 4 && vec4_ok(v, src, dst) && to32(v, n / 4, 4, &v32)) {
        k_strided32_v4<MODE><<<grid_for(d, n / 4), kThreads, 0, st>>>(v32, (const float4 *)src, (float4 *)dst,
                                                                     (uint32_t)(n / 4));
    } else if (to32(v, n, 1, &v32)) {
        if (es == 4) k_strided32<int32_t, MODE><<<grid_for(d, n), kThreads, 0, st>>>(v32, (const int32_t *)src, (int32_t *)dst, (uint32_t)n);
        else if (es == 2) k_strided32<int16_t, MODE><<<grid_for(d, n), kThreads, 0, st>>>(v32, (const int16_t *)src, (int16_t *)dst, (uint32_t)n);
        else k_strided32<int8_t, MODE><<<grid_for(d, n), kThreads, 0, st>>>(v32, (const int8_t *)src, (int8_t *)dst, (uint32_t)n);
    } else {
        if (es == 4) k_strided64<int32_t, MODE><<<grid_for(d, n), kThreads, 0, st>>>(v, (const int32_t *)src, (int32_t *)dst, n);
        else if (es == 2) k_strided64<int16_t, MODE><<<grid_for(d, n), kThreads, 0, st>>>(v, (const int16_t *)src, (int16_t *)dst, n);
        else k_strided64<int8_t, MODE><<<grid_for(d, n), kThreads, 0, st>>>(v, (const int8_t *)src, (int8_t *)dst, n);
    }
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_copy_strided(nck_dev *d, int es, int ndim, const int64_t *shape, const int64_t *stride,
                                 const void *src, void *dst) {
    int64_t n = 1;
    for (int k = 0; k < ndim; k++) n *= shape[k];
    if (n <= 0) return;
    Strided v = simplify(ndim, shape, stride);
    Scope s(d, "copy_strided", 0.0, 2.0 * es * n);
    if (v.nd == 1 && v.stride[0] == 1) {
        cudaMemcpyAsync(dst, src, (size_t)n * es, cudaMemcpyDeviceToDevice, NCK_STREAM(d));
        return;
    }
    if (es == 4) {
        /* integers and floats move alike; the float4 path reads them as floats */
        strided_launch<0>(d, 4, v, n, src, dst);
    } else {
        strided_launch<0>(d, es, v, n, src, dst);
    }
}

// dst[view(i)] (+)= src[i]. Every destination element is hit at most once (views of a permutation
// or a slice), so there is no write conflict.
extern "C" void nck_acc_strided(nck_dev *d, int ndim, const int64_t *shape, const int64_t *dst_stride,
                                const float *src, float *dst, int acc) {
    int64_t n = 1;
    for (int k = 0; k < ndim; k++) n *= shape[k];
    if (n <= 0) return;
    Strided v = simplify(ndim, shape, dst_stride);
    Scope s(d, "acc_strided", 0.0, (acc ? 12.0 : 8.0) * n);
    if (v.nd == 1 && v.stride[0] == 1) {
        if (acc) nck_axpy(d, n, 1.0f, src, dst);
        else cudaMemcpyAsync(dst, src, (size_t)n * 4, cudaMemcpyDeviceToDevice, NCK_STREAM(d));
        return;
    }
    if (acc) strided_launch<1>(d, 4, v, n, src, dst);
    else strided_launch<2>(d, 4, v, n, src, dst);
}

// ---- dtype conversion (newch ops_shape.c:463-504: truncation toward zero, saturation, NaN -> 0) -------

__device__ __forceinline__ double load_as_double(const void *p, int dt, int64_t i) {
    switch (dt) {
    case 0: return (double)((const float *)p)[i];
    case 1: return (double)((const int32_t *)p)[i];
    case 3: return (double)((const int8_t *)p)[i];
    default: return (double)((const uint8_t *)p)[i];
    }
}

__device__ __forceinline__ double saturate(double v, double lo, double hi) {
    if (v != v) return 0.0;
    return v < lo ? lo : v > hi ? hi : v;
}

__global__ void k_convert(int from, int to, const void *__restrict__ src, void *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        double v = load_as_double(src, from, i);
        if (to == 0) ((float *)dst)[i] = (float)v;
        else if (to == 1) ((int32_t *)dst)[i] = (int32_t)saturate(v, -2147483648.0, 2147483647.0);
        else if (to == 3) ((int8_t *)dst)[i] = (int8_t)saturate(v, -128.0, 127.0);
        else ((uint8_t *)dst)[i] = (uint8_t)saturate(v, 0.0, 255.0);
    }
}

extern "C" void nck_convert(nck_dev *d, int from, int to, const void *src, void *dst, int64_t n) {
    if (n <= 0) return;
    Scope s(d, "convert");
    if (from == to) {
        size_t es = (from == 0 || from == 1) ? 4 : 1;
        cudaMemcpyAsync(dst, src, (size_t)n * es, cudaMemcpyDeviceToDevice, NCK_STREAM(d));
        return;
    }
    k_convert<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(from, to, src, dst, n);
    NCK_LAUNCHED(d, 1);
}
