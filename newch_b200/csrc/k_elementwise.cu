// Elementwise kernels: unary math and activations (forward / backward), broadcasting binary ops
// and their reduce-to-shape gradients, comparisons, masked_fill.
//
// Formulas and evaluation order follow newch engine/src/ops/ops_elementwise.c (unary :229-266,
// unary backward :289-338, binary backward :129-186). This file is compiled without FMA
// contraction so products and sums round as newch's plain C loops do; fmaf is written out where
// newch's vector axpy fuses.
#include <math.h>

#include "k_common.cuh"
#include "k_math.cuh"
#include "k_unary.cuh"

using namespace nck;

template <int M>
__device__ __forceinline__ float unary_grad(int kind, float s, float x, float y, float g) {
    switch (kind) {
    case NCK_UN_NEG: return -1.0f * g;
    case NCK_UN_EXP: return g * y;
    case NCK_UN_LOG: return g / x;
    case NCK_UN_SQRT: return g * 0.5f / y;
    case NCK_UN_RELU: return x > 0.0f ? g : 0.0f;
    case NCK_UN_SIGMOID: return g * y * (1.0f - y);
    case NCK_UN_TANH: return g * (1.0f - y * y);
    case NCK_UN_SCALE: return s * g;
    case NCK_UN_ADD_SCALAR: return g;
    case NCK_UN_POW: return g * s * powf(x, s - 1.0f);
    case NCK_UN_LEAKY_RELU: return x > 0.0f ? g : s * g;
    case NCK_UN_RELU6: return (x > 0.0f && x < 6.0f) ? g : 0.0f;
    case NCK_UN_HARDSIGMOID: return (x > -3.0f && x < 3.0f) ? g * (1.0f / 6.0f) : 0.0f;
    case NCK_UN_HARDSWISH: return x < -3.0f ? 0.0f : x <= 3.0f ? g * (x * (1.0f / 3.0f) + 0.5f) : g;
    case NCK_UN_SILU: {
        float t = m_sigmoid<M>(x);
        return g * t * (1.0f + x * (1.0f - t));
    }
    case NCK_UN_GELU: {
        float t = m_erf<M>(NC_SQRT1_2 * x), t2 = m_exp<M>(-0.5f * x * x);
        return g * (0.5f * (1.0f + t) + x * NC_INV_SQRT_2PI * t2);
    }
    case NCK_UN_GELU_TANH: {
        float t = m_tanh<M>(NC_SQRT_2_PI * (x + NC_GELU_C * x * x * x));
        float dt = (1.0f - t * t) * NC_SQRT_2_PI * (1.0f + 3.0f * NC_GELU_C * x * x);
        return g * (0.5f * (1.0f + t) + 0.5f * x * dt);
    }
    }
    return 0.0f;
}

// the accumulation gi += v: axpy-style kinds fuse (newch's vector axpy), the others add
__device__ __forceinline__ float accumulate(int kind, float s, float gi, float g, float v) {
    if (kind == NCK_UN_SCALE) return fmaf(s, g, gi);
    if (kind == NCK_UN_NEG) return fmaf(-1.0f, g, gi);
    if (kind == NCK_UN_ADD_SCALAR) return fmaf(1.0f, g, gi);
    return gi + v;
}

template <int M>
__global__ void k_unary_fwd(int kind, float s, const float *__restrict__ x, float *__restrict__ y, int64_t n,
                            int vec) {
    int64_t stride = (int64_t)gridDim.x * blockDim.x, t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (vec) {
        int64_t n4 = n >> 2;
        for (int64_t i = t; i < n4; i += stride) {
            float4 v = ((const float4 *)x)[i];
            v.x = unary_f<M>(kind, s, v.x), v.y = unary_f<M>(kind, s, v.y), v.z = unary_f<M>(kind, s, v.z);
            v.w = unary_f<M>(kind, s, v.w);
            ((float4 *)y)[i] = v;
        }
        for (int64_t i = (n4 << 2) + t; i < n; i += stride) y[i] = unary_f<M>(kind, s, x[i]);
    } else {
        for (int64_t i = t; i < n; i += stride) y[i] = unary_f<M>(kind, s, x[i]);
    }
}

// nx / ny: the derivative reads x / y (a stream the derivative does not use is not loaded)
template <int M>
__global__ void k_unary_bwd(int kind, float s, const float *__restrict__ x, const float *__restrict__ y,
                            const float *__restrict__ g, float *__restrict__ gi, int64_t n, int vec, int acc, int nx,
                            int ny) {
    int64_t stride = (int64_t)gridDim.x * blockDim.x, t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (vec) {
        int64_t n4 = n >> 2;
        for (int64_t i = t; i < n4; i += stride) {
            const float4 z4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            float4 xv = nx ? __ldg((const float4 *)x + i) : z4, yv = ny ? __ldg((const float4 *)y + i) : z4;
            float4 gv = __ldg((const float4 *)g + i);
            float4 o = acc ? ((float4 *)gi)[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            o.x = accumulate(kind, s, o.x, gv.x, unary_grad<M>(kind, s, xv.x, yv.x, gv.x));
            o.y = accumulate(kind, s, o.y, gv.y, unary_grad<M>(kind, s, xv.y, yv.y, gv.y));
            o.z = accumulate(kind, s, o.z, gv.z, unary_grad<M>(kind, s, xv.z, yv.z, gv.z));
            o.w = accumulate(kind, s, o.w, gv.w, unary_grad<M>(kind, s, xv.w, yv.w, gv.w));
            ((float4 *)gi)[i] = o;
        }
        for (int64_t i = (n4 << 2) + t; i < n; i += stride)
            gi[i] = accumulate(kind, s, acc ? gi[i] : 0.0f, g[i], unary_grad<M>(kind, s, x[i], y[i], g[i]));
    } else {
        for (int64_t i = t; i < n; i += stride)
            gi[i] = accumulate(kind, s, acc ? gi[i] : 0.0f, g[i], unary_grad<M>(kind, s, x[i], y[i], g[i]));
    }
}

static const char *unary_name(int kind, int bwd) {
    static const char *f[] = {"un_neg", "un_exp", "un_log", "un_sqrt", "un_relu", "un_sigmoid", "un_tanh",
                              "un_scale", "un_add_scalar", "un_pow", "un_leaky_relu", "un_relu6",
                              "un_hardsigmoid", "un_hardswish", "un_silu", "un_gelu", "un_gelu_tanh"};
    static const char *b[] = {"unbwd_neg", "unbwd_exp", "unbwd_log", "unbwd_sqrt", "unbwd_relu", "unbwd_sigmoid",
                              "unbwd_tanh", "unbwd_scale", "unbwd_add_scalar", "unbwd_pow", "unbwd_leaky_relu",
                              "unbwd_relu6", "unbwd_hardsigmoid", "unbwd_hardswish", "unbwd_silu", "unbwd_gelu",
                              "unbwd_gelu_tanh"};
    return (kind >= 0 && kind <= NCK_UN_GELU_TANH) ? (bwd ? b[kind] : f[kind]) : "unary";
}

extern "C" void nck_unary_fwd(nck_dev *d, int kind, float s, const float *x, float *y, int64_t n) {
    if (n <= 0) return;
    Scope sc(d, unary_name(kind, 0), 0.0, 8.0 * n);
    int vec = (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
    auto k = d->math_mode == MATH_LIBM ? k_unary_fwd<MATH_LIBM> : k_unary_fwd<MATH_POLY>;
    k<<<grid_for(d, vec ? (n + 3) / 4 : n), kThreads, 0, NCK_STREAM(d)>>>(kind, s, x, y, n, vec);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_unary_bwd(nck_dev *d, int kind, float s, const float *x, const float *y, const float *g,
                              float *gi, int acc, int64_t n) {
    if (n <= 0) return;
    /* reads x, g and the accumulator (and y where the derivative uses it), writes the accumulator */
    int uses_y = kind == NCK_UN_EXP || kind == NCK_UN_SQRT || kind == NCK_UN_SIGMOID || kind == NCK_UN_TANH;
    int uses_x = !uses_y && kind != NCK_UN_SCALE && kind != NCK_UN_NEG && kind != NCK_UN_ADD_SCALAR;
    Scope sc(d, unary_name(kind, 1), 0.0, (8.0 + (acc ? 4.0 : 0.0) + (uses_x ? 4.0 : 0.0) + (uses_y ? 4.0 : 0.0)) * n);
    int vec = (((uintptr_t)x | (uintptr_t)y | (uintptr_t)g | (uintptr_t)gi) & 15) == 0;
    auto k = d->math_mode == MATH_LIBM ? k_unary_bwd<MATH_LIBM> : k_unary_bwd<MATH_POLY>;
    k<<<grid_for(d, vec ? (n + 3) / 4 : n), kThreads, 0, NCK_STREAM(d)>>>(kind, s, x, y, g, gi, n, vec, acc, uses_x,
                                                                         uses_y);
    NCK_LAUNCHED(d, 1);
}

// ---- binary --------------------------------------------------------------------------------------

__device__ __forceinline__ float bin_f(int kind, float a, float b) {
    switch (kind) {
    case NCK_BIN_ADD: return a + b;
    case NCK_BIN_SUB: return a - b;
    case NCK_BIN_MUL: return a * b;
    default: return a / b;
    }
}

__global__ void k_binary_flat(int kind, const float *__restrict__ a, const float *__restrict__ b,
                              float *__restrict__ o, int64_t n, int vec) {
    int64_t stride = (int64_t)gridDim.x * blockDim.x, t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (vec) {
        int64_t n4 = n >> 2;
        for (int64_t i = t; i < n4; i += stride) {
            float4 x = ((const float4 *)a)[i], y = ((const float4 *)b)[i], r;
            r.x = bin_f(kind, x.x, y.x), r.y = bin_f(kind, x.y, y.y), r.z = bin_f(kind, x.z, y.z);
            r.w = bin_f(kind, x.w, y.w);
            ((float4 *)o)[i] = r;
        }
        for (int64_t i = (n4 << 2) + t; i < n; i += stride) o[i] = bin_f(kind, a[i], b[i]);
    } else {
        for (int64_t i = t; i < n; i += stride) o[i] = bin_f(kind, a[i], b[i]);
    }
}

extern "C" void nck_binary_fwd_flat(nck_dev *d, int kind, const float *a, const float *b, float *o, int64_t n) {
    if (n <= 0) return;
    Scope sc(d, "binary");
    int vec = (((uintptr_t)a | (uintptr_t)b | (uintptr_t)o) & 15) == 0;
    k_binary_flat<<<grid_for(d, vec ? (n + 3) / 4 : n), kThreads, 0, NCK_STREAM(d)>>>(kind, a, b, o, n, vec);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_binary_bcast(int kind, nck_bcast bc, const float *__restrict__ a, const float *__restrict__ b,
                               float *__restrict__ o, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i, oa = 0, ob = 0, oo = 0;
        for (int k = bc.ndim - 1; k >= 0; k--) {
            int64_t q = r / bc.shape[k], idx = r - q * bc.shape[k];
            r = q;
            oa += idx * bc.sa[k], ob += idx * bc.sb[k], oo += idx * bc.so[k];
        }
        o[oo] = bin_f(kind, a[oa], b[ob]);
    }
}

static int64_t bc_numel(const nck_bcast *bc) {
    int64_t n = 1;
    for (int k = 0; k < bc->ndim; k++) n *= bc->shape[k];
    return n;
}

extern "C" void nck_binary_fwd(nck_dev *d, int kind, const nck_bcast *bc, const float *a, const float *b, float *o) {
    int64_t n = bc_numel(bc);
    if (n <= 0) return;
    Scope sc(d, "binary");
    k_binary_bcast<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(kind, *bc, a, b, o, n);
    NCK_LAUNCHED(d, 1);
}

// gradient contribution of output position (a, b at their offsets) to input `which`
__device__ __forceinline__ float bin_grad(int kind, int which, float g, float a, float b) {
    switch (kind) {
    case NCK_BIN_ADD: return g;
    case NCK_BIN_SUB: return which ? -g : g;
    case NCK_BIN_MUL: return which ? g * a : g * b;
    default: return which ? -(g * a / (b * b)) : g / b;
    }
}

// One thread per element of gx: the output positions that broadcast onto it are visited in
// row-major order and added one by one, the order newch's strided loop uses.
struct KeptRed {
    int nk, nr;
    int64_t kshape[NCK_MAXD], kso[NCK_MAXD], ksa[NCK_MAXD], ksb[NCK_MAXD], ksx[NCK_MAXD];
    int64_t rshape[NCK_MAXD], rso[NCK_MAXD], rsa[NCK_MAXD], rsb[NCK_MAXD];
    int64_t R;
};

__global__ void k_binary_bwd(int kind, int which, KeptRed kr, const float *__restrict__ g, const float *__restrict__ a,
                             const float *__restrict__ b, float *__restrict__ gx, int64_t m) {
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < m; j += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = j, go = 0, ao = 0, bo = 0, xo = 0;
        for (int k = kr.nk - 1; k >= 0; k--) {
            int64_t q = r / kr.kshape[k], idx = r - q * kr.kshape[k];
            r = q;
            go += idx * kr.kso[k], ao += idx * kr.ksa[k], bo += idx * kr.ksb[k], xo += idx * kr.ksx[k];
        }
        float acc = gx[xo];
        for (int64_t p = 0; p < kr.R; p++) {
            int64_t rr = p, g2 = go, a2 = ao, b2 = bo;
            for (int k = kr.nr - 1; k >= 0; k--) {
                int64_t q = rr / kr.rshape[k], idx = rr - q * kr.rshape[k];
                rr = q;
                g2 += idx * kr.rso[k], a2 += idx * kr.rsa[k], b2 += idx * kr.rsb[k];
            }
            float av = (kind == NCK_BIN_MUL || kind == NCK_BIN_DIV) ? a[a2] : 0.0f;
            float bv = (kind == NCK_BIN_MUL || kind == NCK_BIN_DIV) ? b[b2] : 0.0f;
            acc = acc + bin_grad(kind, which, g[g2], av, bv);
        }
        gx[xo] = acc;
    }
}

// no broadcast and every operand laid out like gx: gx[i] += d/dx f at element i
__global__ void k_binary_bwd_flat(int kind, int which, const float *__restrict__ g, const float *__restrict__ a,
                                  const float *__restrict__ b, float *__restrict__ gx, int64_t n, int vec, int acc) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x, t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const bool ab = kind == NCK_BIN_MUL || kind == NCK_BIN_DIV;
    int64_t done = 0;
    if (vec) {
        const int64_t n4 = n >> 2;
        for (int64_t i = t; i < n4; i += stride) {
            float4 gv = __ldg((const float4 *)g + i), o = acc ? ((float4 *)gx)[i] : make_float4(0, 0, 0, 0);
            float4 av = ab ? __ldg((const float4 *)a + i) : make_float4(0, 0, 0, 0);
            float4 bv = ab ? __ldg((const float4 *)b + i) : make_float4(0, 0, 0, 0);
            o.x = o.x + bin_grad(kind, which, gv.x, av.x, bv.x);
            o.y = o.y + bin_grad(kind, which, gv.y, av.y, bv.y);
            o.z = o.z + bin_grad(kind, which, gv.z, av.z, bv.z);
            o.w = o.w + bin_grad(kind, which, gv.w, av.w, bv.w);
            ((float4 *)gx)[i] = o;
        }
        done = n4 << 2;
    }
    for (int64_t i = done + t; i < n; i += stride)
        gx[i] = (acc ? gx[i] : 0.0f) + bin_grad(kind, which, g[i], ab ? a[i] : 0.0f, ab ? b[i] : 0.0f);
}

static bool contiguous_like(const KeptRed &kr, const int64_t *st) {
    int64_t expect = 1;
    for (int k = kr.nk - 1; k >= 0; k--) {
        if (st[k] != expect) return false;
        expect *= kr.kshape[k];
    }
    return true;
}

extern "C" void nck_binary_bwd(nck_dev *d, int kind, int which, const nck_bcast *bc, const float *g, const float *a,
                               const float *b, float *gx, const int64_t *gx_stride, int64_t gx_numel, int acc) {
    if (gx_numel <= 0) return;
    if (bc_numel(bc) <= 0) {
        if (!acc) cudaMemsetAsync(gx, 0, (size_t)gx_numel * sizeof(float), NCK_STREAM(d));
        return;
    }
    KeptRed kr;
    kr.nk = kr.nr = 0;
    kr.R = 1;
    for (int k = 0; k < bc->ndim; k++) {
        if (bc->shape[k] == 1) continue;
        if (gx_stride[k] == 0) {
            kr.rshape[kr.nr] = bc->shape[k], kr.rso[kr.nr] = bc->so[k], kr.rsa[kr.nr] = bc->sa[k];
            kr.rsb[kr.nr] = bc->sb[k];
            kr.R *= bc->shape[k];
            kr.nr++;
        } else {
            kr.kshape[kr.nk] = bc->shape[k], kr.kso[kr.nk] = bc->so[k], kr.ksa[kr.nk] = bc->sa[k];
            kr.ksb[kr.nk] = bc->sb[k], kr.ksx[kr.nk] = gx_stride[k];
            kr.nk++;
        }
    }
    Scope sc(d, "binary_bwd");
    const bool ab = kind == NCK_BIN_MUL || kind == NCK_BIN_DIV;
    if (kr.nr == 0 && contiguous_like(kr, kr.kso) && contiguous_like(kr, kr.ksx) &&
        (!ab || (contiguous_like(kr, kr.ksa) && contiguous_like(kr, kr.ksb)))) {
        int vec = (((uintptr_t)g | (uintptr_t)gx | (ab ? ((uintptr_t)a | (uintptr_t)b) : 0)) & 15) == 0;
        k_binary_bwd_flat<<<grid_for(d, vec ? (gx_numel + 3) / 4 : gx_numel), kThreads, 0, NCK_STREAM(d)>>>(
            kind, which, g, a, b, gx, gx_numel, vec, acc);
        NCK_LAUNCHED(d, 1);
        return;
    }
    if (!acc) cudaMemsetAsync(gx, 0, (size_t)gx_numel * sizeof(float), NCK_STREAM(d));
    k_binary_bwd<<<grid_for(d, gx_numel), kThreads, 0, NCK_STREAM(d)>>>(kind, which, kr, g, a, b, gx, gx_numel);
    NCK_LAUNCHED(d, 1);
}

// ---- compare / masked_fill ---------------------------------------------------------------------------

__global__ void k_compare(int op, nck_bcast bc, const void *__restrict__ a, int ai, const void *__restrict__ b, int bi,
                          int32_t *__restrict__ o, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i, oa = 0, ob = 0, oo = 0;
        for (int k = bc.ndim - 1; k >= 0; k--) {
            int64_t q = r / bc.shape[k], idx = r - q * bc.shape[k];
            r = q;
            oa += idx * bc.sa[k], ob += idx * bc.sb[k], oo += idx * bc.so[k];
        }
        double x = ai ? (double)((const int32_t *)a)[oa] : (double)((const float *)a)[oa];
        double y = bi ? (double)((const int32_t *)b)[ob] : (double)((const float *)b)[ob];
        int res = op == 0 ? x == y : op == 1 ? x != y : op == 2 ? x < y : op == 3 ? x <= y : op == 4 ? x > y : x >= y;
        o[oo] = res;
    }
}

extern "C" void nck_compare(nck_dev *d, int op, const nck_bcast *bc, const void *a, int a_i32, const void *b,
                            int b_i32, int32_t *o) {
    int64_t n = bc_numel(bc);
    if (n <= 0) return;
    Scope sc(d, "compare");
    k_compare<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(op, *bc, a, a_i32, b, b_i32, o, n);
    NCK_LAUNCHED(d, 1);
}

__global__ void k_masked_fill(nck_bcast bc, const float *__restrict__ x, const int32_t *__restrict__ m, float v,
                              float *__restrict__ o, int64_t n, int bwd) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i, ox = 0, om = 0, oo = 0;
        for (int k = bc.ndim - 1; k >= 0; k--) {
            int64_t q = r / bc.shape[k], idx = r - q * bc.shape[k];
            r = q;
            ox += idx * bc.sa[k], om += idx * bc.sb[k], oo += idx * bc.so[k];
        }
        int32_t mk = m[om];
        if (bwd) {
            if (!mk) o[oo] += x[ox];
        } else {
            o[oo] = mk ? v : x[ox];
        }
    }
}

// The common layout (an attention mask over the last dims, repeated over the leading ones, on a
// contiguous tensor): the mask index is i mod Mn. float4 items when both sizes and the pointers allow.
// bwd: gx (+)= mask ? 0 : g; forward: o = mask ? v : x.
template <int V, int BWD>
__global__ void __launch_bounds__(256) k_masked_fill_tail(const float *__restrict__ x, const int32_t *__restrict__ m,
                                                          float v, float *__restrict__ o, uint32_t n, uint32_t Mn,
                                                          FastDiv dmn, int acc) {
    const uint32_t items = n / V;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < items; i += gridDim.x * blockDim.x) {
        const uint32_t e = i * V, mi = e - dmn.div(e) * Mn;
        if constexpr (V == 4) {
            const float4 xv = __ldg(reinterpret_cast<const float4 *>(x) + i);
            const int4 mv = __ldg(reinterpret_cast<const int4 *>(m + mi));
            float4 r;
            if (BWD) {
                float4 base = acc ? reinterpret_cast<float4 *>(o)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                r.x = mv.x ? base.x : base.x + xv.x, r.y = mv.y ? base.y : base.y + xv.y;
                r.z = mv.z ? base.z : base.z + xv.z, r.w = mv.w ? base.w : base.w + xv.w;
            } else {
                r.x = mv.x ? v : xv.x, r.y = mv.y ? v : xv.y, r.z = mv.z ? v : xv.z, r.w = mv.w ? v : xv.w;
            }
            reinterpret_cast<float4 *>(o)[i] = r;
        } else {
            const int32_t mk = __ldg(m + mi);
            if (BWD) {
                const float base = acc ? o[e] : 0.0f;
                o[e] = mk ? base : base + __ldg(x + e);
            } else {
                o[e] = mk ? v : __ldg(x + e);
            }
        }
    }
}

extern "C" int nck_masked_fill_tail(nck_dev *d, int bwd, const float *x, const int32_t *m, float v, float *o,
                                    int64_t n, int64_t Mn, int acc) {
    if (n <= 0) return 1;
    if (Mn <= 0 || n % Mn || n >= ((int64_t)1 << 31)) return 0;
    Scope sc(d, bwd ? "masked_fill_bwd" : "masked_fill", 0.0, (bwd && acc ? 12.0 : 8.0) * n + 4.0 * Mn);
    const bool v4 = Mn % 4 == 0 && (((uintptr_t)x | (uintptr_t)m | (uintptr_t)o) & 15) == 0;
    const FastDiv dmn = make_fastdiv((uint32_t)Mn);
    const int g = grid_for(d, v4 ? n / 4 : n);
    if (bwd) {
        if (v4) k_masked_fill_tail<4, 1><<<g, 256, 0, NCK_STREAM(d)>>>(x, m, v, o, (uint32_t)n, (uint32_t)Mn, dmn, acc);
        else k_masked_fill_tail<1, 1><<<g, 256, 0, NCK_STREAM(d)>>>(x, m, v, o, (uint32_t)n, (uint32_t)Mn, dmn, acc);
    } else {
        if (v4) k_masked_fill_tail<4, 0><<<g, 256, 0, NCK_STREAM(d)>>>(x, m, v, o, (uint32_t)n, (uint32_t)Mn, dmn, acc);
        else k_masked_fill_tail<1, 0><<<g, 256, 0, NCK_STREAM(d)>>>(x, m, v, o, (uint32_t)n, (uint32_t)Mn, dmn, acc);
    }
    NCK_LAUNCHED(d, 1);
    return 1;
}

extern "C" void nck_masked_fill_fwd(nck_dev *d, const nck_bcast *bc, const float *x, const int32_t *m, float v,
                                    float *o) {
    int64_t n = bc_numel(bc);
    if (n <= 0) return;
    Scope sc(d, "masked_fill");
    k_masked_fill<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(*bc, x, m, v, o, n, 0);
    NCK_LAUNCHED(d, 1);
}

extern "C" void nck_masked_fill_bwd(nck_dev *d, const nck_bcast *bc, const float *g, const int32_t *m, float *gx) {
    int64_t n = bc_numel(bc);
    if (n <= 0) return;
    Scope sc(d, "masked_fill_bwd");
    k_masked_fill<<<grid_for(d, n), kThreads, 0, NCK_STREAM(d)>>>(*bc, g, m, 0.0f, gx, n, 1);
    NCK_LAUNCHED(d, 1);
}
