// The forward formulas of the unary ops (newch engine/src/ops/ops_elementwise.c:229-266), shared by
// the elementwise kernels and the kernels that apply an activation on the fly (the int8 path's
// quantization of a pending GELU output). Files including this are compiled without FMA contraction,
// so each product and sum rounds as newch's C does.
#pragma once

#include <math.h>

#include "k_math.cuh"
#include "nck.h"

namespace nck {

#define NC_SQRT1_2 0.70710678118654752f
#define NC_INV_SQRT_2PI 0.39894228040143268f
#define NC_SQRT_2_PI 0.79788456080286536f
#define NC_GELU_C 0.044715f

template <int M>
__device__ __forceinline__ float unary_f(int kind, float s, float x) {
    switch (kind) {
    case NCK_UN_NEG: return -1.0f * x;
    case NCK_UN_EXP: return m_exp<M>(x);
    case NCK_UN_LOG: return logf(x);
    case NCK_UN_SQRT: return sqrtf(x);
    case NCK_UN_RELU: return x > 0.0f ? x : 0.0f;
    case NCK_UN_SIGMOID: return m_sigmoid<M>(x);
    case NCK_UN_TANH: return m_tanh<M>(x);
    case NCK_UN_SCALE: return s * x;
    case NCK_UN_ADD_SCALAR: return x + s;
    case NCK_UN_POW: return powf(x, s);
    case NCK_UN_LEAKY_RELU: return x > 0.0f ? x : s * x;
    case NCK_UN_RELU6: return fminf(fmaxf(x, 0.0f), 6.0f);
    case NCK_UN_HARDSIGMOID: return fminf(fmaxf(x * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
    case NCK_UN_HARDSWISH: return x * fminf(fmaxf(x + 3.0f, 0.0f), 6.0f) * (1.0f / 6.0f);
    case NCK_UN_SILU: return m_sigmoid<M>(x) * x;
    case NCK_UN_GELU: return 0.5f * x * (1.0f + m_erf<M>(NC_SQRT1_2 * x));
    case NCK_UN_GELU_TANH: {
        float t = m_tanh<M>(NC_SQRT_2_PI * (x + NC_GELU_C * x * x * x));
        return 0.5f * x * (1.0f + t);
    }
    }
    return x;
}

}  // namespace nck
