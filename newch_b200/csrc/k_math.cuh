// Transcendental functions of the activations, softmax and cross entropy, in two selectable forms.
//
// NCK_MATH_POLY (the default): newch's own single-precision approximations, the ones its AVX2+FMA
// kernel tier evaluates (newch engine/src/kernels/x86/kernels_avx2.c:75-177: exp8, sigmoid8, tanh8,
// erf8), restated one lane at a time. Each step is the same IEEE operation in the same order: fmaf
// where that code issues a fused multiply-add, a plain (correctly rounded) product, sum or quotient
// where it issues one. The file is compiled with --fmad=false, so nothing else is fused. The AVX2
// tier pads its tail elements through the same vector code, so every element of a newch tensor gets
// exactly this arithmetic, whatever its position; on a host whose newch selects that tier these
// functions reproduce its results bit for bit.
//
// NCK_MATH_LIBM (nc_config.force_reference, or NC_MATH=libm): CUDA's expf / tanhf / erff in the
// forms newch's reference tier writes with the C library (newch
// engine/src/kernels/ref/kernels_ref.c:43-55).
#pragma once

#include <math.h>
#include <stdint.h>

namespace nck {

enum { MATH_POLY = 0, MATH_LIBM = 1 };

// newch's exp: x = n ln2 + r with n = floor(x log2(e) + 1/2), ln2 split in a high and a low part,
// e^r by a degree-7 polynomial (Horner on the six coefficients, then r^2 p + r + 1), 2^n built in
// the exponent bits. Inputs are clamped to [lo, hi] first: n = 128 (only near ln(FLT_MAX)) is
// applied as 2^127 * 2; below lo the result is 0, past hi it overflows to +inf; NaN passes through.
__device__ __forceinline__ float poly_exp(float x0) {
    const float lo = -87.3365448f, hi = 88.8f;
    float x = fminf(fmaxf(x0, lo), hi);  // NaN maps to lo here and is restored at the end
    float fx = floorf(fmaf(x, 1.44269504088896341f, 0.5f));
    x = fmaf(-fx, 0.693359375f, x);
    x = fmaf(-fx, -2.12194440e-4f, x);
    float y = 1.9875691500e-4f;
    y = fmaf(y, x, 1.3981999507e-3f);
    y = fmaf(y, x, 8.3334519073e-3f);
    y = fmaf(y, x, 4.1665795894e-2f);
    y = fmaf(y, x, 1.6666665459e-1f);
    y = fmaf(y, x, 5.0000001201e-1f);
    y = fmaf(y, x * x, x + 1.0f);
    int n = (int)fx;  // fx is integral and within [-126, 128]
    const bool big = n > 127;
    if (big) n -= 1;
    float r = y * __int_as_float((n + 127) << 23);
    r = r * (big ? 2.0f : 1.0f);
    if (x0 < lo) r = 0.0f;
    return x0 != x0 ? x0 : r;
}

// poly_exp for arguments that are <= 0 or NaN (erf's exp(-x^2)): the same operations and results
// without the upper clamp and the 2^128 scaling, which such arguments never reach
__device__ __forceinline__ float poly_exp_nonpos(float x0) {
    const float lo = -87.3365448f;
    float x = fmaxf(x0, lo);  // NaN maps to lo here and is restored at the end
    float fx = floorf(fmaf(x, 1.44269504088896341f, 0.5f));
    x = fmaf(-fx, 0.693359375f, x);
    x = fmaf(-fx, -2.12194440e-4f, x);
    float y = 1.9875691500e-4f;
    y = fmaf(y, x, 1.3981999507e-3f);
    y = fmaf(y, x, 8.3334519073e-3f);
    y = fmaf(y, x, 4.1665795894e-2f);
    y = fmaf(y, x, 1.6666665459e-1f);
    y = fmaf(y, x, 5.0000001201e-1f);
    y = fmaf(y, x * x, x + 1.0f);
    const int n = (int)fx;  // fx is integral and within [-126, 0]
    float r = y * __int_as_float((n + 127) << 23);
    if (x0 < lo) r = 0.0f;
    return x0 != x0 ? x0 : r;
}

__device__ __forceinline__ float copysign_bits(float mag, float sgn) {
    return __int_as_float(__float_as_int(mag) | (__float_as_int(sgn) & (int)0x80000000));
}

// 1 / (1 + e^(0 - x))
__device__ __forceinline__ float poly_sigmoid(float x) { return __frcp_rn(1.0f + poly_exp(0.0f - x)); }

// |x| < 1/4: x + x^3 (t3 + z (t5 + z (t7 + z t9))), z = x^2 (odd Taylor terms, no cancellation);
// otherwise (1 - e) / (1 + e) with e = exp(-2 |x|), given the sign of x.
__device__ __forceinline__ float poly_tanh(float x) {
    const float ax = fabsf(x);
    const float e = poly_exp_nonpos(ax * -2.0f);
    const float big = copysign_bits((1.0f - e) / (1.0f + e), x);
    const float z = x * x;
    float p = fmaf(0.021869489f, z, -0.053968254f);
    p = fmaf(p, z, 0.133333333f);
    p = fmaf(p, z, -0.333333333f);
    p = fmaf(p * z, x, x);
    return ax < 0.25f ? p : big;
}

// erf by the rational form in t = 1 / (1 + p |x|) (Abramowitz-Stegun 7.1.26) times exp(-x^2), with
// the sign of x restored.
__device__ __forceinline__ float poly_erf(float x) {
    const float ax = fabsf(x);
    const float t = __frcp_rn(fmaf(ax, 0.3275911f, 1.0f));  // the correctly rounded 1 / d, as 1.0f / d
    float p = fmaf(1.061405429f, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    const float e = poly_exp_nonpos(0.0f - ax * ax);
    const float r = fmaf(-(p * t), e, 1.0f);
    return copysign_bits(r, x);
}

template <int M>
__device__ __forceinline__ float m_exp(float x) {
    if (M == MATH_POLY) return poly_exp(x);
    return expf(x);
}
template <int M>
__device__ __forceinline__ float m_sigmoid(float x) {
    if (M == MATH_POLY) return poly_sigmoid(x);
    return 1.0f / (1.0f + expf(-x));
}
template <int M>
__device__ __forceinline__ float m_tanh(float x) {
    if (M == MATH_POLY) return poly_tanh(x);
    return tanhf(x);
}
template <int M>
__device__ __forceinline__ float m_erf(float x) {
    if (M == MATH_POLY) return poly_erf(x);
    return erff(x);
}

}  // namespace nck
