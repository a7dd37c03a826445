// Piecewise activations that kernels other than the elementwise ones apply as an epilogue (BatchNorm
// followed by an activation, BatchNorm + activation + max pooling): forward values and the backward
// factor, in newch's formulas (engine/src/ops/ops_elementwise.c unary :229-266, backward :289-338:
// compares, products and sums only, so they are bit-identical to newch on any tier).
#pragma once

#include "nck.h"

namespace nck {

// kind < 0: identity
__device__ __forceinline__ float epi_fwd(int kind, float s, float x) {
    switch (kind) {
    case NCK_UN_RELU: return x > 0.0f ? x : 0.0f;
    case NCK_UN_RELU6: return fminf(fmaxf(x, 0.0f), 6.0f);
    case NCK_UN_LEAKY_RELU: return x > 0.0f ? x : s * x;
    case NCK_UN_HARDSIGMOID: return fminf(fmaxf(x * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
    case NCK_UN_HARDSWISH: return x * fminf(fmaxf(x + 3.0f, 0.0f), 6.0f) * (1.0f / 6.0f);
    default: return x;
    }
}

// the gradient contribution of upstream gradient g through the activation at input x (PyTorch's
// kink conventions, as newch)
__device__ __forceinline__ float epi_grad(int kind, float s, float x, float g) {
    switch (kind) {
    case NCK_UN_RELU: return x > 0.0f ? g : 0.0f;
    case NCK_UN_RELU6: return (x > 0.0f && x < 6.0f) ? g : 0.0f;
    case NCK_UN_LEAKY_RELU: return x > 0.0f ? g : s * g;
    case NCK_UN_HARDSIGMOID: return (x > -3.0f && x < 3.0f) ? g * (1.0f / 6.0f) : 0.0f;
    case NCK_UN_HARDSWISH: return x < -3.0f ? 0.0f : x <= 3.0f ? g * (x * (1.0f / 3.0f) + 0.5f) : g;
    default: return g;
    }
}

}  // namespace nck
