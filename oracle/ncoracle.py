"""CPU restatement (numpy) of the newch engine's training-step arithmetic: the parity oracle.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
use anything under oracle/; the B200 product path never does. Each function states the newch source
(file:line, paths inside the newch project) whose algorithm it restates. Pinned by tests/test_oracle.py
against golden vectors produced by the reference engine itself (tests/golden/make_golden.py) and
against the known answers of newch's own C tests (engine/tests/test_main.c:933-1076).

Floating-point results follow the reference's formulas and accumulation types (float32 arithmetic,
float64 where newch accumulates in double); summation order inside long reductions differs from
newch's SIMD order, so comparisons use tolerances except where the arithmetic is exact (the RNG,
int8 accumulators, argmax indices, quantized values).
"""

from __future__ import annotations

import numpy as np

f32 = np.float32

# ----------------------------------------------------------------------------------------------
# RNG: xoshiro256** seeded with splitmix64 (engine/src/core/ctx.c:270-276, :414-435)
# ----------------------------------------------------------------------------------------------

M64 = (1 << 64) - 1


def _splitmix64(x: int):
    x = (x + 0x9E3779B97F4A7C15) & M64
    z = x
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return x, z ^ (z >> 31)


def _rotl(x: int, k: int) -> int:
    return ((x << k) | (x >> (64 - k))) & M64


class Rng:
    """The context's stream: nc_manual_seed (ctx.c:270-276) and rng_next (ctx.c:416-428)."""

    def __init__(self, seed: int = 0):
        s = seed if seed else 0x6E63
        self.s = []
        for _ in range(4):
            s, z = _splitmix64(s)
            self.s.append(z)

    def next(self) -> int:
        s = self.s
        r = (_rotl((s[1] * 5) & M64, 7) * 9) & M64
        t = (s[1] << 17) & M64
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = _rotl(s[3], 45)
        return r

    def uniform01(self) -> np.float32:
        """(float)(r >> 40) * 2^-24 (ctx.c:430), exact in float32."""
        return f32(self.next() >> 40) * f32(1.0 / 16777216.0)

    def normal(self) -> np.float32:
        """Box-Muller on two uniforms (ctx.c:432-435)."""
        u1, u2 = self.uniform01(), self.uniform01()
        if u1 < f32(1e-7):
            u1 = f32(1e-7)
        return f32(np.sqrt(f32(-2.0) * np.log(u1, dtype=f32), dtype=f32) * np.cos(f32(6.2831853) * u2, dtype=f32))

    def uniform_array(self, n: int) -> np.ndarray:
        return np.array([self.uniform01() for _ in range(n)], dtype=f32)


def rand_uniform(rng: Rng, lo: float, hi: float, n: int) -> np.ndarray:
    """nc_rand_uniform (engine/src/core/tensor.c:179-185): lo + (hi - lo) * u, element order."""
    lo, hi = f32(lo), f32(hi)
    return np.array([lo + (hi - lo) * rng.uniform01() for _ in range(n)], dtype=f32)


# ----------------------------------------------------------------------------------------------
# elementwise (engine/src/ops/ops_elementwise.c:229-338)
# ----------------------------------------------------------------------------------------------

SQRT1_2, INV_SQRT_2PI, SQRT_2_PI, GELU_C = f32(0.70710678118654752), f32(0.39894228040143268), f32(
    0.79788456080286536), f32(0.044715)


def _erf(x):
    import math
    return np.vectorize(lambda v: f32(math.erf(float(v))), otypes=[f32])(x)


# newch's AVX2-tier transcendental functions (engine/src/kernels/x86/kernels_avx2.c:75-177), the ones
# a newch build on an AVX2+FMA host evaluates for exp / sigmoid / tanh / erf. Restated elementwise in
# float32 with each fused multiply-add rounded once (fma32), so results are bit-identical to that
# tier's.

def fma32(a, b, c) -> np.ndarray:
    """float32 a * b + c with one rounding. a * b is exact in float64 (24-bit factors); the float64 sum
    is made round-to-odd from its exact error (TwoSum), so the final conversion to float32 rounds the
    exact value once."""
    a, b, c = (np.asarray(v, dtype=f32).astype(np.float64) for v in (a, b, c))
    p = a * b
    t = p + c
    bb = t - p
    err = (p - (t - bb)) + (c - bb)  # TwoSum: t + err == p + c exactly
    with np.errstate(invalid="ignore", over="ignore"):
        fix = np.isfinite(t) & (err != 0)
        # round to odd: the truncation of the exact value, with its last bit forced to 1
        toward_zero = np.where(np.sign(err) != np.sign(t), np.nextafter(t, 0.0), t)
        bits = toward_zero.view(np.int64)
        odd = (bits | 1).view(np.float64)
        t = np.where(fix, odd, t)
    return t.astype(f32)


_EXP_LO, _EXP_HI = f32(-87.3365448), f32(88.8)
_EXP_P = [f32(v) for v in (1.9875691500e-4, 1.3981999507e-3, 8.3334519073e-3, 4.1665795894e-2, 1.6666665459e-1,
                           5.0000001201e-1)]


def poly_exp(x0: np.ndarray) -> np.ndarray:
    """exp8 (kernels_avx2.c:96-118): range reduction by n = floor(x log2e + 1/2) with ln2 in two parts,
    the degree-7 polynomial, 2^n from the exponent bits (n = 128 as 2^127 * 2), 0 below the input
    window, NaN passed through."""
    x0 = np.asarray(x0, dtype=f32)
    with np.errstate(invalid="ignore", over="ignore"):
        x = np.minimum(np.maximum(np.nan_to_num(x0, nan=_EXP_LO, posinf=_EXP_HI, neginf=_EXP_LO), _EXP_LO), _EXP_HI)
        fx = np.floor(fma32(x, f32(1.44269504088896341), f32(0.5))).astype(f32)
        x = fma32(-fx, f32(0.693359375), x)
        x = fma32(-fx, f32(-2.12194440e-4), x)
        y = np.full_like(x, _EXP_P[0])
        for c in _EXP_P[1:]:
            y = fma32(y, x, c)
        y = fma32(y, (x * x).astype(f32), (x + f32(1)).astype(f32))
        n = fx.astype(np.int32)
        big = n > 127
        n = np.where(big, n - 1, n)
        scale = ((n + 127).astype(np.int32) << 23).view(f32)
        r = (y * scale).astype(f32)
        r = (r * np.where(big, f32(2), f32(1))).astype(f32)
        r = np.where(x0 < _EXP_LO, f32(0), r)
        return np.where(np.isnan(x0), x0, r).astype(f32)


def _copysign_bits(mag, sgn):
    return ((mag.view(np.uint32) | (np.asarray(sgn, f32).view(np.uint32) & np.uint32(0x80000000)))).view(f32)


def poly_sigmoid(x):
    """sigmoid8 (kernels_avx2.c:120-123): 1 / (1 + exp(0 - x))."""
    x = np.asarray(x, dtype=f32)
    with np.errstate(over="ignore", divide="ignore"):
        return (f32(1) / (f32(1) + poly_exp((f32(0) - x).astype(f32)))).astype(f32)


def poly_tanh(x):
    """tanh8 (kernels_avx2.c:125-139): odd polynomial below |x| = 1/4, else (1 - e) / (1 + e) with
    e = exp(-2|x|) and the sign of x."""
    x = np.asarray(x, dtype=f32)
    ax = np.abs(x)
    with np.errstate(invalid="ignore", over="ignore"):
        e = poly_exp((ax * f32(-2)).astype(f32))
        big = _copysign_bits(((f32(1) - e) / (f32(1) + e)).astype(f32), x)
        z = (x * x).astype(f32)
        p = fma32(f32(0.021869489), z, f32(-0.053968254))
        p = fma32(p, z, f32(0.133333333))
        p = fma32(p, z, f32(-0.333333333))
        p = fma32((p * z).astype(f32), x, x)
    return np.where(ax < f32(0.25), p, big).astype(f32)


def poly_erf(x):
    """erf8 (kernels_avx2.c:148-159): 1 - poly(t) t exp(-x^2), t = 1 / (1 + p|x|), sign restored."""
    x = np.asarray(x, dtype=f32)
    ax = np.abs(x)
    with np.errstate(invalid="ignore", over="ignore"):
        t = (f32(1) / fma32(ax, f32(0.3275911), f32(1))).astype(f32)
        p = fma32(f32(1.061405429), t, f32(-1.453152027))
        p = fma32(p, t, f32(1.421413741))
        p = fma32(p, t, f32(-0.284496736))
        p = fma32(p, t, f32(0.254829592))
        e = poly_exp((f32(0) - (ax * ax).astype(f32)).astype(f32))
        r = fma32(-(p * t).astype(f32), e, f32(1))
    return _copysign_bits(r, x)


def unary_avx2(kind: str, x: np.ndarray):
    """Forward and the derivative factors of the exp / tanh / erf activations as newch evaluates them on
    its AVX2 tier (ops_elementwise.c:229-266 with kernels_avx2.c's exp_f32 / sigmoid_f32 / tanh_f32 /
    erf_f32). Returns (y, dfun) where dfun(g) gives the backward contribution (ops_elementwise.c:289-338)."""
    y, d = _unary_avx2(kind, np.asarray(x, dtype=f32))

    def dfun(g):
        with np.errstate(all="ignore"):
            return d(np.asarray(g, dtype=f32))
    return y, dfun


def _unary_avx2(kind: str, x: np.ndarray):
    with np.errstate(all="ignore"):
        if kind == "exp":
            y = poly_exp(x)
            return y, lambda g: (g * y).astype(f32)
        if kind == "sigmoid":
            y = poly_sigmoid(x)
            return y, lambda g: (g * y * (f32(1) - y)).astype(f32)
        if kind == "tanh":
            y = poly_tanh(x)
            return y, lambda g: (g * (f32(1) - y * y)).astype(f32)
        if kind == "silu":
            t = poly_sigmoid(x)
            return (t * x).astype(f32), lambda g: (g * t * (f32(1) + x * (f32(1) - t))).astype(f32)
        if kind == "gelu":
            t = poly_erf((SQRT1_2 * x).astype(f32))
            t2 = poly_exp((f32(-0.5) * x * x).astype(f32))
            y = (f32(0.5) * x * (f32(1) + t)).astype(f32)
            return y, lambda g: (g * (f32(0.5) * (f32(1) + t) + x * INV_SQRT_2PI * t2)).astype(f32)
        if kind == "gelu_tanh":
            t = poly_tanh((SQRT_2_PI * (x + GELU_C * x * x * x)).astype(f32))
            y = (f32(0.5) * x * (f32(1) + t)).astype(f32)

            def d(g):
                dt = (f32(1) - t * t) * SQRT_2_PI * (f32(1) + f32(3) * GELU_C * x * x)
                return (g * (f32(0.5) * (f32(1) + t) + f32(0.5) * x * dt)).astype(f32)
            return y, d
    raise ValueError(kind)


def unary(kind: str, x: np.ndarray, s: float = 0.0) -> np.ndarray:
    """Forward of the unary ops (ops_elementwise.c:229-266)."""
    x = x.astype(f32)
    s = f32(s)
    if kind == "relu":
        return np.where(x > 0, x, f32(0)).astype(f32)
    if kind == "sigmoid":
        return (f32(1) / (f32(1) + np.exp(-x))).astype(f32)
    if kind == "tanh":
        return np.tanh(x).astype(f32)
    if kind == "exp":
        return np.exp(x).astype(f32)
    if kind == "log":
        return np.log(x).astype(f32)
    if kind == "sqrt":
        return np.sqrt(x).astype(f32)
    if kind == "neg":
        return (f32(-1) * x).astype(f32)
    if kind == "scale":
        return (s * x).astype(f32)
    if kind == "add_scalar":
        return (x + s).astype(f32)
    if kind == "pow":
        return np.power(x, s).astype(f32)
    if kind == "leaky_relu":
        return np.where(x > 0, x, s * x).astype(f32)
    if kind == "relu6":
        return np.minimum(np.maximum(x, f32(0)), f32(6)).astype(f32)
    if kind == "hardsigmoid":
        return np.minimum(np.maximum(x * f32(1.0 / 6.0) + f32(0.5), f32(0)), f32(1)).astype(f32)
    if kind == "hardswish":
        return (x * np.minimum(np.maximum(x + f32(3), f32(0)), f32(6)) * f32(1.0 / 6.0)).astype(f32)
    if kind == "silu":
        return ((f32(1) / (f32(1) + np.exp(-x))) * x).astype(f32)
    if kind == "gelu":
        return (f32(0.5) * x * (f32(1) + _erf(SQRT1_2 * x))).astype(f32)
    if kind == "gelu_tanh":
        t = np.tanh(SQRT_2_PI * (x + GELU_C * x * x * x)).astype(f32)
        return (f32(0.5) * x * (f32(1) + t)).astype(f32)
    raise ValueError(kind)


def unary_grad(kind: str, x: np.ndarray, g: np.ndarray, s: float = 0.0) -> np.ndarray:
    """d/dx times g, PyTorch kink conventions (ops_elementwise.c:289-338)."""
    x, g, s = x.astype(f32), g.astype(f32), f32(s)
    y = unary(kind, x, s)
    if kind == "relu":
        return np.where(x > 0, g, f32(0))
    if kind == "sigmoid":
        return g * y * (f32(1) - y)
    if kind == "tanh":
        return g * (f32(1) - y * y)
    if kind == "exp":
        return g * y
    if kind == "log":
        return g / x
    if kind == "sqrt":
        return g * f32(0.5) / y
    if kind == "neg":
        return -g
    if kind == "scale":
        return s * g
    if kind == "add_scalar":
        return g
    if kind == "pow":
        return g * s * np.power(x, s - f32(1))
    if kind == "leaky_relu":
        return np.where(x > 0, g, s * g)
    if kind == "relu6":
        return np.where((x > 0) & (x < 6), g, f32(0))
    if kind == "hardsigmoid":
        return np.where((x > -3) & (x < 3), g * f32(1.0 / 6.0), f32(0))
    if kind == "hardswish":
        return np.where(x < -3, f32(0), np.where(x <= 3, g * (x * f32(1.0 / 3.0) + f32(0.5)), g))
    if kind == "silu":
        t = f32(1) / (f32(1) + np.exp(-x))
        return g * t * (f32(1) + x * (f32(1) - t))
    if kind == "gelu":
        t = _erf(SQRT1_2 * x)
        t2 = np.exp(f32(-0.5) * x * x)
        return g * (f32(0.5) * (f32(1) + t) + x * INV_SQRT_2PI * t2)
    if kind == "gelu_tanh":
        t = np.tanh(SQRT_2_PI * (x + GELU_C * x * x * x))
        dt = (f32(1) - t * t) * SQRT_2_PI * (f32(1) + f32(3) * GELU_C * x * x)
        return g * (f32(0.5) * (f32(1) + t) + f32(0.5) * x * dt)
    raise ValueError(kind)


def binary_grads(op: str, a: np.ndarray, b: np.ndarray, g: np.ndarray):
    """Gradients of a op b summed back to each operand's broadcast shape (ops_elementwise.c:129-186)."""
    if op == "add":
        ga, gb = g, g
    elif op == "sub":
        ga, gb = g, -g
    elif op == "mul":
        ga, gb = g * b, g * a
    else:
        ga, gb = g / b, -(g * a / (b * b))
    return _unbroadcast(ga, a.shape), _unbroadcast(gb, b.shape)


def _unbroadcast(g: np.ndarray, shape) -> np.ndarray:
    g = np.asarray(g, dtype=np.float64)
    while g.ndim > len(shape):
        g = g.sum(axis=0)
    for i, n in enumerate(shape):
        if n == 1 and g.shape[i] != 1:
            g = g.sum(axis=i, keepdims=True)
    return g.astype(f32)


# ----------------------------------------------------------------------------------------------
# GEMM-based ops (engine/src/ops/ops_linalg.c)
# ----------------------------------------------------------------------------------------------

def linear(x, w, b=None):
    """y = x W^T + b (ops_linalg.c:299-309), float64 products rounded to float32."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if b is not None:
        y = y + np.asarray(b, np.float64)
    return y.astype(f32)


def linear_grads(x, w, g):
    """dX = g W, dW = g^T X, dB = sum g (ops_linalg.c:311-331)."""
    x64, w64, g64 = (np.asarray(t, np.float64) for t in (x, w, g))
    g2 = g64.reshape(-1, g64.shape[-1])
    x2 = x64.reshape(-1, x64.shape[-1])
    return (g64 @ w64).astype(f32), (g2.T @ x2).astype(f32), g2.sum(axis=0).astype(f32)


# ----------------------------------------------------------------------------------------------
# convolution and pooling (engine/src/ops/ops_conv.c)
# ----------------------------------------------------------------------------------------------

def _out(n, k, s, p, d):
    return (n + 2 * p - d * (k - 1) - 1) // s + 1


def im2col(x, kh, kw, sh, sw, ph, pw, dh=1, dw=1):
    """col [N, C*KH*KW, OH*OW], rows ordered (c, ki, kj) (ops_conv.c:66-86)."""
    N, C, H, W = x.shape
    OH, OW = _out(H, kh, sh, ph, dh), _out(W, kw, sw, pw, dw)
    xp = np.zeros((N, C, H + 2 * ph, W + 2 * pw), dtype=x.dtype)
    xp[:, :, ph:ph + H, pw:pw + W] = x
    cols = np.empty((N, C, kh, kw, OH, OW), dtype=x.dtype)
    for i in range(kh):
        for j in range(kw):
            cols[:, :, i, j] = xp[:, :, i * dh:i * dh + sh * (OH - 1) + 1:sh, j * dw:j * dw + sw * (OW - 1) + 1:sw]
    return cols.reshape(N, C * kh * kw, OH * OW), OH, OW


def conv2d(x, w, b=None, stride=(1, 1), pad=(0, 0), dil=(1, 1), groups=1):
    """y[n, oc] = b[oc] + W_g col_g (ops_conv.c:290-316; depthwise :192-220 is the groups == C case)."""
    x64, w64 = np.asarray(x, np.float64), np.asarray(w, np.float64)
    N, C, H, W = x.shape
    OC, Cg, KH, KW = w.shape
    col, OH, OW = im2col(x64, KH, KW, stride[0], stride[1], pad[0], pad[1], dil[0], dil[1])
    OCg = OC // groups
    y = np.empty((N, OC, OH * OW))
    for g in range(groups):
        wg = w64[g * OCg:(g + 1) * OCg].reshape(OCg, -1)
        cg = col[:, g * Cg * KH * KW:(g + 1) * Cg * KH * KW]
        y[:, g * OCg:(g + 1) * OCg] = np.einsum("ok,nkl->nol", wg, cg)
    if b is not None:
        y += np.asarray(b, np.float64)[None, :, None]
    return y.reshape(N, OC, OH, OW).astype(f32)


def conv2d_grads(x, w, g, stride=(1, 1), pad=(0, 0), dil=(1, 1), groups=1):
    """dW = dY col^T summed over samples, dX = col2im(W^T dY), dB = sum dY (ops_conv.c:318-357)."""
    x64, w64, g64 = (np.asarray(t, np.float64) for t in (x, w, g))
    N, C, H, W = x.shape
    OC, Cg, KH, KW = w.shape
    col, OH, OW = im2col(x64, KH, KW, stride[0], stride[1], pad[0], pad[1], dil[0], dil[1])
    OCg = OC // groups
    gy = g64.reshape(N, OC, OH * OW)
    dw = np.empty_like(w64)
    dcol = np.empty_like(col)
    for gi in range(groups):
        wg = w64[gi * OCg:(gi + 1) * OCg].reshape(OCg, -1)
        rows = slice(gi * Cg * KH * KW, (gi + 1) * Cg * KH * KW)
        gg = gy[:, gi * OCg:(gi + 1) * OCg]
        dw[gi * OCg:(gi + 1) * OCg] = np.einsum("nol,nkl->ok", gg, col[:, rows]).reshape(OCg, Cg, KH, KW)
        dcol[:, rows] = np.einsum("ok,nol->nkl", wg, gg)
    # col2im (ops_conv.c:89-109)
    dx = np.zeros((N, C, H + 2 * pad[0], W + 2 * pad[1]))
    dc = dcol.reshape(N, C, KH, KW, OH, OW)
    for i in range(KH):
        for j in range(KW):
            dx[:, :, i * dil[0]:i * dil[0] + stride[0] * (OH - 1) + 1:stride[0],
               j * dil[1]:j * dil[1] + stride[1] * (OW - 1) + 1:stride[1]] += dc[:, :, i, j]
    dx = dx[:, :, pad[0]:pad[0] + H, pad[1]:pad[1] + W]
    return dx.astype(f32), dw.astype(f32), gy.sum(axis=(0, 2)).astype(f32)


def pool2d(x, k, s, p, is_max=True):
    """Window max with the first maximum winning and its in-plane index, or the count_include_pad
    average (ops_conv.c:434-468)."""
    N, C, H, W = x.shape
    OH, OW = _out(H, k[0], s[0], p[0], 1), _out(W, k[1], s[1], p[1], 1)
    y = np.empty((N, C, OH, OW), dtype=f32)
    arg = np.full((N, C, OH, OW), -1, dtype=np.int32)
    for oy in range(OH):
        for ox in range(OW):
            best = np.full((N, C), -np.inf, dtype=f32)
            bi = np.full((N, C), -1, dtype=np.int32)
            acc = np.zeros((N, C), dtype=f32)
            for ki in range(k[0]):
                iy = oy * s[0] - p[0] + ki
                if iy < 0 or iy >= H:
                    continue
                for kj in range(k[1]):
                    ix = ox * s[1] - p[1] + kj
                    if ix < 0 or ix >= W:
                        continue
                    v = x[:, :, iy, ix].astype(f32)
                    acc = (acc + v).astype(f32)
                    take = (v > best) | (bi < 0)
                    best = np.where(take, v, best)
                    bi = np.where(take, iy * W + ix, bi).astype(np.int32)
            if is_max:
                y[:, :, oy, ox], arg[:, :, oy, ox] = best, bi
            else:
                y[:, :, oy, ox] = acc * f32(1.0 / (k[0] * k[1]))
    return y, arg


def maxpool_grad(x_shape, arg, g):
    """Each output's gradient goes to its argmax (ops_conv.c:482-496)."""
    N, C, H, W = x_shape
    gx = np.zeros((N, C, H * W), dtype=np.float64)
    a = arg.reshape(N, C, -1)
    gg = np.asarray(g, np.float64).reshape(N, C, -1)
    for n in range(N):
        for c in range(C):
            np.add.at(gx[n, c], a[n, c], gg[n, c])
    return gx.reshape(x_shape).astype(f32)


# ----------------------------------------------------------------------------------------------
# normalisation, softmax and losses (engine/src/ops/ops_nn.c)
# ----------------------------------------------------------------------------------------------

def batch_norm_train(x, w, b, rm, rv, mom, eps):
    """Batch statistics in double, unbiased running variance (ops_nn.c:262-310)."""
    N, C = x.shape[:2]
    xs = np.asarray(x, np.float64).reshape(N, C, -1)
    M = xs.shape[0] * xs.shape[2]
    mu = xs.sum(axis=(0, 2)) / M
    ss = ((xs - mu[None, :, None]) ** 2).sum(axis=(0, 2))
    mean = mu.astype(f32)
    invstd = (1.0 / np.sqrt(ss / M + float(eps))).astype(f32)
    a = (w.astype(f32) * invstd).astype(f32)
    d = (b.astype(f32) - mean * a).astype(f32)
    y = (x.astype(f32).reshape(N, C, -1) * a[None, :, None] + d[None, :, None]).astype(f32).reshape(x.shape)
    mom = f32(mom)
    rm2 = ((f32(1) - mom) * rm.astype(f32) + mom * mu.astype(f32)).astype(f32)
    rv2 = ((f32(1) - mom) * rv.astype(f32) + mom * (ss / (M - 1)).astype(f32)).astype(f32)
    return y, mean, invstd, rm2, rv2


def batch_norm_grads(x, w, g, mean, invstd, training=True):
    """sum g and sum g * xhat in double, then dx (ops_nn.c:312-349)."""
    N, C = x.shape[:2]
    xs = x.astype(f32).reshape(N, C, -1)
    gs = g.astype(f32).reshape(N, C, -1)
    M = xs.shape[0] * xs.shape[2]
    xhat = ((xs - mean[None, :, None]) * invstd[None, :, None]).astype(f32)
    sg = gs.astype(np.float64).sum(axis=(0, 2))
    sgx = (gs * xhat).astype(np.float64).sum(axis=(0, 2))
    k = (w.astype(f32) * invstd).astype(f32)
    if training:
        mg, mgx = (sg / M).astype(f32), (sgx / M).astype(f32)
        dx = k[None, :, None] * (gs - mg[None, :, None] - xhat * mgx[None, :, None])
    else:
        dx = k[None, :, None] * gs
    return dx.astype(f32).reshape(x.shape), sgx.astype(f32), sg.astype(f32)


def layer_norm(x, w, b, eps):
    """Per row over the last dims, double statistics, biased variance (ops_nn.c:463-490)."""
    D = w.size if w is not None else x.shape[-1]
    xr = np.asarray(x, np.float64).reshape(-1, D)
    mean = xr.mean(axis=1)
    var = ((xr - mean[:, None]) ** 2).sum(axis=1) / D
    rstd = (1.0 / np.sqrt(var + float(eps))).astype(f32)
    v = ((x.astype(f32).reshape(-1, D) - mean.astype(f32)[:, None]) * rstd[:, None]).astype(f32)
    y = v * w.astype(f32) if w is not None else v
    if b is not None:
        y = y + b.astype(f32)
    return y.astype(f32).reshape(x.shape), mean.astype(f32), rstd


def layer_norm_grads(x, w, g, mean, rstd):
    """ops_nn.c:492-522."""
    D = x.shape[-1]
    xr, gr = x.astype(f32).reshape(-1, D), g.astype(f32).reshape(-1, D)
    xhat = ((xr - mean[:, None]) * rstd[:, None]).astype(f32)
    gi = gr * w.astype(f32) if w is not None else gr
    mg = (gi.astype(np.float64).sum(axis=1) / D).astype(f32)
    mgx = ((gi * xhat).astype(np.float64).sum(axis=1) / D).astype(f32)
    dx = rstd[:, None] * (gi - mg[:, None] - xhat * mgx[:, None])
    gw = (gr.astype(np.float64) * xhat).sum(axis=0).astype(f32)
    gb = gr.astype(np.float64).sum(axis=0).astype(f32)
    return dx.astype(f32).reshape(x.shape), gw, gb


def log_softmax(x):
    """x - max - log(sum exp(x - max)) per row (ops_nn.c:22-35)."""
    x = x.astype(f32)
    m = x.max(axis=-1, keepdims=True)
    s = np.exp(x - m).astype(np.float64).sum(axis=-1, keepdims=True)
    return (x - m - np.log(s).astype(f32)).astype(f32)


def softmax(x):
    x = x.astype(f32)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m).astype(f32)
    return (e * (f32(1) / e.astype(np.float64).sum(axis=-1, keepdims=True).astype(f32))).astype(f32)


def softmax_grad(y, g, log_form):
    """ops_nn.c:48-71."""
    if log_form:
        return (g - np.exp(y) * g.sum(axis=-1, keepdims=True)).astype(f32)
    return (y * (g - (g * y).sum(axis=-1, keepdims=True))).astype(f32)


def cross_entropy(x, labels):
    """Mean of -log softmax[label] with a double sum (ops_nn.c:107-134); returns (loss, prob)."""
    lp = log_softmax(x)
    loss = -lp[np.arange(len(labels)), labels].astype(np.float64).sum()
    return f32(loss / len(labels)) if len(labels) else f32(np.nan), np.exp(lp).astype(f32)


def cross_entropy_grad(prob, labels, gloss=1.0):
    """(prob - onehot) * g / N (ops_nn.c:136-149)."""
    N = len(labels)
    s = f32(gloss) / f32(max(N, 1))
    gi = (s * prob).astype(f32)
    gi[np.arange(N), labels] -= s
    return gi


def nll_loss(logp, labels, reduce_sum=False):
    """ops_nn.c:387-406."""
    loss = -logp[np.arange(len(labels)), labels].astype(np.float64).sum()
    return f32(loss) if reduce_sum else f32(loss / len(labels))


def dropout(x, p, rng: Rng):
    """Inverted dropout: draw i keeps element i when u >= p (ops_nn.c:182-196)."""
    p = f32(p)
    keep = f32(1) / (f32(1) - p) if p < 1 else f32(0)
    u = rng.uniform_array(x.size)
    mask = np.where(u >= p, keep, f32(0)).astype(f32)
    return (x.astype(f32).reshape(-1) * mask).reshape(x.shape), mask.reshape(x.shape)


# ----------------------------------------------------------------------------------------------
# int8 quantization (engine/src/ops/ops_quant.c)
# ----------------------------------------------------------------------------------------------

def quantize_rows(w):
    """amax / 127 scale, reciprocal, round half to even, clamp +-127 (ops_quant.c:11-21). Exact."""
    w = w.astype(f32)
    amax = np.abs(w).max(axis=1)
    s = np.where(amax > 0, amax / f32(127), f32(1)).astype(f32)
    inv = (f32(1) / s).astype(f32)
    q = np.clip(np.rint((w * inv[:, None]).astype(f32)), -127, 127).astype(np.int8)
    return q, s


def gemm_s8_nt(a, b):
    """C[i, j] = sum_k a[i, k] b[j, k] in exact integer arithmetic (kernels_ref.c:117-128). Evaluated as a
    float64 product: every partial sum is an integer below 127 * 127 * K < 2^53, so the result is
    exact in any summation order."""
    return np.rint(a.astype(np.float64) @ b.astype(np.float64).T).astype(np.int64).astype(np.int32)


def linear_int8(x, wq, ws, bias=None):
    """Per-row activation quantization, exact int32 accumulators, y = (float)acc * xs * ws + b
    (ops_quant.c:71-80). Returns (y, acc, xq, xs)."""
    x2 = x.reshape(-1, x.shape[-1])
    xq, xs = quantize_rows(x2)
    acc = gemm_s8_nt(xq, wq)
    y = (acc.astype(f32) * xs[:, None]).astype(f32) * ws[None, :].astype(f32)
    if bias is not None:
        y = y + bias.astype(f32)
    return y.astype(f32).reshape(*x.shape[:-1], wq.shape[0]), acc, xq, xs


# ----------------------------------------------------------------------------------------------
# optimizers (engine/src/optim/optim.c:161-213)
# ----------------------------------------------------------------------------------------------

def adam_step(w, g, m, v, t, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, decoupled=False, gs=1.0):
    """One Adam / AdamW update in newch's order (optim.c:198-211), float32 throughout."""
    lr, b1, b2, eps, wd, gs = (f32(a) for a in (lr, beta1, beta2, eps, weight_decay, gs))
    bc1 = f32(1) - np.power(b1, f32(t), dtype=f32)
    bc2 = f32(1) - np.power(b2, f32(t), dtype=f32)
    w = w.astype(f32)
    if decoupled:
        w = (w * (f32(1) - lr * wd)).astype(f32)
    l2 = f32(0) if decoupled else wd
    gj = (gs * g.astype(f32) + l2 * w).astype(f32)
    m = (b1 * m + (f32(1) - b1) * gj).astype(f32)
    v = (b2 * v + (f32(1) - b2) * gj * gj).astype(f32)
    w = (w - lr * (m / bc1) / (np.sqrt(v / bc2) + eps)).astype(f32)
    return w, m, v


def sgd_step(w, g, buf, lr, momentum=0.0, weight_decay=0.0, gs=1.0):
    """optim.c:178-186."""
    gj = (f32(gs) * g + f32(weight_decay) * w).astype(f32)
    if buf is not None:
        gj = buf = (f32(momentum) * buf + gj).astype(f32)
    return (w - f32(lr) * gj).astype(f32), buf


def rmsprop_step(w, g, v, buf, lr, alpha, eps, momentum=0.0, weight_decay=0.0, eps_inside=False, gs=1.0):
    """optim.c:187-197: v = a v + (1 - a) g^2, step = g / den, optional momentum buffer."""
    lr, a, eps, mom, wd, gs = (f32(t) for t in (lr, alpha, eps, momentum, weight_decay, gs))
    gj = (gs * g.astype(f32) + wd * w).astype(f32)
    v = (a * v + (f32(1) - a) * gj * gj).astype(f32)
    den = np.sqrt(v + eps).astype(f32) if eps_inside else (np.sqrt(v).astype(f32) + eps).astype(f32)
    step = (gj / den).astype(f32)
    if buf is not None:
        step = buf = (mom * buf + step).astype(f32)
    return (w - lr * step).astype(f32), v, buf


def attention(q, k, v, mask, p, rng, G, fill=-np.inf, scale=None):
    """newch's attention chain (net/__init__.py:811-820) for q [B, L, D], k [B, S, D], v [B, S, Dv],
    mask [L, S] (nonzero = masked) or None, dropout p drawn from rng, upstream gradient G: returns
    y and the gradients of q, k and v (ops_linalg.c bmm, ops_nn.c masked_fill / softmax / dropout)."""
    q, k, v = (t.astype(np.float64) for t in (q, k, v))
    s = np.matmul(q, k.transpose(0, 2, 1)).astype(f32)
    if scale is not None:
        s = (f32(scale) * s).astype(f32)
    m = np.zeros(s.shape[1:], bool) if mask is None else mask.astype(bool)
    s = np.where(m, f32(fill), s).astype(f32)
    y = softmax(s)
    if p > 0:
        pd, keep = dropout(y, p, rng)
    else:
        pd, keep = y, np.ones_like(y)
    out = np.matmul(pd.astype(np.float64), v).astype(f32)
    G = G.astype(np.float64)
    gpd = np.matmul(G, v.transpose(0, 2, 1)).astype(f32)
    gy = (gpd * keep).astype(f32)
    gs = np.where(m, f32(0), softmax_grad(y, gy, False)).astype(f32)
    if scale is not None:
        gs = (f32(scale) * gs).astype(f32)
    gs = gs.astype(np.float64)
    dq = np.matmul(gs, k).astype(f32)
    dk = np.matmul(gs.transpose(0, 2, 1), q).astype(f32)
    dv = np.matmul(pd.astype(np.float64).transpose(0, 2, 1), G).astype(f32)
    return out, dq, dk, dv
