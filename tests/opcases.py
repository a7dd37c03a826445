"""Op-level parity cases run through the nc.h C ABI on any engine.

Each case builds seeded inputs, runs one op forward and its backward with a seeded upstream
gradient, and returns named numpy outputs. tests/golden/make_golden.py records them from the
reference engine (tests/golden/ops.npz); the GPU tests run the same cases on the B200 engine and the
CPU tests recompute them with the numpy oracle.
"""

from __future__ import annotations

import numpy as np

from nchelp import Eng, capi, seeded

ALL = capi.ALL_AXES


def _conv(e: Eng, xs, ws, bias, stride, pad, dil, groups, seed):
    x = e.param(seeded(seed, xs))
    w = e.param(seeded(seed + 1, ws, 0.5))
    b = e.param(seeded(seed + 2, (ws[0],))) if bias else None
    y = e.check(e.L.nc_conv2d_ex(x, w, b, stride[0], stride[1], pad[0], pad[1], dil[0], dil[1], groups))
    out = {"x": e.np(x), "w": e.np(w), "y": e.np(y)}
    G = seeded(seed + 3, e.shape(y))
    e.backward_with(y, G)
    out.update(G=G, dx=e.grad(x), dw=e.grad(w))
    if bias:
        out.update(b=e.np(b), db=e.grad(b))
    return out


def case_conv_basic(e):
    return _conv(e, (2, 2, 5, 5), (3, 2, 3, 3), True, (1, 1), (1, 1), (1, 1), 1, 10)


def case_conv_s2_groups(e):
    return _conv(e, (2, 4, 7, 6), (6, 2, 3, 3), True, (2, 2), (1, 1), (1, 1), 2, 20)


def case_conv_dilation(e):
    return _conv(e, (1, 2, 8, 9), (2, 2, 3, 2), False, (1, 1), (2, 1), (2, 1), 1, 30)


def case_conv_depthwise(e):
    return _conv(e, (2, 3, 7, 6), (3, 1, 3, 3), True, (1, 1), (1, 1), (1, 1), 3, 40)


def case_conv_depthwise_w8(e):  # rows a multiple of 4 wide: the strip kernels
    return _conv(e, (3, 5, 9, 8), (5, 1, 3, 3), True, (1, 1), (1, 1), (1, 1), 5, 42)


def case_conv_depthwise_valid(e):  # no padding: strip forward and weight gradient, tiled input gradient
    return _conv(e, (2, 3, 10, 10), (3, 1, 3, 3), True, (1, 1), (0, 0), (1, 1), 3, 43)


def case_conv_depthwise_s2(e):
    return _conv(e, (2, 4, 9, 8), (4, 1, 3, 3), False, (2, 2), (1, 1), (2, 1), 4, 45)


def case_conv_pointwise(e):
    return _conv(e, (2, 5, 4, 4), (3, 5, 1, 1), True, (1, 1), (0, 0), (1, 1), 1, 50)


def case_conv_im2col(e):
    return _conv(e, (4, 8, 12, 12), (16, 8, 3, 3), True, (1, 1), (1, 1), (1, 1), 1, 60)


def case_conv_stem(e):
    return _conv(e, (3, 3, 16, 16), (8, 3, 3, 3), True, (2, 2), (1, 1), (1, 1), 1, 65)


def _pool(e, xs, k, s, p, is_max, seed):
    x = e.param(seeded(seed, xs))
    fn = e.L.nc_max_pool2d if is_max else e.L.nc_avg_pool2d
    y = e.check(fn(x, k[0], k[1], s[0], s[1], p[0], p[1]))
    G = seeded(seed + 1, e.shape(y))
    out = {"x": e.np(x), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["dx"] = e.grad(x)
    return out


def case_maxpool_2x2(e):
    return _pool(e, (2, 3, 8, 8), (2, 2), (2, 2), (0, 0), True, 70)


def _pool_fresh(e, xs, seed):
    """2x2 / stride-2 max pooling of an intermediate (scale by 1): its gradient is a fresh buffer, so the
    backward takes the kernels that store every input gradient instead of adding."""
    x = e.param(seeded(seed, xs))
    h = e.check(e.L.nc_scale(x, 1.0))
    y = e.check(e.L.nc_max_pool2d(h, 2, 2, 2, 2, 0, 0))
    G = seeded(seed + 1, e.shape(y))
    out = {"x": e.np(x), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["dx"] = e.grad(x)
    return out


def case_maxpool_2x2_w4(e):
    return _pool_fresh(e, (2, 3, 9, 12), 71)  # width a multiple of 4, odd height


def case_maxpool_2x2_w2(e):
    return _pool_fresh(e, (3, 4, 14, 14), 72)  # even width (cfg2's second pooling)


def case_maxpool_2x2_odd(e):
    return _pool_fresh(e, (2, 2, 7, 9), 73)  # odd width and height


def case_maxpool_overlap(e):
    return _pool(e, (1, 2, 5, 6), (3, 3), (1, 1), (1, 1), True, 80)


def case_avgpool(e):
    return _pool(e, (2, 2, 6, 6), (2, 2), (2, 2), (0, 0), False, 90)


def case_batch_norm_train(e):
    x = e.param(seeded(100, (4, 3, 5, 5), 2.0) + 1.0)
    w = e.param(seeded(101, (3,)))
    b = e.param(seeded(102, (3,)))
    e.L.nc_persistent_begin(e.ctx)
    rm = e.t(seeded(103, (3,), 0.1))
    rv = e.t(np.abs(seeded(104, (3,))) + 0.5)
    e.L.nc_persistent_end(e.ctx)
    out = {"x": e.np(x), "w": e.np(w), "b": e.np(b), "rm0": e.np(rm), "rv0": e.np(rv)}
    y = e.check(e.L.nc_batch_norm(x, w, b, rm, rv, 1, 0.1, 1e-5))
    G = seeded(105, e.shape(y))
    out.update(y=e.np(y), rm=e.np(rm), rv=e.np(rv), G=G)
    e.backward_with(y, G)
    out.update(dx=e.grad(x), dw=e.grad(w), db=e.grad(b))
    return out


def _bn_chain(e, seed, shape, act, pool, reuse=False):
    """BatchNorm (training) -> activation -> (2 x 2 max pool): the chain the B200 engine runs as a
    deferred epilogue and one fused backward. reuse: the BatchNorm output is read a second time (added
    to the result), which forces the unfused paths."""
    x = e.param(seeded(seed, shape, 2.0) + 0.5)
    C = shape[1]
    w = e.param(seeded(seed + 1, (C,)))
    b = e.param(seeded(seed + 2, (C,)))
    e.L.nc_persistent_begin(e.ctx)
    rm = e.t(np.zeros(C, np.float32))
    rv = e.t(np.ones(C, np.float32))
    e.L.nc_persistent_end(e.ctx)
    y = e.check(e.L.nc_batch_norm(x, w, b, rm, rv, 1, 0.1, 1e-5))
    z = e.check(_unary_call(e, act, y) if act != "none" else y)
    if reuse:
        z = e.check(e.L.nc_add(z, y))
    out = e.check(e.L.nc_max_pool2d(z, 2, 2, 2, 2, 0, 0)) if pool else z
    G = seeded(seed + 3, e.shape(out))
    res = {"x": e.np(x), "w": e.np(w), "b": e.np(b), "y": e.np(out), "G": G}
    e.backward_with(out, G)
    res.update(dx=e.grad(x), dw=e.grad(w), db=e.grad(b), rm=e.np(rm), rv=e.np(rv))
    return res


def case_conv3_bn_relu_pool(e):
    """Conv2d(1, C, 3, padding 1) of an image (no gradient) -> BatchNorm -> ReLU -> 2 x 2 max pool: the
    B200 engine computes the convolution's weight and bias gradients inside the chain's fused backward."""
    img = e.t(seeded(760, (5, 1, 10, 12), 1.0))
    cw = e.param(seeded(761, (6, 1, 3, 3), 0.3))
    cb = e.param(seeded(762, (6,), 0.1))
    x = e.check(e.L.nc_conv2d_ex(img, cw, cb, 1, 1, 1, 1, 1, 1, 1))
    w = e.param(seeded(763, (6,)))
    b = e.param(seeded(764, (6,)))
    e.L.nc_persistent_begin(e.ctx)
    rm = e.t(np.zeros(6, np.float32))
    rv = e.t(np.ones(6, np.float32))
    e.L.nc_persistent_end(e.ctx)
    y = e.check(e.L.nc_batch_norm(x, w, b, rm, rv, 1, 0.1, 1e-5))
    out = e.check(e.L.nc_max_pool2d(e.check(e.L.nc_relu(y)), 2, 2, 2, 2, 0, 0))
    G = seeded(765, e.shape(out))
    res = {"y": e.np(out), "G": G}
    e.backward_with(out, G)
    # the convolution bias feeds BatchNorm, so its gradient is rounding noise around zero (compared on
    # the trace workloads with their exemption for such biases, not against a golden value here)
    res.update(dcw=e.grad(cw), dw=e.grad(w), db=e.grad(b), rm=e.np(rm), rv=e.np(rv))
    return res


def case_bn_relu_pool(e):
    return _bn_chain(e, 700, (4, 6, 10, 12), "relu", True)


def case_bn_pool(e):
    return _bn_chain(e, 710, (3, 5, 8, 8), "none", True)


def case_bn_hardswish(e):
    return _bn_chain(e, 720, (4, 6, 7, 9), "hardswish", False)


def case_bn_relu6_pool(e):
    return _bn_chain(e, 730, (2, 4, 6, 10), "relu6", True)


def case_bn_relu_reused(e):
    return _bn_chain(e, 740, (3, 4, 8, 8), "relu", True, reuse=True)


def case_bn_relu_pool_odd(e):
    return _bn_chain(e, 750, (2, 3, 9, 7), "relu", True)


def case_batch_norm_eval(e):
    x = e.param(seeded(110, (3, 4, 6)))
    w = e.param(seeded(111, (4,)))
    b = e.param(seeded(112, (4,)))
    e.L.nc_persistent_begin(e.ctx)
    rm = e.t(seeded(113, (4,), 0.1))
    rv = e.t(np.abs(seeded(114, (4,))) + 0.5)
    e.L.nc_persistent_end(e.ctx)
    y = e.check(e.L.nc_batch_norm(x, w, b, rm, rv, 0, 0.1, 1e-5))
    G = seeded(115, e.shape(y))
    out = {"x": e.np(x), "w": e.np(w), "b": e.np(b), "rm": e.np(rm), "rv": e.np(rv), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out.update(dx=e.grad(x), dw=e.grad(w), db=e.grad(b))
    return out


def case_layer_norm(e):
    x = e.param(seeded(120, (6, 16), 3.0) + 0.5)
    w = e.param(seeded(121, (16,)))
    b = e.param(seeded(122, (16,)))
    y = e.check(e.L.nc_layer_norm(x, 1, w, b, 1e-5))
    G = seeded(123, e.shape(y))
    out = {"x": e.np(x), "w": e.np(w), "b": e.np(b), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out.update(dx=e.grad(x), dw=e.grad(w), db=e.grad(b))
    return out


def case_linear(e):
    x = e.param(seeded(130, (2, 5, 7)))
    w = e.param(seeded(131, (4, 7)))
    b = e.param(seeded(132, (4,)))
    y = e.check(e.L.nc_linear_fn(x, w, b))
    G = seeded(133, e.shape(y))
    out = {"x": e.np(x), "w": e.np(w), "b": e.np(b), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out.update(dx=e.grad(x), dw=e.grad(w), db=e.grad(b))
    return out


def case_bmm_transposed(e):
    a = e.param(seeded(140, (3, 4, 5)))
    b = e.param(seeded(141, (3, 6, 5)))
    bt = e.check(e.L.nc_transpose(b, 1, 2))  # [3, 5, 6] view: passed to the GEMM as a transpose flag
    y = e.check(e.L.nc_matmul(a, bt))
    G = seeded(142, e.shape(y))
    out = {"a": e.np(a), "b": e.np(b), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out.update(da=e.grad(a), db=e.grad(b))
    return out


def case_bmm_broadcast(e):
    a = e.param(seeded(145, (2, 3, 4, 5)))
    b = e.param(seeded(146, (3, 5, 2)))
    y = e.check(e.L.nc_matmul(a, b))
    G = seeded(147, e.shape(y))
    out = {"a": e.np(a), "b": e.np(b), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out.update(da=e.grad(a), db=e.grad(b))
    return out


def _attention(e, seed, BH, L, S, D, Dv, p, mask="random", scale=None, layout="plain", read_probs=False):
    """scores = q @ k^T (k through a transposed view) -> [scale] -> masked_fill(-inf) -> softmax ->
    [dropout] -> @ v: newch's multi-head attention chain, which the B200 engine keeps as recipes and
    runs as one fused forward and one fused backward. layout "mha": q, k, v are the [T, BH, Dh] ->
    [BH, T, Dh] transposed views nn.MultiheadAttention makes (q scaled first, as it does).
    read_probs: the softmax output is read back, which forces the unfused paths."""
    e.L.nc_manual_seed(e.ctx, seed)
    res = {}
    if layout == "mha":
        qb, kb, vb = (e.param(seeded(seed + i, (L, BH, D if i < 2 else Dv))) for i in range(3))
        q = e.check(e.L.nc_scale(e.check(e.L.nc_transpose(qb, 0, 1)), 1.0 / np.sqrt(D)))
        k = e.check(e.L.nc_transpose(kb, 0, 1))
        v = e.check(e.L.nc_transpose(vb, 0, 1))
        leaves = {"q": qb, "k": kb, "v": vb}
    else:
        q = e.param(seeded(seed, (BH, L, D)))
        k = e.param(seeded(seed + 1, (BH, S, D)))
        v = e.param(seeded(seed + 2, (BH, S, Dv)))
        leaves = {"q": q, "k": k, "v": v}
    for n, t in leaves.items():
        res[n] = e.np(t)
    s = e.check(e.L.nc_matmul(q, e.check(e.L.nc_transpose(k, 1, 2))))
    if scale is not None:
        s = e.check(e.L.nc_scale(s, scale))
    if mask == "causal":
        m = (np.arange(S)[None, :] > np.arange(L)[:, None]).astype(np.int32)
    elif mask == "random":
        m = (np.random.default_rng(seed + 3).random((L, S)) > 0.6).astype(np.int32)
        m[:, 0] = 0  # no row fully masked
    else:
        m = None
    if m is not None:
        res["mask"] = m
        s = e.check(e.L.nc_masked_fill(s, e.t(m), -np.inf))
    pr = e.check(e.L.nc_softmax(s))
    if read_probs:
        res["probs"] = e.np(pr)
    pd = e.check(e.L.nc_dropout(pr, p)) if p > 0 else pr
    y = e.check(e.L.nc_matmul(pd, v))
    G = seeded(seed + 4, e.shape(y))
    res.update(y=e.np(y), G=G)
    e.backward_with(y, G)
    for n, t in leaves.items():
        res["d" + n] = e.grad(t)
    return res


def case_attention_chain(e):
    return _attention(e, 800, 6, 10, 12, 8, 6, 0.2)


def case_attention_mha(e):
    return _attention(e, 810, 6, 20, 20, 8, 8, 0.1, mask="causal", layout="mha")


def case_attention_mha_128(e):
    return _attention(e, 820, 4, 128, 128, 32, 32, 0.1, mask="causal", layout="mha")


def case_attention_sdpa(e):
    return _attention(e, 830, 5, 33, 40, 16, 12, 0.0, mask="random", scale=0.25)


def case_attention_unmasked(e):
    return _attention(e, 840, 3, 7, 9, 5, 3, 0.3, mask=None)


def case_attention_probs_read(e):
    return _attention(e, 850, 4, 12, 12, 8, 8, 0.2, mask="causal", read_probs=True)


def case_softmax(e):
    x = e.param(seeded(150, (5, 9), 3.0))
    y = e.check(e.L.nc_softmax(x))
    G = seeded(151, (5, 9))
    out = {"x": e.np(x), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["dx"] = e.grad(x)
    return out


def case_log_softmax(e):
    x = e.param(seeded(155, (5, 9), 3.0))
    y = e.check(e.L.nc_log_softmax(x))
    G = seeded(156, (5, 9))
    out = {"x": e.np(x), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["dx"] = e.grad(x)
    return out


def case_cross_entropy(e):
    x = e.param(seeded(160, (8, 10), 2.0))
    lab = np.random.default_rng(161).integers(0, 10, 8).astype(np.int32)
    loss = e.check(e.L.nc_cross_entropy(x, e.t(lab)))
    out = {"x": e.np(x), "labels": lab, "loss": e.np(loss)}
    assert e.L.nc_backward(loss) == 0, e.err()
    out["dx"] = e.grad(x)
    return out


def case_nll_loss(e):
    x = e.param(seeded(165, (6, 5)))
    lab = np.random.default_rng(166).integers(0, 5, 6).astype(np.int32)
    loss = e.check(e.L.nc_nll_loss(x, e.t(lab), 0))
    out = {"x": e.np(x), "labels": lab, "loss": e.np(loss)}
    assert e.L.nc_backward(loss) == 0, e.err()
    out["dx"] = e.grad(x)
    return out


UNARY = ["relu", "sigmoid", "tanh", "exp", "neg", "scale", "add_scalar", "leaky_relu", "relu6", "hardsigmoid",
         "hardswish", "silu", "gelu", "gelu_tanh"]


def _unary_call(e, kind, x):
    L = e.L
    if kind in ("scale", "add_scalar", "leaky_relu"):
        return getattr(L, f"nc_{kind}")(x, 0.3)
    if kind == "gelu":
        return L.nc_gelu(x, 0)
    if kind == "gelu_tanh":
        return L.nc_gelu(x, 1)
    return getattr(L, f"nc_{kind}")(x)


def case_unary(e):
    base = np.concatenate([seeded(170, (239,), 3.0), np.array([-3, 3, 0, 6, -6, 0.5, -0.5, 2.9, -2.9, 6.1, 1e-3,
                                                               -1e-3, 10, -10, 3.0001, -3.0001, 5.999, 0.0],
                                                              dtype=np.float32)])
    out = {"x": base}
    for kind in UNARY:
        x = e.param(base)
        y = e.check(_unary_call(e, kind, x))
        G = seeded(171, base.shape)
        out[f"{kind}_y"] = e.np(y)
        e.backward_with(y, G)
        out[f"{kind}_dx"] = e.grad(x)
        out["G"] = G
        e.step_end()
    return out


TRANSCENDENTAL = ["sigmoid", "tanh", "exp", "silu", "gelu", "gelu_tanh"]


def case_transcendental(e):
    """The activations built on exp / tanh / erf over their whole range: a dense sweep of [-12, 12],
    both sides of every branch and clamp of newch's polynomial forms (|x| = 1/4 for tanh, the exp
    input window [-87.34, 88.8] and the 2^128 scale step near ln(FLT_MAX)), denormal and signed
    zero inputs, +-inf and NaN."""
    sweep = np.linspace(-12.0, 12.0, 1201, dtype=np.float32)
    edges = np.array([0.0, -0.0, 1e-40, -1e-40, 1e-30, -1e-30, 0.25, -0.25, np.nextafter(np.float32(0.25), 0),
                      -np.nextafter(np.float32(0.25), 0), 0.2500001, 88.0, 88.37, 88.5, 88.72, 88.73, 88.8, 88.81,
                      89.0, 100.0, -87.0, -87.33, -87.3365448, -87.34, -87.5, -88.0, -103.0, -104.0, -150.0,
                      np.inf, -np.inf, np.nan, 1e30, -1e30, 44.0, -44.0, 9.0, -9.0, 13.2, -13.2, 3.0, -3.0],
                     dtype=np.float32)
    base = np.concatenate([sweep, edges]).astype(np.float32)
    out = {"x": base}
    G = seeded(172, base.shape)
    out["G"] = G
    for kind in TRANSCENDENTAL:
        x = e.param(base)
        y = e.check(_unary_call(e, kind, x))
        out[f"{kind}_y"] = e.np(y)
        e.backward_with(y, G)
        out[f"{kind}_dx"] = e.grad(x)
        e.step_end()
    return out


def case_binary_broadcast(e):
    out = {}
    A, B = seeded(180, (3, 1, 4)), np.abs(seeded(181, (5, 1))) + 0.5
    out["a"], out["b"] = A, B
    for op in ("add", "sub", "mul", "div"):
        a, b = e.param(A), e.param(B)
        y = e.check(getattr(e.L, f"nc_{op}")(a, b))
        G = seeded(182, e.shape(y))
        out[f"{op}_y"] = e.np(y)
        e.backward_with(y, G)
        out[f"{op}_da"], out[f"{op}_db"], out["G"] = e.grad(a), e.grad(b), G
        e.step_end()
    return out


def case_reductions(e):
    X = seeded(190, (3, 4, 5))
    out = {"x": X}
    for nm, fn in (("sum", e.L.nc_sum), ("mean", e.L.nc_mean), ("max", e.L.nc_max)):
        for axis in (0, 1, 2, ALL):
            x = e.param(X)
            y = e.check(fn(x, axis, 1))
            G = seeded(191 + axis % 7, e.shape(y))
            key = f"{nm}_{'all' if axis == ALL else axis}"
            out[f"{key}_y"] = e.np(y)
            e.backward_with(y, G)
            out[f"{key}_dx"], out[f"{key}_G"] = e.grad(x), G
            e.step_end()
    x = e.t(X)
    out["argmax_1"] = e.np(e.check(e.L.nc_argmax(x, 1)))
    return out


def case_index_select(e):
    x = e.param(seeded(200, (6, 4)))
    idx = np.array([3, 0, 3, 5, 1, 3], dtype=np.int32)
    y = e.check(e.L.nc_index_select(x, e.t(idx)))
    G = seeded(201, e.shape(y))
    out = {"x": e.np(x), "idx": idx, "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["dx"] = e.grad(x)
    return out


def case_masked_fill(e):
    x = e.param(seeded(210, (2, 3, 4)))
    mask = (np.random.default_rng(211).random((3, 4)) > 0.5).astype(np.int32)
    y = e.check(e.L.nc_masked_fill(x, e.t(mask), -np.inf))
    G = seeded(212, e.shape(y))
    out = {"x": e.np(x), "mask": mask, "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["dx"] = e.grad(x)
    return out


def case_views(e):
    x = e.param(seeded(220, (3, 4, 5)))
    t = e.check(e.L.nc_transpose(x, 0, 2))          # [5, 4, 3] view
    s = e.check(e.L.nc_slice(t, 1, 1, 2, 2))        # [5, 2, 3] strided view
    c = e.check(e.L.nc_contiguous(s))
    n, shp = capi.shape_arg((10, 3))
    r = e.check(e.L.nc_reshape(c, n, shp))
    y = e.check(e.L.nc_mul(r, r))
    G = seeded(221, (10, 3))
    out = {"x": e.np(x), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["dx"] = e.grad(x)
    return out


def case_cat(e):
    a, b = e.param(seeded(230, (2, 3, 2))), e.param(seeded(231, (2, 1, 2)))
    arr = capi.ptr_array([a, b])
    y = e.check(e.L.nc_cat(2, arr, 1))
    G = seeded(232, e.shape(y))
    out = {"a": e.np(a), "b": e.np(b), "y": e.np(y), "G": G}
    e.backward_with(y, G)
    out["da"], out["db"] = e.grad(a), e.grad(b)
    return out


def case_to_dtype(e):
    u = np.arange(0, 256, 7, dtype=np.uint8)
    f = np.array([-3.7, 2.9, 1e10, -1e10, np.nan, 127.9, -128.9, 0.5], dtype=np.float32)
    return {"u8": u, "u8_f32": e.np(e.check(e.L.nc_to_dtype(e.t(u), capi.F32))),
            "f": f, "f_i32": e.np(e.check(e.L.nc_to_dtype(e.t(f), capi.I32))),
            "f_i8": e.np(e.check(e.L.nc_to_dtype(e.t(f), capi.I8)))}


def case_dropout(e):
    e.L.nc_manual_seed(e.ctx, 4242)
    x = e.param(np.ones(50000, dtype=np.float32))
    y1 = e.check(e.L.nc_dropout(x, 0.25))
    y2 = e.check(e.L.nc_dropout(x, 0.5))  # continues the same stream
    G = seeded(240, (50000,))
    out = {"y1": e.np(y1), "y2": e.np(y2), "G": G}
    e.backward_with(y1, G)
    out["dx"] = e.grad(x)
    return out


def case_random(e):
    e.L.nc_manual_seed(e.ctx, 7)
    n, shp = capi.shape_arg((1000,))
    u = e.np(e.check(e.L.nc_rand_uniform(e.ctx, -0.5, 2.0, n, shp)))
    g = e.np(e.check(e.L.nc_randn(e.ctx, 1.5, n, shp)))
    return {"uniform": u, "normal": g}


def case_int8(e):
    w = seeded(250, (13, 70), 0.2)
    x = seeded(251, (7, 70))
    b = seeded(252, (13,))
    sp = capi.ptr_array([None])
    q = e.check(e.L.nc_quantize_rows(e.t(w), sp))
    s = sp[0]
    y = e.check(e.L.nc_linear_int8(e.t(x), q, s, e.t(b)))
    return {"w": w, "x": x, "b": b, "q": e.np(q), "scale": e.np(s), "y": e.np(y)}


def case_int8_gelu_chain(e):
    """Inference (no tape) int8 MLP block: linear_int8 -> GELU -> linear_int8, 1024 features: the B200
    engine quantizes the pending GELU output on the fly (no fp32 GELU tensor is written unless read)."""
    e.L.nc_set_grad_enabled(e.ctx, 0)
    out = {}
    x = seeded(255, (33, 1024))
    h = e.t(x)
    for i, (o, k) in enumerate(((1024, 1024), (10, 1024))):
        w = seeded(256 + i, (o, k), 0.05)
        b = seeded(258 + i, (o,), 0.1)
        sp = capi.ptr_array([None])
        q = e.check(e.L.nc_quantize_rows(e.t(w), sp))
        h = e.check(e.L.nc_linear_int8(h, q, sp[0], e.t(b)))
        if i == 0:
            pre = h
            h = e.check(e.L.nc_gelu(h, 0))
            e.L.nc_release_temp(pre)  # as newch's inference loop does: the GELU input goes first
    out.update(x=x, y=e.np(h))
    e.L.nc_set_grad_enabled(e.ctx, 1)
    return out


def _adam(e, decoupled, seed):
    w0 = seeded(seed, (50,))
    w = e.param(w0)
    opts = capi.OptimOpts(1e-2, 0.0, 0.05, 0.9, 0.999, 1e-8)
    arr = capi.ptr_array([w])
    opt = e.check((e.L.nc_adamw if decoupled else e.L.nc_adam)(e.ctx, arr, 1, opts))
    out = {"w0": w0}
    for k in range(3):
        G = seeded(seed + 1 + k, (50,))
        e.L.nc_optim_clear_grad(opt)
        wt = e.check(e.L.nc_mul(w, e.t(G)))
        assert e.L.nc_backward(e.check(e.L.nc_sum(wt, ALL, 0))) == 0
        e.L.nc_optim_step(opt)
        out[f"G{k}"] = G
        out[f"w{k + 1}"] = e.np(w)
        e.step_end()
    e.L.nc_optim_free(opt)
    return out


def _optim(e, make, opts, seed, steps=4):
    """Several update steps of one optimizer on a seeded weight vector with seeded gradients."""
    w0 = seeded(seed, (50,))
    w = e.param(w0)
    opt = e.check(make(capi.ptr_array([w]), opts))
    out = {"w0": w0}
    for k in range(steps):
        G = seeded(seed + 1 + k, (50,))
        e.L.nc_optim_clear_grad(opt)
        wt = e.check(e.L.nc_mul(w, e.t(G)))
        assert e.L.nc_backward(e.check(e.L.nc_sum(wt, ALL, 0))) == 0
        e.L.nc_optim_step(opt)
        out[f"G{k}"] = G
        out[f"w{k + 1}"] = e.np(w)
        e.step_end()
    e.L.nc_optim_free(opt)
    return out


def case_sgd(e):
    return _optim(e, lambda a, o: e.L.nc_sgd(e.ctx, a, 1, o), capi.OptimOpts(0.1, 0.0, 0.01, 0.9, 0.999, 1e-8), 270)


def case_sgd_momentum(e):
    return _optim(e, lambda a, o: e.L.nc_sgd(e.ctx, a, 1, o), capi.OptimOpts(0.05, 0.9, 0.02, 0.9, 0.999, 1e-8), 280)


def case_rmsprop(e):
    return _optim(e, lambda a, o: e.L.nc_rmsprop(e.ctx, a, 1, o, 0),
                  capi.OptimOpts(1e-2, 0.0, 0.01, 0.9, 0.99, 1e-8), 290)


def case_rmsprop_momentum_eps_inside(e):
    return _optim(e, lambda a, o: e.L.nc_rmsprop(e.ctx, a, 1, o, 1),
                  capi.OptimOpts(1e-2, 0.8, 0.0, 0.9, 0.95, 1e-6), 300)


def case_adam(e):
    return _adam(e, False, 260)


def case_adamw(e):
    return _adam(e, True, 270)


CASES = {name[5:]: fn for name, fn in globals().items() if name.startswith("case_")}


def run_case(which: str, name: str, force_reference: bool = False) -> dict:
    with Eng(which, seed=1, force_reference=int(force_reference)) as e:
        out = CASES[name](e)
        assert e.ok(), e.err()
        return {k: np.asarray(v) for k, v in out.items() if v is not None}
