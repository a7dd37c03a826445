"""Pins the numpy oracle (oracle/ncoracle.py) to the reference engine: golden vectors recorded from
newch's own C engine (tests/golden/ops.npz) and the known answers of newch's C tests
(engine/tests/test_main.c:933-1076). CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import ncoracle as O
from nchelp import rel_err

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "ops.npz")


def g(case, key):
    return GOLD[f"{case}/{key}"]


CONV = {
    "conv_basic": dict(stride=(1, 1), pad=(1, 1), dil=(1, 1), groups=1),
    "conv_s2_groups": dict(stride=(2, 2), pad=(1, 1), dil=(1, 1), groups=2),
    "conv_dilation": dict(stride=(1, 1), pad=(2, 1), dil=(2, 1), groups=1),
    "conv_depthwise": dict(stride=(1, 1), pad=(1, 1), dil=(1, 1), groups=3),
    "conv_depthwise_s2": dict(stride=(2, 2), pad=(1, 1), dil=(2, 1), groups=4),
    "conv_depthwise_w8": dict(stride=(1, 1), pad=(1, 1), dil=(1, 1), groups=5),
    "conv_depthwise_valid": dict(stride=(1, 1), pad=(0, 0), dil=(1, 1), groups=3),
    "conv_pointwise": dict(stride=(1, 1), pad=(0, 0), dil=(1, 1), groups=1),
    "conv_im2col": dict(stride=(1, 1), pad=(1, 1), dil=(1, 1), groups=1),
    "conv_stem": dict(stride=(2, 2), pad=(1, 1), dil=(1, 1), groups=1),
}


@pytest.mark.parametrize("case", sorted(CONV))
def test_conv(case):
    kw = CONV[case]
    x, w = g(case, "x"), g(case, "w")
    b = GOLD[f"{case}/b"] if f"{case}/b" in GOLD else None
    y = O.conv2d(x, w, b, **kw)
    assert rel_err(y, g(case, "y")) < 2e-6
    dx, dw, db = O.conv2d_grads(x, w, g(case, "G"), **kw)
    assert rel_err(dx, g(case, "dx")) < 2e-6
    assert rel_err(dw, g(case, "dw")) < 2e-6
    if b is not None:
        assert rel_err(db, g(case, "db")) < 2e-6


@pytest.mark.parametrize("case,args", [("maxpool_2x2", ((2, 2), (2, 2), (0, 0), True)),
                                       ("maxpool_overlap", ((3, 3), (1, 1), (1, 1), True)),
                                       ("avgpool", ((2, 2), (2, 2), (0, 0), False))])
def test_pool(case, args):
    x = g(case, "x")
    y, arg = O.pool2d(x, *args)
    assert np.array_equal(y, g(case, "y")) if args[3] else rel_err(y, g(case, "y")) < 1e-6
    if args[3]:
        dx = O.maxpool_grad(x.shape, arg, g(case, "G"))
        assert rel_err(dx, g(case, "dx")) < 1e-6


def test_batch_norm_train():
    c = "batch_norm_train"
    y, mean, invstd, rm, rv = O.batch_norm_train(g(c, "x"), g(c, "w"), g(c, "b"), g(c, "rm0"), g(c, "rv0"), 0.1, 1e-5)
    assert rel_err(y, g(c, "y")) < 1e-6
    assert rel_err(rm, g(c, "rm")) < 1e-6 and rel_err(rv, g(c, "rv")) < 1e-6
    dx, dw, db = O.batch_norm_grads(g(c, "x"), g(c, "w"), g(c, "G"), mean, invstd)
    assert rel_err(dx, g(c, "dx")) < 1e-5 and rel_err(dw, g(c, "dw")) < 1e-5 and rel_err(db, g(c, "db")) < 1e-5


def test_layer_norm():
    c = "layer_norm"
    y, mean, rstd = O.layer_norm(g(c, "x"), g(c, "w"), g(c, "b"), 1e-5)
    assert rel_err(y, g(c, "y")) < 1e-6
    dx, dw, db = O.layer_norm_grads(g(c, "x"), g(c, "w"), g(c, "G"), mean, rstd)
    assert rel_err(dx, g(c, "dx")) < 1e-5 and rel_err(dw, g(c, "dw")) < 1e-5 and rel_err(db, g(c, "db")) < 1e-5


def test_linear():
    c = "linear"
    assert rel_err(O.linear(g(c, "x"), g(c, "w"), g(c, "b")), g(c, "y")) < 1e-6
    dx, dw, db = O.linear_grads(g(c, "x"), g(c, "w"), g(c, "G"))
    assert rel_err(dx, g(c, "dx")) < 1e-6 and rel_err(dw, g(c, "dw")) < 1e-6 and rel_err(db, g(c, "db")) < 1e-6


def test_softmax_family_and_losses():
    assert rel_err(O.softmax(g("softmax", "x")), g("softmax", "y")) < 1e-6
    assert rel_err(O.softmax_grad(g("softmax", "y"), g("softmax", "G"), False), g("softmax", "dx")) < 1e-5
    assert rel_err(O.log_softmax(g("log_softmax", "x")), g("log_softmax", "y")) < 1e-6
    assert rel_err(O.softmax_grad(g("log_softmax", "y"), g("log_softmax", "G"), True), g("log_softmax", "dx")) < 1e-5
    loss, prob = O.cross_entropy(g("cross_entropy", "x"), g("cross_entropy", "labels"))
    assert abs(loss - g("cross_entropy", "loss")) < 1e-6 * abs(loss)
    assert rel_err(O.cross_entropy_grad(prob, g("cross_entropy", "labels")), g("cross_entropy", "dx")) < 1e-6
    assert abs(O.nll_loss(g("nll_loss", "x"), g("nll_loss", "labels")) - g("nll_loss", "loss")) < 1e-6


@pytest.mark.parametrize("kind", ["relu", "sigmoid", "tanh", "exp", "neg", "scale", "add_scalar", "leaky_relu",
                                  "relu6", "hardsigmoid", "hardswish", "silu", "gelu", "gelu_tanh"])
def test_unary(kind):
    s = 0.3 if kind in ("scale", "add_scalar", "leaky_relu") else 0.0
    x = g("unary", "x")
    # the reference's SIMD tier uses polynomial exp / tanh / erf (about 1e-7 relative)
    tol = 2e-6 if kind in ("sigmoid", "tanh", "exp", "silu", "gelu", "gelu_tanh") else 0.0
    y = O.unary(kind, x, s)
    assert rel_err(y, g("unary", f"{kind}_y")) <= tol
    assert rel_err(O.unary_grad(kind, x, g("unary", "G"), s), g("unary", f"{kind}_dx")) <= max(tol, 1e-7)


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_binary_broadcast(op):
    a, b = g("binary_broadcast", "a"), g("binary_broadcast", "b")
    y = {"add": a + b, "sub": a - b, "mul": a * b, "div": a / b}[op]
    assert np.array_equal(y.astype(np.float32), g("binary_broadcast", f"{op}_y"))
    da, db = O.binary_grads(op, a, b, g("binary_broadcast", "G"))
    assert rel_err(da, g("binary_broadcast", f"{op}_da")) < 1e-6
    assert rel_err(db, g("binary_broadcast", f"{op}_db")) < 1e-6


def test_rng_uniform_and_normal_bit_exact():
    rng = O.Rng(7)
    u = O.rand_uniform(rng, -0.5, 2.0, 1000)
    assert np.array_equal(u, g("random", "uniform"))
    nrm = np.array([np.float32(1.5) * rng.normal() for _ in range(1000)], dtype=np.float32)
    assert rel_err(nrm, g("random", "normal")) < 1e-6  # libm log/cos may differ in the last bit


def test_dropout_mask_bit_exact():
    rng = O.Rng(4242)
    x = np.ones(50000, dtype=np.float32)
    y1, m1 = O.dropout(x, 0.25, rng)
    y2, _ = O.dropout(x, 0.5, rng)
    assert np.array_equal(y1, g("dropout", "y1")) and np.array_equal(y2, g("dropout", "y2"))
    assert np.array_equal((g("dropout", "G") * m1).astype(np.float32), g("dropout", "dx"))
    assert abs(float((y1 == 0).mean()) - 0.25) < 0.02


def test_int8_bit_exact():
    q, s = O.quantize_rows(g("int8", "w"))
    assert np.array_equal(q, g("int8", "q")) and np.array_equal(s, g("int8", "scale"))
    y, acc, xq, xs = O.linear_int8(g("int8", "x"), q, s, g("int8", "b"))
    assert np.array_equal(y, g("int8", "y"))
    ref = O.linear(g("int8", "x"), g("int8", "w"), g("int8", "b"))
    assert np.sqrt(((y - ref) ** 2).sum() / (ref ** 2).sum()) < 0.02  # test_main.c:1046-1065


def test_int8_gemm_known_pattern():
    """test_main.c:1066-1073: the exact int8 GEMM on a fixed pattern."""
    A = np.array([(i * 37) % 255 - 127 for i in range(5 * 37)], dtype=np.int8).reshape(5, 37)
    B = np.array([(i * 91) % 255 - 127 for i in range(6 * 37)], dtype=np.int8).reshape(6, 37)
    C = O.gemm_s8_nt(A, B)
    ref = np.array([[sum(int(A[i, k]) * int(B[j, k]) for k in range(37)) for j in range(6)] for i in range(5)])
    assert np.array_equal(C, ref)


@pytest.mark.parametrize("case,decoupled", [("adam", False), ("adamw", True)])
def test_adam(case, decoupled):
    w = g(case, "w0")
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    for k in range(3):
        w, m, v = O.adam_step(w, g(case, f"G{k}"), m, v, k + 1, 1e-2, weight_decay=0.05, decoupled=decoupled)
        assert rel_err(w, g(case, f"w{k + 1}")) < 1e-6


@pytest.mark.parametrize("case,momentum,wd,lr", [("sgd", 0.0, 0.01, 0.1), ("sgd_momentum", 0.9, 0.02, 0.05)])
def test_sgd(case, momentum, wd, lr):
    w = g(case, "w0")
    buf = np.zeros_like(w) if momentum else None
    for k in range(4):
        w, buf = O.sgd_step(w, g(case, f"G{k}"), buf, lr, momentum=momentum, weight_decay=wd)
        assert rel_err(w, g(case, f"w{k + 1}")) < 1e-6


@pytest.mark.parametrize("case,mom,wd,alpha,eps,inside", [("rmsprop", 0.0, 0.01, 0.99, 1e-8, False),
                                                          ("rmsprop_momentum_eps_inside", 0.8, 0.0, 0.95, 1e-6, True)])
def test_rmsprop(case, mom, wd, alpha, eps, inside):
    w = g(case, "w0")
    v = np.zeros_like(w)
    buf = np.zeros_like(w) if mom else None
    for k in range(4):
        w, v, buf = O.rmsprop_step(w, g(case, f"G{k}"), v, buf, 1e-2, alpha, eps, momentum=mom, weight_decay=wd,
                                   eps_inside=inside)
        assert rel_err(w, g(case, f"w{k + 1}")) < 1e-6


@pytest.mark.parametrize("case,seed,p,scale,mha", [("attention_chain", 800, 0.2, None, False),
                                                   ("attention_mha", 810, 0.1, None, True),
                                                   ("attention_sdpa", 830, 0.0, 0.25, False),
                                                   ("attention_unmasked", 840, 0.3, None, False)])
def test_attention_chain(case, seed, p, scale, mha):
    q, k, v = g(case, "q"), g(case, "k"), g(case, "v")
    if mha:  # [T, BH, Dh] leaves seen through transposes, q scaled by 1 / sqrt(Dh)
        q = (np.float32(1.0 / np.sqrt(q.shape[-1])) * q.transpose(1, 0, 2)).astype(np.float32)
        k, v = k.transpose(1, 0, 2), v.transpose(1, 0, 2)
    mask = g(case, "mask") if f"{case}/mask" in GOLD.files else None
    y, dq, dk, dv = O.attention(q, k, v, mask, p, O.Rng(seed), g(case, "G"), scale=scale)
    if mha:
        s = np.float32(1.0 / np.sqrt(q.shape[-1]))
        dq = (s * dq).transpose(1, 0, 2)
        dk, dv = dk.transpose(1, 0, 2), dv.transpose(1, 0, 2)
    for name, got in (("y", y), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert rel_err(got, g(case, name)) < 1e-5, (case, name, rel_err(got, g(case, name)))


def test_known_answers_from_reference_tests():
    """Known values of newch's C tests (test_main.c:937-942, :1011-1021)."""
    x = np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3)
    y = O.conv2d(x, np.ones((1, 1, 2, 2), np.float32))
    assert y[0, 0, 1, 1] == 5 + 6 + 8 + 9
    mp, _ = O.pool2d(x, (2, 2), (1, 1), (0, 0))
    assert mp[0, 0, 0, 1] == 6
    bx = np.array([1, 2, 3, 6], np.float32).reshape(4, 1)
    yb, _, _, rm, rv = O.batch_norm_train(bx, np.ones(1, np.float32), np.zeros(1, np.float32),
                                          np.zeros(1, np.float32), np.ones(1, np.float32), 1.0, 0.0)
    assert abs(rm[0] - 3.0) < 1e-6 and abs(rv[0] - 14.0 / 3.0) < 1e-5
    assert abs(yb[3, 0] - 3.0 / np.sqrt(3.5)) < 1e-5


@pytest.mark.parametrize("kind", ["sigmoid", "tanh", "exp", "silu", "gelu", "gelu_tanh"])
@pytest.mark.parametrize("case", ["unary", "transcendental"])
def test_avx2_transcendentals_bit_exact(case, kind):
    """The restated AVX2-tier exp / sigmoid / tanh / erf forms reproduce the reference engine's outputs
    and gradients bit for bit, over the dense sweep and the edge values (clamps, overflow, denormals,
    signed zeros, infinities, NaN)."""
    x = g(case, "x")
    y, d = O.unary_avx2(kind, x)
    assert np.array_equal(y, g(case, f"{kind}_y"), equal_nan=True)
    assert np.array_equal(d(g(case, "G")), g(case, f"{kind}_dx"), equal_nan=True)
