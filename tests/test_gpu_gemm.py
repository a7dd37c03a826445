"""The FP32 GEMM in its three modes (NC_GEMM=ffma | tf32 | 3xtf32): every transpose combination,
strided batches, batch reduction (conv weight gradients) and split-K shapes, against float64 numpy.

Tolerances (normwise, max|err| / max|ref|): FFMA 1e-5, 3xTF32 1e-5, TF32 2e-3 (10-bit mantissa
inputs, fp32 accumulation)."""

from __future__ import annotations

import os

import numpy as np
import pytest

from nchelp import Eng, capi, rel_err, seeded
from opcases import CASES, run_case
from pathlib import Path

pytestmark = pytest.mark.gpu
TOL = {"ffma": 1e-5, "3xtf32": 1e-5, "tf32": 2e-3}
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "ops.npz")


@pytest.fixture(params=["ffma", "tf32", "3xtf32"])
def mode(request, monkeypatch):
    monkeypatch.setenv("NC_GEMM", request.param)
    # small products would take the one-thread / one-warp-per-output kernels; these tests keep them on
    # the tiled FFMA and tensor-core kernels (test_small_products covers the small path)
    monkeypatch.setenv("NC_GEMM_SMALL", "0")
    return request.param


def engine(mode):
    e = Eng("b200")
    assert e.L.nc_ext_gemm_mode(e.ctx).decode() == mode
    return e


SHAPES = [(128, 128, 64), (200, 72, 288), (64, 196, 288), (512, 128, 3136), (10, 128, 512), (333, 250, 97),
          (8, 8, 8192)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_matmul_transposes(mode, M, N, K, ta, tb):
    A = seeded(M * 7 + K, (K, M) if ta else (M, K))
    B = seeded(N * 13 + K, (N, K) if tb else (K, N))
    with engine(mode) as e:
        a, b = e.t(A), e.t(B)
        if ta:
            a = e.check(e.L.nc_transpose(a, 0, 1))
        if tb:
            b = e.check(e.L.nc_transpose(b, 0, 1))
        y = e.np(e.check(e.L.nc_matmul(a, b)))
    ref = (A.T if ta else A).astype(np.float64) @ (B.T if tb else B).astype(np.float64)
    assert rel_err(y, ref) < TOL[mode]


@pytest.mark.parametrize("bs,M,N,K", [(6, 128, 128, 32), (512, 64, 32, 16), (3, 130, 70, 200)])
def test_batched_and_grads(mode, bs, M, N, K):
    A, B, G = seeded(1, (bs, M, K)), seeded(2, (bs, K, N)), seeded(3, (bs, M, N))
    with engine(mode) as e:
        a, b = e.param(A), e.param(B)
        y = e.check(e.L.nc_matmul(a, b))
        out = e.np(y)
        e.backward_with(y, G)
        da, db = e.grad(a), e.grad(b)
    A64, B64, G64 = (x.astype(np.float64) for x in (A, B, G))
    assert rel_err(out, A64 @ B64) < TOL[mode]
    assert rel_err(da, G64 @ B64.transpose(0, 2, 1)) < TOL[mode]
    assert rel_err(db, A64.transpose(0, 2, 1) @ G64) < TOL[mode]


@pytest.mark.parametrize("case", ["conv_basic", "conv_im2col", "conv_pointwise", "conv_stem", "conv_s2_groups",
                                  "linear", "bmm_transposed", "bmm_broadcast"])
def test_gemm_ops_against_reference(mode, case):
    out = run_case("b200", case)
    for k, v in out.items():
        ref = GOLD[f"{case}/{k}"]
        assert rel_err(v, ref) <= TOL[mode], (case, k, rel_err(v, ref))


def test_conv_weight_grad_batch_reduction_large(mode):
    """dW of a 3x3 conv over 256 samples: the batch sum runs inside the GEMM (split over CTAs)."""
    X, W = seeded(4, (256, 16, 14, 14)), seeded(5, (32, 16, 3, 3), 0.2)
    with engine(mode) as e:
        x, w = e.t(X), e.param(W)
        y = e.check(e.L.nc_conv2d(x, w, None, 1, 1, 1, 1))
        G = seeded(6, e.shape(y))
        e.backward_with(y, G)
        dw = e.grad(w)
    import ncoracle as O
    _, dw_ref, _ = O.conv2d_grads(X, W, G, pad=(1, 1))
    # a sum over 50k positions: in 3xTF32 each reduction slice adds ~1000 tensor-core products into one
    # tensor-memory accumulator (fp32 additions that are not round-to-nearest), ~1e-5 normwise
    tol = 4e-5 if mode == "3xtf32" else TOL[mode]
    assert rel_err(dw, dw_ref) < tol


@pytest.mark.parametrize("M,N,K", [(10, 128, 512), (512, 10, 128), (512, 128, 10), (8, 8, 8192), (1, 1, 1),
                                   (37, 19, 70), (64, 196, 288), (24, 45, 777)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_small_products(mode, monkeypatch, M, N, K, ta, tb):
    """Products with at most 64k outputs and 4M multiply-adds take the small kernels (one thread per
    output for a reduction of at most 64; a block per 32 columns of a row for a transposed A and a
    reduction of at least 256, ragged columns and rows included; else one warp per output), exact fp32
    in every mode: the FFMA tolerance applies whatever NC_GEMM says. Forward and both gradients (dA, dB
    are small too)."""
    monkeypatch.setenv("NC_GEMM_SMALL", "1")
    A = seeded(M * 7 + K, (K, M) if ta else (M, K))
    B = seeded(N * 13 + K, (N, K) if tb else (K, N))
    G = seeded(5, (M, N))
    with engine(mode) as e:
        a, b = e.param(A), e.param(B)
        at = e.check(e.L.nc_transpose(a, 0, 1)) if ta else a
        bt = e.check(e.L.nc_transpose(b, 0, 1)) if tb else b
        y = e.check(e.L.nc_matmul(at, bt))
        out = e.np(y)
        e.backward_with(y, G)
        da, db = e.grad(a), e.grad(b)
    A64, B64, G64 = (x.astype(np.float64) for x in (A, B, G))
    Am, Bm = (A64.T if ta else A64), (B64.T if tb else B64)
    assert rel_err(out, Am @ Bm) < 1e-5
    dAm, dBm = G64 @ Bm.T, Am.T @ G64
    assert rel_err(da, dAm.T if ta else dAm) < 1e-5
    assert rel_err(db, dBm.T if tb else dBm) < 1e-5


def test_small_linear_bias_and_batch_sum():
    """The small kernels' epilogue (bias, accumulation into an existing gradient) through Linear, and the
    batch-summed reduction through a small convolution weight gradient."""
    import ncoracle as O

    X, W, Bv = seeded(1, (64, 40)), seeded(2, (10, 40), 0.2), seeded(3, (10,))
    with Eng("b200") as e:
        x, w, b = e.param(X), e.param(W), e.param(Bv)
        y = e.check(e.L.nc_linear_fn(x, w, b))
        out = e.np(y)
        G = seeded(4, out.shape)
        for _ in range(2):  # the second backward adds into the gradients
            y = e.check(e.L.nc_linear_fn(x, w, b))
            e.backward_with(y, G)
        dx, dw, db = e.grad(x), e.grad(w), e.grad(b)
    X64, W64, G64 = (v.astype(np.float64) for v in (X, W, G))
    assert rel_err(out, X64 @ W64.T + Bv) < 1e-5
    assert rel_err(dx, 2 * G64 @ W64) < 1e-5
    assert rel_err(dw, 2 * G64.T @ X64) < 1e-5
    assert rel_err(db, 2 * G64.sum(0)) < 1e-5
    Xc, Wc = seeded(5, (6, 3, 5, 5)), seeded(6, (4, 3, 1, 1), 0.3)
    with Eng("b200") as e:
        x, w = e.param(Xc), e.param(Wc)
        y = e.check(e.L.nc_conv2d(x, w, None, 1, 1, 0, 0))
        Gc = seeded(7, e.shape(y))
        e.backward_with(y, Gc)
        dwc = e.grad(w)
    _, dw_ref, _ = O.conv2d_grads(Xc, Wc, Gc)
    assert rel_err(dwc, dw_ref) < 1e-5


def test_small_weight_gradient_accumulates():
    """A Linear weight gradient over a long batch (dY^T X: transposed A, 600 rows, 45 columns, the
    row-streaming small kernel) written by the first backward and added into by the second."""
    X, W = seeded(21, (600, 45)), seeded(22, (10, 45), 0.2)
    with Eng("b200") as e:
        x, w = e.param(X), e.param(W)
        G = seeded(23, (600, 10))
        for _ in range(2):
            e.backward_with(e.check(e.L.nc_linear_fn(x, w, None)), G)
        dw = e.grad(w)
    assert rel_err(dw, 2 * G.astype(np.float64).T @ X.astype(np.float64)) < 1e-5
