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
