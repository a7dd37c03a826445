"""Convolution forward, dX, dW and dB on the B200 engine against the numpy oracle (float64), over
geometries that exercise the implicit-GEMM tensor-core path (groups 1, more than 32 taps): strides,
padding, dilation, non-square kernels, position counts that are not a multiple of the 128-row
tile, channel counts above one 128-wide tile, reductions split across CTAs. Unit-stride dX runs on
the implicit path too; strided dX and the FFMA mode take the unfolded path, checked the same way.

Every case runs on three convolution paths: tap-shifted GEMMs over the packed padded grid (the
default, NC_CONV=tap; strided convolutions fall through to the unfolded path), unfolded (im2col +
GEMM + col2im, NC_CONV=unfolded) and implicit (NC_CONV=implicit). Tolerances (normwise,
max|err| / max|ref|): FFMA 1e-5; 3xTF32 4e-5 (the tap-shifted dX sums taps x output channels, up to
1800 products here, in one tensor-memory accumulator, whose fp32 additions are not round-to-nearest);
TF32 2e-3. The contract for the tensor-core path is 1e-3."""

from __future__ import annotations

import numpy as np
import pytest

from nchelp import Eng, rel_err, seeded

pytestmark = pytest.mark.gpu
TOL = {"ffma": 1e-5, "3xtf32": 4e-5, "tf32": 2e-3}

# (N, C, H, W), (OC, KH, KW), stride, pad, dilation
GEOMS = [
    ((3, 4, 9, 11), (5, 3, 3), (1, 1), (1, 1), (1, 1)),
    ((3, 8, 14, 14), (16, 3, 3), (1, 1), (1, 1), (1, 1)),
    ((2, 16, 13, 17), (40, 3, 3), (2, 2), (1, 1), (1, 1)),
    ((2, 12, 12, 12), (24, 5, 5), (1, 1), (2, 2), (1, 1)),
    ((2, 8, 15, 15), (20, 3, 3), (1, 1), (2, 2), (2, 2)),
    ((1, 32, 7, 7), (200, 3, 3), (1, 1), (1, 1), (1, 1)),
    ((4, 64, 6, 5), (33, 1, 3), (1, 1), (0, 1), (1, 1)),
    ((2, 150, 5, 6), (20, 3, 3), (1, 1), (1, 1), (1, 1)),
    ((16, 32, 14, 14), (64, 3, 3), (1, 1), (1, 1), (1, 1)),
    ((5, 20, 10, 9), (12, 3, 2), (1, 2), (0, 1), (1, 1)),
    # few taps (C * KH * KW <= 32): direct kernels, four positions per thread where the output width is
    # a multiple of 4 and the stride 1, one position per thread otherwise
    ((4, 1, 28, 28), (32, 3, 3), (1, 1), (1, 1), (1, 1)),
    ((2, 1, 9, 10), (16, 3, 3), (1, 1), (1, 1), (2, 2)),
    ((2, 1, 6, 8), (8, 1, 3), (1, 1), (0, 1), (1, 1)),
    ((3, 1, 10, 14), (8, 3, 3), (1, 1), (2, 2), (2, 2)),
    ((2, 1, 12, 12), (16, 3, 3), (1, 1), (0, 0), (1, 1)),
    ((2, 3, 16, 16), (8, 3, 3), (2, 2), (1, 1), (1, 1)),
]


@pytest.fixture(params=["ffma", "tf32", "3xtf32"])
def mode(request, monkeypatch):
    monkeypatch.setenv("NC_GEMM", request.param)
    return request.param


@pytest.fixture(params=["tap", "unfolded", "implicit"], autouse=True)
def conv_path(request, monkeypatch):
    """NC_CONV=tap: tap-shifted GEMMs over packed x / dY; implicit: tensor-core convolutions gathered
    straight from x / dY; unfolded: im2col + GEMM + col2im."""
    monkeypatch.setenv("NC_CONV", request.param)
    return request.param


@pytest.mark.parametrize("xs,wk,stride,pad,dil", GEOMS)
def test_conv_forward_and_grads(mode, xs, wk, stride, pad, dil):
    import ncoracle as O

    ws = (wk[0], xs[1], wk[1], wk[2])
    X, W, B = seeded(1, xs), seeded(2, ws, 0.3), seeded(3, (wk[0],))
    with Eng("b200") as e:
        assert e.L.nc_ext_gemm_mode(e.ctx).decode() == mode
        x, w, b = e.param(X), e.param(W), e.param(B)
        y = e.check(e.L.nc_conv2d_ex(x, w, b, stride[0], stride[1], pad[0], pad[1], dil[0], dil[1], 1))
        out = e.np(y)
        G = seeded(4, out.shape)
        e.backward_with(y, G)
        dx, dw, db = e.grad(x), e.grad(w), e.grad(b)
        assert e.ok(), e.err()
    y_ref = O.conv2d(X, W, B, stride=stride, pad=pad, dil=dil)
    dx_ref, dw_ref, db_ref = O.conv2d_grads(X, W, G, stride=stride, pad=pad, dil=dil)
    tol = TOL[mode]
    assert rel_err(out, y_ref) < tol
    assert rel_err(dx, dx_ref) < tol
    assert rel_err(dw, dw_ref) < tol
    assert rel_err(db, db_ref) < 1e-5


def test_conv_grads_accumulate(mode):
    """Two backward passes add into the same gradients (dX and dW accumulate, never overwrite)."""
    import ncoracle as O

    xs, ws = (4, 16, 10, 10), (24, 16, 3, 3)
    X, W = seeded(5, xs), seeded(6, ws, 0.3)
    with Eng("b200") as e:
        x, w = e.param(X), e.param(W)
        for seed in (7, 8):
            y = e.check(e.L.nc_conv2d_ex(x, w, None, 1, 1, 1, 1, 1, 1, 1))
            e.backward_with(y, seeded(seed, e.shape(y)))
        dx, dw = e.grad(x), e.grad(w)
        shape_y = e.shape(y)
    G = seeded(7, shape_y) + seeded(8, shape_y)
    dx_ref, dw_ref, _ = O.conv2d_grads(X, W, G, pad=(1, 1))
    assert rel_err(dx, dx_ref) < TOL[mode]
    assert rel_err(dw, dw_ref) < TOL[mode]


def test_conv_large_batch_against_unfolded_path(monkeypatch):
    """cfg2's second convolution at batch 128: the tensor-core path (3xTF32) against FFMA."""
    xs, ws = (128, 32, 14, 14), (64, 32, 3, 3)
    X, W, B = seeded(9, xs), seeded(10, ws, 0.2), seeded(11, (64,))
    res = {}
    for m in ("ffma", "3xtf32"):
        monkeypatch.setenv("NC_GEMM", m)
        with Eng("b200") as e:
            x, w, b = e.param(X), e.param(W), e.param(B)
            y = e.check(e.L.nc_conv2d_ex(x, w, b, 1, 1, 1, 1, 1, 1, 1))
            G = seeded(12, e.shape(y))
            out = e.np(y)
            e.backward_with(y, G)
            res[m] = (out, e.grad(x), e.grad(w), e.grad(b))
    for a, r in zip(res["3xtf32"], res["ffma"]):
        assert rel_err(a, r) < TOL["3xtf32"]


@pytest.mark.parametrize("xs,oc", [((64, 16, 28, 28), 16), ((37, 24, 20, 20), 40)])
def test_conv_off_the_tape_packs_a_few_samples_at_a_time(xs, oc, conv_path):
    """A forward nothing will differentiate (no input needs a gradient) keeps no packed copy for a
    backward, so the tap-shifted path packs a few samples at a time (ragged last chunk here): the
    output is bit-identical to the whole-batch forward on the tape, and the arena's peak stays below
    the output plus half of it (4 MiB at least) plus the packed weights, where the whole-batch pack
    (channels padded to 32, two planes) would be several times the output. The other paths: values."""
    import ncoracle as O

    ws = (oc, xs[1], 3, 3)
    X, W, B = seeded(13, xs), seeded(14, ws, 0.3), seeded(15, (oc,))
    with Eng("b200") as e:
        x, w, b = e.param(X), e.param(W), e.param(B)
        on_tape = e.np(e.check(e.L.nc_conv2d_ex(x, w, b, 1, 1, 1, 1, 1, 1, 1)))
        e.step_end()
        xc, wc, bc = e.t(X, persistent=True), e.t(W, persistent=True), e.t(B, persistent=True)
        before = e.L.nc_get_mem_stats(e.ctx).arena_bytes_in_use
        e.L.nc_reset_peak(e.ctx)
        y = e.check(e.L.nc_conv2d_ex(xc, wc, bc, 1, 1, 1, 1, 1, 1, 1))
        assert not e.L.nc_requires_grad(y)
        off_tape = e.np(y)
        peak = e.L.nc_get_mem_stats(e.ctx).arena_peak_bytes - before
        assert e.ok(), e.err()
    out_bytes = off_tape.nbytes
    wpack = oc * 9 * 32 * ((xs[1] + 31) // 32) * 2 * 4
    if conv_path == "tap":
        assert peak <= out_bytes + max(out_bytes // 2, 4 << 20) + wpack + (1 << 20), peak
        assert np.array_equal(off_tape, on_tape)
    assert rel_err(off_tape, O.conv2d(X, W, B, pad=(1, 1))) < TOL["3xtf32"]
