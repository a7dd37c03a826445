"""End-to-end parity of the five benchmark configurations: the recorded newch call sequences replayed
on the B200 engine and on the reference engine (CPU), step by step.

Checked: every nc_item result (the per-step losses, BatchNorm's num_batches_tracked), and the copied-out
results after training (final parameters, or the int8 model's logits). Losses must agree to 1e-5
relative on the CUDA-core GEMM path (NC_GEMM=ffma) and to 1e-3 relative on the tensor-core paths
(3xTF32, the default, and TF32), whose contractions round differently from the reference's loops;
in TF32 mode only the first loss (identical weights) is held to 1e-3, later ones to 1e-2.
Final parameters after Adam are compared normwise against the reference with a
tolerance for Adam's normalisation: for a parameter whose true gradient is zero (a conv bias in front
of BatchNorm, the key bias of attention), the update lr * m / sqrt(v) is the sign of rounding noise and
can differ by up to 2 * lr per step between any two correct implementations; every other parameter
must agree to 1e-3 relative after the three recorded steps.
"""

from __future__ import annotations

import numpy as np
import pytest

from nchelp import REF_LIB, capi, rel_err
from newch_b200 import replay

pytestmark = pytest.mark.gpu
LR = {"cfg1": 1e-3, "cfg2": 1e-3, "cfg2_stream": 1e-3, "cfg3": 1e-3, "cfg4": 3e-4}


def run(lib, name):
    t = replay.Trace(name)
    r = replay.Replayer(lib, t)
    r.run_all()
    return t, r


LOSS_TOL = {"ffma": 1e-5, "3xtf32": 1e-3, "tf32": 1e-3}
# TF32 rounding (rel ~1e-3 per GEMM) moves the weights after the first update; on these short,
# high-learning-rate runs over random labels the losses that follow drift apart by up to ~0.5%.
TF32_DRIFT = 1e-2


@pytest.fixture(params=["ffma", "3xtf32", "tf32"])
def mode(request, monkeypatch):
    monkeypatch.setenv("NC_GEMM", request.param)
    return request.param


def compare(name, mode="ffma"):
    ref = capi.load(REF_LIB)
    gpu = capi.load_b200()
    t, rg = run(gpu, name)
    _, rr = run(ref, name)
    assert gpu.nc_ok(rg.ctx), gpu.nc_error(rg.ctx)
    gi, ri = [v for _, v in rg.items], [v for _, v in rr.items]
    assert len(gi) == len(ri)
    first_loss = next((k for k, b in enumerate(ri) if b != round(b)), len(ri))
    for k, (a, b) in enumerate(zip(gi, ri)):
        tol = LOSS_TOL[mode]
        if mode == "tf32" and k > first_loss:
            tol = TF32_DRIFT  # later losses come from weights that already differ by TF32 updates
        assert a == pytest.approx(b, rel=tol, abs=1e-6), (mode, k, gi, ri)
    assert len(rg.outputs) == len(rr.outputs)
    base = name.replace("_small", "")
    steps = len(t.steps())
    for (_, a), (_, b) in zip(rg.outputs, rr.outputs):
        x, y = np.frombuffer(a, np.float32), np.frombuffer(b, np.float32)
        if base == "cfg5":
            assert rel_err(x, y) < 2e-2  # GELU between int8 layers re-quantizes: see test_gpu_engine int8
            continue
        err = np.abs(x.astype(np.float64) - y)
        ok = err <= 1e-3 * np.max(np.abs(y)) + 2.0 * LR[base] * steps
        assert ok.all(), f"{name}: parameter differs beyond Adam noise: {err.max():.3g}"
        if mode == "ffma":  # tensor-core gradients (rel 1e-6..1e-3) flip near-zero-gradient Adam updates
            assert rel_err(x, y) < 0.1
    gpu.nc_free_ctx(rg.ctx)
    ref.nc_free_ctx(rr.ctx)


@pytest.mark.parametrize("name", ["cfg1_small", "cfg2_small", "cfg3_small", "cfg4_small", "cfg5_small"])
def test_small_configs(name, mode):
    compare(name, mode)


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg2_stream", "cfg3", "cfg4", "cfg5"])
def test_full_size_configs(name, mode):
    compare(name, mode)


def test_full_size_against_recorded_losses(monkeypatch):
    """The B200 replay of config 2 reproduces the losses newch itself logged when the trace was made."""
    monkeypatch.setenv("NC_GEMM", "ffma")
    gpu = capi.load_b200()
    t, r = run(gpu, "cfg2")
    got = [v for _, v in r.items]
    assert got == pytest.approx(t.golden_items(), rel=1e-5, abs=1e-6)
    gpu.nc_free_ctx(r.ctx)
