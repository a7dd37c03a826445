"""nc_ext_cross_entropy_fwd_noalloc (the cross entropy that keeps its scratch in a static device array
and allocates nothing) against the engine's own nc_cross_entropy on the same data, two calls in a
row, plus its size limit. Device buffers for the no-allocation call come from PyTorch (plumbing
only); the call goes through the C ABI."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from nchelp import Eng, capi, rel_err, seeded

pytestmark = pytest.mark.gpu
MAX_ROWS = 262144  # NC_EXT_CE_NOALLOC_MAX_ROWS in include/nc_ext.h
NC_OK, NC_ERR_ARG = 0, 4


def engine_loss(X, lab):
    with Eng("b200") as e:
        loss = e.check(e.L.nc_cross_entropy(e.t(X), e.t(lab)))
        out = float(e.np(loss).reshape(()))
        assert e.ok(), e.err()
    return out


def softmax64(X):
    z = X.astype(np.float64) - X.max(axis=1, keepdims=True)
    p = np.exp(z)
    return p / p.sum(axis=1, keepdims=True)


def test_matches_engine_cross_entropy_twice_in_a_row():
    import torch

    L = capi.load_b200()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    for seed, (rows, classes) in [(11, (512, 10)), (12, (8192, 96))]:
        X = seeded(seed, (rows, classes), 3.0)
        lab = np.random.default_rng(seed).integers(0, classes, rows).astype(np.int32)
        want = engine_loss(X, lab)
        x = torch.from_numpy(X).to(dev)
        y = torch.from_numpy(lab).to(dev)
        prob = torch.empty_like(x)
        loss = torch.full((1,), float("nan"), dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        rc = L.nc_ext_cross_entropy_fwd_noalloc(x.data_ptr(), y.data_ptr(), rows, classes, prob.data_ptr(),
                                                loss.data_ptr(), status.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == NC_OK
        stream.synchronize()
        assert int(status.item()) == 0
        got = float(loss.item())
        assert got == pytest.approx(want, rel=1e-6, abs=1e-7), (rows, classes, got, want)
        assert rel_err(prob.cpu().numpy(), softmax64(X)) < 1e-5


def test_rejects_rows_beyond_the_static_scratch():
    import torch

    L = capi.load_b200()
    dev = torch.device("cuda", 0)
    loss = torch.zeros(1, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    one = torch.zeros(1, dtype=torch.float32, device=dev)
    lab = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = L.nc_ext_cross_entropy_fwd_noalloc(one.data_ptr(), lab.data_ptr(), MAX_ROWS + 1, 1, one.data_ptr(),
                                            loss.data_ptr(), status.data_ptr(), None)
    assert rc == NC_ERR_ARG
    rc = L.nc_ext_cross_entropy_fwd_noalloc(one.data_ptr(), lab.data_ptr(), 1, 1, one.data_ptr(), loss.data_ptr(),
                                            None, None)
    assert rc == NC_ERR_ARG
    torch.cuda.synchronize()
    assert float(loss.item()) == 0.0  # nothing was launched
