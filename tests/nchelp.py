"""Small driver over the nc.h C ABI for tests: numpy in, numpy out, on any nc-ABI library (the B200
engine, or the reference engine built under oracle/_ref as the checker)."""

from __future__ import annotations

import ctypes
import math
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

from newch_b200 import capi  # noqa: E402

REF_LIB = REPO / "oracle" / "_ref" / "libnc_ref.so"
NP2NC = {np.dtype(np.float32): capi.F32, np.dtype(np.int32): capi.I32, np.dtype(np.int8): capi.I8,
         np.dtype(np.uint8): capi.U8}
NC2NP = {v: k for k, v in NP2NC.items()}

_libs: dict = {}


def lib(which: str):
    """'ref' (reference engine, CPU) or 'b200' (this engine)."""
    if which not in _libs:
        _libs[which] = capi.load(REF_LIB) if which == "ref" else capi.load_b200()
    return _libs[which]


class Eng:
    """One engine context."""

    def __init__(self, which: str = "b200", seed: int = 1, force_reference: int = 0):
        self.L = lib(which)
        cfg = capi.Config(0, seed, force_reference, 0)
        self.ctx = self.L.nc_init(ctypes.byref(cfg))
        assert self.ctx, "nc_init failed"
        self._keep = []

    def close(self):
        if self.ctx:
            self.L.nc_free_ctx(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # -- tensors ---------------------------------------------------------------------------
    def t(self, arr, persistent: bool = False):
        arr = np.ascontiguousarray(arr)
        n, shp = capi.shape_arg(arr.shape)
        if persistent:
            self.L.nc_persistent_begin(self.ctx)
        p = self.L.nc_from_data(self.ctx, NP2NC[arr.dtype], arr.ctypes.data if arr.size else None, n, shp)
        if persistent:
            self.L.nc_persistent_end(self.ctx)
        self.check(p)
        return p

    def param(self, arr):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        self.L.nc_persistent_begin(self.ctx)
        src = self.t(arr)
        self.L.nc_persistent_end(self.ctx)
        n, shp = capi.shape_arg(arr.shape)
        p = self.L.nc_parameter(self.ctx, src, n, shp)
        self.check(p)
        self.L.nc_release(src)
        return p

    def shape(self, t):
        nd = self.L.nc_ndim(t)
        s = self.L.nc_shape(t)
        return tuple(s[i] for i in range(nd))

    def np(self, t):
        self.check(t)
        dt = NC2NP[self.L.nc_get_dtype(t)]
        shape = self.shape(t)
        out = np.empty(shape, dtype=dt)
        if out.size:
            ok = self.L.nc_copy_to(t, out.ctypes.data, out.nbytes)
            assert ok, self.err()
        return out

    def grad(self, t):
        g = self.L.nc_grad(t)
        return None if not g else self.np(g)

    def err(self) -> str:
        return self.L.nc_error(self.ctx).decode(errors="replace")

    def check(self, p):
        if not p:
            raise RuntimeError(f"engine returned NULL: {self.err()}")
        return p

    def ok(self) -> bool:
        return bool(self.L.nc_ok(self.ctx))

    def backward_with(self, y, G):
        """Backpropagates with upstream gradient G: loss = sum(y * G)."""
        gt = self.t(np.ascontiguousarray(G, dtype=np.float32))
        loss = self.check(self.L.nc_sum(self.check(self.L.nc_mul(y, gt)), capi.ALL_AXES, 0))
        st = self.L.nc_backward(loss)
        assert st == 0, self.err()
        return loss

    def step_end(self):
        self.L.nc_step_end(self.ctx)


def rel_err(a, b) -> float:
    """max |a - b| / max |b| (normwise over the tensor), 0 for empty tensors."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    if a.size == 0:
        return 0.0
    den = np.max(np.abs(b))
    return float(np.max(np.abs(a - b)) / (den if den > 0 else 1.0))


def seeded(seed, shape, scale=1.0, dtype=np.float32):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(dtype)


def numel(shape) -> int:
    return int(math.prod(shape))
