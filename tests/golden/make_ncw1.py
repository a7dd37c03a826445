"""Generates tests/golden/ref_state.ncw: an NCW1 named-tensor file written by the reference engine
(newch's own C sources, built by oracle/Makefile into oracle/_ref/libnc_ref.so) with nc_save, for the
interchange tests in tests/test_gpu_engine.py (the B200 engine reads it, and writes the same bytes).

    make -C oracle && python tests/golden/make_ncw1.py
"""

from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from nchelp import Eng, capi, seeded  # noqa: E402

OUT = HERE / "ref_state.ncw"


def ncw1_tensors():
    """(name, array) pairs of the file: float32 of several ranks, int32, int8, uint8, a one-element and
    an empty tensor."""
    return [
        ("fc1.weight", seeded(9000, (6, 10))),
        ("fc1.bias", seeded(9001, (6,))),
        ("conv.weight", seeded(9002, (4, 3, 3, 3))),
        ("steps", np.array([3, -7, 2**31 - 1], np.int32)),
        ("qweight", np.array([-127, 0, 5, 127, -1], np.int8)),
        ("bytes", np.arange(0, 250, 25, dtype=np.uint8)),
        ("scalar", np.array([2.5], np.float32)),
        ("empty", np.zeros((0, 4), np.float32)),
    ]


def main() -> int:
    items = ncw1_tensors()
    with Eng("ref") as e:
        ts = [e.t(a, persistent=True) for _, a in items]
        names = (ctypes.c_char_p * len(items))(*[n.encode() for n, _ in items])
        st = e.L.nc_save(e.ctx, str(OUT).encode(), len(items), names, capi.ptr_array(ts))
        assert st == 0, e.err()
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
