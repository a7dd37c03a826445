"""Generates tests/golden/ops.npz: every case of tests/opcases.py run on the reference engine (newch's
own C sources, built by oracle/Makefile into oracle/_ref/libnc_ref.so).

    make -C oracle && python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from opcases import CASES, run_case  # noqa: E402


def main() -> int:
    data = {}
    for name in CASES:
        out = run_case("ref", name)
        for k, v in out.items():
            data[f"{name}/{k}"] = v
        print(f"{name}: {len(out)} arrays")
    np.savez_compressed(HERE / "ops.npz", **data)
    print(f"wrote {HERE / 'ops.npz'} ({(HERE / 'ops.npz').stat().st_size / 1e3:.1f} kB)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
