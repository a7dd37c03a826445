"""Generates tests/golden/trace_spread.json: how far the reference engine's two CPU kernel tiers (its
AVX2+FMA tier and its scalar reference tier, selected by nc_config.force_reference) lie apart on each
workload trace: per backward pass and parameter, the gradients computed from the same parameters
(the scalar-tier run is given the AVX2 run's parameters after every step), and per parameter, the
parameters after the whole run (each tier on its own trajectory), max-norm and Frobenius.

Both tiers are newch's own correct fp32 arithmetic; they differ only in summation order. Where a
gradient is a long sum with heavy cancellation (a convolution weight whose output feeds BatchNorm
sums ~10^5 products to a result far smaller than its terms), that spread is far above 1e-5, and any
third correct implementation, the B200 engine included, lands at the same distance.
tests/test_gpu_traces.py uses it as the floor of its per-parameter tolerances.

    make -C oracle REF=<newch checkout> && python tests/golden/make_trace_spread.py [names...]
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent.parent))

from nchelp import REF_LIB, capi  # noqa: E402
from newch_b200 import replay  # noqa: E402

OUT = HERE / "trace_spread.json"
NAMES = ["cfg1_small", "cfg2_small", "cfg3_small", "cfg4_small", "cfg1", "cfg2", "cfg2_stream", "cfg3", "cfg4"]


def normwise(a: np.ndarray, b: np.ndarray) -> float:
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30)) if b.size else 0.0


def frobenius(a: np.ndarray, b: np.ndarray) -> float:
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(np.linalg.norm(a - b) / max(float(np.linalg.norm(b)), 1e-30)) if b.size else 0.0


def spread(name: str) -> dict:
    lib = capi.load(REF_LIB)
    t = replay.Trace(name)
    a = replay.Replayer(lib, t, grads=True, capture_params=True)
    a.run_all()
    synced = replay.Replayer(lib, t, grads=True, force_reference=1, set_params=a.params_after)
    synced.run_all()
    free = replay.Replayer(lib, t, force_reference=1)
    free.run_all()
    grads = []
    for (_, ga), (_, gb) in zip(a.grads, synced.grads):
        grads.append([normwise(np.frombuffer(y, np.float32), np.frombuffer(x, np.float32))
                      if x is not None and y is not None else 0.0 for x, y in zip(ga, gb)])
    pa = [(np.frombuffer(x, np.float32), np.frombuffer(y, np.float32)) for (_, x), (_, y) in zip(a.outputs, free.outputs)]
    out = {"grads": grads, "params": [normwise(y, x) for x, y in pa], "params_frob": [frobenius(y, x) for x, y in pa]}
    for r in (a, synced, free):
        lib.nc_free_ctx(r.ctx)
    return out


def main() -> int:
    names = sys.argv[1:] or NAMES
    data = json.loads(OUT.read_text()) if OUT.exists() else {}
    for n in names:
        t0 = time.time()
        data[n] = spread(n)
        print(f"{n}: {time.time() - t0:.1f} s, worst gradient spread "
              f"{max((max(r) for r in data[n]['grads']), default=0.0):.3g}", flush=True)
        OUT.write_text(json.dumps(data, indent=0))
    return 0


if __name__ == "__main__":
    sys.exit(main())
