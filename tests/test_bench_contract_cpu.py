"""bench.py's reference arm on CPU: one short run, its JSON line carries the keys the benchmark
contract names (the B200 arm's line, checked on the GPU box by the benchmark itself, carries the same
plus roofline, clocks and gpu_launches)."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def test_reference_arm_json_line():
    if not (REPO / "oracle" / "_ref" / "libnc_ref.so").exists():
        pytest.skip("reference engine not built (make -C oracle)")
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
                         capture_output=True, text=True, timeout=600, cwd=str(REPO))
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    # the B200 arm's line carries the same config dict (bench.config_dict), so the two arms compare
    assert line["config"] == {"workload": line["config"]["workload"], "global_batch": 512, "per_gpu_batch": 512,
                              "parallelism": "dp1"}
    assert {"value", "unit", "cores", "kind", "sample"} <= set(line["cpu_baseline"])
    assert line["cpu_baseline"]["kind"] == "reference"
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
