"""newch's own unittest suite (its Python package unchanged, 140 tests over `tests/test_*.py` of the
newch project: torch-style models, fit(), callbacks, DataLoader, optimizers and their raw state
pointers, NCW1 checkpoints with bit-exact resume, RNN and transformer blocks) run against a library
chosen by NEWCH_LIB, the one hook newch's `_lib.py:58-73` offers.

The package and suite are staged by `make -C oracle REF=<newch checkout>` into oracle/_ref/suite
(test infrastructure, kept out of history). The CPU test runs the suite on the reference engine
built beside it, which pins the staging and this harness; the GPU test runs the same suite, in a
child process, on the B200 engine (newch_b200/libnc.so) and requires every test to pass.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
SUITE = REPO / "oracle" / "_ref" / "suite"
B200_LIB = REPO / "newch_b200" / "libnc.so"
REF_LIB = REPO / "oracle" / "_ref" / "libnc_ref.so"

HEAD = re.compile(r"^(\w+) \(([\w.]+)\)")
OUTCOME = re.compile(r" \.\.\. (ok|FAIL|ERROR|skipped.*|expected failure|unexpected success)$")


def run_suite(lib: Path, timeout: int = 900) -> tuple[dict, str, int]:
    """Runs the staged suite with NEWCH_LIB=lib; returns ({test id: outcome}, output, tests run)."""
    assert (SUITE / "newch" / "_lib.py").exists() and (SUITE / "tests").is_dir(), (
        "newch's Python package and tests are not staged under oracle/_ref/suite: "
        "run make -C oracle REF=<newch checkout>")
    assert lib.exists(), f"{lib} is not built"
    env = dict(os.environ, NEWCH_LIB=str(lib), PYTHONDONTWRITEBYTECODE="1")
    env.pop("PYTHONPATH", None)
    proc = subprocess.run([sys.executable, "-m", "unittest", "discover", "-s", "tests", "-v"], cwd=SUITE, env=env,
                          capture_output=True, text=True, timeout=timeout)
    out = proc.stderr + proc.stdout
    results, current = {}, None
    for ln in out.splitlines():  # "name (id)" then, on it or after a docstring line, "... outcome"
        h = HEAD.match(ln)
        if h:
            current = h.group(2)
        o = OUTCOME.search(ln)
        if o and current is not None:
            results[current] = o.group(1)
            current = None
    ran = re.search(r"^Ran (\d+) tests? in", out, re.M)
    return results, out, int(ran.group(1)) if ran else -1


def failures(results: dict) -> list:
    return sorted(k for k, v in results.items() if v in ("FAIL", "ERROR", "unexpected success"))


def report(out: str, limit: int = 12000) -> str:
    i = out.find("=" * 70)
    return out[i:i + limit] if i >= 0 else out[-limit:]


def test_suite_green_on_the_reference_engine():
    """The staged package and suite, on the reference engine they came with: all 140 pass."""
    results, out, ran = run_suite(REF_LIB)
    assert ran == 140 and len(results) == ran, out[-4000:]
    assert not failures(results), report(out)


@pytest.mark.gpu
def test_suite_green_on_the_b200_engine():
    """The same unchanged suite with NEWCH_LIB pointing at the B200 library: every test passes."""
    results, out, ran = run_suite(B200_LIB)
    assert ran == 140 and len(results) == ran, out[-4000:]
    bad = failures(results)
    assert not bad, f"{len(bad)} failing: {bad}\n" + report(out)
