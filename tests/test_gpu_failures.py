"""Failure detection on the B200 engine, made without faulting or hanging a GPU:

- a tensor-core pipeline wait that nothing completes gives up after its bound and surfaces as
  NC_ERR_STATE at the next synchronization, and the context keeps working after nc_clear_error;
- a data-parallel rank whose NCCL id never arrives (no rank 0), or whose id file is a stale one from
  another launch, gives up after NC_DP_TIMEOUT seconds with NC_ERR_STATE instead of waiting forever.
  No communicator is created in these cases.
"""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap
import time
from pathlib import Path

import numpy as np
import pytest

from nchelp import Eng

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent
NC_ERR_STATE = 5


def test_pipeline_wait_gives_up_and_context_survives():
    with Eng("b200") as e:
        t0 = time.time()
        st = e.L.nc_ext_pipeline_wait_probe(e.ctx)
        elapsed = time.time() - t0
        assert st == NC_ERR_STATE, st
        assert "pipeline wait timed out" in e.err()
        assert 1.5 < elapsed < 30.0, elapsed  # the wait's bound is 2 s
        e.L.nc_clear_error(e.ctx)
        a, b = e.t(np.arange(6, dtype=np.float32)), e.t(np.full(6, 2.0, np.float32))
        y = e.np(e.check(e.L.nc_mul(a, b)))
        assert e.ok(), e.err()
        np.testing.assert_array_equal(y, np.arange(6, dtype=np.float32) * 2.0)


_INIT = textwrap.dedent("""
    import ctypes, sys, time
    sys.path.insert(0, {repo!r})
    from newch_b200 import capi
    L = capi.load_b200()
    t0 = time.time()
    ctx = L.nc_init(ctypes.byref(capi.Config(0, 1, 0, 0)))
    print(L.nc_status_code(ctx), round(time.time() - t0, 2), L.nc_error(ctx).decode())
""")


def _rank1_init(tmp_path, token=None, stale=None):
    idf = tmp_path / "nccl.id"
    if stale is not None:
        idf.write_bytes(stale)
    env = dict(os.environ, NC_WORLD_SIZE="2", NC_RANK="1", NC_NCCL_ID_FILE=str(idf), NC_DP_TIMEOUT="1")
    env.pop("TORCHELASTIC_RUN_ID", None)
    if token:
        env["NC_NCCL_ID_TOKEN"] = token
    else:
        env.pop("NC_NCCL_ID_TOKEN", None)
    out = subprocess.run([sys.executable, "-c", _INIT.format(repo=str(REPO))], env=env, capture_output=True,
                         text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    code, secs, msg = out.stdout.strip().split(" ", 2)
    return int(code), float(secs), msg


def test_dp_rank_gives_up_when_the_id_never_arrives(tmp_path):
    code, secs, msg = _rank1_init(tmp_path)
    assert code == NC_ERR_STATE and "gave up waiting" in msg, (code, msg)
    assert secs < 30.0


def test_dp_rank_ignores_an_id_file_from_another_launch(tmp_path):
    stale = b"NCDPID1\0" + b"earlier-run".ljust(56, b"\0") + bytes(128)
    code, secs, msg = _rank1_init(tmp_path, token="this-run", stale=stale)
    assert code == NC_ERR_STATE and "gave up waiting" in msg and "this-run" in msg, (code, msg)
    assert secs < 30.0
