"""Data-parallel parity on two B200s: two ranks, each training on its own micro-batch with the engine's
NCCL gradient averaging, end with the parameters, BatchNorm running statistics and per-rank losses
that the reference engine computes with gradient accumulation over the same two micro-batches
(newch engine/src/optim/optim.c:161-167: gs = 1 / accumulation steps; BatchNorm's running statistics
updated once per micro-batch in order, ops_nn.c:291-292; dropout masks drawn from one stream in
micro-batch order, ops_nn.c:182-204).

The engine reproduces each piece: rank r's dropout draws start where the reference's r-th micro-batch
draws start (nc_ext_dp_rng_stride), gradients are averaged over ranks before the update, and every
rank applies all ranks' BatchNorm statistics to its running statistics in rank order.

Runs when the box has at least two GPUs (skipped otherwise). CUDA-core GEMMs (NC_GEMM=ffma): losses,
running statistics and every parameter to 1e-5 (normwise).
"""

from __future__ import annotations

import os
import subprocess
import sys
import uuid
from pathlib import Path

import numpy as np
import pytest

from nchelp import REF_LIB, capi, rel_err

import dp_model

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def _gpus() -> int:
    try:
        return capi.load_b200().nc_ext_device_count()
    except OSError:
        return 0


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference engine not built")
def test_two_ranks_match_reference_accumulation(tmp_path):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    env_base = dict(os.environ, NC_WORLD_SIZE=str(world), NC_NCCL_ID_FILE=str(tmp_path / "nccl.id"),
                    NC_NCCL_ID_TOKEN=uuid.uuid4().hex, NC_GEMM="ffma", NC_DP_TIMEOUT="60", NCCL_NVLS_ENABLE="0")
    procs = []
    for r in range(world):
        env = dict(env_base, NC_RANK=str(r), NC_DEVICE=str(r))
        procs.append(subprocess.Popen([sys.executable, str(HERE / "dp_model.py"), str(tmp_path / f"rank{r}.npz")],
                                      env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=300)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            logs.append(p.communicate()[0])
    for r, p in enumerate(procs):
        assert p.returncode == 0, f"rank {r} failed:\n{logs[r][-3000:]}"
    ranks = [dict(np.load(tmp_path / f"rank{r}.npz")) for r in range(world)]
    ref = dp_model.run_accumulated("ref", world)

    # the losses: rank r's step-s loss is the reference's loss of micro-batch (s, r)
    ref_losses = ref["losses"].reshape(dp_model.STEPS, world)
    for r in range(world):
        np.testing.assert_allclose(ranks[r]["losses"], ref_losses[:, r], rtol=1e-5, atol=1e-6)
    for r in range(world):
        got = ranks[r]
        for k in ("bn_rm", "bn_rv"):
            assert rel_err(got[k], ref[k]) <= 1e-5, (r, k, got[k], ref[k])
        for k in ("conv_w", "bn_w", "bn_b", "fc_w", "fc_b"):
            assert rel_err(got[k], ref[k]) <= 1e-5, (r, k, rel_err(got[k], ref[k]))
    # every rank holds the same model
    for k in ranks[0]:
        if k != "losses":
            assert np.array_equal(ranks[0][k], ranks[1][k]), k
