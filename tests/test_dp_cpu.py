"""Data-parallel host logic on CPU with two gloo ranks (no GPU): the NCCL-id hand-off every rank
makes before joining the engine's all-reduce group, and the averaging contract that group
implements (mean over ranks of per-shard mean-loss gradients equals the full-batch gradient for a
batch-independent model), checked on the reference engine."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
HERE = Path(__file__).resolve().parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    return dist.group.WORLD


class _FakeLib:
    """Stands in for the engine's NCCL entry points: records what each rank joined with."""

    def __init__(self):
        self.joined = None

    def nc_ext_nccl_unique_id(self, buf, cap):
        data = bytes(range(7, 7 + 128))
        buf[:128] = data
        return 128

    def nc_ext_dp_init(self, ctx, rank, world, idb, n):
        self.joined = (rank, world, bytes(idb[:n]))
        return 0

    def nc_error(self, ctx):
        return b""


def _id_worker(rank, world, port, q):
    sys.path.insert(0, str(REPO))
    from newch_b200 import dist as dh

    pg = _init(rank, world, port)
    lib = _FakeLib()
    dh.join_engine_group(lib, None, pg, rank, world)
    other = dh.broadcast_bytes(pg, rank, b"" if rank == 0 else None)
    q.put((rank, lib.joined, other, dh.shard_seed_offset(rank)))
    import torch.distributed as d
    d.destroy_process_group()


def _run(target, world, *extra):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + extra) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


def test_every_rank_joins_with_rank0_nccl_id():
    res = _run(_id_worker, 2)
    ids = {joined[2] for _, joined, _, _ in res}
    assert len(ids) == 1 and len(next(iter(ids))) == 128
    assert [joined[:2] for _, joined, _, _ in res] == [(0, 2), (1, 2)]
    assert all(other == b"" for _, _, other, _ in res)
    assert res[0][3] != res[1][3]  # ranks draw different input shards


def _grad_worker(rank, world, port, q, X, Y, W, B):
    sys.path.insert(0, str(HERE))
    import torch
    import torch.distributed as dist
    from nchelp import Eng

    pg = _init(rank, world, port)
    shard = slice(rank * len(X) // world, (rank + 1) * len(X) // world)
    with Eng("ref") as e:
        x, w, b = e.t(X[shard]), e.param(W), e.param(B)
        y = e.t(Y[shard])
        loss = e.check(e.L.nc_cross_entropy(e.check(e.L.nc_linear_fn(x, w, b)), y))
        assert e.L.nc_backward(loss) == 0, e.err()
        g = np.concatenate([e.grad(w).ravel(), e.grad(b).ravel()])
    t = torch.from_numpy(g.astype(np.float64))
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=pg)  # the engine's ncclAvg: sum / world
    q.put((rank, (t / world).numpy()))
    dist.destroy_process_group()


def test_rank_average_equals_full_batch_gradient():
    sys.path.insert(0, str(HERE))
    from nchelp import REF_LIB, Eng

    if not REF_LIB.exists():
        pytest.skip("reference engine not built (make -C oracle)")
    rng = np.random.default_rng(3)
    X = rng.standard_normal((64, 20)).astype(np.float32)
    Y = rng.integers(0, 7, 64).astype(np.int32)
    W = (rng.standard_normal((7, 20)) * 0.3).astype(np.float32)
    B = rng.standard_normal(7).astype(np.float32)
    res = _run(_grad_worker, 2, X, Y, W, B)
    with Eng("ref") as e:
        x, w, b = e.t(X), e.param(W), e.param(B)
        loss = e.check(e.L.nc_cross_entropy(e.check(e.L.nc_linear_fn(x, w, b)), e.t(Y)))
        assert e.L.nc_backward(loss) == 0
        full = np.concatenate([e.grad(w).ravel(), e.grad(b).ravel()])
    for _, avg in res:
        np.testing.assert_allclose(avg, full, rtol=1e-5, atol=1e-7)


def _exit_worker(rank, world, port, q):
    """Rank 0 leaves right after the group forms (between steps: nothing in flight); rank 1's set-up
    exchange must end with an error, not wait for good."""
    import time
    from datetime import timedelta

    import torch.distributed as dist

    sys.path.insert(0, str(REPO))
    from newch_b200 import dist as dh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 0:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()  # the item is delivered before the process vanishes
        os._exit(0)
    t0 = time.time()
    try:
        dh.join_engine_group(_FakeLib(), None, dist.group.WORLD, rank, world)
        q.put((rank, "joined", time.time() - t0))
    except Exception as ex:  # the broadcast from the departed rank fails
        q.put((rank, f"error {type(ex).__name__}", time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_departed_rank_ends_the_exchange_with_an_error():
    res = _run(_exit_worker, 2)
    assert res[0][1] == "left"
    status, secs = res[1][1], res[1][2]
    assert status.startswith("error"), status
    assert secs < 60.0, secs
