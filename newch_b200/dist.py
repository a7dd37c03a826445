"""Host side of data-parallel runs: one process per GPU under torch.distributed (the harness's
process group, gloo, carries only set-up bytes); gradients are averaged by the engine itself with
one NCCL all-reduce of its flat gradient buffer per optimizer step (include/nc_ext.h).

Each rank replays the same recorded newch calls with its own input shard (generator seed offset per
rank) and the same initial weights (the same context seed)."""

from __future__ import annotations

import ctypes

SHARD_SEED_STRIDE = 7919  # input generator offset between ranks


def shard_seed_offset(rank: int) -> int:
    return rank * SHARD_SEED_STRIDE


def broadcast_bytes(pg, rank: int, payload: bytes | None, cap: int = 512) -> bytes:
    """Rank 0's payload (at most cap bytes) on every rank of the process group."""
    import torch
    import torch.distributed as dist

    t = torch.zeros(cap + 2, dtype=torch.uint8)
    if rank == 0:
        if payload is None or len(payload) > cap:
            raise ValueError("rank 0 needs a payload of at most cap bytes")
        n = len(payload)
        t[0], t[1] = n & 0xFF, n >> 8
        if n:
            t[2:2 + n] = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
    dist.broadcast(t, 0, group=pg)
    n = int(t[0]) | (int(t[1]) << 8)
    return bytes(t[2:2 + n].tolist())


def join_engine_group(lib, ctx, pg, rank: int, world: int) -> None:
    """Rank 0 creates the NCCL id, every rank receives it and joins the engine's all-reduce group."""
    payload = None
    if rank == 0:
        buf = (ctypes.c_char * 512)()
        n = lib.nc_ext_nccl_unique_id(buf, 512)
        if n <= 0:
            raise RuntimeError("nc_ext_nccl_unique_id failed")
        payload = buf.raw[:n]
    idb = broadcast_bytes(pg, rank, payload)
    st = lib.nc_ext_dp_init(ctx, rank, world, idb, len(idb))
    if st != 0:
        raise RuntimeError(f"dp init failed: {lib.nc_error(ctx)}")
