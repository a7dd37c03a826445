"""A small two-block-CNN training loop written against the nc.h C ABI, shared by the data-parallel
parity test (tests/test_gpu_dp.py): the reference engine runs it with gradient accumulation over the
ranks' micro-batches, each B200 rank runs its own micro-batch of every step.

Model (config 2's first block at a small size): Conv2d(1, 8, 3, p=1, no bias) -> BatchNorm2d(8) -> ReLU ->
MaxPool2d(2) -> flatten -> Dropout(0.25) -> Linear(1568, 10) -> cross_entropy; AdamW lr 1e-3,
weight decay 0.01. Initial weights come from the context's seeded stream, so every engine and every
rank starts from the same ones. The convolution has no bias: a bias in front of BatchNorm gets only a
rounding-noise gradient, Adam moves it by lr times the sign of that noise, and the BatchNorm running
mean tracks the bias, so it would compare the two engines' rounding noise rather than the data-parallel
update.

Run as a script, it is one B200 rank of a data-parallel group (the engine joins the group from the
NC_RANK / NC_WORLD_SIZE / NC_NCCL_ID_FILE environment at nc_init) and writes its results to the
.npz path given on the command line.
"""

from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent))

from nchelp import Eng, capi  # noqa: E402

B, C1, STEPS, P_DROP = 16, 8, 3, 0.25
FLAT = C1 * 14 * 14
DRAWS_PER_STEP = B * FLAT  # one dropout over [B, FLAT] per micro-batch step


def batch(step: int, part: int):
    """Micro-batch `part` of step `step`: images uniform in [0, 1), labels in [0, 10)."""
    rng = np.random.default_rng(1000 * step + part)
    return rng.random((B, 1, 28, 28), dtype=np.float32), rng.integers(0, 10, B).astype(np.int32)


def _uniform_param(e: Eng, shape, bound):
    n, shp = capi.shape_arg(shape)
    init = e.check(e.L.nc_rand_uniform(e.ctx, -bound, bound, n, shp))
    return e.check(e.L.nc_parameter(e.ctx, init, n, shp))


def build(e: Eng):
    L = e.L
    L.nc_persistent_begin(e.ctx)
    p = {"conv_w": _uniform_param(e, (C1, 1, 3, 3), 1 / 3),
         "bn_w": e.check(L.nc_parameter(e.ctx, e.t(np.ones(C1, np.float32)), *capi.shape_arg((C1,)))),
         "bn_b": e.check(L.nc_parameter(e.ctx, None, *capi.shape_arg((C1,)))),
         "fc_w": _uniform_param(e, (10, FLAT), FLAT ** -0.5), "fc_b": _uniform_param(e, (10,), FLAT ** -0.5)}
    stats = {"bn_rm": e.t(np.zeros(C1, np.float32)), "bn_rv": e.t(np.ones(C1, np.float32))}
    L.nc_persistent_end(e.ctx)
    names = list(p)
    arr = capi.ptr_array([p[k] for k in names])
    opt = e.check(L.nc_adamw(e.ctx, arr, len(names), capi.OptimOpts(1e-3, 0.0, 0.01, 0.0, 0.0, 0.0)))
    return p, stats, opt


def forward_loss(e: Eng, p, stats, x, y):
    L = e.L
    h = e.check(L.nc_conv2d_ex(e.t(x), p["conv_w"], None, 1, 1, 1, 1, 1, 1, 1))
    h = e.check(L.nc_batch_norm(h, p["bn_w"], p["bn_b"], stats["bn_rm"], stats["bn_rv"], 1, 0.1, 1e-5))
    h = e.check(L.nc_max_pool2d(e.check(L.nc_relu(h)), 2, 2, 2, 2, 0, 0))
    h = e.check(L.nc_reshape(h, *capi.shape_arg((B, FLAT))))
    h = e.check(L.nc_dropout(h, P_DROP))
    logits = e.check(L.nc_linear_fn(h, p["fc_w"], p["fc_b"]))
    return e.check(L.nc_cross_entropy(logits, e.t(y)))


def results(e: Eng, p, stats, losses):
    out = {k: e.np(v) for k, v in p.items()}
    out.update({k: e.np(v) for k, v in stats.items()})
    out["losses"] = np.array(losses, np.float32)
    return out


def run_accumulated(which: str, world: int) -> dict:
    """One context steps through every rank's micro-batch in rank order with gradient accumulation
    over `world` micro-batches: the update data-parallel training must reproduce."""
    with Eng(which, seed=7) as e:
        p, stats, opt = build(e)
        e.L.nc_optim_set_accumulation(opt, world)
        losses = []
        for s in range(STEPS):
            for r in range(world):
                e.L.nc_optim_zero_grad(opt)
                loss = forward_loss(e, p, stats, *batch(s, r))
                losses.append(e.L.nc_item(loss))
                assert e.L.nc_backward(loss) == 0, e.err()
                e.L.nc_optim_step(opt)
                e.step_end()
        out = results(e, p, stats, losses)
        assert e.ok(), e.err()
        e.L.nc_optim_free(opt)
        return out


def run_rank(rank: int, world: int) -> dict:
    """This process's rank: its own micro-batch of every step; gradients averaged by the engine."""
    with Eng("b200", seed=7) as e:
        assert e.L.nc_ext_dp_world(e.ctx) == world, e.err()
        p, stats, opt = build(e)
        assert e.L.nc_ext_dp_rng_stride(e.ctx, DRAWS_PER_STEP) == 0, e.err()
        losses = []
        for s in range(STEPS):
            e.L.nc_optim_zero_grad(opt)
            loss = forward_loss(e, p, stats, *batch(s, rank))
            losses.append(e.L.nc_item(loss))
            assert e.L.nc_backward(loss) == 0, e.err()
            e.L.nc_optim_step(opt)
            e.step_end()
        out = results(e, p, stats, losses)
        assert e.ok(), e.err()
        e.L.nc_optim_free(opt)
        return out


if __name__ == "__main__":
    import os
    rank, world = int(os.environ["NC_RANK"]), int(os.environ["NC_WORLD_SIZE"])
    np.savez(sys.argv[1], **run_rank(rank, world))
    sys.stdout.flush()
    _ = ctypes  # the engine library is released with the process
