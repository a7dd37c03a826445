#!/usr/bin/env python3
"""Training-step throughput of the B200 newch engine (train samples/sec), with its roofline and the
reference engine's multithreaded CPU path timed on the same host.

The workload is a recorded nc.h call sequence of the unchanged newch Python package (recorded by
tests/golden/record_traces.py): by default configuration 2, the two-block CNN trained through
compile/fit with AdamW at batch 512 per GPU. One timed step replays exactly the calls newch's fit()
makes for one batch (forward, cross entropy, zero_grad, backward, optimizer step, loss.item(),
step_end) through the C ABI.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config cfg2]
                  [--extra cfg1,cfg3,cfg4,cfg5 | --extra none]

The JSON line's headline (value, e2e, roofline, cpu_baseline) is the --config workload. Under
"configs" the same line carries shorter measurements of the other configurations (--extra): their
samples/s (rows/s for the int8 inference of config 5), host wall-clock end-to-end rate, dominant
kernel against its roof and, at N=1, the reference engine's CPU rate on a bounded sample.

Multi-GPU: launched by torch.distributed.run, one process per GPU; each rank trains on its own data
shard and the engine all-reduces the flat gradient buffer over NCCL before every update (weak
scaling; config 5 is batch-sharded inference, config 1 runs at N=1 only). Rank 0 prints one JSON
line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from newch_b200 import capi, replay  # noqa: E402
from newch_b200 import dist as dist_host  # noqa: E402

METRIC = "train samples/sec at 1/2/4/8 B200 (CNN, transformer); % HBM/tensor roofline"
REF_LIB = REPO / "oracle" / "_ref" / "libnc_ref.so"
BATCH = {"cfg1": 64, "cfg2": 512, "cfg3": 256, "cfg4": 64, "cfg5": 8192, "cfg2_stream": 512}
DESC = {
    "cfg1": "small CNN step (Conv16+ReLU+MaxPool+Linear, log_softmax+nll, Adam), batch 64",
    "cfg2": "two-block CNN via compile/fit (Conv32/64+BN+ReLU+Pool, Dropout, Linear 3136-128-10, AdamW), "
            "batch 512 per GPU",
    "cfg3": "depthwise-separable MobileNet-style step (Adam), batch 256 per GPU",
    "cfg4": "causal char TransformerEncoder LM step (4 layers, d 256, T 128, AdamW), batch 64 per GPU",
    "cfg5": "int8 quantize_ MLP inference, 8192 rows",
}
E2E_TRACE = {"cfg2": "cfg2_stream"}
UNIT = {"cfg4": "sequences/s", "cfg5": "rows/s"}
DATA = {"cfg1": "synthetic (seeded uint8 images [B,1,28,28], 10 uniform labels)",
        "cfg2": "synthetic (seeded, MNIST-shaped)", "cfg3": "synthetic (seeded N(0,1) [B,3,64,64], 100 labels)",
        "cfg4": "synthetic (seeded token ids uniform in [0,96), T=128)",
        "cfg5": "synthetic (seeded N(0,1) activations [8192,1024])"}
SETUP_DRIVER = "recorded newch call sequence replayed through the nc.h C ABI"
L2_NOTE = "flushed between timed steps (256 MiB write, outside the timed events)"
INPUTS_NOTE = ("value: the step's host-data uploads (nc_from_data) made once before the timed region, inputs "
               "resident in HBM; e2e: every step uploads its batch from pinned host memory and reads its result")


def config_dict(cfg: str, world: int) -> dict:
    """The workload description both arms report (identical keys and values)."""
    b = BATCH.get(cfg, 1)
    return {"workload": f"{cfg}: {DESC.get(cfg, cfg)}", "global_batch": b * world, "per_gpu_batch": b,
            "parallelism": f"dp{world}"}


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.25)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.out = self.proc.communicate(timeout=5)[0]
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def load_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "sm_max_mhz": d.get("sm_max_mhz", 1965.0),
                "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0, "src": "fallback"}


def compute_roof(scope: str, peaks: dict):
    """The arithmetic roof of a timed scope: (TFLOP/s, bound, how it is derived). The tensor roofs scale
    the measured bf16 GEMM by the dense-rate ratios of the B200's tensor cores (TF32 1/2, int8 2x);
    CUDA-core kernels (FFMA) take 128 fp32 FMAs per clock per SM on 148 SMs at the maximum clock."""
    b = peaks["bf16_tflops"]
    if scope.startswith("qgemm_i8"):
        return 2.0 * b, "tensor", "int8 tensor roof = 2 x measured bf16 (dense-rate ratio)"
    if "tf32" in scope or scope.startswith("conv_tap"):
        return 0.5 * b, "tensor", ("tf32 tensor roof = measured bf16 / 2 (dense-rate ratio); 3xTF32 issues three "
                                   "TF32 products per fp32 product, so its useful-FLOP ceiling is a third of it")
    return 148 * 128 * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12, "fp32", "fp32 CUDA-core roof (148 SMs x 128 FMA/clk)"


def step_io_bytes(trace: replay.Trace, start: int, end: int):
    """Host->device and device->host bytes of one step's calls (inputs uploaded, results read)."""
    h2d = d2h = 0
    for c in trace.calls[start:end]:
        name, args = c[0], c[1]
        if name in ("nc_from_data", "nc_copy_from"):
            for a in args:
                if isinstance(a, dict) and "b" in a:
                    h2d += trace.blobs[a["b"]]["n"]
        elif name == "nc_item":
            d2h += 4
        elif name == "nc_copy_to":
            d2h += int(args[2])
    return h2d, d2h


class Run:
    """A trace replayed on the B200 engine: prologue and recorded steps once, then the last recorded
    step repeated."""

    def __init__(self, lib, trace_name: str, rank: int, world: int, pg, pinned: bool = False,
                 resident: bool = False):
        self.lib = lib
        self.name = trace_name
        self.trace = replay.Trace(trace_name)
        self.rep = replay.Replayer(lib, self.trace, seed_offset=dist_host.shard_seed_offset(rank), pinned=pinned)
        self.rep.run(0, 1)  # nc_init
        self.ctx = self.rep.ctx
        if not self.ctx or not lib.nc_ok(self.ctx):
            raise RuntimeError(f"nc_init failed: {lib.nc_error(self.ctx) if self.ctx else 'NULL'}")
        if world > 1:
            dist_host.join_engine_group(lib, self.ctx, pg, rank, world)
        steps = self.trace.steps()
        self.rep.run(1, steps[-1][1])  # model set-up and every recorded step
        self.step = steps[-1]
        # resident: the repeated step's host-data uploads (nc_from_data) are made once here, so the
        # timed steps start with their inputs in HBM
        self.resident_bytes = self.rep.make_resident(*self.step) if resident else 0

    def one(self):
        self.rep.run(*self.step)


def timed_steps(run: Run, k: int, stream, flush):
    """Device time of k steps (CUDA events on the engine's stream), L2 flushed between steps."""
    import torch
    evs = []
    for _ in range(k):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        run.one()
        b.record(stream)
        evs.append((a, b))
        with torch.cuda.stream(stream):
            flush.zero_()
    torch.cuda.synchronize()
    run.lib.nc_ext_synchronize(run.ctx)
    return sum(a.elapsed_time(b) for a, b in evs) / 1e3


def wall_steps(run: Run, k: int, stream, flush):
    """Host wall-clock time of k steps through the public calls, each step timed from its first call to
    the device finishing its work (the step's loss read waits for it; a final synchronize covers calls
    after it), the L2 flush between steps outside the timed spans."""
    import torch
    total = 0.0
    for _ in range(k):
        t0 = time.perf_counter()
        run.one()
        run.lib.nc_ext_synchronize(run.ctx)
        total += time.perf_counter() - t0
        with torch.cuda.stream(stream):
            flush.zero_()
        torch.cuda.synchronize()
    return total


def roofline(run: Run, peaks: dict, steps: int = 3) -> dict:
    lib, ctx = run.lib, run.ctx
    lib.nc_ext_timing(ctx, 1)
    lib.nc_ext_timing_reset(ctx)
    for _ in range(steps):
        run.one()
    table = capi.kernel_table(lib, ctx)
    lib.nc_ext_timing(ctx, 0)
    total = sum(t[1] for t in table) or 1.0
    name, ms, cnt, fl, by = max(table, key=lambda t: t[1])
    per_launch_ms = ms / max(cnt, 1)
    # the binding roof: a kernel with FLOPs is tensor-bound only when its arithmetic takes longer at the
    # tensor peak than its algorithmic bytes take at the HBM peak
    cpeak, cbound, cnote = compute_roof(name, peaks)
    t_compute = fl / (cpeak * 1e12)
    t_hbm = by / (peaks["hbm_gbs"] * 1e9)
    if fl > 0 and t_compute >= t_hbm:
        achieved = fl / max(cnt, 1) / (per_launch_ms / 1e3) / 1e12
        peak, unit, bound, note = round(cpeak, 1), "TFLOP/s", cbound, cnote
    else:
        achieved = by / max(cnt, 1) / (per_launch_ms / 1e3) / 1e9
        peak, unit, bound, note = peaks["hbm_gbs"], "GB/s", "hbm", "measured HBM copy bandwidth"
    # DRAM bytes per call of this scope in this workload, from one-kernel ncu captures (profiles/)
    traffic = None
    tf = REPO / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(run.name, {}).get(name)
    kernels = sorted(table, key=lambda t: -t[1])[:16]
    sec = max(per_launch_ms, 1e-9) / 1e3
    return {"kernel": name, "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic, "peak_src": peaks["src"] + " (MEASURED_PEAKS.json): " + note,
            "algorithmic_bytes_per_launch": round(by / max(cnt, 1)), "flops_per_launch": round(fl / max(cnt, 1)),
            "achieved_gbs": round(by / max(cnt, 1) / sec / 1e9, 1),
            "achieved_tflops": round(fl / max(cnt, 1) / sec / 1e12, 2),
            "share_of_step_kernel_time": round(ms / total, 3), "launches_per_step": cnt / steps,
            "top_kernels": [{"name": t[0], "ms_per_step": round(t[1] / steps, 4), "share": round(t[1] / total, 3)}
                            for t in kernels]}


def cpu_reference(trace_name: str, budget_s: float, max_steps: int, warmup: int = 1):
    """The reference engine (its multithreaded AVX2 tier, all host cores) replaying the same trace;
    returns the step times, the thread count and the kernel tier, and frees its context."""
    lib = capi.load(REF_LIB)
    tr = replay.Trace(trace_name)
    rep = replay.Replayer(lib, tr)
    steps = tr.steps()
    rep.run(0, steps[-1][1])
    s = steps[-1]
    for _ in range(warmup):
        rep.run(*s)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max_steps and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        rep.run(*s)
        times.append(time.perf_counter() - t0)
    ctx = rep.ctx
    cores = lib.nc_num_threads(ctx)
    backend = lib.nc_kernel_backend(ctx).decode()
    lib.nc_free_ctx(ctx)
    return times, cores, backend


def max_over_ranks(pg, secs: float) -> float:
    if not pg:
        return secs
    import torch
    import torch.distributed as dist
    t = torch.tensor([secs], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
    return float(t[0])


def measure(lib, cfg: str, rank: int, world: int, pg, local: int, steps: int, warmup: int, flush, *,
            extras: bool = True, cpu_budget_s: float = 20.0, cpu_steps: int = 30, clocks=None) -> dict:
    """One workload on this rank's GPU: device-timed steps (max over ranks), then the wall-clock
    end-to-end rate, the dominant kernel against its roof and (rank 0 at N=1) the CPU reference."""
    import torch
    import torch.distributed as dist
    batch = BATCH.get(cfg, 1)
    run = Run(lib, cfg, rank, world, pg, resident=True)
    stream = torch.cuda.ExternalStream(lib.nc_ext_stream(run.ctx), device=torch.device("cuda", local))
    for _ in range(warmup):
        run.one()
    lib.nc_ext_synchronize(run.ctx)
    if pg:
        dist.barrier(pg)
    torch.cuda.synchronize()
    l0 = lib.nc_ext_launch_count(run.ctx)
    if clocks is not None:  # nvidia-smi samples span the timed steps only
        with clocks:
            secs = timed_steps(run, steps, stream, flush)
    else:
        secs = timed_steps(run, steps, stream, flush)
    launches = (lib.nc_ext_launch_count(run.ctx) - l0) // max(steps, 1)
    if pg:
        dist.barrier(pg)
    secs = max_over_ranks(pg, secs)
    if not lib.nc_ok(run.ctx):
        raise SystemExit(f"{cfg}: engine error: {lib.nc_error(run.ctx).decode()}")
    res = {"value": round(batch * world * steps / secs, 3), "unit": UNIT.get(cfg, "samples/s"),
           "ms_per_step": round(1e3 * secs / steps, 4), "steps": steps, "warmup": warmup,
           "gpu_launches": int(launches), "gemm": lib.nc_ext_gemm_mode(run.ctx).decode(),
           "config": config_dict(cfg, world), "resident_input_bytes": run.resident_bytes}
    if extras:
        # end to end: the step's batch uploaded from pinned host memory through the public calls
        et = E2E_TRACE.get(cfg, cfg)
        erun = Run(lib, et, rank, world, pg, pinned=True)
        estream = torch.cuda.ExternalStream(lib.nc_ext_stream(erun.ctx), device=torch.device("cuda", local))
        for _ in range(max(warmup, 3)):
            erun.one()
        ek = max(10, min(steps, 200))
        if pg:
            dist.barrier(pg)
        ewall = max_over_ranks(pg, wall_steps(erun, ek, estream, flush))
        edev = max_over_ranks(pg, timed_steps(erun, ek, estream, flush))
        h2d, d2h = step_io_bytes(erun.trace, *erun.step)
        res["e2e"] = {"value": round(batch * world * ek / ewall, 3), "unit": res["unit"], "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": d2h, "trace": et, "steps": ek,
                      "timing": "host wall clock around each step's public calls, to the device finishing",
                      "value_device_events": round(batch * world * ek / edev, 3)}
        lib.nc_ext_synchronize(erun.ctx)
        lib.nc_free_ctx(erun.ctx)
        # every rank steps (each step all-reduces gradients); rank 0 reports its kernel table
        res["roofline"] = roofline(run, load_peaks())
        res["cpu_baseline"] = None
        if rank == 0 and world == 1 and REF_LIB.exists():
            times, cores, backend = cpu_reference(cfg, budget_s=cpu_budget_s, max_steps=cpu_steps)
            res["cpu_baseline"] = {
                "value": round(batch * len(times) / sum(times), 3), "unit": res["unit"], "cores": cores,
                "kind": "reference",
                "sample": f"{len(times)} steps of {cfg} (median {1e3 * statistics.median(times):.1f} ms), "
                          f"newch engine {backend} tier built from its sources, same recorded calls"}
    lib.nc_ext_synchronize(run.ctx)
    lib.nc_free_ctx(run.ctx)
    return res


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="cfg2")
    ap.add_argument("--extra", default="cfg1,cfg3,cfg4,cfg5",
                    help="other configurations measured briefly into the line's 'configs' ('none': skip)")
    ap.add_argument("--no-extras", action="store_true", help="skip e2e, roofline, CPU baseline and --extra")
    args = ap.parse_args()
    rank, world, local = dist_env()
    cfg = args.config
    batch = BATCH.get(cfg, 1)
    extra = [] if args.no_extras or args.extra == "none" else [c for c in args.extra.split(",") if c and c != cfg]
    if world > 1:
        extra = [c for c in extra if c != "cfg1"]  # config 1 is a single-GPU configuration

    if args.impl == "reference":
        if rank != 0:
            return 0
        if not REF_LIB.exists():
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libnc_ref.so was not built"}))
            return 0
        times, cores, backend = cpu_reference(cfg, budget_s=120.0, max_steps=max(args.steps, 1),
                                               warmup=max(args.warmup, 1))
        t = sum(times)
        value = batch * len(times) / t
        out = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT.get(cfg, "samples/s"),
               "n_gpus": world, "steps": len(times), "warmup": args.warmup, "ms_per_step": round(1e3 * t / len(times), 3),
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
               "data": DATA.get(cfg, "synthetic"), "config": config_dict(cfg, world),
               "setup": {"driver": SETUP_DRIVER, "engine": f"newch reference engine, {backend} tier, {cores} threads"},
               "cpu_baseline": {"value": round(value, 3), "unit": UNIT.get(cfg, "samples/s"), "cores": cores,
                                "kind": "reference",
                                "sample": f"{len(times)} {cfg} steps of {batch} samples on one host process, newch "
                                          f"engine ({backend} tier) built from its sources, same recorded calls"},
               "e2e": {"value": round(value, 3), "unit": UNIT.get(cfg, "samples/s"), "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(out), flush=True)
        return 0

    os.environ["NC_DEVICE"] = str(local)
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        os.environ.setdefault("NC_DP_TIMEOUT", "60")  # a rank that never joins ends the run, not hangs it
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
        pg = dist.group.WORLD
    lib = capi.load_b200()
    if lib.nc_ext_device_count() < 1:
        raise SystemExit("no CUDA device")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")

    clk = Clocks(local)
    head = measure(lib, cfg, rank, world, pg, local, args.steps, args.warmup, flush, extras=not args.no_extras,
                   clocks=clk)
    others = {}
    for c in extra:
        k = max(3, min(args.steps, {"cfg1": 50, "cfg5": 10}.get(c, 10)))
        others[c] = measure(lib, c, rank, world, pg, local, k, max(3, min(args.warmup, 5)), flush,
                            cpu_budget_s={"cfg1": 5.0}.get(c, 12.0), cpu_steps={"cfg1": 30}.get(c, 3))
    if rank == 0:
        out = {"metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": DATA.get(cfg, "synthetic"),
               "config": config_dict(cfg, world),
               "setup": {"gemm": head["gemm"], "l2": L2_NOTE, "driver": SETUP_DRIVER, "inputs": INPUTS_NOTE},
               "gpu_launches": head["gpu_launches"], "clocks": clk.summary(), "e2e": head.get("e2e"),
               "roofline": head.get("roofline"), "cpu_baseline": head.get("cpu_baseline"), "configs": others}
        print(json.dumps(out), flush=True)
    if pg:
        dist.barrier(pg)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
