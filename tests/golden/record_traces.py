"""Records the nc.h call sequence that the unchanged newch Python package issues for each benchmark
configuration, so the B200 engine can be driven (and checked) through exactly the calls a newch
user's script makes, on a machine where the newch package itself is not installed.

How: the configuration's PyTorch-style script (``import newch as torch``) runs against the reference
engine with every ctypes entry point of ``newch._lib.lib`` wrapped. Each call is stored with its
arguments, tensor pointers are replaced by handle numbers, host buffers by blobs (seeded synthetic
inputs by their generator spec instead of their bytes), and scalar results (losses from
``nc_item``) and copied-out buffers are kept as golden values.

Test-fixture tooling: run it on a machine where a newch checkout (its Python package and the
engine built from its sources) is available:

    make -C oracle REF=<newch checkout>
    python tests/golden/record_traces.py --ref <newch checkout> [--lib oracle/_ref/libnc_ref.so] [names...]

Output: ``newch_b200/workloads/<name>.json.gz`` (the workload definitions bench.py, smoke() and the
tests replay).
"""

from __future__ import annotations

import argparse
import base64
import ctypes
import gzip
import hashlib
import importlib
import json
import math
import os
import sys
import zlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from newch_b200 import synth  # noqa: E402

DT_SIZE = {0: 4, 1: 4, 2: 2, 3: 1, 4: 1}
INLINE_MAX = 1 << 16  # golden outputs above this are kept as summaries


class Recorder:
    """Wraps every function of a ctypes library (in place) and logs the calls."""

    def __init__(self, lib, signatures):
        self.lib = lib
        self.calls: list = []
        self.addr2h: dict = {}
        self.next_h = 1
        self.blobs: dict = {}
        self.blob_by_hash: dict = {}
        self.marks: dict = {}
        self.warnings: list = []
        self.active = True
        for name, (res, args) in signatures.items():
            orig = getattr(lib, name)
            setattr(lib, name, self._wrap(name, orig, res, args))

    # -- handles and blobs ------------------------------------------------------------------
    def _h(self, addr):
        if addr is None or addr == 0:
            return None
        if isinstance(addr, ctypes.c_void_p):
            addr = addr.value
            if not addr:
                return None
        h = self.addr2h.get(int(addr))
        if h is None:
            raise RuntimeError(f"pointer {addr:#x} was never returned by a recorded call")
        return h

    def _new_h(self, addr):
        if not addr:
            return None
        h = self.next_h
        self.next_h += 1
        self.addr2h[int(addr)] = h
        return h

    def _blob(self, data: bytes) -> str:
        key = hashlib.sha256(data).hexdigest()
        if key in self.blob_by_hash:
            return self.blob_by_hash[key]
        bid = f"b{len(self.blobs)}"
        spec = synth.spec_for(data)
        if spec is not None:
            self.blobs[bid] = {"gen": spec, "n": len(data)}
        else:
            self.blobs[bid] = {"zlib": base64.b64encode(zlib.compress(data, 6)).decode(), "n": len(data)}
        self.blob_by_hash[key] = bid
        return bid

    @staticmethod
    def _summary(data: bytes) -> dict:
        a = np.frombuffer(data, dtype=np.float32)
        step = max(1, a.size // 4096)
        return {"sha256": hashlib.sha256(data).hexdigest(), "n": len(data), "sum": float(a.astype(np.float64).sum()),
                "sumsq": float((a.astype(np.float64) ** 2).sum()), "stride": step,
                "sample": base64.b64encode(a[::step].tobytes()).decode()}

    def mark(self, name: str) -> None:
        self.marks[name] = len(self.calls)

    # -- wrapping -------------------------------------------------------------------------
    def _wrap(self, name, orig, res, argtypes):
        rec = self

        def call(*args):
            if not rec.active:
                return orig(*args)
            enc, post = rec._encode(name, args, argtypes)
            r = orig(*args)
            entry = [name, enc, rec._encode_ret(name, r, res)]
            if post is not None:
                extra = post(r)
                if extra is not None:
                    entry.append(extra)
            rec.calls.append(entry)
            return r

        call.__name__ = name
        return call

    def _encode_ret(self, name, r, res):
        if res is ctypes.c_void_p:
            if name in ("nc_data_f32", "nc_data_i32", "nc_optim_state"):
                self.warnings.append(f"{name}: host pointer handed out; direct memory access is not recorded")
                return None
            return {"h": self._new_h(r)} if r else None
        if res is ctypes.c_char_p:
            return r.decode(errors="replace") if r is not None else None
        if res in (ctypes.c_float,):
            return float(r)
        if res in (ctypes.c_int, ctypes.c_int64):
            return int(r)
        return None  # structs, pointers to host structs, void

    def _encode(self, name, args, argtypes):
        enc = []
        post = None
        for i, (a, t) in enumerate(zip(args, argtypes)):
            enc.append(self._encode_arg(name, i, a, t, args))
        if name == "nc_copy_to":
            dst, nbytes = args[1], int(args[2])

            def post(r, dst=dst, nbytes=nbytes):
                if not r:
                    return None
                data = ctypes.string_at(dst, nbytes)
                if nbytes <= INLINE_MAX:
                    return {"out": self._blob(data)}
                return {"out_summary": self._summary(data)}
        elif name == "nc_quantize_rows":
            outp = args[1]

            def post(r, outp=outp):
                return {"out_h": self._new_h(outp[0]) if outp[0] else None}
        return enc, post

    def _encode_arg(self, name, i, a, t, args):
        P, I64P = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)
        PP = ctypes.POINTER(ctypes.c_void_p)
        if name == "nc_from_data" and i == 2:
            n = math.prod(int(args[4][k]) for k in range(int(args[3])))
            nbytes = n * DT_SIZE[int(args[1])]
            return {"b": self._blob(ctypes.string_at(a, nbytes))} if a else None
        if name == "nc_copy_from" and i == 1:
            return {"b": self._blob(ctypes.string_at(a, int(args[2])))} if a else None
        if name == "nc_copy_to" and i == 1:
            return {"o": int(args[2])}
        if name == "nc_quantize_rows" and i == 1:
            return {"o": 1}
        if t is PP:
            counts = {"nc_cat": 0, "nc_backward_ex": 3, "nc_sgd": 2, "nc_adam": 2, "nc_adamw": 2, "nc_rmsprop": 2,
                      "nc_clip_grad_norm": 1, "nc_save": 2, "nc_load": 2, "nc_sequential": 1, "nc_parameters": 2}
            n = int(args[counts[name]]) if name in counts else 0
            if a is None or n == 0:
                return {"hl": []}
            return {"hl": [self._h(a[k]) for k in range(n)]}
        if t is P:
            return {"h": self._h(a)} if a else None
        if t is I64P:
            return {"s": [int(v) for v in a]} if a is not None else None
        if t is ctypes.c_char_p:
            return {"str": a.decode() if isinstance(a, bytes) else a}
        if isinstance(t, type) and issubclass(t, ctypes.Structure):
            return {"st": [float(getattr(a, f)) for f, _ in t._fields_]}
        if getattr(t, "_type_", None) is not None and isinstance(getattr(t, "_type_"), type) and issubclass(
                t._type_, ctypes.Structure):  # POINTER(Config) via byref
            obj = getattr(a, "_obj", a)
            return {"st": [getattr(obj, f) for f, _ in obj._fields_]}
        if getattr(t, "__name__", "") == "LP_c_char_p":
            n = int(args[2])
            return {"strs": [a[k].decode() for k in range(n)]}
        if isinstance(a, float):
            return {"f": a} if not math.isfinite(a) else a
        return a

    def to_json(self, meta: dict) -> dict:
        steps = [i for i, c in enumerate(self.calls) if c[0] == "nc_step_end"]
        return {"format": "nc-trace-1", "meta": meta, "marks": self.marks, "step_ends": steps,
                "calls": self.calls, "blobs": self.blobs, "warnings": sorted(set(self.warnings))}


# ---------------------------------------------------------------------------------------------
# The configurations, written the way a newch user writes them (only the imports differ from a
# PyTorch script). ``nc`` is the newch package, ``nn`` newch.net, ``F`` newch.net.functional.
# ---------------------------------------------------------------------------------------------

def cfg1_small_cnn(nc, nn, F, rec, *, batch=64, steps=3, seed=1):
    """Conv2d(1,16,3,1,1)+bias -> ReLU -> MaxPool2d(2) -> flatten -> Linear(3136,10) -> log_softmax ->
    nll_loss, Adam lr 1e-3; input uint8 [B,1,28,28] / 255, labels in [0,10)."""
    ctx = nc.Context(seed=seed)
    nc.set_default_context(ctx)
    conv = nn.Conv2d(1, 16, 3, 1, 1)
    fc = nn.Linear(16 * 14 * 14, 10)
    params = [conv.weight, conv.bias, fc.weight, fc.bias]
    opt = nc.optim.Adam(params, lr=1e-3)
    rec.mark("train_begin")
    for s in range(steps):
        xb = synth.uniform_u8(seed * 1000 + s, (batch, 1, 28, 28))
        yb = synth.labels(seed * 1000 + s, batch, 10)
        x = nc.tensor(xb)
        y = nc.tensor(yb)
        h = F.max_pool2d(F.relu(conv(x.float() / 255)), 2)
        out = F.log_softmax(fc(h.flatten(1)), dim=1)
        loss = F.nll_loss(out, y)
        opt.zero_grad()
        loss.backward()
        opt.step()
        loss.item()
        ctx.step_end()
    rec.mark("train_end")
    for p in params:
        p.tolist()
    return ctx


def cfg2_two_block_cnn(nc, nn, F, rec, *, batch=512, batches=4, seed=2):
    """Two-block CNN via compile/fit: Conv(1,32)+BN+ReLU+Pool, Conv(32,64)+BN+ReLU+Pool, Flatten,
    Dropout(0.25), Linear(3136,128), ReLU, Linear(128,10); cross_entropy; AdamW lr 1e-3 wd 0.01."""
    ctx = nc.Context(seed=seed)
    nc.set_default_context(ctx)
    model = nn.Sequential(
        nn.Conv2d(1, 32, 3, padding=1), nn.BatchNorm2d(32), nn.ReLU(), nn.MaxPool2d(2),
        nn.Conv2d(32, 64, 3, padding=1), nn.BatchNorm2d(64), nn.ReLU(), nn.MaxPool2d(2),
        nn.Flatten(), nn.Dropout(0.25), nn.Linear(64 * 7 * 7, 128), nn.ReLU(), nn.Linear(128, 10))
    model.compile(nc.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.01), "cross_entropy")
    n = batch * batches
    x = synth.uniform_f32(seed * 1000, (n, 1, 28, 28))
    y = synth.labels(seed * 1000, n, 10)
    rec.mark("train_begin")
    model.fit(x, y, batch_size=batch, epochs=1, shuffle=True, seed=seed, verbose=0)
    rec.mark("train_end")
    for p in model.parameters():
        p.tolist()
    return ctx


def cfg2_stream(nc, nn, F, rec, *, batch=512, batches=4, seed=2):
    """Config 2's model and optimizer fed through fit() from host batches: each step uploads its
    batch [B,1,28,28] f32 and labels from host memory (the end-to-end path)."""
    ctx = nc.Context(seed=seed)
    nc.set_default_context(ctx)
    model = nn.Sequential(
        nn.Conv2d(1, 32, 3, padding=1), nn.BatchNorm2d(32), nn.ReLU(), nn.MaxPool2d(2),
        nn.Conv2d(32, 64, 3, padding=1), nn.BatchNorm2d(64), nn.ReLU(), nn.MaxPool2d(2),
        nn.Flatten(), nn.Dropout(0.25), nn.Linear(64 * 7 * 7, 128), nn.ReLU(), nn.Linear(128, 10))
    model.compile(nc.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.01), "cross_entropy")
    xs, ys = [], []
    for b in range(batches):
        xs.append(synth.uniform_f32(seed * 1000 + 17 + b, (batch, 1, 28, 28)))
        ys.append(synth.labels(seed * 1000 + 17 + b, batch, 10))

    class Loader:
        def __iter__(self):
            return iter(list(zip(xs, ys)))

    rec.mark("train_begin")
    model.fit(Loader(), epochs=1, verbose=0)
    rec.mark("train_end")
    for p in model.parameters():
        p.tolist()
    return ctx


def cfg3_depthwise(nc, nn, F, rec, *, batch=256, steps=3, seed=3, chans=(32, 64, 128, 256, 256), hw=64):
    """MobileNet-style: Conv(3,32,3,s2,p1)+BN+Hardswish, 4x [dw Conv(C,C,3,groups=C,'same')+BN+Hardswish,
    pw Conv(C,C',1)+BN+Hardswish], mean over H,W, Linear(256,100); cross_entropy; Adam."""
    ctx = nc.Context(seed=seed)
    nc.set_default_context(ctx)

    class Net(nn.Module):
        def __init__(self):
            super().__init__()
            layers = [nn.Conv2d(3, chans[0], 3, stride=2, padding=1), nn.BatchNorm2d(chans[0]), nn.Hardswish()]
            for c, c2 in zip(chans[:-1], chans[1:]):
                layers += [nn.Conv2d(c, c, 3, groups=c, padding="same"), nn.BatchNorm2d(c), nn.Hardswish(),
                           nn.Conv2d(c, c2, 1), nn.BatchNorm2d(c2), nn.Hardswish()]
            self.features = nn.Sequential(*layers)
            self.head = nn.Linear(chans[-1], 100)

        def forward(self, x):
            return self.head(self.features(x).mean((2, 3)))

    model = Net()
    opt = nc.optim.Adam(model.parameters(), lr=1e-3)
    rec.mark("train_begin")
    for s in range(steps):
        x = nc.tensor(synth.normal_f32(seed * 1000 + s, (batch, 3, hw, hw)))
        y = nc.tensor(synth.labels(seed * 1000 + s, batch, 100))
        loss = F.cross_entropy(model(x), y)
        opt.zero_grad()
        loss.backward()
        opt.step()
        loss.item()
        ctx.step_end()
    rec.mark("train_end")
    for p in model.parameters():
        p.tolist()
    return ctx


def cfg4_transformer(nc, nn, F, rec, *, batch=64, T=128, steps=3, seed=4, d=256, heads=8, ff=1024, layers=4,
                     vocab=96):
    """Causal char-level TransformerEncoder LM: Embedding(96,256), 4x TransformerEncoderLayer(256, 8, 1024,
    GELU, batch_first, post-norm, dropout 0.1) with an integer causal mask, Linear(256,96);
    next-token cross_entropy; AdamW lr 3e-4."""
    ctx = nc.Context(seed=seed)
    nc.set_default_context(ctx)

    class LM(nn.Module):
        def __init__(self):
            super().__init__()
            self.tok = nn.Embedding(vocab, d)
            layer = nn.TransformerEncoderLayer(d, heads, ff, activation=nn.GELU(), batch_first=True)
            self.encoder = nn.TransformerEncoder(layer, layers)
            self.head = nn.Linear(d, vocab)
            rows = nc.tensor(list(range(T))).reshape(T, 1)
            with nc.persistent():
                self.causal = nc.tensor(list(range(T))) > rows  # 1 = future position, not attended

        def forward(self, idx):
            return self.head(self.encoder(self.tok(idx), mask=self.causal))

    model = LM()
    opt = nc.optim.AdamW(model.parameters(), lr=3e-4)
    rec.mark("train_begin")
    for s in range(steps):
        ids = synth.labels(seed * 1000 + s, batch * (T + 1), vocab).reshape(batch, T + 1)
        x = nc.tensor(np.ascontiguousarray(ids[:, :T]))
        y = nc.tensor(np.ascontiguousarray(ids[:, 1:]))
        opt.zero_grad()
        logits = model(x)
        loss = F.cross_entropy(logits.reshape(-1, vocab), y.reshape(-1))
        loss.backward()
        opt.step()
        loss.item()
        ctx.step_end()
    rec.mark("train_end")
    for p in model.parameters():
        p.tolist()
    return ctx


def cfg5_int8_mlp(nc, nn, F, rec, *, rows=8192, steps=2, seed=5, dims=(1024, 4096, 4096, 1024, 10)):
    """int8 quantize_ inference: Linear(1024,4096)->GELU->Linear(4096,4096)->GELU->Linear(4096,1024)->GELU->
    Linear(1024,10), converted by newch.quantize_; fp32 N(0,1) activations, forward under no_grad."""
    ctx = nc.Context(seed=seed)
    nc.set_default_context(ctx)
    layers = []
    for i in range(len(dims) - 1):
        layers.append(nn.Linear(dims[i], dims[i + 1]))
        if i < len(dims) - 2:
            layers.append(nn.GELU())
    model = nn.Sequential(*layers)
    nc.quantize_(model)
    rec.mark("train_begin")
    with nc.no_grad():
        for s in range(steps):
            x = nc.tensor(synth.normal_f32(seed * 1000 + s, (rows, dims[0])))
            out = model(x)
            out.tolist()
            del out, x
            ctx.step_end()
    rec.mark("train_end")
    return ctx


CONFIGS = {
    # full sizes (the five benchmark configurations)
    "cfg1": (cfg1_small_cnn, {}),
    "cfg2": (cfg2_two_block_cnn, {}),
    "cfg3": (cfg3_depthwise, {}),
    "cfg4": (cfg4_transformer, {}),
    "cfg5": (cfg5_int8_mlp, {}),
    "cfg2_stream": (cfg2_stream, {}),
    # small cases of the same graphs for fast parity tests
    "cfg1_small": (cfg1_small_cnn, {"batch": 8}),
    "cfg2_small": (cfg2_two_block_cnn, {"batch": 16, "batches": 3}),
    "cfg3_small": (cfg3_depthwise, {"batch": 4, "hw": 16, "chans": (8, 16, 16)}),
    "cfg4_small": (cfg4_transformer, {"batch": 2, "T": 16, "d": 32, "heads": 4, "ff": 64, "layers": 2}),
    "cfg5_small": (cfg5_int8_mlp, {"rows": 32, "dims": (64, 128, 32, 10)}),
}


def record(name: str, ref: Path, libpath: Path, out_dir: Path) -> Path:
    os.environ["NEWCH_LIB"] = str(libpath)
    sys.path.insert(0, str(ref))
    for m in [m for m in sys.modules if m == "newch" or m.startswith("newch.")]:
        del sys.modules[m]
    nc = importlib.import_module("newch")
    nn = importlib.import_module("newch.net")
    F = importlib.import_module("newch.net.functional")
    L = importlib.import_module("newch._lib")
    rec = Recorder(L.lib, L._SIGNATURES)
    fn, kw = CONFIGS[name]
    ctx = fn(nc, nn, F, rec, **kw)
    rec.active = False
    meta = {"name": name, "doc": (fn.__doc__ or "").strip(), "kwargs": {k: list(v) if isinstance(v, tuple) else v
                                                                        for k, v in kw.items()},
            "recorded_with": "newch reference engine (" + L.lib.nc_kernel_backend(ctx._p).decode() + " tier)",
            "synth": synth.VERSION}
    out = out_dir / f"{name}.json.gz"
    with gzip.open(out, "wt") as f:
        json.dump(rec.to_json(meta), f, separators=(",", ":"))
    os._exit_code = 0
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="newch source checkout (its Python package is imported)")
    ap.add_argument("--lib", default=str(REPO / "oracle" / "_ref" / "libnc_ref.so"))
    ap.add_argument("--out", default=str(REPO / "newch_b200" / "workloads"))
    ap.add_argument("names", nargs="*", default=list(CONFIGS))
    args = ap.parse_args()
    import subprocess
    if len(args.names) > 1:  # one process per config: the engine context and its RNG start fresh
        rc = 0
        for n in args.names:
            rc |= subprocess.call([sys.executable, __file__, "--ref", args.ref, "--lib", args.lib, "--out", args.out, n])
        return rc
    out = record(args.names[0], Path(args.ref), Path(args.lib), Path(args.out))
    print(f"{out} ({out.stat().st_size / 1e3:.1f} kB)", flush=True)
    os._exit(0)  # the reference package can crash in Tensor.__del__ at interpreter shutdown


if __name__ == "__main__":
    sys.exit(main())
