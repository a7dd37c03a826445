"""Replays a recorded nc.h call sequence (a workload trace) against any library with the newch C ABI.

A trace is what the unchanged newch Python package called for one benchmark configuration (see
newch_b200/workloads/record_traces.py). Replaying it against the B200 library runs exactly the
calls a newch user's script makes; replaying it against the reference engine reproduces the
reference's results for the same calls. Handles are re-bound to whatever pointers the library under
test returns, host buffers are rebuilt from the trace's blobs (seeded synthetic inputs are
regenerated), and every scalar result and copied-out buffer is kept for comparison.
"""

from __future__ import annotations

import base64
import ctypes
import gzip
import json
import zlib
from ctypes import c_char_p, c_int64, c_void_p
from pathlib import Path

import numpy as np

from . import capi, synth

WORKLOADS = Path(__file__).resolve().parent / "workloads"


class ReplayMismatch(RuntimeError):
    pass


class Trace:
    def __init__(self, path):
        path = Path(path)
        if not path.exists():
            path = WORKLOADS / f"{path}.json.gz"
        with gzip.open(path, "rt") as f:
            t = json.load(f)
        if t.get("format") != "nc-trace-1":
            raise ValueError(f"{path}: not an nc trace")
        self.path = path
        self.meta = t["meta"]
        self.calls = t["calls"]
        self.blobs = t["blobs"]
        self.marks = t["marks"]
        self.step_ends = t["step_ends"]

    def blob(self, bid: str, seed_offset: int = 0) -> np.ndarray:
        b = self.blobs[bid]
        if "gen" in b:
            spec = synth.with_seed_offset(b["gen"], seed_offset) if seed_offset else b["gen"]
            return np.frombuffer(synth.generate(spec).tobytes(), dtype=np.uint8).copy()
        return np.frombuffer(zlib.decompress(base64.b64decode(b["zlib"])), dtype=np.uint8).copy()

    def steps(self):
        """(start, end) call ranges of the training/inference steps, each ending with nc_step_end."""
        begin = self.marks.get("train_begin", 0)
        out, start = [], begin
        for e in self.step_ends:
            if e >= begin:
                out.append((start, e + 1))
                start = e + 1
        return out

    def golden_items(self):
        """Scalar results the reference returned from nc_item during the steps (the losses)."""
        b, e = self.marks.get("train_begin", 0), self.marks.get("train_end", len(self.calls))
        return [c[2] for c in self.calls[b:e] if c[0] == "nc_item"]

    def golden_outputs(self):
        """Buffers the reference copied out after the steps (final parameters / predictions)."""
        e = self.marks.get("train_end", len(self.calls))
        out = []
        for c in self.calls[e:]:
            if c[0] == "nc_copy_to" and len(c) > 3:
                out.append(c[3])
        return out

    def output_bytes(self, entry) -> bytes | None:
        if "out" in entry:
            return self.blob(entry["out"]).tobytes()
        return None


_STRUCTS = {"nc_init": capi.Config}


class Replayer:
    """Executes trace calls on `lib`. `seed_offset` regenerates synthetic inputs with another seed
    (per-rank data shards); `check` raises when a call's success differs from the recording."""

    OPTIMIZERS = ("nc_sgd", "nc_adam", "nc_adamw", "nc_rmsprop")

    def __init__(self, lib, trace: Trace, seed_offset: int = 0, check: bool = True, pinned: bool = False,
                 grads: bool = False, capture=(), force_reference: int | None = None, capture_params: bool = False,
                 set_params=None):
        self.lib = lib
        self.trace = trace
        self.check = check
        self.pinned = pinned  # host inputs in page-locked memory (as a data loader would stage them)
        self.h: dict = {}
        self.items: list = []    # (call index, value) of nc_item results
        self.outputs: list = []  # (call index, bytes) of nc_copy_to results
        # grads=True: after every backward call, each optimizer parameter's gradient (bytes, or None
        # when it has none) as (call index, [per parameter]); parameters in the optimizer's order
        self.capture_grads = grads
        self.grads: list = []
        self._param_handles: list = []
        # capture: names of calls whose returned tensor (and nc_quantize_rows' scale output) is copied
        # out right after the call: self.captured lists (call index, name, argument handles, result
        # handle) and self.tensors maps those result handles (trace numbering) to the bytes
        self.capture = frozenset(capture)
        self.captured: list = []
        self.tensors: dict = {}
        self._keep: list = []
        self._blobs: dict = {}
        self.seed_offset = seed_offset
        self.force_reference = force_reference  # overrides nc_init's config field when not None
        # capture_params: each optimizer parameter's bytes after every optimizer step, in
        # self.params_after (one list per step); set_params: such a list of lists, written into the
        # parameters after each step instead (the step's update is replaced by the given values)
        self.capture_params = capture_params
        self.set_params = set_params
        self.params_after: list = []
        self.param_shapes: list = []  # shapes of the optimizer's parameters, taken when it is created
        self._steps_done = 0
        self._resident: dict = {}  # call index -> device tensor made once (make_resident)
        self._resident_ptrs: set = set()
        self._fns = {name: getattr(lib, name) for name in {c[0] for c in trace.calls}}
        self._prepared = [self._prepare(i, c) for i, c in enumerate(trace.calls)]

    # -- preparation: everything that does not depend on live handles is built once ------------
    def _blob_ptr(self, bid):
        arr = self._blobs.get(bid)
        if arr is None:
            arr = self.trace.blob(bid, self.seed_offset)
            if self.pinned:
                import torch  # page-locked host allocation only
                t = torch.empty(max(arr.size, 1), dtype=torch.uint8, pin_memory=True)
                t.numpy()[: arr.size] = arr
                self._keep.append(t)
                arr = t.numpy()
            self._blobs[bid] = arr
        return arr.ctypes.data

    def _prepare(self, idx, call):
        name, args, ret = call[0], call[1], call[2]
        extra = call[3] if len(call) > 3 else None
        conv = []
        fn = self._fns[name]
        argtypes = capi.SIGNATURES[name][1] if name in capi.SIGNATURES else []
        for k, a in enumerate(args):
            t = argtypes[k] if k < len(argtypes) else None
            if a is None:
                conv.append((0, None))
            elif isinstance(a, dict):
                if "h" in a:
                    conv.append((1, a["h"]))
                elif "s" in a:
                    arr = (c_int64 * max(len(a["s"]), 1))(*a["s"])
                    self._keep.append(arr)
                    conv.append((0, arr))
                elif "b" in a:
                    conv.append((0, self._blob_ptr(a["b"])))
                elif "o" in a:
                    conv.append((2, int(a["o"])))
                elif "hl" in a:
                    conv.append((3, list(a["hl"])))
                elif "st" in a:
                    st_t = t if isinstance(t, type) and issubclass(t, ctypes.Structure) else _STRUCTS.get(name)
                    if st_t is None and t is not None and hasattr(t, "_type_"):
                        st_t = t._type_
                    obj = st_t(*a["st"])
                    if name == "nc_init" and self.force_reference is not None:
                        obj.force_reference = int(self.force_reference)
                    self._keep.append(obj)
                    conv.append((0, ctypes.byref(obj) if name == "nc_init" else obj))
                elif "str" in a:
                    conv.append((0, a["str"].encode()))
                elif "strs" in a:
                    arr = (c_char_p * max(len(a["strs"]), 1))(*[s.encode() for s in a["strs"]])
                    self._keep.append(arr)
                    conv.append((0, arr))
                elif "f" in a:
                    conv.append((0, float(a["f"])))
                else:
                    raise ValueError(f"call {idx} {name}: unknown argument {a}")
            else:
                conv.append((0, a))
        ret_h = ret["h"] if isinstance(ret, dict) and "h" in ret else None
        ret_null = ret is None and capi.SIGNATURES.get(name, (None,))[0] is c_void_p and name not in (
            "nc_data_f32", "nc_data_i32", "nc_optim_state")
        out_h = extra.get("out_h") if isinstance(extra, dict) else None
        return (fn, name, conv, ret_h, ret_null, out_h)

    def make_resident(self, start: int, end: int) -> int:
        """Inputs resident on the device: every nc_from_data call of calls [start, end) that uploads host
        data is made once now, between nc_persistent_begin/end, and later runs of the range hand its
        tensor to the following calls instead of uploading again (its releases inside the range are
        skipped). Returns the bytes made resident."""
        ctx, total = self.ctx, 0
        for i in range(start, end):
            fn, name, conv, ret_h, ret_null, out_h = self._prepared[i]
            if name != "nc_from_data" or ret_h is None or not any(isinstance(a, dict) and "b" in a
                                                                  for a in self.trace.calls[i][1]):
                continue
            self.lib.nc_persistent_begin(ctx)
            try:
                self.run(i, i + 1)
            finally:
                self.lib.nc_persistent_end(ctx)
            self._resident[i] = self.h[ret_h]
            total += int(self.lib.nc_numel(self.h[ret_h])) * {0: 4, 1: 4, 2: 2, 3: 1, 4: 1}[
                int(self.lib.nc_get_dtype(self.h[ret_h]))]
        self._resident_ptrs = set(self._resident.values())
        return total

    # -- execution --------------------------------------------------------------------------
    def run(self, start: int = 0, end: int | None = None) -> None:
        h = self.h
        prepared = self._prepared
        resident, rptrs = self._resident, self._resident_ptrs
        end = len(prepared) if end is None else end
        for i in range(start, end):
            fn, name, conv, ret_h, ret_null, out_h = prepared[i]
            if resident:
                if i in resident:
                    h[ret_h] = resident[i]
                    continue
                if name in ("nc_release", "nc_release_temp") and conv and conv[0][0] == 1 and h[conv[0][1]] in rptrs:
                    continue
            vals = []
            outbuf = None
            for kind, v in conv:
                if kind == 0:
                    vals.append(v)
                elif kind == 1:
                    vals.append(h[v])
                elif kind == 2:
                    outbuf = (ctypes.c_char * v)() if name == "nc_copy_to" else (c_void_p * 1)()
                    vals.append(outbuf)
                else:
                    vals.append((c_void_p * max(len(v), 1))(*[h[x] if x is not None else None for x in v]))
            r = fn(*vals)
            if ret_h is not None:
                if not r:
                    raise ReplayMismatch(f"call {i} {name}: returned NULL where the reference succeeded: "
                                         f"{self._error()}")
                h[ret_h] = r
            elif ret_null and r and self.check:
                raise ReplayMismatch(f"call {i} {name}: succeeded where the reference returned NULL")
            if out_h is not None:
                h[out_h] = outbuf[0]
            if name in self.capture and r and ret_h is not None:
                self.captured.append((i, name, [v if kind == 1 else None for kind, v in conv], ret_h))
                self.tensors[ret_h] = self._tensor_bytes(r)
                if out_h is not None:
                    self.tensors[out_h] = self._tensor_bytes(outbuf[0])
            if name == "nc_item":
                self.items.append((i, r))
            elif name == "nc_copy_to" and outbuf is not None:
                self.outputs.append((i, bytes(outbuf)))
            if name in self.OPTIMIZERS:
                self._param_handles = next((list(v) for kind, v in conv if kind == 3), [])
                self.param_shapes = [self._shape(h[p]) for p in self._param_handles]
            elif name == "nc_optim_step" and (self.capture_params or self.set_params is not None):
                self._after_step()
            if self.capture_grads:
                if name in self.OPTIMIZERS:
                    self._param_handles = next((list(v) for kind, v in conv if kind == 3), [])
                elif name in ("nc_backward", "nc_backward_ex"):
                    self.grads.append((i, [self._grad_bytes(h[p]) for p in self._param_handles]))

    def _shape(self, t):
        nd = int(self.lib.nc_ndim(t))
        s = self.lib.nc_shape(t)
        return tuple(int(s[k]) for k in range(nd))

    def _after_step(self):
        k = self._steps_done
        self._steps_done += 1
        if self.set_params is not None and k < len(self.set_params):
            for p, data in zip(self._param_handles, self.set_params[k]):
                buf = (ctypes.c_char * len(data)).from_buffer_copy(data)
                if not self.lib.nc_copy_from(self.h[p], buf, len(data)):
                    raise ReplayMismatch(f"nc_copy_from of a parameter failed: {self._error()}")
        if self.capture_params:
            self.params_after.append([self._tensor_bytes(self.h[p]) for p in self._param_handles])

    def _tensor_bytes(self, t):
        n = int(self.lib.nc_numel(t)) * {0: 4, 1: 4, 2: 2, 3: 1, 4: 1}[int(self.lib.nc_get_dtype(t))]
        buf = (ctypes.c_char * max(n, 1))()
        if not self.lib.nc_copy_to(t, buf, n):
            raise ReplayMismatch(f"nc_copy_to of a captured tensor failed: {self._error()}")
        return bytes(buf)[:n]

    def _grad_bytes(self, p):
        g = self.lib.nc_grad(p)
        return self._tensor_bytes(g) if g else None

    def _error(self) -> str:
        ctx = self.h.get(1)  # nc_init is every trace's first call
        try:
            return self.lib.nc_error(ctx).decode(errors="replace") if ctx else "?"
        except Exception:  # pragma: no cover - diagnostics only
            return "?"

    def run_all(self) -> None:
        self.run(0, None)

    @property
    def ctx(self):
        return self.h.get(1)
