"""Workload traces: replaying a recorded newch call sequence on the reference engine reproduces the
recording bit for bit, so a trace is a faithful stand-in for newch's Python layer driving the C ABI.
CPU only (uses the reference engine built under oracle/_ref)."""

from __future__ import annotations

import numpy as np
import pytest

from nchelp import REF_LIB, capi
from newch_b200 import replay

SMALL = ["cfg1_small", "cfg2_small", "cfg3_small", "cfg4_small", "cfg5_small"]
pytestmark = pytest.mark.skipif(not REF_LIB.exists(), reason="reference engine not built (make -C oracle)")


@pytest.mark.parametrize("name", SMALL)
def test_reference_replay_is_bit_exact(name):
    lib = capi.load(REF_LIB)
    t = replay.Trace(name)
    r = replay.Replayer(lib, t)
    r.run_all()
    assert [v for _, v in r.items] == t.golden_items()
    gouts = t.golden_outputs()
    got = [b for _, b in r.outputs][-len(gouts):] if gouts else []
    for g, b in zip(gouts, got):
        ref = t.output_bytes(g)
        if ref is not None:
            assert ref == b
        else:
            a = np.frombuffer(b, np.float32).astype(np.float64)
            assert a.sum() == pytest.approx(g["out_summary"]["sum"], rel=1e-12, abs=1e-12)
    lib.nc_free_ctx(r.ctx)


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg2_stream", "cfg3", "cfg4", "cfg5"] + SMALL)
def test_trace_structure(name):
    t = replay.Trace(name)
    assert t.calls[0][0] == "nc_init"
    steps = t.steps()
    assert steps and all(t.calls[e - 1][0] == "nc_step_end" for _, e in steps)
    names = {c[0] for c in t.calls}
    assert names <= set(capi.SIGNATURES), names - set(capi.SIGNATURES)
    # a repeatable step only refers to handles made before it or inside it
    s, e = steps[-1]
    made = set()
    for c in t.calls[:s]:
        if isinstance(c[2], dict) and "h" in c[2]:
            made.add(c[2]["h"])
        if len(c) > 3 and isinstance(c[3], dict) and c[3].get("out_h"):
            made.add(c[3]["out_h"])
    inside = set()
    for c in t.calls[s:e]:
        for a in c[1]:
            if isinstance(a, dict) and "h" in a:
                assert a["h"] in made or a["h"] in inside
        if isinstance(c[2], dict) and "h" in c[2]:
            inside.add(c[2]["h"])


@pytest.mark.parametrize("name", ["cfg3_small", "cfg5_small"])
def test_resident_inputs_replay_the_same_step(name):
    """The benchmark's resident-input mode (the repeated step's nc_from_data uploads made once, before
    timing) gives the step the same results as uploading every time."""
    lib = capi.load(REF_LIB)
    t = replay.Trace(name)
    s = t.steps()[-1]
    runs = []
    for resident in (False, True):
        r = replay.Replayer(lib, t)
        r.run(0, s[1])
        made = r.make_resident(*s) if resident else 0
        assert (made > 0) == resident
        n0 = len(r.items), len(r.outputs)
        for _ in range(2):
            r.run(*s)
        runs.append(([v for _, v in r.items[n0[0]:]], [b for _, b in r.outputs[n0[1]:]]))
        lib.nc_free_ctx(r.ctx)
    assert runs[0] == runs[1]


def test_smoke_parameter_check_on_the_reference():
    """__graft_entry__.smoke()'s final-parameter check (byte-kept and summarized outputs) gives zero on the
    reference engine's own replay of the smoke trace."""
    import sys as _sys
    from pathlib import Path as _P
    _sys.path.insert(0, str(_P(__file__).resolve().parent.parent))
    import __graft_entry__ as ge
    lib = capi.load(REF_LIB)
    t = replay.Trace("cfg1_small")
    r = replay.Replayer(lib, t)
    r.run_all()
    assert ge.param_error(t, r.outputs) == 0.0
    lib.nc_free_ctx(r.ctx)
