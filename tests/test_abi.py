"""The B200 library presents the newch C ABI: it loads without a GPU, exports every entry point that
include/nc.h and include/nc_ext.h declare (and every name newch's ctypes layer binds), and its
structs have newch's layouts. No compute calls. CPU only."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from nchelp import REF_LIB, capi

REPO = Path(__file__).resolve().parent.parent


def declared(header: str) -> set:
    text = (REPO / "include" / header).read_text()
    return set(re.findall(r"NC_API[^;{]*?\b(nc_\w+)\s*\(", text, flags=re.S))


def exported(path: Path) -> set:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.split() and line.split()[-1].startswith("nc_")}


@pytest.fixture(scope="module")
def lib_path():
    p = capi.b200_library_path()
    assert p.exists(), "newch_b200/libnc.so is not built (run __graft_entry__.build())"
    return p


def test_library_loads_without_a_gpu(lib_path):
    lib = capi.load(lib_path, ext=True)  # applies every signature: a missing name raises
    assert lib.nc_ext_device_count() >= 0


def test_exports_every_declared_symbol(lib_path):
    names = declared("nc.h") | declared("nc_ext.h")
    assert len(declared("nc.h")) >= 120
    missing = names - exported(lib_path)
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_exports_exactly_the_header(lib_path):
    assert exported(lib_path) == declared("nc.h") | declared("nc_ext.h")


def test_covers_the_signature_table(lib_path):
    assert set(capi.SIGNATURES) <= exported(lib_path)
    assert set(capi.EXT_SIGNATURES) <= exported(lib_path)


@pytest.mark.skipif(not REF_LIB.exists(), reason="reference engine not built (make -C oracle)")
def test_same_symbols_as_the_reference_engine(lib_path):
    ours, ref = exported(lib_path), exported(REF_LIB)
    assert ref <= ours, f"reference symbols missing: {sorted(ref - ours)}"
    assert {n for n in ours - ref if not n.startswith("nc_ext_")} == set()


def test_struct_layouts():
    assert ctypes.sizeof(capi.Config) == 24
    assert ctypes.sizeof(capi.MemStats) == 32
    assert ctypes.sizeof(capi.OptimOpts) == 24
    assert ctypes.sizeof(capi.CpuInfo) == 8 + 4 * 8


def test_enum_values_in_header():
    text = (REPO / "include" / "nc.h").read_text()
    for name, val in [("NC_F32", 0), ("NC_I32", 1), ("NC_F16", 2), ("NC_I8", 3), ("NC_U8", 4), ("NC_ERR_STATE", 5),
                      ("NC_BACKWARD_FREE_GRAPH", 1), ("NC_BACKWARD_RETAIN", 2)]:
        assert re.search(rf"\b{name}\s*=\s*{val}\b", text), name
    assert "#define NC_ALL_AXES (-128)" in text and "#define NC_MAX_DIMS 6" in text
