"""Op parity on the B200: every case of tests/opcases.py through the C ABI against the reference
engine's golden vectors (tests/golden/ops.npz).

Tolerances: normwise max|got - ref| / max|ref| <= 1e-5 for float results (the FP32 FFMA GEMM mode,
ulp-level differences from summation order and from the reference's polynomial exp/tanh/erf), and
bit-exact equality for integer results, argmax indices, the RNG stream, dropout masks, int8
quantization and accumulators, and pure data movement."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from nchelp import rel_err
from opcases import CASES, run_case

pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "ops.npz")

EXACT = {
    "dropout": {"y1", "y2", "dx"},
    "random": {"uniform"},
    "int8": {"q", "scale", "y"},
    "reductions": {"argmax_1", "max_0_y", "max_1_y", "max_2_y", "max_all_y", "max_0_dx", "max_1_dx", "max_2_dx",
                   "max_all_dx"},
    "maxpool_2x2": {"y"},
    "maxpool_2x2_w4": {"y", "dx"},
    "maxpool_2x2_w2": {"y", "dx"},
    "maxpool_2x2_odd": {"y", "dx"},
    "maxpool_overlap": {"y"},
    "to_dtype": {"u8", "f", "u8_f32", "f_i32", "f_i8"},
    "index_select": {"y"},
    "masked_fill": {"y", "dx"},
    "views": {"y"},
    "cat": {"y", "da", "db"},
    "binary_broadcast": {"add_y", "sub_y", "mul_y", "div_y"},
    "unary": {"relu_y", "neg_y", "scale_y", "add_scalar_y", "leaky_relu_y", "relu6_y", "hardsigmoid_y",
              "hardswish_y", "relu_dx", "neg_dx", "scale_dx", "add_scalar_dx", "leaky_relu_dx", "relu6_dx",
              "hardsigmoid_dx", "hardswish_dx"},
}
TOL = 1e-5


@pytest.mark.parametrize("case", sorted(CASES))
def test_op_matches_reference(case):
    out = run_case("b200", case)
    keys = [k[len(case) + 1:] for k in GOLD.files if k.startswith(case + "/")]
    assert set(keys) == set(out), (set(keys) ^ set(out))
    exact = EXACT.get(case, set())
    for k in keys:
        ref, got = GOLD[f"{case}/{k}"], out[k]
        assert got.shape == ref.shape and got.dtype == ref.dtype, (k, got.shape, ref.shape)
        if k in exact or got.dtype.kind in "iu":
            assert np.array_equal(got, ref, equal_nan=True), f"{case}/{k} differs"
        else:
            err = rel_err(got, ref)
            assert err <= TOL, f"{case}/{k}: rel err {err:.3g}"
