"""Op parity on the B200: every case of tests/opcases.py through the C ABI against the reference
engine's golden vectors (tests/golden/ops.npz).

Tolerances: normwise max|got - ref| / max|ref| <= 1e-5 for float results (ulp-level differences from
summation order), and bit-exact equality for integer results, argmax indices, the RNG stream, dropout
masks, int8 quantization and accumulators, pure data movement, and the activations built on exp /
tanh / erf (the engine evaluates newch's own AVX2-tier polynomials, which is what the reference
engine runs on an AVX2+FMA host such as the one the golden vectors came from)."""

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
    "int8_gelu_chain": {"x", "y"},
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
              "hardsigmoid_dx", "hardswish_dx"}
    | {f"{k}_{o}" for k in ("sigmoid", "tanh", "exp", "silu", "gelu", "gelu_tanh") for o in ("y", "dx")},
    "transcendental": {"x", "G"} | {f"{k}_{o}" for k in ("sigmoid", "tanh", "exp", "silu", "gelu", "gelu_tanh")
                                    for o in ("y", "dx")},
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


@pytest.mark.parametrize("how", ["env", "force_reference"])
def test_libm_math_mode(how, monkeypatch):
    """NC_MATH=libm (or force_reference, as newch selects its reference tier) evaluates exp / tanh / erf
    with CUDA's libm, as newch's reference tier calls the C library: within 1e-5 of the AVX2-tier
    goldens on the sweep, and the same special values (+-inf, NaN, 0) at the edges."""
    if how == "env":
        monkeypatch.setenv("NC_MATH", "libm")
    out = run_case("b200", "transcendental", force_reference=(how == "force_reference"))
    x = GOLD["transcendental/x"]
    finite = np.isfinite(x) & (np.abs(x) < 80)
    for k in [k for k in out if k.endswith("_y") or k.endswith("_dx")]:
        ref, got = GOLD[f"transcendental/{k}"], out[k]
        assert rel_err(got[finite], ref[finite]) <= TOL, k
        special = ~finite & np.isfinite(ref)
        assert np.allclose(got[special], ref[special], rtol=1e-5, atol=1e-30), k


@pytest.mark.parametrize("case", ["bn_relu_pool", "bn_pool", "bn_hardswish", "bn_relu6_pool", "bn_relu_reused",
                                  "bn_relu_pool_odd", "conv3_bn_relu_pool", "attention_chain", "attention_mha", "attention_mha_128",
                                  "attention_sdpa", "attention_unmasked", "attention_probs_read", "int8_gelu_chain"])
def test_chains_unfused(case, monkeypatch):
    """NC_FUSE=0: the BatchNorm and attention chains through the unfused kernels (every intermediate
    written), held to the same goldens as the fused default (test_op_matches_reference)."""
    monkeypatch.setenv("NC_FUSE", "0")
    out = run_case("b200", case)
    for k in out:
        ref = GOLD[f"{case}/{k}"]
        assert rel_err(out[k], ref) <= TOL, (case, k)


@pytest.mark.parametrize("case", ["batch_norm_train", "bn_relu_pool", "bn_pool", "bn_hardswish", "bn_relu6_pool",
                                  "bn_relu_reused", "bn_relu_pool_odd"])
@pytest.mark.parametrize("stage", ["0", "8", "16"])
def test_bn_reductions_other_forms(case, stage, monkeypatch):
    """NC_BN_BULK=0 (register-fed BatchNorm statistics and backward sums), =8 and =16 (every eligible
    pass fed by bulk copies in 8 / 16 KiB stages, aligned and unaligned planes): the same goldens as
    the default policy (test_op_matches_reference)."""
    monkeypatch.setenv("NC_BN_BULK", stage)
    out = run_case("b200", case)
    for k in out:
        ref = GOLD[f"{case}/{k}"]
        assert rel_err(out[k], ref) <= TOL, (case, k)


@pytest.mark.parametrize("case", ["dropout", "attention_chain", "attention_mha_128"])
@pytest.mark.parametrize("side", ["0", "1"])
def test_masks_on_either_stream(case, side, monkeypatch):
    """NC_RNG_SIDE=0: dropout masks drawn on the main stream; =1: every mask drawn on the side stream
    (by default only masks of at least 1M draws are); both held to the same goldens (bit-exact where
    test_op_matches_reference is)."""
    monkeypatch.setenv("NC_RNG_SIDE", side)
    out = run_case("b200", case)
    exact = EXACT.get(case, set())
    for k in out:
        ref = GOLD[f"{case}/{k}"]
        if k in exact:
            assert np.array_equal(out[k], ref, equal_nan=True), (case, k)
        else:
            assert rel_err(out[k], ref) <= TOL, (case, k)
