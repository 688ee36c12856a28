"""Pins the CPU oracle against the reference's own known-answer tests.

Every case in ``golden/reference_kats.json`` is a literal from a
``crates/mote-reference/tests/*.rs`` test (the ``source`` field names the
file:line).  Expected values are compared exactly where the Rust test uses
``assert_eq!`` and with the Rust test's own tolerance where it uses one.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import checker

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())["cases"]
FORMATS = {"Q8_0": 0, "Q4_0": 1, "Q4_K": 2, "Q6_K": 3}
LAYOUTS = {"HalfSplit": 0, "Interleaved": 1}


def _eps(v):
    return float(v) if not isinstance(v, str) else float(v)


def _run(ref, case):
    op = case["op"]
    if op == "dequantize":
        return ref.dequantize_quantized_row(np.array(case["bytes"], np.uint8),
                                            FORMATS[case["format"]], case["row_elements"])
    if op == "linear":
        return ref.quantized_linear_f32(np.array(case["input"], np.float32),
                                        np.array(case["weights"], np.uint8),
                                        FORMATS[case["format"]], case["rows"],
                                        case["output_features"], case["input_features"])
    if op == "rms_norm":
        return ref.rms_norm_f32(case["input"], case["weight"], case["hidden"],
                                _eps(case["epsilon"]))
    if op == "fused_add_rms_norm":
        return ref.fused_add_rms_norm_f32(case["input"], case["residual"], case["weight"],
                                          case["hidden"], _eps(case["epsilon"]))
    if op == "rope":
        return ref.rope_f32(case["input"], case["cos"], case["sin"], case["tokens"],
                            case["heads"], case["head_dim"], case["rotary_dim"],
                            LAYOUTS[case["layout"]])
    if op == "matmul":
        return ref.matmul_f32(case["lhs"], case["rhs"], case["m"], case["n"], case["k"])
    raise AssertionError(op)


@pytest.mark.parametrize("case", KATS, ids=[f"{i}-{c['op']}" for i, c in enumerate(KATS)])
def test_reference_known_answer(oracle_lib, case):
    ref = oracle_lib
    if "error" in case:
        with pytest.raises(ref.OracleError) as info:
            _run(ref, case)
        want = dict(case["error"])
        assert info.value.kind == want.pop("kind"), case["source"]
        for name, value in want.items():
            assert info.value.fields[name] == value, (case["source"], name)
        return
    got = _run(ref, case)
    if case["op"] == "fused_add_rms_norm":
        normalized, residual = got
        np.testing.assert_array_equal(residual, np.array(case["expected_residual"], np.float32))
        got = normalized
    if "expected" in case:
        np.testing.assert_array_equal(got, np.array(case["expected"], np.float32),
                                      err_msg=case["source"])
    if "anchors" in case:
        for index, want in case["anchors"]:
            assert abs(float(got[index]) - want) < case["anchor_tolerance"], case["source"]
    if "f64_tolerance" in case:
        hidden = case["hidden"]
        if case["op"] == "rms_norm":
            expect = checker.rms_norm_f64(case["input"], case["weight"], hidden, case["epsilon"])
        else:
            expect, _ = checker.fused_add_rms_norm_f64(case["input"], case["residual"],
                                                       case["weight"], hidden, case["epsilon"])
        expect = expect.reshape(-1).astype(np.float32)
        assert np.all(np.abs(got - expect) < case["f64_tolerance"]), case["source"]


def test_every_reference_test_file_is_represented():
    sources = {c["source"].split(":")[0].rsplit("/", 1)[-1] for c in KATS}
    assert sources == {"quantized_rows.rs", "rms_norm_f32.rs", "fused_add_rms_norm_f32.rs",
                       "rope_f32.rs", "matmul_f32.rs"}


def test_f16_conversions_match_ieee_round_to_nearest_even(oracle_lib):
    ref = oracle_lib
    # every binary16 pattern widens exactly (NaNs compared as NaN)
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    ours = ref.f16_to_f32(bits)
    numpy_ = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(numpy_)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan].view(np.uint32), numpy_[~nan].view(np.uint32))
    # narrowing: random f32 patterns plus every tie between adjacent f16 values
    rng = np.random.default_rng(7)
    pats = rng.integers(0, 1 << 32, size=1 << 20, dtype=np.uint64).astype(np.uint32)
    vals = pats.view(np.float32)
    finite16 = bits.view(np.float16)[np.isfinite(bits.view(np.float16))].astype(np.float64)
    finite16 = np.unique(finite16)
    ties = ((finite16[:-1] + finite16[1:]) / 2).astype(np.float32)
    vals = np.concatenate([vals, ties, np.float32([0.0, -0.0, 65504.0, 65520.0, 1e-8, 6e-8])])
    vals = vals[~np.isnan(vals)]
    got = ref.f32_to_f16(vals)
    want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_multithreaded_linear_is_bit_identical(oracle_lib):
    ref = oracle_lib
    rng = np.random.default_rng(3)
    rows, n, k = 3, 37, 256
    w = ref.q4_0_quantize(rng.normal(0, 0.02, (n, k)).astype(np.float32), n, k)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    one = ref.quantized_linear_f32(x, w, ref.Q4_0, rows, n, k)
    many = ref.quantized_linear_f32(x, w, ref.Q4_0, rows, n, k, threads=5)
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))
