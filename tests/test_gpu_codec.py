"""Bit-exactness of the device Q4_0 codec.

* decode: equal bit for bit to mote-reference's dequantize_quantized_row
  (crates/mote-reference/src/quantized.rs:58-74), including the reference's
  known-answer blocks (tests/quantized_rows.rs:16-41);
* encode: equal byte for byte to the oracle's restatement of ggml's Q4_0
  reference quantizer, on N(0, 0.02) rows and on edge blocks (all zero,
  negative and positive absmax, ties at the rounding boundary, huge and
  subnormal magnitudes).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from tests import _fixtures as fx

pytestmark = pytest.mark.gpu

from mote_b200 import ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain, quantized  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def device_decode(ctx, w, n, k):
    wt = ctx.from_bytes(quantized((n, k)), w)
    out = ctx.empty(plain((n, k), DType.F32))
    ops.q4_0_decode_f32(ctx, wt, out)
    return np.frombuffer(ctx.read_bytes(out), np.float32).reshape(n, k)


def device_encode(ctx, x, n, k):
    xt = ctx.from_bytes(plain((n, k), DType.F32), np.asarray(x, np.float32))
    wt = ctx.empty(quantized((n, k)))
    ops.q4_0_encode_f32(ctx, xt, wt)
    return np.frombuffer(ctx.read_bytes(wt), np.uint8)


def test_decode_reference_known_answers(ctx, oracle_lib):
    kats = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())
    for case in kats["cases"]:
        if case["op"] != "dequantize" or case["format"] != "Q4_0" or "expected" not in case:
            continue
        k = case["row_elements"]
        got = device_decode(ctx, np.array(case["bytes"], np.uint8), 1, k)
        assert np.array_equal(got.reshape(-1), np.array(case["expected"], np.float32))


@pytest.mark.parametrize("n,k", [(7, 32), (64, 4096), (2048, 2048)])
def test_decode_bit_exact(ctx, oracle_lib, n, k):
    w = fx.q4_0_weights(oracle_lib, n, k, seed=n + k)
    got = device_decode(ctx, w, n, k)
    want = oracle_lib.dequantize_matrix(w, n, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_decode_every_nibble_and_scale_pattern(ctx, oracle_lib):
    rng = np.random.default_rng(1)
    n, k = 256, 256
    blocks = rng.integers(0, 256, (n, k // 32, 18), dtype=np.uint8)
    # finite scales only: f16 exponent field != 31
    blocks[:, :, 1] &= 0x7B
    w = blocks.reshape(-1)
    got = device_decode(ctx, w, n, k)
    want = oracle_lib.dequantize_matrix(w, n, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n,k", [(3, 32), (512, 4096), (1000, 2048)])
def test_encode_bit_exact_on_gaussian_rows(ctx, oracle_lib, n, k):
    x = np.random.default_rng(n).normal(0, 0.02, (n, k)).astype(np.float32)
    got = device_encode(ctx, x, n, k)
    want = oracle_lib.q4_0_quantize(x, n, k)
    assert np.array_equal(got, want)


def test_encode_edge_blocks(ctx, oracle_lib):
    rows = []
    rows.append(np.zeros(32))                                     # all zero: d = -0
    rows.append(np.linspace(-1, 1, 32))                           # ties in magnitude
    r = np.full(32, 0.5)
    r[5] = -4.0
    rows.append(r)                                                # negative absmax
    r = np.full(32, -0.25)
    r[31] = 3.0
    rows.append(r)                                                # positive absmax, last
    rows.append(np.arange(32) - 16.0)                              # integers, boundary ties
    rows.append(np.full(32, 1e-30))                                # subnormal f16 scale
    rows.append(np.full(32, 6e4) * np.sign(np.arange(32) - 15.5))  # near f16 max
    rows.append((np.arange(32) % 17) * 0.0625 - 0.5)                # exact .5 boundaries
    x = np.stack(rows).astype(np.float32)
    n = x.shape[0]
    got = device_encode(ctx, x, n, 32)
    want = oracle_lib.q4_0_quantize(x, n, 32)
    assert np.array_equal(got, want)


def test_encode_decode_round_trip_error_bound(ctx, oracle_lib):
    """Property at full config-3 size: every element is within one quantization
    step |d| of its decoded value (half a step when not clamped at q = 15),
    plus the f16 rounding of d."""
    n, k = 14336, 4096
    x = np.random.default_rng(3).normal(0, 0.02, (n, k)).astype(np.float32)
    w = device_encode(ctx, x, n, k)
    back = device_decode(ctx, w, n, k)
    blocks = x.reshape(n, k // 32, 32)
    amax = np.abs(blocks).max(axis=2, keepdims=True)
    d = amax / 8.0
    err = np.abs(back.reshape(n, k // 32, 32) - blocks)
    f16_slack = d * 8 * 2.0 ** -10
    clamped = np.abs(blocks) / np.where(d == 0, 1, d) > 7.5
    assert np.all(err <= np.where(clamped, d, d * 0.5) * 1.0001 + f16_slack)
