"""K-quant oracle (Q4_K, Q6_K) against golden vectors from gguf 0.19.0.

mote-reference rejects K-quants (crates/mote-reference/src/quantized.rs:152-157);
the golden vectors in tests/golden/kquant_golden.npz come from the published
ggml dequantization as the gguf package implements it
(tests/golden/make_kquant_golden.py).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import ref

GOLDEN = np.load(Path(__file__).parent / "golden" / "kquant_golden.npz")
FORMATS = {"q4_k": (ref.Q4_K, 144), "q6_k": (ref.Q6_K, 210)}


@pytest.mark.parametrize("name", sorted(FORMATS))
def test_dequantize_matches_gguf_bit_for_bit(name):
    fmt, bb = FORMATS[name]
    blocks = GOLDEN[f"{name}_blocks"]
    want = GOLDEN[f"{name}_values"]
    got = ref.kquant_dequantize(blocks.reshape(-1), fmt, 1, blocks.shape[0] * 256)
    assert got.view(np.uint32).reshape(-1).tolist() == want.tolist()


@pytest.mark.parametrize("name", sorted(FORMATS))
def test_dequantize_rows_are_independent(name):
    # the same blocks as 4 rows decode to the same values
    fmt, bb = FORMATS[name]
    blocks = GOLDEN[f"{name}_blocks"][:48]
    want = GOLDEN[f"{name}_values"][: 48 * 256]
    got = ref.kquant_dequantize(blocks.reshape(-1), fmt, 4, 12 * 256)
    assert got.view(np.uint32).reshape(-1).tolist() == want.tolist()


def test_q4_k_edge_blocks():
    blocks = GOLDEN["q4_k_blocks"]
    vals = GOLDEN["q4_k_values"].view(np.float32)
    assert not blocks[0].any() and not vals[:256].any()  # all-zero block decodes to zeros
    # all-ones bytes with d = dmin = 1: every scale and min is 63, q = 15
    assert np.all(vals[256:512] == np.float32(63 * 15 - 63))


def test_kquant_linear_f64_is_the_dot_product_of_decoded_rows():
    rng = np.random.default_rng(3)
    for name, (fmt, bb) in FORMATS.items():
        blocks = GOLDEN[f"{name}_blocks"][:8]
        w = blocks.reshape(-1)  # 4 rows of K = 512
        x = rng.normal(0, 1, (3, 512)).astype(np.float32)
        y = ref.kquant_linear_f64(x, w, fmt, 3, 4, 512)
        dec = ref.kquant_dequantize(w, fmt, 4, 512).astype(np.float64)
        np.testing.assert_allclose(y, x.astype(np.float64) @ dec.T, rtol=1e-12, atol=1e-12)


def test_kquant_rejections():
    w = np.zeros(144, np.uint8)
    with pytest.raises(ref.OracleError):
        ref.kquant_dequantize(w, ref.Q4_0, 1, 256)
    with pytest.raises(ref.OracleError):
        ref.kquant_linear_f64(np.zeros(128, np.float32), w, ref.Q4_K, 1, 1, 128)
