"""Writes ``reference_kats.json``: the known-answer tests of ``mote-reference``.

The Rust reference cannot be built in this environment (no cargo/rustc), so
its own tests cannot run.  Their known answers are plain literals in the
test sources; this script transcribes each one -- inputs, expected outputs
and expected error variants -- together with the file:line it comes from.
The oracle is pinned by passing every case (tests/test_oracle_kats.py), and
the CUDA kernels are pinned transitively through the oracle.

Run:  python tests/golden/make_golden.py   (rewrites the JSON next to it)
"""
from __future__ import annotations

import json
from pathlib import Path

USIZE_MAX = (1 << 64) - 1


def q4_0_block(scale_bits: int, quants: list[int]) -> list[int]:
    """quantized_rows.rs:4-8: little-endian f16 scale then 16 quant bytes."""
    return [scale_bits & 0xFF, scale_bits >> 8] + list(quants)


def q8_0_block(scale_bits: int, quants: list[int]) -> list[int]:
    """quantized_rows.rs:10-14."""
    return [scale_bits & 0xFF, scale_bits >> 8] + [q & 0xFF for q in quants]


def cases() -> list[dict]:
    out: list[dict] = []
    R = "crates/mote-reference/tests/"

    # ---- quantized_rows.rs -------------------------------------------------
    quants = [0x88] * 16
    quants[0] = 0xF0
    quants[1] = 0x78
    expected = [0.0] * 32
    expected[0], expected[16], expected[17] = -16.0, 14.0, -2.0
    out.append(dict(source=R + "quantized_rows.rs:16-30", op="dequantize", format="Q4_0",
                    bytes=q4_0_block(0x4000, quants), row_elements=32, expected=expected))

    out.append(dict(source=R + "quantized_rows.rs:32-41", op="dequantize", format="Q4_0",
                    bytes=q4_0_block(0x3C00, [0x99] * 16) + q4_0_block(0x3800, [0x66] * 16),
                    row_elements=64, expected=[1.0] * 32 + [-1.0] * 32))

    q8 = [0] * 32
    q8[:5] = [-128, -1, 0, 1, 127]
    out.append(dict(source=R + "quantized_rows.rs:43-52", op="dequantize", format="Q8_0",
                    bytes=q8_0_block(0x3800, q8), row_elements=32,
                    expected=[-64.0, -0.5, 0.0, 0.5, 63.5] + [0.0] * 27))

    out.append(dict(source=R + "quantized_rows.rs:54-66", op="linear", format="Q4_0",
                    input=[1.0] * 32 + [2.0] * 16 + [-1.0] * 16,
                    weights=q4_0_block(0x3C00, [0x89] * 16) + q4_0_block(0x3800, [0xA8] * 16),
                    rows=2, output_features=2, input_features=32,
                    expected=[16.0, 16.0, 32.0, -16.0]))

    first = [0] * 32
    first[0], first[31] = 2, -4
    second = [0] * 32
    second[0], second[31] = -3, 5
    inp = [0.0] * 32
    inp[0], inp[31] = 3.0, 2.0
    out.append(dict(source=R + "quantized_rows.rs:68-83", op="linear", format="Q8_0", input=inp,
                    weights=q8_0_block(0x3800, first) + q8_0_block(0x3C00, second),
                    rows=1, output_features=2, input_features=32, expected=[-1.0, 1.0]))

    out.append(dict(source=R + "quantized_rows.rs:85-90", op="linear", format="Q4_0", input=[],
                    weights=[], rows=3, output_features=2, input_features=0,
                    expected=[0.0] * 6))
    out.append(dict(source=R + "quantized_rows.rs:91-96", op="linear", format="Q8_0", input=[],
                    weights=q8_0_block(0x3C00, [0] * 32) * 2, rows=0, output_features=2,
                    input_features=32, expected=[]))
    out.append(dict(source=R + "quantized_rows.rs:97-101", op="dequantize", format="Q8_0",
                    bytes=[], row_elements=0, expected=[]))

    for fmt in ("Q4_K", "Q6_K"):
        out.append(dict(source=R + "quantized_rows.rs:104-116", op="dequantize", format=fmt,
                        bytes=[], row_elements=0,
                        error={"kind": "UnsupportedFormat"}))
        out.append(dict(source=R + "quantized_rows.rs:104-116", op="linear", format=fmt,
                        input=[], weights=[], rows=0, output_features=0, input_features=0,
                        error={"kind": "UnsupportedFormat"}))

    out.append(dict(source=R + "quantized_rows.rs:120-127", op="dequantize", format="Q4_0",
                    bytes=[], row_elements=31,
                    error={"kind": "RowMisaligned", "row_elements": 31, "block_elements": 32}))
    out.append(dict(source=R + "quantized_rows.rs:128-134", op="dequantize", format="Q4_0",
                    bytes=[0] * 17, row_elements=32,
                    error={"kind": "RowByteLengthMismatch", "expected": 18, "actual": 17}))
    out.append(dict(source=R + "quantized_rows.rs:135-141", op="linear", format="Q4_0",
                    input=[0.0] * 31, weights=[0] * 18, rows=1, output_features=1,
                    input_features=32,
                    error={"kind": "InputLengthMismatch", "expected": 32, "actual": 31}))
    out.append(dict(source=R + "quantized_rows.rs:142-148", op="linear", format="Q4_0",
                    input=[0.0] * 32, weights=[0] * 17, rows=1, output_features=1,
                    input_features=32,
                    error={"kind": "WeightLengthMismatch", "expected": 18, "actual": 17}))
    out.append(dict(source=R + "quantized_rows.rs:153-160", op="linear", format="Q4_0",
                    input=[], weights=[], rows=USIZE_MAX, output_features=1, input_features=32,
                    error={"kind": "DimensionsOverflow", "rows": USIZE_MAX,
                           "output_features": 1, "input_features": 32}))
    huge = (USIZE_MAX // 32) * 32
    out.append(dict(source=R + "quantized_rows.rs:162-170", op="dequantize", format="Q8_0",
                    bytes=[], row_elements=huge,
                    error={"kind": "DimensionsOverflow", "rows": 1, "output_features": 1,
                           "input_features": huge}))

    # ---- rms_norm_f32.rs ---------------------------------------------------
    x = [1.0, 2.0, 3.0, 4.0, -2.0, 0.0, 2.0, -4.0]
    w = [1.0, 2.0, 0.5, 1.5]
    out.append(dict(source=R + "rms_norm_f32.rs:26-66", op="rms_norm", input=x, weight=w,
                    hidden=4, epsilon=1e-6, f64_tolerance=1e-5, anchor_tolerance=1e-4,
                    anchors=[[0, 0.3651484], [1, 1.4605935], [4, -0.8164966],
                             [6, 0.4082483], [7, -2.4494897]]))
    out.append(dict(source=R + "rms_norm_f32.rs:68-72", op="rms_norm", input=[],
                    weight=[1.0, 2.0, 3.0, 4.0], hidden=4, epsilon=1e-6, expected=[]))
    out.append(dict(source=R + "rms_norm_f32.rs:74-78", op="rms_norm", input=[1.0, 2.0],
                    weight=[1.0, 1.0], hidden=0, epsilon=1e-6,
                    error={"kind": "ZeroHiddenSize"}))
    out.append(dict(source=R + "rms_norm_f32.rs:80-90", op="rms_norm", input=[1.0, 2.0],
                    weight=[1.0], hidden=2, epsilon=1e-6,
                    error={"kind": "WeightLengthMismatch", "weight_len": 1, "hidden_size": 2}))
    out.append(dict(source=R + "rms_norm_f32.rs:92-102", op="rms_norm", input=[1.0, 2.0, 3.0],
                    weight=[1.0, 1.0], hidden=2, epsilon=1e-6,
                    error={"kind": "InputNotMultiple", "input_len": 3, "hidden_size": 2}))
    for eps in (-1e-6, "nan", "inf", "-inf"):
        out.append(dict(source=R + "rms_norm_f32.rs:104-119", op="rms_norm", input=[1.0, 2.0],
                        weight=[1.0, 1.0], hidden=2, epsilon=eps,
                        error={"kind": "InvalidEpsilon"}))

    # ---- fused_add_rms_norm_f32.rs ----------------------------------------
    r = [0.5, -1.0, 2.0, 1.0, 2.0, 1.0, -1.0, 4.0]
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:41-105", op="fused_add_rms_norm",
                    input=x, residual=r, weight=w, hidden=4, epsilon=1e-6, f64_tolerance=1e-5,
                    anchor_tolerance=1e-4,
                    anchors=[[0, 0.4111132], [3, 2.055566], [4, 0.0], [5, 2.8284243],
                             [6, 0.7071061]],
                    expected_residual=[1.5, 1.0, 5.0, 5.0, 0.0, 1.0, 1.0, 0.0]))
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:107-121", op="fused_add_rms_norm",
                    input=[1.0, 2.0, -3.0, 4.0], residual=[4.0, -3.0, 2.0, -1.0],
                    weight=[0.0] * 4, hidden=4, epsilon=1e-6, expected=[0.0] * 4,
                    expected_residual=[5.0, -1.0, -1.0, 3.0]))
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:123-136", op="fused_add_rms_norm",
                    input=[3.0], residual=[1.0], weight=[2.0], hidden=1, epsilon=0.0,
                    expected=[2.0], expected_residual=[4.0]))
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:138-143", op="fused_add_rms_norm",
                    input=[], residual=[], weight=[1.0, 2.0, 3.0, 4.0], hidden=4, epsilon=1e-6,
                    expected=[], expected_residual=[]))
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:145-150", op="fused_add_rms_norm",
                    input=[1.0, 2.0], residual=[1.0, 1.0], weight=[1.0, 1.0], hidden=0,
                    epsilon=1e-6, error={"kind": "ZeroHiddenSize"}))
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:152-162", op="fused_add_rms_norm",
                    input=[1.0, 2.0], residual=[1.0, 1.0], weight=[1.0], hidden=2,
                    epsilon=1e-6,
                    error={"kind": "WeightLengthMismatch", "weight_len": 1, "hidden_size": 2}))
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:164-174", op="fused_add_rms_norm",
                    input=[1.0, 2.0], residual=[1.0], weight=[1.0, 1.0], hidden=2,
                    epsilon=1e-6,
                    error={"kind": "ResidualLengthMismatch", "residual_len": 1, "input_len": 2}))
    out.append(dict(source=R + "fused_add_rms_norm_f32.rs:176-187", op="fused_add_rms_norm",
                    input=[1.0, 2.0, 3.0], residual=[1.0, 1.0, 1.0], weight=[1.0, 1.0],
                    hidden=2, epsilon=1e-6,
                    error={"kind": "InputNotMultiple", "input_len": 3, "hidden_size": 2}))
    for eps in (-1e-6, "nan", "inf", "-inf"):
        out.append(dict(source=R + "fused_add_rms_norm_f32.rs:189-205", op="fused_add_rms_norm",
                        input=[1.0, 2.0], residual=[1.0, 1.0], weight=[1.0, 1.0], hidden=2,
                        epsilon=eps, error={"kind": "InvalidEpsilon"}))

    # ---- rope_f32.rs ---------------------------------------------------------
    out.append(dict(source=R + "rope_f32.rs:4-21", op="rope", input=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0],
                    cos=[0.0, 1.0], sin=[1.0, 0.0], tokens=1, heads=1, head_dim=6,
                    rotary_dim=4, layout="HalfSplit", expected=[-3.0, 2.0, 1.0, 4.0, 5.0, 6.0]))
    out.append(dict(source=R + "rope_f32.rs:23-40", op="rope",
                    input=[1.0, 2.0, 3.0, 4.0, 10.0, 20.0, 30.0, 40.0], cos=[0.0, 1.0],
                    sin=[1.0, 0.0], tokens=1, heads=2, head_dim=4, rotary_dim=4,
                    layout="Interleaved",
                    expected=[-2.0, 1.0, 3.0, 4.0, -20.0, 10.0, 30.0, 40.0]))
    out.append(dict(source=R + "rope_f32.rs:42-53", op="rope", input=[], cos=[], sin=[],
                    tokens=0, heads=3, head_dim=8, rotary_dim=8, layout="HalfSplit",
                    expected=[]))
    out.append(dict(source=R + "rope_f32.rs:42-53", op="rope", input=[1.0, 2.0], cos=[], sin=[],
                    tokens=1, heads=1, head_dim=2, rotary_dim=0, layout="Interleaved",
                    expected=[1.0, 2.0]))
    out.append(dict(source=R + "rope_f32.rs:55-68", op="rope", input=[], cos=[], sin=[],
                    tokens=0, heads=0, head_dim=4, rotary_dim=3, layout="HalfSplit",
                    error={"kind": "OddRotaryDimension", "rotary_dim": 3}))
    out.append(dict(source=R + "rope_f32.rs:55-68", op="rope", input=[], cos=[], sin=[],
                    tokens=0, heads=0, head_dim=4, rotary_dim=6, layout="HalfSplit",
                    error={"kind": "RotaryDimensionTooLarge", "rotary_dim": 6, "head_dim": 4}))
    out.append(dict(source=R + "rope_f32.rs:70-93", op="rope", input=[0.0], cos=[1.0],
                    sin=[0.0], tokens=1, heads=1, head_dim=4, rotary_dim=2, layout="HalfSplit",
                    error={"kind": "InputLengthMismatch", "expected": 4, "actual": 1}))
    out.append(dict(source=R + "rope_f32.rs:70-93", op="rope", input=[0.0] * 4, cos=[],
                    sin=[0.0], tokens=1, heads=1, head_dim=4, rotary_dim=2, layout="HalfSplit",
                    error={"kind": "CosLengthMismatch", "expected": 1, "actual": 0}))
    out.append(dict(source=R + "rope_f32.rs:70-93", op="rope", input=[0.0] * 4, cos=[1.0],
                    sin=[], tokens=1, heads=1, head_dim=4, rotary_dim=2, layout="HalfSplit",
                    error={"kind": "SinLengthMismatch", "expected": 1, "actual": 0}))

    # ---- matmul_f32.rs -------------------------------------------------------
    out.append(dict(source=R + "matmul_f32.rs:3-11", op="matmul",
                    lhs=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0], rhs=[7.0, 8.0, 9.0, 10.0, 11.0, 12.0],
                    m=2, n=2, k=3, expected=[58.0, 64.0, 139.0, 154.0]))
    out.append(dict(source=R + "matmul_f32.rs:13-16", op="matmul", lhs=[], rhs=[], m=2, n=3,
                    k=0, expected=[0.0] * 6))
    out.append(dict(source=R + "matmul_f32.rs:18-25", op="matmul", lhs=[],
                    rhs=[1.0, 2.0, 3.0, 4.0], m=0, n=2, k=2, expected=[]))
    out.append(dict(source=R + "matmul_f32.rs:27-42", op="matmul", lhs=[1.0], rhs=[1.0] * 6,
                    m=2, n=2, k=3,
                    error={"kind": "LhsLengthMismatch", "expected": 6, "actual": 1}))
    out.append(dict(source=R + "matmul_f32.rs:27-42", op="matmul", lhs=[1.0] * 6, rhs=[1.0],
                    m=2, n=2, k=3,
                    error={"kind": "RhsLengthMismatch", "expected": 6, "actual": 1}))
    out.append(dict(source=R + "matmul_f32.rs:44-54", op="matmul", lhs=[], rhs=[],
                    m=USIZE_MAX, n=1, k=2, error={"kind": "DimensionsOverflow"}))
    return out


def main() -> None:
    path = Path(__file__).resolve().parent / "reference_kats.json"
    doc = {
        "about": "Known-answer tests transcribed from RiversJin/mote "
                 "crates/mote-reference/tests/*.rs by make_golden.py",
        "cases": cases(),
    }
    path.write_text(json.dumps(doc, indent=1) + "\n")
    print(f"wrote {len(doc['cases'])} cases to {path}")


if __name__ == "__main__":
    main()
