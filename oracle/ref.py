"""ctypes bindings for the C restatement of ``mote-reference``.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Each wrapper names
the reference function it restates; the C source carries the file:line
citations.  Errors come back as :class:`OracleError` whose ``kind`` is the
reference's error-variant name and whose ``fields`` are that variant's
fields, so tests can assert the same taxonomy the Rust tests assert.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_build" / "libmote_oracle.so"

Q8_0, Q4_0, Q4_K, Q6_K = 0, 1, 2, 3
HALF_SPLIT, INTERLEAVED = 0, 1

_STATUS = {
    1: ("UnsupportedFormat", ("format",)),
    2: ("RowMisaligned", ("format", "row_elements", "block_elements")),
    3: ("DimensionsOverflow", ("rows", "output_features", "input_features")),
    4: ("InputLengthMismatch", ("expected", "actual")),
    5: ("WeightLengthMismatch", ("expected", "actual")),
    6: ("RowByteLengthMismatch", ("expected", "actual")),
    10: ("ZeroHiddenSize", ()),
    11: ("WeightLengthMismatch", ("weight_len", "hidden_size")),
    12: ("InputNotMultiple", ("input_len", "hidden_size")),
    13: ("ResidualLengthMismatch", ("residual_len", "input_len")),
    14: ("InvalidEpsilon", ()),
    20: ("OddRotaryDimension", ("rotary_dim",)),
    21: ("RotaryDimensionTooLarge", ("rotary_dim", "head_dim")),
    22: ("DimensionsOverflow", ()),
    23: ("InputLengthMismatch", ("expected", "actual")),
    24: ("CosLengthMismatch", ("expected", "actual")),
    25: ("SinLengthMismatch", ("expected", "actual")),
    30: ("DimensionsOverflow", ()),
    31: ("LhsLengthMismatch", ("expected", "actual")),
    32: ("RhsLengthMismatch", ("expected", "actual")),
    40: ("ArgumentInvalid", ()),
}


class OracleError(Exception):
    def __init__(self, status: int, err: "_Err"):
        kind, names = _STATUS.get(status, ("Unknown", ()))
        values = (err.a, err.b, err.c)
        self.status = status
        self.kind = kind
        self.fields = {name: int(values[i]) for i, name in enumerate(names)}
        super().__init__(f"{kind} {self.fields}")


class _Err(ctypes.Structure):
    _fields_ = [("a", ctypes.c_uint64), ("b", ctypes.c_uint64), ("c", ctypes.c_uint64)]


def build(force: bool = False) -> Path:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    src = _HERE / "mote_oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(_HERE), "-s"], check=True)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        l = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        S = ctypes.c_size_t
        E = ctypes.POINTER(_Err)
        I = ctypes.c_int
        F = ctypes.c_float
        sig = {
            "oracle_f16_to_f32": (F, [ctypes.c_uint16]),
            "oracle_f32_to_f16": (ctypes.c_uint16, [F]),
            "oracle_f16_to_f32_array": (None, [P, P, S]),
            "oracle_f32_to_f16_array": (None, [P, P, S]),
            "oracle_dequantize_quantized_row": (I, [P, S, I, S, P, E]),
            "oracle_quantized_linear_f32": (I, [P, S, P, S, I, S, S, S, P, E]),
            "oracle_quantized_linear_f32_mt": (I, [P, S, P, S, I, S, S, S, P, I, E]),
            "oracle_matmul_f32": (I, [P, S, P, S, S, S, S, P, E]),
            "oracle_rope_f32": (I, [P, S, P, S, P, S, S, S, S, S, I, P, E]),
            "oracle_rms_norm_f32": (I, [P, S, P, S, S, F, P, E]),
            "oracle_fused_add_rms_norm_f32": (I, [P, S, P, S, P, S, S, F, P, P, E]),
            "oracle_q4_0_quantize_rows": (I, [P, S, S, P]),
            "oracle_embedding_gather_f16": (I, [P, S, S, P, S, P, P]),
            "oracle_swiglu_f64": (None, [P, P, S, P]),
            "oracle_rope_cos_sin_f64": (I, [P, S, S, ctypes.c_double, P, P]),
            "oracle_kquant_dequantize_row": (I, [P, S, I, S, P]),
            "oracle_kquant_linear_f64": (I, [P, P, I, S, S, S, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None or a.size == 0:
        # The Rust API takes slices; an empty slice has a dangling but
        # non-null pointer.  A 1-byte dummy keeps C from ever seeing NULL.
        return ctypes.addressof(_DUMMY)
    return a.ctypes.data


_DUMMY = ctypes.c_uint64(0)


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype).reshape(-1))


def _check(status: int, err: _Err) -> None:
    if status != 0:
        raise OracleError(status, err)


# ---------------------------------------------------------------- f16 ----
def f16_to_f32(bits) -> np.ndarray:
    b = _c(bits, np.uint16)
    out = np.empty(b.size, np.float32)
    lib().oracle_f16_to_f32_array(_ptr(b), _ptr(out), b.size)
    return out


def f32_to_f16(values) -> np.ndarray:
    v = _c(values, np.float32)
    out = np.empty(v.size, np.uint16)
    lib().oracle_f32_to_f16_array(_ptr(v), _ptr(out), v.size)
    return out


# ------------------------------------------------------ mote-reference ----
def dequantize_quantized_row(row_bytes, fmt: int, row_elements: int) -> np.ndarray:
    """``mote_reference::dequantize_quantized_row`` (quantized.rs:58-74)."""
    b = _c(row_bytes, np.uint8)
    # Geometry that cannot be allocated is rejected by the C side before it
    # writes anything, so a dummy output buffer is enough there.
    out = np.empty(row_elements if row_elements < (1 << 40) else 0, np.float32)
    err = _Err()
    _check(lib().oracle_dequantize_quantized_row(_ptr(b), b.size, fmt, row_elements,
                                                 _ptr(out), ctypes.byref(err)), err)
    return out


def dequantize_matrix(weights, rows: int, k: int, fmt: int = Q4_0) -> np.ndarray:
    """Row-by-row dequantization of a [rows, k] block-encoded matrix."""
    w = _c(weights, np.uint8)
    rb = (k // 32) * (18 if fmt == Q4_0 else 34)
    out = np.empty((rows, k), np.float32)
    for r in range(rows):
        out[r] = dequantize_quantized_row(w[r * rb:(r + 1) * rb], fmt, k)
    return out


def quantized_linear_f32(inp, weights, fmt: int, rows: int, output_features: int,
                         input_features: int, threads: int = 1) -> np.ndarray:
    """``mote_reference::quantized_linear_f32`` (quantized.rs:89-144).

    ``threads > 1`` partitions the output features over POSIX threads; the
    per-element arithmetic is unchanged, so results are bit-identical.
    """
    x = _c(inp, np.float32)
    w = _c(weights, np.uint8)
    n_out = rows * output_features if rows * output_features < (1 << 62) else 0
    out = np.empty(n_out, np.float32)
    err = _Err()
    if threads > 1:
        st = lib().oracle_quantized_linear_f32_mt(_ptr(x), x.size, _ptr(w), w.size, fmt, rows,
                                                  output_features, input_features, _ptr(out),
                                                  threads, ctypes.byref(err))
    else:
        st = lib().oracle_quantized_linear_f32(_ptr(x), x.size, _ptr(w), w.size, fmt, rows,
                                               output_features, input_features, _ptr(out),
                                               ctypes.byref(err))
    _check(st, err)
    return out


# ------------------------------------------------------------- K-quants ----
KQUANT_BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}


def kquant_dequantize(weights, fmt: int, rows: int, k: int) -> np.ndarray:
    """[rows, k] f32 values of a Q4_K / Q6_K matrix (ggml's dequantization
    as gguf 0.19.0 states it; the reference itself rejects these formats)."""
    w = _c(weights, np.uint8)
    rb = k // 256 * KQUANT_BLOCK_BYTES.get(fmt, 0)
    out = np.empty((rows, k), np.float32)
    for r in range(rows):
        st = lib().oracle_kquant_dequantize_row(_ptr(w[r * rb:(r + 1) * rb]), rb, fmt, k,
                                                _ptr(out[r]))
        if st != 0:
            raise OracleError(st, _Err())
    return out


def kquant_linear_f64(inp, weights, fmt: int, rows: int, n: int, k: int) -> np.ndarray:
    """Y = X . dequant(W)^T with f64 accumulation (tolerance reference)."""
    x = _c(inp, np.float32)
    w = _c(weights, np.uint8)
    out = np.empty(rows * n, np.float64)
    st = lib().oracle_kquant_linear_f64(_ptr(x), _ptr(w), fmt, rows, n, k, _ptr(out))
    if st != 0:
        raise OracleError(st, _Err())
    return out.reshape(rows, n)


def matmul_f32(lhs, rhs, m: int, n: int, k: int) -> np.ndarray:
    """``mote_reference::matmul_f32`` (lib.rs:116-156)."""
    a = _c(lhs, np.float32)
    b = _c(rhs, np.float32)
    out = np.empty(m * n if m * n < (1 << 40) else 0, np.float32)
    err = _Err()
    _check(lib().oracle_matmul_f32(_ptr(a), a.size, _ptr(b), b.size, m, n, k, _ptr(out),
                                   ctypes.byref(err)), err)
    return out


def rope_f32(inp, cos, sin, tokens: int, heads: int, head_dim: int, rotary_dim: int,
             layout: int) -> np.ndarray:
    """``mote_reference::rope_f32`` (lib.rs:170-244)."""
    x = _c(inp, np.float32)
    c = _c(cos, np.float32)
    s = _c(sin, np.float32)
    out = np.empty(x.size, np.float32)
    err = _Err()
    _check(lib().oracle_rope_f32(_ptr(x), x.size, _ptr(c), c.size, _ptr(s), s.size, tokens,
                                 heads, head_dim, rotary_dim, layout, _ptr(out),
                                 ctypes.byref(err)), err)
    return out


def rms_norm_f32(inp, weight, hidden_size: int, epsilon: float) -> np.ndarray:
    """``mote_reference::rms_norm_f32`` (lib.rs:262-301)."""
    x = _c(inp, np.float32)
    w = _c(weight, np.float32)
    out = np.empty(x.size, np.float32)
    err = _Err()
    _check(lib().oracle_rms_norm_f32(_ptr(x), x.size, _ptr(w), w.size, hidden_size,
                                     ctypes.c_float(epsilon), _ptr(out), ctypes.byref(err)), err)
    return out


def fused_add_rms_norm_f32(inp, residual, weight, hidden_size: int, epsilon: float):
    """``mote_reference::fused_add_rms_norm_f32`` (lib.rs:333-384).

    Returns ``(normalized, residual)`` like ``FusedAddRmsNormOutput``.
    """
    x = _c(inp, np.float32)
    r = _c(residual, np.float32)
    w = _c(weight, np.float32)
    normalized = np.empty(x.size, np.float32)
    res_out = np.empty(x.size, np.float32)
    err = _Err()
    _check(lib().oracle_fused_add_rms_norm_f32(_ptr(x), x.size, _ptr(r), r.size, _ptr(w),
                                               w.size, hidden_size, ctypes.c_float(epsilon),
                                               _ptr(normalized), _ptr(res_out),
                                               ctypes.byref(err)), err)
    return normalized, res_out


# ------------------------------------------------------- new operators ----
def q4_0_quantize(values, rows: int, k: int) -> np.ndarray:
    """Q4_0 encoder (ggml's published reference quantizer, restated)."""
    x = _c(values, np.float32)
    assert x.size == rows * k and k % 32 == 0
    out = np.empty(rows * (k // 32) * 18, np.uint8)
    st = lib().oracle_q4_0_quantize_rows(_ptr(x), rows, k, _ptr(out))
    if st != 0:
        raise OracleError(st, _Err())
    return out


def embedding_gather_f16(table_bits, vocab: int, hidden: int, ids):
    t = _c(table_bits, np.uint16)
    i = _c(ids, np.int32)
    out = np.empty(i.size * hidden, np.uint16)
    flag = np.zeros(1, np.uint32)
    lib().oracle_embedding_gather_f16(_ptr(t), vocab, hidden, _ptr(i), i.size, _ptr(out),
                                      _ptr(flag))
    return out, int(flag[0])


def swiglu_f64(gate, up) -> np.ndarray:
    g = _c(gate, np.float32)
    u = _c(up, np.float32)
    out = np.empty(g.size, np.float32)
    lib().oracle_swiglu_f64(_ptr(g), _ptr(u), g.size, _ptr(out))
    return out


def rope_cos_sin_f64(positions, rotary_dim: int, theta: float):
    p = _c(positions, np.int32)
    half = rotary_dim // 2
    c = np.empty(p.size * half, np.float32)
    s = np.empty(p.size * half, np.float32)
    st = lib().oracle_rope_cos_sin_f64(_ptr(p), p.size, rotary_dim, ctypes.c_double(theta),
                                       _ptr(c), _ptr(s))
    if st != 0:
        raise OracleError(st, _Err())
    return c.reshape(p.size, half), s.reshape(p.size, half)


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
