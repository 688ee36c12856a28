"""Independent float64 checkers and the error metrics of the parity tests.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference's own tests judge GPU output against the f32 oracle with
``|actual - expected| <= max(abs_tol, rel_tol * |expected|)``
(crates/mote-backend-hip/tests/quantized_linear.rs:53-61,
tests/rms_norm.rs:50-61, tests/rope.rs:416-421);
:func:`within_reference_tolerance` is that rule.

The specification's bound is "max relative error <= 1e-3 against an f64
accumulation".  A dot product can cancel to (nearly) zero, so an
element-wise relative error needs a floor; the two metrics used are

* ``rel_err_elementwise_tau``: ``max_i |y_i - r_i| / max(|r_i|, tau)`` with
  ``tau = 1e-3 * rms(r)`` -- the strict element-wise definition: only
  outputs within a thousandth of the RMS of zero are judged on absolute
  error;
* ``rel_err_elementwise``: ``max_i |y_i - r_i| / max(|r_i|, rms(r))`` --
  element-wise, floored at the RMS of the reference (looser: an output
  smaller than the RMS is judged on its absolute error / RMS);
* ``rel_err_normwise``: ``max_i |y_i - r_i| / max_i |r_i|``.

All are reported; each test states which bound it asserts.  Paths that
compute with the exact decoded weights (the decode GEMVs) meet the strict
tau-floored bound: their only rounding is the f32 accumulation and the
final f16 output rounding, which is relative.  The tensor-core prefill path
rounds every dequantized weight to f16 (as a dense f16 weight matrix is),
an absolute error per output of ~3e-4 * rms, so it is held to the
normwise and rms-floored bounds.
"""
from __future__ import annotations

import numpy as np

LINEAR_REL_TOL = 1e-3


def f16_round(values) -> np.ndarray:
    """Round to binary16 (round-to-nearest-even) and widen back to f32."""
    return np.asarray(values, np.float32).astype(np.float16).astype(np.float32)


def rms(values) -> float:
    v = np.asarray(values, np.float64)
    return float(np.sqrt(np.mean(v * v))) if v.size else 0.0


TAU_FRACTION = 1e-3


def rel_err_elementwise_tau(actual, ref, tau_fraction: float = TAU_FRACTION) -> float:
    a = np.asarray(actual, np.float64).reshape(-1)
    r = np.asarray(ref, np.float64).reshape(-1)
    if r.size == 0:
        return 0.0
    floor = max(tau_fraction * rms(r), np.finfo(np.float64).tiny)
    return float(np.max(np.abs(a - r) / np.maximum(np.abs(r), floor)))


def rel_err_elementwise(actual, ref) -> float:
    a = np.asarray(actual, np.float64).reshape(-1)
    r = np.asarray(ref, np.float64).reshape(-1)
    if r.size == 0:
        return 0.0
    floor = max(rms(r), np.finfo(np.float64).tiny)
    return float(np.max(np.abs(a - r) / np.maximum(np.abs(r), floor)))


def rel_err_normwise(actual, ref) -> float:
    a = np.asarray(actual, np.float64).reshape(-1)
    r = np.asarray(ref, np.float64).reshape(-1)
    if r.size == 0:
        return 0.0
    denom = max(float(np.max(np.abs(r))), np.finfo(np.float64).tiny)
    return float(np.max(np.abs(a - r)) / denom)


def within_reference_tolerance(actual, expected, abs_tol: float, rel_tol: float):
    """The reference tests' rule; returns (ok, index_of_first_failure)."""
    a = np.asarray(actual, np.float64).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    tol = np.maximum(abs_tol, rel_tol * np.abs(e))
    bad = np.nonzero(~(np.abs(a - e) <= tol))[0]
    return (bad.size == 0, int(bad[0]) if bad.size else -1)


# ------------------------------------------------------------ float64 ops --
def linear_f64(x, w_dequant) -> np.ndarray:
    """``y = x @ W^T`` accumulated in float64 from the decoded weights."""
    return np.asarray(x, np.float64) @ np.asarray(w_dequant, np.float64).T


def q4_0_dequant_np(weights: np.ndarray, rows: int, k: int) -> np.ndarray:
    """Vectorised Q4_0 decode (independent of the C restatement)."""
    blocks = np.asarray(weights, np.uint8).reshape(rows, k // 32, 18)
    d = blocks[:, :, 0:2].copy().view(np.float16).astype(np.float32)  # [rows, nb, 1]
    qs = blocks[:, :, 2:]
    lo = (qs & 0x0F).astype(np.int8) - 8
    hi = (qs >> 4).astype(np.int8) - 8
    q = np.concatenate([lo, hi], axis=2).astype(np.float32)  # [rows, nb, 32]
    return (q * d).reshape(rows, k)


def rms_norm_f64(x, w, hidden: int, eps: float) -> np.ndarray:
    x64 = np.asarray(x, np.float64).reshape(-1, hidden)
    ms = np.mean(x64 * x64, axis=1, keepdims=True)
    return x64 / np.sqrt(ms + float(np.float32(eps))) * np.asarray(w, np.float64)


def fused_add_rms_norm_f64(x, r, w, hidden: int, eps: float):
    s = np.asarray(x, np.float64) + np.asarray(r, np.float64)
    return rms_norm_f64(s, w, hidden, eps), s


def rope_f64(x, cos, sin, tokens: int, heads: int, head_dim: int, rotary_dim: int,
             layout: int) -> np.ndarray:
    v = np.asarray(x, np.float64).reshape(tokens, heads, head_dim).copy()
    half = rotary_dim // 2
    c = np.asarray(cos, np.float64).reshape(tokens, 1, half)
    s = np.asarray(sin, np.float64).reshape(tokens, 1, half)
    if layout == 0:
        a = v[:, :, :half].copy()
        b = v[:, :, half:rotary_dim].copy()
        v[:, :, :half] = a * c - b * s
        v[:, :, half:rotary_dim] = b * c + a * s
    else:
        a = v[:, :, 0:rotary_dim:2].copy()
        b = v[:, :, 1:rotary_dim:2].copy()
        v[:, :, 0:rotary_dim:2] = a * c - b * s
        v[:, :, 1:rotary_dim:2] = b * c + a * s
    return v.reshape(-1)


def swiglu_f64(g, u) -> np.ndarray:
    g64 = np.asarray(g, np.float64)
    return g64 / (1.0 + np.exp(-g64)) * np.asarray(u, np.float64)


def ulp_distance_f32(a, b) -> np.ndarray:
    """Distance in units in the last place between two f32 arrays."""
    ai = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    bi = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


def gqa_attention_f64(q, k, v, query_positions, scale: float) -> np.ndarray:
    """Grouped-query attention in float64 (no reference operator: the
    reference names attention with a KV cache as planned,
    docs/roadmap.md:58-60; this is the standard definition).

    ``q`` [T, Hq, D]; ``k``, ``v`` [S, Hkv, D] for key positions 0..S-1;
    query ``t`` sits at position ``query_positions[t]`` and attends keys
    ``0..query_positions[t]`` (inclusive); query head ``h`` reads KV head
    ``h // (Hq // Hkv)``.  Returns [T, Hq, D]."""
    q64 = np.asarray(q, np.float64)
    k64 = np.asarray(k, np.float64)
    v64 = np.asarray(v, np.float64)
    t, hq, d = q64.shape
    s_len, hkv, _ = k64.shape
    g = hq // hkv
    pos = np.asarray(query_positions, np.int64).reshape(t, 1)
    mask = np.arange(s_len)[None, :] > pos  # [T, S]
    out = np.zeros((t, hq, d), np.float64)
    for h in range(hq):
        kh = k64[:, h // g, :]
        sc = (q64[:, h, :] @ kh.T) * scale  # [T, S]
        sc[mask] = -np.inf
        mx = np.max(sc, axis=1, keepdims=True)
        mx[~np.isfinite(mx)] = 0.0
        p = np.exp(sc - mx)
        denom = p.sum(axis=1, keepdims=True)
        denom[denom == 0] = 1.0
        out[:, h, :] = (p / denom) @ v64[:, h // g, :]
    return out
