"""Input generators shared by the tests.

Two families:
* the reference's own deterministic index-formula fixtures
  (crates/mote-backend-hip/tests/*.rs, benches/quantized_linear.rs), so the
  GPU tests read like the reference's GPU tests;
* seeded synthetic inputs with the BASELINE configs' distributions
  (weights ~ N(0, 0.02) Q4_0-encoded, activations ~ N(0, 1)).
"""
from __future__ import annotations

import numpy as np


def f16(values) -> np.ndarray:
    return np.asarray(values, np.float32).astype(np.float16)


def f16_bits(values) -> np.ndarray:
    return f16(values).view(np.uint16)


# ---- reference formula fixtures --------------------------------------------
def hip_linear_input(rows: int, k: int) -> np.ndarray:
    """tests/quantized_linear.rs:16-18: f16((index % 23) / 7 - 1.5)."""
    idx = np.arange(rows * k)
    return f16((idx % 23).astype(np.float32) / np.float32(7.0) - np.float32(1.5)).reshape(rows, k)


def hip_linear_weights(n: int, k: int) -> np.ndarray:
    """tests/quantized_linear.rs:160-177."""
    out = bytearray()
    for of in range(n):
        for block in range(k // 32):
            scale = np.float16(0.125 * ((of + block) % 4 + 1))
            out += scale.tobytes()
            for j in range(16):
                low = (of * 3 + block * 5 + j) % 16
                high = (of * 7 + block * 2 + j * 3 + 1) % 16
                out.append(low | (high << 4))
    return np.frombuffer(bytes(out), np.uint8)


def hip_bench_weights(n: int, k: int) -> np.ndarray:
    """benches/quantized_linear.rs:134-152 (vectorised)."""
    nb = k // 32
    of = np.arange(n)[:, None, None]
    blk = np.arange(nb)[None, :, None]
    j = np.arange(16)[None, None, :]
    scale = (np.float32(0.015625) * (((of[:, :, 0] * 3 + blk[:, :, 0]) % 4) + 1)).astype(np.float16)
    low = (of * 5 + blk * 3 + j) % 16
    high = (of * 7 + blk + j * 3 + 1) % 16
    qs = (low | (high << 4)).astype(np.uint8)
    out = np.empty((n, nb, 18), np.uint8)
    out[:, :, 0:2] = scale.view(np.uint8).reshape(n, nb, 2)
    out[:, :, 2:] = qs
    return out.reshape(-1)


def hip_bench_input(rows: int, k: int) -> np.ndarray:
    """benches/quantized_linear.rs:128-132: f16((index % 29) / 14 - 1)."""
    idx = np.arange(rows * k)
    return f16((idx % 29).astype(np.float32) / np.float32(14.0) - np.float32(1.0)).reshape(rows, k)


def norm_input(n: int) -> np.ndarray:
    """tests/rms_norm.rs:161-163 and rope.rs: ((i*37+5) % 19) / 6 - 1.5."""
    i = np.arange(n)
    return ((i * 37 + 5) % 19).astype(np.float32) / np.float32(6.0) - np.float32(1.5)


def norm_weight(n: int) -> np.ndarray:
    """tests/rms_norm.rs:165-167: 0.5 + ((i*7+3) % 13) / 12."""
    i = np.arange(n)
    return np.float32(0.5) + ((i * 7 + 3) % 13).astype(np.float32) / np.float32(12.0)


def residual_input(n: int) -> np.ndarray:
    """tests/fused_add_rms_norm.rs:485-487: ((i*11+7) % 23) / 8 - 1.4."""
    i = np.arange(n)
    return ((i * 11 + 7) % 23).astype(np.float32) / np.float32(8.0) - np.float32(1.4)


def rope_cos(n: int) -> np.ndarray:
    """tests/rope.rs (cos_element): ((i*11+3) % 13) / 12."""
    i = np.arange(n)
    return ((i * 11 + 3) % 13).astype(np.float32) / np.float32(12.0)


def rope_sin(n: int) -> np.ndarray:
    """tests/rope.rs (sin_element): ((i*7+1) % 17) / 16."""
    i = np.arange(n)
    return ((i * 7 + 1) % 17).astype(np.float32) / np.float32(16.0)


# ---- seeded synthetic -------------------------------------
def q4_0_weights(oracle_ref, n: int, k: int, seed: int, std: float = 0.02) -> np.ndarray:
    """W ~ N(0, std) f32, Q4_0-encoded by the oracle's encoder."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, std, (n, k)).astype(np.float32)
    return oracle_ref.q4_0_quantize(w, n, k)


def activations(m: int, k: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).normal(0.0, 1.0, (m, k)).astype(np.float32)
