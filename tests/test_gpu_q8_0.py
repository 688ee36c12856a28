"""GPU parity of the Q8_0 linear (mote_cuda_quantized_linear_q8_0_f16*).

Weights are seeded Q8_0 blocks (random f16 scales, signed bytes in
[-127, 127]); the oracle is mote-reference's quantized_linear_f32 for Q8_0
restated in C (decode = f32(q) * f32(d), quantized.rs:191-195), bit-exact
with the Rust crate.  Bounds, as for the Q4_0 decode path: the reference
test rule (abs 0.01 / rel 0.002) against the f16-rounded f32 oracle, and
1e-3 normwise and element-wise (rms floor) against a float64 accumulation
of the exactly decoded weights.  The fast path (K % 256 == 0, aligned),
the generic kernel (other K, unaligned input), ragged N, every token count
up to 16, chunked launches beyond 16 (N % 16 != 0), the tcgen05 prefill
path (more than 16 tokens, N % 16 == 0) and the f32 output are covered.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker

pytestmark = pytest.mark.gpu

from mote_b200 import errors, ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, QuantFormat, plain, quantized  # noqa: E402

BOUND = 1e-3


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def q8_0_weights(n: int, k: int, seed: int) -> np.ndarray:
    """[N, K/32] blocks: f16 scale ~ 0.02/127 * U(0.5, 1.5) * (+-1), int8 in [-127, 127]."""
    rng = np.random.default_rng(seed)
    nb = k // 32
    d = (rng.uniform(0.5, 1.5, (n, nb)) * rng.choice([-1.0, 1.0], (n, nb)) * 0.02 / 127)
    q = rng.integers(-127, 128, (n, nb, 32)).astype(np.int8)
    out = np.empty((n, nb, 34), np.uint8)
    out[:, :, 0:2] = d.astype(np.float16).view(np.uint8).reshape(n, nb, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def q8_0_dequant(w: np.ndarray, n: int, k: int) -> np.ndarray:
    blocks = w.reshape(n, k // 32, 34)
    d = blocks[:, :, 0:2].copy().view(np.float16).astype(np.float64)
    q = blocks[:, :, 2:].view(np.int8).astype(np.float64)
    return (q * d).reshape(n, k)


def run(ctx, x, w, m, n, k, out_dtype=DType.F16):
    xt = ctx.from_bytes(plain((m, k), DType.F16), x.astype(np.float16))
    wt = ctx.from_bytes(quantized((n, k), QuantFormat.Q8_0), w)
    yt = ctx.empty(plain((m, n), out_dtype))
    ops.quantized_linear_q8_0(ctx, xt, wt, yt, out_dtype)
    np_out = np.float16 if out_dtype is DType.F16 else np.float32
    got = np.frombuffer(ctx.read_bytes(yt), np_out).astype(np.float32).reshape(m, n)
    assert ctx.device_status() == 0
    return got


def tensor_core_path(m, n, k):
    """More than 16 tokens with N % 16 == 0 and K % 256 == 0 run on the
    tcgen05 GEMM, which rounds each weight q * d to f16 (<= 2^-11 relative):
    element-wise bound 2e-3 there, as for the Q4_0 prefill path."""
    return m > 16 and n % 16 == 0 and k % 256 == 0


def check(oracle_lib, got, x, w, m, n, k, f16_out=True, rows=None):
    x32 = x.astype(np.float16).astype(np.float32)
    if rows is None:
        want = oracle_lib.quantized_linear_f32(x32, w, oracle_lib.Q8_0, m, n, k,
                                               threads=8).reshape(m, n)
        ok, bad = checker.within_reference_tolerance(
            got, checker.f16_round(want) if f16_out else want, 0.01, 0.002)
        assert ok, bad
    else:  # sampled rows of a large problem
        got, x32 = got[rows], x32[rows]
    ref64 = checker.linear_f64(x32, q8_0_dequant(w, n, k))
    assert checker.rel_err_normwise(got, ref64) <= BOUND
    elementwise = 2e-3 if tensor_core_path(m, n, k) else BOUND
    assert checker.rel_err_elementwise(got, ref64) <= elementwise


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9, 12, 16, 17, 40])
@pytest.mark.parametrize("n,k", [(2048, 2048), (40, 256), (300, 4096)])
def test_q8_0_matches_oracle(ctx, oracle_lib, m, n, k):
    w = q8_0_weights(n, k, seed=n + k)
    x = np.random.default_rng(m).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, run(ctx, x, w, m, n, k), x, w, m, n, k)


@pytest.mark.parametrize("m,n,k", [(1, 1000, 8192), (4, 528, 14336), (16, 64, 6144),
                                   (1, 16032, 4096)])
def test_q8_0_long_k_and_splits(ctx, oracle_lib, m, n, k):
    w = q8_0_weights(n, k, seed=7 + n)
    x = np.random.default_rng(9 + m).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, run(ctx, x, w, m, n, k), x, w, m, n, k)


@pytest.mark.parametrize("m,n,k", [(17, 256, 256), (64, 4096, 4096), (200, 528, 1024),
                                   (129, 16, 768), (300, 2048, 2048)])
def test_q8_0_prefill_tensor_cores(ctx, oracle_lib, m, n, k):
    """More than 16 tokens on the tcgen05 GEMM with Q8_0 conversion (TMA of
    272-byte rows as 2-byte units, exact byte decode, q * d rounded to f16);
    N % 16 == 0 and K % 256 == 0, ragged M."""
    w = q8_0_weights(n, k, seed=40 + m)
    x = np.random.default_rng(41 + m).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, run(ctx, x, w, m, n, k), x, w, m, n, k)


def test_q8_0_prefill_full_size_sampled(ctx):
    """M=2048, K=4096, N=14336 on the tensor cores, 64 sampled rows x all N
    in float64."""
    m, n, k = 2048, 14336, 4096
    w = q8_0_weights(n, k, seed=77)
    x = np.random.default_rng(78).normal(0, 1, (m, k)).astype(np.float16)
    got = run(ctx, x, w, m, n, k)
    rows = np.random.default_rng(0).choice(m, 64, replace=False)
    check(None, got, x, w, m, n, k, rows=rows)


@pytest.mark.parametrize("m,n,k", [(3, 100, 96), (9, 33, 1056), (1, 7, 32)])
def test_q8_0_generic_path(ctx, oracle_lib, m, n, k):
    """K not a multiple of 256: the warp-per-row kernel."""
    w = q8_0_weights(n, k, seed=3 + n)
    x = np.random.default_rng(5).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, run(ctx, x, w, m, n, k), x, w, m, n, k)


def test_q8_0_f32_output(ctx, oracle_lib):
    m, n, k = 5, 512, 2048
    w = q8_0_weights(n, k, seed=11)
    x = np.random.default_rng(12).normal(0, 1, (m, k)).astype(np.float16)
    check(oracle_lib, run(ctx, x, w, m, n, k, DType.F32), x, w, m, n, k, f16_out=False)


def test_q8_0_unaligned_input_takes_generic_path(ctx, oracle_lib):
    """An input 2 bytes past a 16-byte boundary: same results as aligned."""
    import ctypes

    from mote_b200._native import lib

    m, n, k = 2, 256, 512
    w = q8_0_weights(n, k, seed=21)
    x = np.random.default_rng(22).normal(0, 1, (m, k)).astype(np.float16)
    buf = ctx.from_bytes(plain((m * k + 8,), DType.F16),
                         np.concatenate([np.zeros(1, np.float16), x.reshape(-1),
                                         np.zeros(7, np.float16)]))
    wt = ctx.from_bytes(quantized((n, k), QuantFormat.Q8_0), w)
    yt = ctx.empty(plain((m, n), DType.F16))
    assert lib().mote_cuda_quantized_linear_q8_0_f16(buf.pointer + 2, wt.pointer, yt.pointer, m,
                                                     n, k, ctx.stream) == 0
    got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, n)
    check(oracle_lib, got, x, w, m, n, k)


def test_q8_0_exact_integer_blocks(ctx):
    """Blocks with scale 1.0 and small integer quants (0..31, and -1
    repeated): exact integer dot products, representable in f16."""
    n, k, m = 2, 32, 1
    w = np.zeros((n, 34), np.uint8)
    w[:, 0:2] = np.array([1.0], np.float16).view(np.uint8)
    w[0, 2:] = np.arange(32, dtype=np.int8).view(np.uint8)
    w[1, 2:] = np.full(32, -1, np.int8).view(np.uint8)
    x = np.ones((m, k), np.float16)
    got = run(ctx, x, w.reshape(-1), m, n, k)
    assert got.tolist() == [[496.0, -32.0]]


def test_q8_0_argument_rules(ctx):
    x = ctx.from_bytes(plain((1, 256), DType.F16), np.zeros(256, np.float16))
    w4 = ctx.empty(quantized((16, 256)))
    y = ctx.empty(plain((1, 16), DType.F16))
    with pytest.raises(errors.UnsupportedEncoding):  # a Q4_0 tensor
        ops.quantized_linear_q8_0(ctx, x, w4, y)
    w8 = ctx.empty(quantized((16, 256), QuantFormat.Q8_0))
    with pytest.raises(errors.DTypeMismatch):
        ops.quantized_linear_q8_0(ctx, x, w8, y, DType.I32)
