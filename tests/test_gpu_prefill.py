"""GPU parity of the prefill-shaped Q4_0 GEMM (tcgen05/TMEM path).

Problems with more tokens than one GEMV launch stages (M > 16), N % 16 == 0
and K % 256 == 0 run on the tensor-core kernel.  It dequantizes weights to
f16 (q - 8) * d -- correctly rounded, so each weight carries <= 2^-11
relative error -- and accumulates in f32.  Bounds, against a float64
accumulation of the exactly decoded weights:
* normwise max relative error (max|y - r| / max|r|) <= 1e-3 (north star);
* element-wise relative error with an rms floor <= 2e-3 (the f16 weight
  rounding adds ~2e-4 rms to the f16 output rounding's 4.9e-4 bound);
* the reference test rule abs 0.01 / rel 0.002 against the f16-rounded f32
  oracle (crates/mote-backend-hip/tests/quantized_linear.rs:53-61).
Config 5b (M=2048, K=4096, N=14336) is checked on 96 sampled rows x all N.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker
from tests import _fixtures as fx

pytestmark = pytest.mark.gpu

from mote_b200 import ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain, quantized  # noqa: E402

NORMWISE = 1e-3
ELEMENTWISE = 2e-3


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def run(ctx, x, w, m, n, k, out_dtype=DType.F16):
    xt = ctx.from_bytes(plain((m, k), DType.F16), x.astype(np.float16))
    wt = ctx.from_bytes(quantized((n, k)), w)
    yt = ctx.empty(plain((m, n), out_dtype))
    ops.quantized_linear_q4_0(ctx, xt, wt, yt, DType.F16, out_dtype)
    np_out = np.float16 if out_dtype is DType.F16 else np.float32
    got = np.frombuffer(ctx.read_bytes(yt), np_out).astype(np.float32).reshape(m, n)
    assert ctx.device_status() == 0
    return got


@pytest.mark.parametrize("m,n,k", [(17, 256, 256), (128, 256, 4096), (200, 528, 1024),
                                   (64, 4096, 4096), (256, 512, 2048), (129, 16, 768)])
def test_prefill_matches_f64(ctx, oracle_lib, m, n, k):
    w = fx.q4_0_weights(oracle_lib, n, k, seed=m * 7 + n)
    x = fx.activations(m, k, seed=n + k).astype(np.float16)
    got = run(ctx, x, w, m, n, k)
    ref = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w, n, k))
    assert checker.rel_err_normwise(got, ref) <= NORMWISE
    assert checker.rel_err_elementwise(got, ref) <= ELEMENTWISE
    want32 = oracle_lib.quantized_linear_f32(x.astype(np.float32), w, oracle_lib.Q4_0, m, n, k,
                                             threads=8).reshape(m, n)
    ok, bad = checker.within_reference_tolerance(got, checker.f16_round(want32), 0.01, 0.002)
    assert ok, bad


def test_prefill_f32_output(ctx, oracle_lib):
    m, n, k = 96, 256, 2048
    w = fx.q4_0_weights(oracle_lib, n, k, seed=5)
    x = fx.activations(m, k, seed=6).astype(np.float16)
    got = run(ctx, x, w, m, n, k, DType.F32)
    ref = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w, n, k))
    assert checker.rel_err_normwise(got, ref) <= 5e-4


def test_prefill_exact_on_small_integers(ctx):
    """Weights (q - 8) * d with d a power of two and integer activations:
    every product and partial sum is exact in f16/f32, so the GEMM must match
    an integer reference exactly."""
    rng = np.random.default_rng(1)
    m, n, k = 130, 64, 512
    q = rng.integers(0, 16, (n, k // 32, 32))
    blocks = np.zeros((n, k // 32, 18), np.uint8)
    blocks[:, :, 0:2] = np.array([np.float16(0.25)]).view(np.uint8)
    lo, hi = q[:, :, :16], q[:, :, 16:]
    blocks[:, :, 2:] = (lo | (hi << 4)).astype(np.uint8)
    w = blocks.reshape(-1)
    x = rng.integers(-3, 4, (m, k)).astype(np.float16)
    got = run(ctx, x, w, m, n, k, DType.F32)
    ref = x.astype(np.float64) @ ((q.reshape(n, k) - 8) * 0.25).T
    assert np.array_equal(got, ref.astype(np.float32))


def test_config5_prefill_full_size_sampled(ctx, oracle_lib):
    """Config 5b: M=2048, K=4096, N=14336, checked on 96 rows x all N in f64."""
    m, n, k = 2048, 14336, 4096
    w = fx.q4_0_weights(oracle_lib, n, k, seed=55)
    x = fx.activations(m, k, seed=56).astype(np.float16)
    got = run(ctx, x, w, m, n, k)
    rows = np.random.default_rng(0).choice(m, 96, replace=False)
    dec = checker.q4_0_dequant_np(w, n, k)
    ref = checker.linear_f64(x[rows].astype(np.float32), dec)
    assert checker.rel_err_normwise(got[rows], ref) <= NORMWISE
    assert checker.rel_err_elementwise(got[rows], ref) <= ELEMENTWISE


@pytest.mark.parametrize("m,n,k", [(512, 10240, 2048), (128, 38400, 2048), (64, 39680, 1024),
                                   (2048, 14336, 4096)])
def test_prefill_split_last_wave(ctx, oracle_lib, m, n, k):
    """Through the workspace entry the tiles of a partial last wave are split
    along K (on 148 SMs: 12 tiles x 8 parts, 4 x 8, 14 x 4 and 8 x 16 here)
    and their f32 parts added in part order by a second kernel: two calls
    give identical outputs, which agree with the unsplit kernel (the plain
    entry) and, on sampled rows, with a float64 accumulation."""
    import ctypes

    from mote_b200._native import lib

    w = fx.q4_0_weights(oracle_lib, n, k, seed=900 + m)
    x = fx.activations(m, k, seed=901 + m).astype(np.float16)
    xt = ctx.from_bytes(plain((m, k), DType.F16), x)
    wt = ctx.from_bytes(quantized((n, k)), w)
    need = ctypes.c_uint64(0)
    assert lib().mote_cuda_q4_0_linear_workspace_bytes(m, n, k, ctypes.byref(need)) == 0
    ws = ctx.from_bytes(plain((need.value,), DType.U8), np.zeros(need.value, np.uint8))
    nan = np.full(m * n, np.nan, np.float16)
    outs = []
    for split in (True, True, False):
        yt = ctx.from_bytes(plain((m, n), DType.F16), nan)
        if split:
            st = lib().mote_cuda_quantized_linear_q4_0_f16_ws(
                xt.pointer, wt.pointer, yt.pointer, m, n, k, ws.pointer, need.value, ctx.stream)
        else:
            st = lib().mote_cuda_quantized_linear_q4_0_f16(xt.pointer, wt.pointer, yt.pointer,
                                                           m, n, k, ctx.stream)
        assert st == 0
        outs.append(np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32)
                    .reshape(m, n))
    assert ctx.device_status() == 0
    assert np.array_equal(outs[0], outs[1]) and not np.isnan(outs[0]).any()
    ok, bad = checker.within_reference_tolerance(outs[0], outs[2], 0.01, 0.002)
    assert ok, bad
    rows = np.random.default_rng(1).choice(m, min(m, 48), replace=False)
    ref = checker.linear_f64(x[rows].astype(np.float32), checker.q4_0_dequant_np(w, n, k))
    assert checker.rel_err_normwise(outs[0][rows], ref) <= NORMWISE
    assert checker.rel_err_elementwise(outs[0][rows], ref) <= ELEMENTWISE
