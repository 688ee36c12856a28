"""GPU parity of the dense f16 x f16 -> f32 matmul (cuBLASLt), the CUDA
counterpart of the HIP backend's hipBLASLt matmul.

The first case restates the reference's own test
(crates/mote-backend-hip/tests/matmul.rs:12-48: M=48, N=64, K=32,
deterministic values, |a - e| <= max(0.05, 0.002 |e|) against
mote-reference's matmul_f32, here the pinned C oracle).  The others hold
seeded N(0, 1) shapes to 1e-3 element-wise (rms floor) against a float64
product, and check the empty and K = 0 rules, the cached plan on repeat
calls and the error path."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import checker

pytestmark = pytest.mark.gpu

from mote_b200 import errors, ops  # noqa: E402
from mote_b200._native import lib  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def matmul(ctx, a, b):
    m, k = a.shape
    n = b.shape[1]
    lt = ctx.from_bytes(plain((m, k), DType.F16), a.astype(np.float16))
    rt = ctx.from_bytes(plain((k, n), DType.F16), b.astype(np.float16))
    ot = ctx.empty(plain((m, n), DType.F32))
    ops.matmul_f16_f32(ctx, lt, rt, ot)
    return np.frombuffer(ctx.read_bytes(ot), np.float32).reshape(m, n)


def test_reference_case(ctx, oracle_lib):
    m, n, k = 48, 64, 32
    r, c = np.meshgrid(np.arange(m), np.arange(k), indexing="ij")
    a = (((r * 7 + c * 3) % 17) / 8.0 - 1.0).astype(np.float16)
    r, c = np.meshgrid(np.arange(k), np.arange(n), indexing="ij")
    b = (((r * 5 + c * 11) % 19) / 8.0 - 1.0).astype(np.float16)
    got = matmul(ctx, a, b)
    want = oracle_lib.matmul_f32(a.astype(np.float32), b.astype(np.float32), m, n, k).reshape(m, n)
    assert np.all(np.abs(want - got) <= np.maximum(0.05, np.abs(want) * 0.002))


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 5, 7), (64, 128, 256), (17, 33, 65),
                                   (256, 4096, 2048), (2048, 2048, 2048)])
def test_matches_f64(ctx, m, n, k):
    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.normal(0, 1, (m, k)).astype(np.float16)
    b = rng.normal(0, 1, (k, n)).astype(np.float16)
    got = matmul(ctx, a, b)
    ref = checker.linear_f64(a.astype(np.float32), b.astype(np.float32).T)
    assert checker.rel_err_elementwise(got, ref) <= 1e-3
    again = matmul(ctx, a, b)  # the cached plan gives the same result
    assert np.array_equal(got, again)


def test_empty_and_zero_k(ctx):
    lt = ctx.empty(plain((4, 0), DType.F16))
    rt = ctx.empty(plain((0, 6), DType.F16))
    ot = ctx.from_bytes(plain((4, 6), DType.F32), np.full((4, 6), 7.0, np.float32))
    ops.matmul_f16_f32(ctx, lt, rt, ot)
    assert not np.frombuffer(ctx.read_bytes(ot), np.float32).any()
    e = ctx.empty(plain((0, 3), DType.F32))
    ops.matmul_f16_f32(ctx, ctx.empty(plain((0, 2), DType.F16)),
                       ctx.empty(plain((2, 3), DType.F16)), e)


def test_checks_and_null_arguments(ctx):
    with pytest.raises(errors.ShapeMismatch):
        ops.matmul_f16_f32(ctx, ctx.empty(plain((2, 3), DType.F16)),
                           ctx.empty(plain((4, 5), DType.F16)), ctx.empty(plain((2, 5), DType.F32)))
    with pytest.raises(errors.DTypeMismatch):
        ops.matmul_f16_f32(ctx, ctx.empty(plain((2, 3), DType.F16)),
                           ctx.empty(plain((3, 5), DType.F16)), ctx.empty(plain((2, 5), DType.F16)))
    handle, ws, ws_bytes = ctx.blas()
    st = lib().mote_cuda_blaslt_matmul_f16_f32(handle, 2, 2, 2, None, ws, ws, ws, ws_bytes,
                                                ctx.stream)
    assert st == -1
    assert b"null" in lib().mote_cuda_blaslt_last_error(handle)
