"""mote_cuda_quantized_linear_q4_0_f16_noalloc: the workspace linear with its
split-K scratch in a static per-device array.

Compared with the existing entry point mote_cuda_quantized_linear_q4_0_f16_ws
(given a zeroed workspace) over two calls in a row: the outputs must be
identical, complete (the outputs start as NaN) and the same on the second
call, which works only if the first left the static counters at zero.  The
shapes cover the decode GEMV with and without its K split over CTAs, and
the tensor-core GEMM with its last-wave K split inside the static scratch
(64 tokens, 346 tiles: 2 or 4 parts on 148 SMs) and unsplit (2048 tokens).
A decode request whose split needs more than the static scratch is
rejected with status 10200 before anything is enqueued.  The file is
collected last and also passes on its own.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from mote_b200._native import lib, status_string  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain, quantized  # noqa: E402
from tests import _fixtures as fx  # noqa: E402

SCRATCH_TOO_SMALL = 10200


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (12, 2048, 4096), (9, 300, 8192),
                                   (1, 4096, 4096), (16, 1000, 2048), (64, 44288, 4096),
                                   (2048, 4096, 4096)])
def test_noalloc_matches_workspace_entry_twice(ctx, oracle_lib, m, n, k):
    w = fx.q4_0_weights(oracle_lib, n, k, seed=800 + n)
    x = fx.activations(m, k, seed=801 + m).astype(np.float16)
    xt = ctx.from_bytes(plain((m, k), DType.F16), x)
    wt = ctx.from_bytes(quantized((n, k)), w)
    need = ctypes.c_uint64(0)
    assert lib().mote_cuda_q4_0_linear_workspace_bytes(m, n, k, ctypes.byref(need)) == 0
    ws = ctx.from_bytes(plain((max(need.value, 256),), DType.U8),
                        np.zeros(max(need.value, 256), np.uint8))
    nan = np.full(m * n, np.nan, np.float16)

    def run(noalloc: bool) -> np.ndarray:
        yt = ctx.from_bytes(plain((m, n), DType.F16), nan)
        if noalloc:
            st = lib().mote_cuda_quantized_linear_q4_0_f16_noalloc(
                xt.pointer, wt.pointer, yt.pointer, m, n, k, ctx.stream)
        else:
            st = lib().mote_cuda_quantized_linear_q4_0_f16_ws(
                xt.pointer, wt.pointer, yt.pointer, m, n, k, ws.pointer, need.value, ctx.stream)
        assert st == 0, status_string(st)
        return np.frombuffer(ctx.read_bytes(yt), np.uint16).reshape(m, n)

    for _ in range(2):  # two calls in a row each
        a, b = run(True), run(False)
        assert np.array_equal(a, b)
        assert not np.isnan(a.view(np.float16)).any()
    assert ctx.device_status() == 0


def test_noalloc_rejects_oversized_split(ctx):
    # 9 tokens, 4096 row tiles: the 2-way K split needs 256 KiB of counters
    # + 2 x 4096 x 256 x 4 B of partial sums = 8.25 MiB > 8 MiB
    m, n, k = 9, 65536, 4096
    x = ctx.empty(plain((m, k), DType.F16))
    w = ctx.empty(quantized((n, k)))
    y = ctx.empty(plain((m, n), DType.F16))
    st = lib().mote_cuda_quantized_linear_q4_0_f16_noalloc(x.pointer, w.pointer, y.pointer, m, n,
                                                           k, ctx.stream)
    assert st == SCRATCH_TOO_SMALL
    assert "static scratch" in status_string(st)
    ctx.sync()
    assert ctx.device_status() == 0
