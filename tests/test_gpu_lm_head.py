"""Config 5a at full size: the Q4_0 lm_head, K=4096, N=128256, M in {1, 16, 64}.

These are the shapes the lm_head figures are measured on, and they reach
code no smaller test does:
* M=1 and M=16 run the decode GEMV with its lm_head-sized warp split (pairs
  of warps per 16-row tile once the tiles outnumber the warps: N above
  ~22k rows) over 8016 tiles;
* M=64 runs the tcgen05 GEMM with 64-token tiles, whose partial last wave
  (1002 tiles on the resident slots) is split along K through the context's
  workspace and added in part order by the reduction kernel.

Weights ~ N(0, 0.02) Q4_0-encoded by the oracle's encoder (bit-exact with
the device encoder, test_gpu_codec.py), activations ~ N(0, 1) f16, through
``mote_b200.ops.quantized_linear_q4_0`` (the workspace entry).  Every one of
the M x 128256 outputs is compared with a float64 accumulation of the
decoded weights, computed in row chunks:
* M = 1, 16 (exact decode): element-wise relative error <= 1e-3 with the
  strict floor tau = 1e-3 * rms(ref), and normwise <= 1e-3;
* M = 64 (f16-rounded weights on the tensor cores): normwise <= 1e-3 and
  rms-floored element-wise <= 2e-3, as for every prefill shape.
On sampled row windows (the first, two middle and the last 512 output
features, the last one ending at the ragged end of the tile grid), the
outputs also meet the reference test rule abs 0.01 / rel 0.002 against the
f16-rounded f32 oracle (crates/mote-backend-hip/tests/quantized_linear.rs:53-61).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker

pytestmark = pytest.mark.gpu

from mote_b200 import ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain, quantized  # noqa: E402

M_MAX, N, K = 64, 128256, 4096
ROW_BYTES = K // 32 * 18
CHUNK = 8192
WINDOWS = [(0, 512), (40000, 40512), (80064, 80576), (N - 512, N)]
DECODE_BOUND = 1e-3
PREFILL_ELEMENTWISE = 2e-3


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


@pytest.fixture(scope="module")
def lm_head(oracle_lib):
    """Q4_0 weight bytes, 64 activation rows and their float64 outputs."""
    rng = np.random.default_rng(5128)
    x = rng.standard_normal((M_MAX, K), dtype=np.float32).astype(np.float16)
    x64 = x.astype(np.float64)
    w = np.empty(N * ROW_BYTES, np.uint8)
    ref = np.empty((M_MAX, N), np.float64)
    for r0 in range(0, N, CHUNK):
        r1 = min(N, r0 + CHUNK)
        f = rng.standard_normal((r1 - r0, K), dtype=np.float32) * np.float32(0.02)
        wb = oracle_lib.q4_0_quantize(f, r1 - r0, K)
        w[r0 * ROW_BYTES:r1 * ROW_BYTES] = wb
        ref[:, r0:r1] = x64 @ checker.q4_0_dequant_np(wb, r1 - r0, K).astype(np.float64).T
    return w, x, ref


@pytest.fixture(scope="module")
def weights_on_device(ctx, lm_head):
    w, _, _ = lm_head
    return ctx.from_bytes(quantized((N, K)), w)


@pytest.mark.parametrize("m", [1, 16, 64])
def test_config5_lm_head_full_size(ctx, oracle_lib, lm_head, weights_on_device, m):
    w, x_all, ref_all = lm_head
    x, ref = x_all[:m], ref_all[:m]
    xt = ctx.from_bytes(plain((m, K), DType.F16), x)
    yt = ctx.from_bytes(plain((m, N), DType.F16), np.full(m * N, np.nan, np.float16))
    ops.quantized_linear_q4_0(ctx, xt, weights_on_device, yt, DType.F16, DType.F16)
    got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, N)
    assert ctx.device_status() == 0
    assert not np.isnan(got).any()
    assert checker.rel_err_normwise(got, ref) <= DECODE_BOUND
    if m <= 16:
        assert checker.rel_err_elementwise_tau(got, ref) <= DECODE_BOUND
    else:
        assert checker.rel_err_elementwise(got, ref) <= PREFILL_ELEMENTWISE
    threads = min(8, max(1, oracle_lib.host_threads()))
    x32 = x.astype(np.float32)
    for r0, r1 in WINDOWS:
        want = oracle_lib.quantized_linear_f32(x32, w[r0 * ROW_BYTES:r1 * ROW_BYTES],
                                               oracle_lib.Q4_0, m, r1 - r0, K,
                                               threads=threads).reshape(m, r1 - r0)
        ok, bad = checker.within_reference_tolerance(got[:, r0:r1], checker.f16_round(want),
                                                     0.01, 0.002)
        assert ok, (r0, bad)
