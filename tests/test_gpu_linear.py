"""GPU parity of the Q4_0 linear against the CPU oracle (mote-reference restated).

Mirrors crates/mote-backend-hip/tests/quantized_linear.rs (fixtures,
tolerance abs 0.01 / rel 0.002 against the f16-rounded f32 oracle, empty
outputs, K == 0, aliasing and encoding validation) and adds the BASELINE
shapes with seeded N(0, 0.02) Q4_0 weights and N(0, 1) activations.

Bounds asserted, with ``checker`` metrics against a float64 accumulation of
the decoded weights:
* f16 outputs of the decode paths (<= 16 tokens, or shapes the tensor-core
  kernel does not take): element-wise relative error <= 1e-3 with the
  strict floor tau = 1e-3 * rms(ref) (``rel_err_elementwise_tau``) -- the
  f16 output rounding alone contributes up to 4.9e-4, and it is relative;
* f32 outputs: element-wise relative error (floor rms) <= 1e-5, and the
  tau-floored error <= 1e-3;
* the tensor-core prefill path (more than 16 tokens): the bounds of
  test_gpu_prefill.py (normwise 1e-3, rms-floored 2e-3).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker
from tests import _fixtures as fx

pytestmark = pytest.mark.gpu

from mote_b200 import errors, ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, QuantFormat, plain, quantized  # noqa: E402

F16_BOUND = 1e-3
F32_BOUND = 1e-5
# tcgen05 path: (q - 8) * d rounded to f16 (<= 2^-11 relative per weight)
# plus the f16 output rounding; element-wise (rms floor) bound 2e-3.
PREFILL_ELEMENTWISE_BOUND = 2e-3


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def run_linear(ctx, x, w_bytes, m, n, k, in_dtype=DType.F16, out_dtype=DType.F16):
    np_in = np.float16 if in_dtype is DType.F16 else np.float32
    np_out = np.float16 if out_dtype is DType.F16 else np.float32
    xt = ctx.from_bytes(plain((m, k), in_dtype), np.asarray(x, np_in))
    wt = ctx.from_bytes(quantized((n, k)), np.asarray(w_bytes, np.uint8))
    yt = ctx.empty(plain((m, n), out_dtype))
    ops.quantized_linear_q4_0(ctx, xt, wt, yt, in_dtype, out_dtype)
    out = np.frombuffer(ctx.read_bytes(yt), np_out).astype(np.float32).reshape(m, n)
    assert ctx.device_status() == 0
    return out


def oracle_linear(oracle_ref, x_f32, w_bytes, m, n, k):
    threads = min(8, max(1, oracle_ref.host_threads()))
    return oracle_ref.quantized_linear_f32(x_f32, w_bytes, oracle_ref.Q4_0, m, n, k,
                                           threads=threads).reshape(m, n)


def test_reference_fixture_3x5x64(ctx, oracle_lib):
    """quantized_linear.rs:13-62, verbatim fixture and tolerance (generic path)."""
    rows, n, k = 3, 5, 64
    x = fx.hip_linear_input(rows, k)
    w = fx.hip_linear_weights(n, k)
    wt = ctx.from_bytes(quantized((n, k)), w)
    assert ctx.read_bytes(wt) == w.tobytes()  # bytes stay as uploaded
    got = run_linear(ctx, x, w, rows, n, k)
    want = checker.f16_round(oracle_linear(oracle_lib, x.astype(np.float32), w, rows, n, k))
    ok, bad = checker.within_reference_tolerance(got, want, 0.01, 0.002)
    assert ok, (bad, got.reshape(-1)[bad], want.reshape(-1)[bad])


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9, 16, 17, 33, 64, 70])
@pytest.mark.parametrize("n,k", [(40, 256), (2048, 2048), (96, 1280)])
def test_fast_path_matches_oracle(ctx, oracle_lib, m, n, k):
    _check_fast_path(ctx, oracle_lib, m, n, k)


# Odd and long K (K/256 = 9, 24, 32, 33, 56 units of 256) with few tiles:
# every warp split (2, 4 or 8 warps per tile) divides K unevenly somewhere.
@pytest.mark.parametrize("m,n,k", [(1, 1000, 2304), (8, 304, 6144), (9, 304, 6144),
                                   (1, 520, 8192), (16, 520, 8192), (2, 64, 8448),
                                   (1, 528, 14336), (12, 528, 14336)])
def test_fast_path_kernel_splits(ctx, oracle_lib, m, n, k):
    _check_fast_path(ctx, oracle_lib, m, n, k)


def _check_fast_path(ctx, oracle_lib, m, n, k):
    w = fx.q4_0_weights(oracle_lib, n, k, seed=1000 + n + k)
    x = fx.activations(m, k, seed=7 + m).astype(np.float16)
    got = run_linear(ctx, x, w, m, n, k)
    x32 = x.astype(np.float32)
    want32 = oracle_linear(oracle_lib, x32, w, m, n, k)
    ok, bad = checker.within_reference_tolerance(got, checker.f16_round(want32), 0.01, 0.002)
    assert ok, bad
    ref64 = checker.linear_f64(x32, checker.q4_0_dequant_np(w, n, k))
    # M > 16 with N % 16 == 0 runs on the tcgen05 prefill path, whose weights
    # are rounded to f16 (see test_gpu_prefill.py for its bounds).
    prefill = m > 16 and n % 16 == 0
    bound = PREFILL_ELEMENTWISE_BOUND if prefill else F16_BOUND
    assert checker.rel_err_elementwise(got, ref64) <= bound
    assert checker.rel_err_normwise(got, ref64) <= F16_BOUND
    if not prefill:
        assert checker.rel_err_elementwise_tau(got, ref64) <= F16_BOUND


@pytest.mark.parametrize("m", [1, 3, 4, 5, 16])
def test_f32_activations_keep_full_precision(ctx, oracle_lib, m):
    """Config 1 (M=1, K=N=2048) and neighbours: f32 in, f32 out."""
    n, k = 2048, 2048
    w = fx.q4_0_weights(oracle_lib, n, k, seed=11)
    x = fx.activations(m, k, seed=12)
    got = run_linear(ctx, x, w, m, n, k, DType.F32, DType.F32)
    want32 = oracle_linear(oracle_lib, x, w, m, n, k)
    ref64 = checker.linear_f64(x, checker.q4_0_dequant_np(w, n, k))
    assert checker.rel_err_elementwise(got, ref64) <= F32_BOUND
    assert checker.rel_err_elementwise_tau(got, ref64) <= F16_BOUND
    assert checker.rel_err_elementwise(want32, ref64) <= F32_BOUND
    ok, bad = checker.within_reference_tolerance(got, want32, 1e-5, 1e-5)
    assert ok, bad


def test_f32_output_variant(ctx, oracle_lib):
    m, n, k = 4, 1024, 4096
    w = fx.q4_0_weights(oracle_lib, n, k, seed=21)
    x = fx.activations(m, k, seed=22).astype(np.float16)
    got = run_linear(ctx, x, w, m, n, k, DType.F16, DType.F32)
    ref64 = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w, n, k))
    assert checker.rel_err_elementwise(got, ref64) <= F32_BOUND


_CONFIG3 = {}


def _config3_case(oracle_lib, n, k=4096):
    """Weights, decoded f64 weights and the 16 activation rows of config 3
    for one N (cached: every M of the sweep uses the same matrix)."""
    if n not in _CONFIG3:
        w = fx.q4_0_weights(oracle_lib, n, k, seed=300 + n)
        x = fx.activations(16, k, seed=301).astype(np.float16)
        ref64 = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w, n, k))
        _CONFIG3.clear()
        _CONFIG3[n] = (w, x, ref64)
    return _CONFIG3[n]


@pytest.mark.parametrize("n", [4096, 11008, 14336])
@pytest.mark.parametrize("m", [1, 2, 4, 8, 16])
def test_config3_batch_decode_shapes(ctx, oracle_lib, m, n):
    """Config 3 at full size: every M of the sweep (1, 2, 4, 8, 16) at
    K=4096 and N = 4096, 11008, 14336 -- the shapes and kernel instantiations
    (column packing MC = 1, 2, 4, 8 and two n8 tiles with the K split over
    CTAs) the headline measures -- through the workspace entry that
    mote_b200.ops uses, against f64 (strict tau floor) and the f32 oracle
    with the reference rule."""
    k = 4096
    w, x_all, ref_all = _config3_case(oracle_lib, n, k)
    x, ref64 = x_all[:m], ref_all[:m]
    got = run_linear(ctx, x, w, m, n, k)
    assert checker.rel_err_elementwise_tau(got, ref64) <= F16_BOUND
    assert checker.rel_err_normwise(got, ref64) <= F16_BOUND
    want32 = oracle_linear(oracle_lib, x.astype(np.float32), w, m, n, k)
    ok, bad = checker.within_reference_tolerance(got, checker.f16_round(want32), 0.01, 0.002)
    assert ok, bad


def test_reference_bench_fixture_sampled(ctx, oracle_lib):
    """benches/quantized_linear.rs:89-126 validation of 3 sampled outputs."""
    rows, n, k = 16, 4096, 4096
    w = fx.hip_bench_weights(n, k)
    x = fx.hip_bench_input(rows, k)
    got = run_linear(ctx, x, w, rows, n, k)
    rb = (k // 32) * 18
    for row, of in [(0, 0), (rows // 2, n // 3), (rows - 1, n - 1)]:
        dec = oracle_lib.dequantize_quantized_row(w[of * rb:(of + 1) * rb], oracle_lib.Q4_0, k)
        exp = np.float32(0)
        for inner in range(k):
            exp = np.float32(exp + np.float32(x[row, inner]) * dec[inner])
        exp = float(np.float16(exp))
        assert abs(got[row, of] - exp) <= max(0.25, abs(exp) * 0.005)


def test_gate_up_swiglu_fused(ctx, oracle_lib):
    m, f, k = 3, 1000, 2048
    wg = fx.q4_0_weights(oracle_lib, f, k, seed=41)
    wu = fx.q4_0_weights(oracle_lib, f, k, seed=42)
    x = fx.activations(m, k, seed=43).astype(np.float16)
    xt = ctx.from_bytes(plain((m, k), DType.F16), x)
    gt = ctx.from_bytes(quantized((f, k)), wg)
    ut = ctx.from_bytes(quantized((f, k)), wu)
    yt = ctx.empty(plain((m, f), DType.F16))
    ops.q4_0_gate_up_swiglu_f16(ctx, xt, gt, ut, yt)
    got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, f)
    x32 = x.astype(np.float32)
    g64 = checker.linear_f64(x32, checker.q4_0_dequant_np(wg, f, k))
    u64 = checker.linear_f64(x32, checker.q4_0_dequant_np(wu, f, k))
    ref = checker.swiglu_f64(g64, u64)
    assert checker.rel_err_elementwise(got, ref) <= 2e-3
    assert checker.rel_err_normwise(got, ref) <= 1e-3


def test_empty_outputs_return_without_launch(ctx):
    """quantized_linear.rs:124-140."""
    xt = ctx.from_bytes(plain((0, 32), DType.F16), b"")
    wt = ctx.from_bytes(quantized((2, 32)), fx.hip_linear_weights(2, 32))
    yt = ctx.empty(plain((0, 2), DType.F16))
    ops.quantized_linear_q4_0_f16(ctx, xt, wt, yt)
    assert ctx.read_bytes(yt) == b""


def test_zero_input_features_writes_zeros(ctx):
    """quantized_linear.rs:142-158."""
    xt = ctx.from_bytes(plain((3, 0), DType.F16), b"")
    wt = ctx.from_bytes(quantized((2, 0)), b"")
    yt = ctx.from_bytes(plain((3, 2), DType.F16), np.full(6, 7.0, np.float16))
    ops.quantized_linear_q4_0_f16(ctx, xt, wt, yt)
    assert np.all(np.frombuffer(ctx.read_bytes(yt), np.float16) == 0)


def test_validates_geometry_encoding_and_aliasing(ctx):
    """quantized_linear.rs:64-122."""
    x = ctx.from_bytes(plain((1, 32), DType.F16), np.zeros(32, np.float16))
    w = ctx.from_bytes(quantized((32, 32)), fx.hip_linear_weights(32, 32))
    y = ctx.empty(plain((1, 32), DType.F16))
    with pytest.raises(errors.AliasedStorage) as e:
        ops.quantized_linear_q4_0_f16(ctx, x, w, x)
    assert (e.value.tensor, e.value.other) == ("output", "input")
    from mote_b200.context import Tensor

    y_on_w = Tensor(plain((1, 32), DType.F16), w.storage, 0)
    with pytest.raises(errors.AliasedStorage) as e:
        ops.quantized_linear_q4_0_f16(ctx, x, w, y_on_w)
    assert (e.value.tensor, e.value.other) == ("output", "weights")
    q8 = ctx.from_bytes(quantized((32, 32), QuantFormat.Q8_0), np.zeros(32 * 34, np.uint8))
    with pytest.raises(errors.UnsupportedEncoding):
        ops.quantized_linear_q4_0_f16(ctx, x, q8, y)
    short = ctx.from_bytes(quantized((32, 64)), fx.hip_linear_weights(32, 64))
    with pytest.raises(errors.ShapeMismatch) as e:
        ops.quantized_linear_q4_0_f16(ctx, x, short, y)
    assert e.value.tensor == "weights"
    other = CudaContext(0)
    y2 = other.empty(plain((1, 32), DType.F16))
    with pytest.raises(errors.WrongStorage):
        ops.quantized_linear_q4_0_f16(ctx, x, w, y2)


def test_unaligned_weights_use_generic_path(ctx, oracle_lib):
    """A weight tensor that is not 16-byte aligned still computes correctly."""
    n, k = 24, 512
    w = fx.q4_0_weights(oracle_lib, n, k, seed=5)
    x = fx.activations(2, k, seed=6).astype(np.float16)
    from mote_b200.context import CudaStorage, Tensor

    storage = CudaStorage(ctx.inner, w.nbytes + 2, np.concatenate([np.zeros(2, np.uint8), w]))
    wt = Tensor(quantized((n, k)), storage, 2)
    xt = ctx.from_bytes(plain((2, k), DType.F16), x)
    yt = ctx.empty(plain((2, n), DType.F16))
    # The typed API only takes zero-offset tensors (context.rs:150-176) ...
    with pytest.raises(errors.UnsupportedByteOffset):
        ops.quantized_linear_q4_0_f16(ctx, xt, wt, yt)
    # ... the C ABI takes any pointer.
    from mote_b200._native import lib

    assert lib().mote_cuda_quantized_linear_q4_0_f16(xt.pointer, wt.pointer, yt.pointer, 2, n, k,
                                                     ctx.stream) == 0
    got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(2, n)
    ref64 = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w, n, k))
    assert checker.rel_err_elementwise(got, ref64) <= F16_BOUND


@pytest.mark.parametrize("m,n,k,in_place", [(1, 2048, 8192, False), (4, 2048, 8192, True),
                                            (16, 200, 512, False), (24, 96, 1280, True),
                                            (3, 40, 96, False)])
def test_residual_epilogue(ctx, oracle_lib, m, n, k, in_place):
    """``y = x @ W^T + r`` with one f16 rounding (fast, multi-launch and
    generic paths; output aliasing the residual)."""
    w = fx.q4_0_weights(oracle_lib, n, k, seed=90 + m)
    x = fx.activations(m, k, seed=91 + m).astype(np.float16)
    r = np.random.default_rng(92 + m).normal(0, 1, (m, n)).astype(np.float16)
    xt = ctx.from_bytes(plain((m, k), DType.F16), x)
    wt = ctx.from_bytes(quantized((n, k)), w)
    rt = ctx.from_bytes(plain((m, n), DType.F16), r)
    yt = rt if in_place else ctx.empty(plain((m, n), DType.F16))
    ops.quantized_linear_q4_0_f16_residual(ctx, xt, wt, rt, yt)
    got = np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, n)
    assert ctx.device_status() == 0
    acc = oracle_linear(oracle_lib, x.astype(np.float32), w, m, n, k)
    want = checker.f16_round(acc + r.astype(np.float32))
    ok, bad = checker.within_reference_tolerance(got, want, 0.01, 0.002)
    assert ok, bad
    ref64 = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w, n, k)) + r
    assert checker.rel_err_normwise(got, ref64) <= 1e-3


def test_residual_zero_input_features_copies_residual(ctx):
    xt = ctx.from_bytes(plain((3, 0), DType.F16), b"")
    wt = ctx.from_bytes(quantized((2, 0)), b"")
    r = np.arange(6, dtype=np.float16)
    rt = ctx.from_bytes(plain((3, 2), DType.F16), r)
    yt = ctx.from_bytes(plain((3, 2), DType.F16), np.full(6, 7.0, np.float16))
    ops.quantized_linear_q4_0_f16_residual(ctx, xt, wt, rt, yt)
    assert np.array_equal(np.frombuffer(ctx.read_bytes(yt), np.float16), r)


# K split over CTAs (9-16 tokens, up to 4096 tiles); the other shapes take
# the unsplit kernel with the workspace present (1-16 tokens, 3-896 tiles).
@pytest.mark.parametrize("m,n,k", [(5, 4096, 4096), (8, 1000, 4096), (9, 4096, 4096),
                                   (16, 14336, 4096), (16, 300, 8192), (12, 528, 14336),
                                   (16, 64, 1024), (1, 40, 2304), (1, 4016, 4096),
                                   (3, 11008, 4096), (1, 14336, 4096), (4, 2000, 12288)])
def test_split_k_workspace_path(ctx, oracle_lib, m, n, k):
    """mote_cuda_quantized_linear_q4_0_f16_ws: K split over CTAs through the
    workspace.  Two calls in a row (into NaN-filled outputs) give identical,
    complete outputs -- the second only works if the first reset every tile
    counter -- and a too-small workspace falls back to the unsplit kernel."""
    import ctypes

    from mote_b200._native import lib

    w = fx.q4_0_weights(oracle_lib, n, k, seed=500 + n)
    x = fx.activations(m, k, seed=501 + m).astype(np.float16)
    xt = ctx.from_bytes(plain((m, k), DType.F16), x)
    wt = ctx.from_bytes(quantized((n, k)), w)
    need = ctypes.c_uint64(0)
    assert lib().mote_cuda_q4_0_linear_workspace_bytes(m, n, k, ctypes.byref(need)) == 0
    assert need.value > 0
    ws = ctx.from_bytes(plain((need.value,), DType.U8), np.zeros(need.value, np.uint8))
    outs = []
    nan = np.full(m * n, np.nan, np.float16)  # any tile left unstored stays NaN
    for ws_bytes in (need.value, need.value, 16):
        yt = ctx.from_bytes(plain((m, n), DType.F16), nan)
        assert lib().mote_cuda_quantized_linear_q4_0_f16_ws(
            xt.pointer, wt.pointer, yt.pointer, m, n, k, ws.pointer, ws_bytes, ctx.stream) == 0
        outs.append(np.frombuffer(ctx.read_bytes(yt), np.float16).astype(np.float32).reshape(m, n))
    assert ctx.device_status() == 0
    assert np.array_equal(outs[0], outs[1]) and not np.isnan(outs[1]).any()
    want = oracle_linear(oracle_lib, x.astype(np.float32), w, m, n, k)
    ref64 = checker.linear_f64(x.astype(np.float32), checker.q4_0_dequant_np(w, n, k))
    for got in (outs[0], outs[2]):
        ok, bad = checker.within_reference_tolerance(got, checker.f16_round(want), 0.01, 0.002)
        assert ok, bad
        assert checker.rel_err_elementwise(got, ref64) <= F16_BOUND


def test_overlapped_downloads_match_the_outputs(ctx, oracle_lib):
    """Host-buffer pipeline of the end-to-end bench: activations uploaded
    from pinned memory, linears on the compute stream, each output copied
    back on the context's copy stream right after its linear (the later
    linears run meanwhile); after sync() every host buffer holds exactly the
    device output, on every one of several back-to-back steps."""
    from mote_b200.context import PinnedBuffer

    rng = np.random.default_rng(91)
    k = 4096
    shapes = [(1, 4096), (4, 11008), (16, 2048)]
    ws = {n: ctx.from_bytes(quantized((n, k)), fx.q4_0_weights(oracle_lib, n, k, seed=300 + n))
          for _, n in shapes}
    xs = {m: ctx.empty(plain((m, k), DType.F16)) for m, _ in shapes}
    ys = {(m, n): ctx.empty(plain((m, n), DType.F16)) for m, n in shapes}
    hx = {m: PinnedBuffer(m * k * 2) for m, _ in shapes}
    hy = {(m, n): PinnedBuffer(m * n * 2) for m, n in shapes}
    for step in range(3):
        for m, _ in shapes:
            hx[m].view(np.float16)[:] = rng.normal(0, 1, m * k).astype(np.float16)
            ctx.upload_async(xs[m], hx[m])
        for m, n in shapes:
            ops.quantized_linear_q4_0_f16(ctx, xs[m], ws[n], ys[(m, n)])
            ctx.download_overlapped(hy[(m, n)], ys[(m, n)])
        ctx.sync()
        for m, n in shapes:
            want = np.frombuffer(ctx.read_bytes(ys[(m, n)]), np.uint16)
            got = hy[(m, n)].view(np.uint16)
            assert np.array_equal(got, want), (step, m, n)
