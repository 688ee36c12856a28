"""Decoder-layer fusions: RMSNorm in the projection's staging, RoPE in the
QKV epilogue, and the four-kernel decoder layer.

The oracle chain is mote-reference restated: ``rms_norm_f32`` rounded to
f16 (what the fused kernels stage), ``quantized_linear_f32``, and
``rope_f32``.  The fused QKV rotates the f32 accumulators before its single
f16 rounding, so it is compared with RoPE applied in float64 to the
unrounded projection.  Tolerances: the reference's rule (abs 0.01 / rel
0.002) and the north-star normwise bound 1e-3 against float64.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker
from tests import _fixtures as fx

pytestmark = pytest.mark.gpu

from mote_b200 import decoder, errors, ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain, quantized  # noqa: E402

EPS = 1e-5


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def _f16(ctx, t, shape):
    return np.frombuffer(ctx.read_bytes(t), np.float16).astype(np.float32).reshape(shape)


def _normed(oracle_lib, x, gamma):
    m, k = x.shape
    n = oracle_lib.rms_norm_f32(x.astype(np.float32), gamma.astype(np.float32), k, EPS)
    return checker.f16_round(n).reshape(m, k)


def _setup(ctx, oracle_lib, m, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (m, k)).astype(np.float16)
    gamma = (1 + rng.normal(0, 0.1, k)).astype(np.float16)
    xt = ctx.from_bytes(plain((m, k), DType.F16), x)
    gt = ctx.from_bytes(plain((k,), DType.F16), gamma)
    return x, gamma, xt, gt


@pytest.mark.parametrize("m,n,k", [(1, 2048, 2048), (3, 1000, 4096), (16, 512, 2048),
                                   (20, 304, 1280)])
def test_rms_norm_linear(ctx, oracle_lib, m, n, k):
    x, gamma, xt, gt = _setup(ctx, oracle_lib, m, k, seed=m + n)
    w = fx.q4_0_weights(oracle_lib, n, k, seed=n + k)
    wt = ctx.from_bytes(quantized((n, k)), w)
    yt = ctx.empty(plain((m, n), DType.F16))
    ops.q4_0_rms_norm_linear_f16(ctx, xt, gt, wt, yt, EPS)
    got = _f16(ctx, yt, (m, n))
    assert ctx.device_status() == 0
    xn = _normed(oracle_lib, x, gamma)
    want = oracle_lib.quantized_linear_f32(xn, w, oracle_lib.Q4_0, m, n, k, threads=8).reshape(m, n)
    ok, bad = checker.within_reference_tolerance(got, checker.f16_round(want), 0.01, 0.002)
    assert ok, bad
    ref64 = checker.linear_f64(xn, checker.q4_0_dequant_np(w, n, k))
    assert checker.rel_err_normwise(got, ref64) <= 1e-3


@pytest.mark.parametrize("m", [1, 4, 9])
def test_rms_norm_gate_up_swiglu(ctx, oracle_lib, m):
    f, k = 1000, 2048
    x, gamma, xt, gt = _setup(ctx, oracle_lib, m, k, seed=70 + m)
    wg = fx.q4_0_weights(oracle_lib, f, k, seed=71)
    wu = fx.q4_0_weights(oracle_lib, f, k, seed=72)
    gtt, utt = ctx.from_bytes(quantized((f, k)), wg), ctx.from_bytes(quantized((f, k)), wu)
    yt = ctx.empty(plain((m, f), DType.F16))
    ops.q4_0_rms_norm_gate_up_swiglu_f16(ctx, xt, gt, gtt, utt, yt, EPS)
    got = _f16(ctx, yt, (m, f))
    xn = _normed(oracle_lib, x, gamma)
    ref = checker.swiglu_f64(checker.linear_f64(xn, checker.q4_0_dequant_np(wg, f, k)),
                             checker.linear_f64(xn, checker.q4_0_dequant_np(wu, f, k)))
    assert checker.rel_err_elementwise(got, ref) <= 2e-3
    assert checker.rel_err_normwise(got, ref) <= 1e-3


@pytest.mark.parametrize("m,qh,kvh,hd,k", [(1, 32, 8, 64, 2048), (4, 4, 2, 128, 1024),
                                           (17, 2, 1, 64, 512)])
def test_rms_norm_qkv_rope(ctx, oracle_lib, m, qh, kvh, hd, k):
    n = (qh + 2 * kvh) * hd
    x, gamma, xt, gt = _setup(ctx, oracle_lib, m, k, seed=90 + m)
    w = fx.q4_0_weights(oracle_lib, n, k, seed=91)
    wt = ctx.from_bytes(quantized((n, k)), w)
    pos = np.arange(7, 7 + m, dtype=np.int32)
    cos, sin = oracle_lib.rope_cos_sin_f64(pos, hd, 500000.0)
    ct = ctx.from_bytes(plain((m, hd // 2), DType.F32), cos.astype(np.float32))
    st = ctx.from_bytes(plain((m, hd // 2), DType.F32), sin.astype(np.float32))
    yt = ctx.empty(plain((m, n), DType.F16))
    ops.q4_0_rms_norm_qkv_rope_f16(ctx, xt, gt, wt, ct, st, yt, qh, kvh, hd, EPS)
    got = _f16(ctx, yt, (m, n))
    assert ctx.device_status() == 0
    xn = _normed(oracle_lib, x, gamma)
    proj = checker.linear_f64(xn, checker.q4_0_dequant_np(w, n, k))  # [m, n] float64
    want = proj.copy()
    rope_rows = (qh + kvh) * hd
    want[:, :rope_rows] = checker.rope_f64(proj[:, :rope_rows], cos, sin, m, qh + kvh, hd, hd,
                                           0).reshape(m, rope_rows)
    ok, bad = checker.within_reference_tolerance(got, checker.f16_round(want), 0.01, 0.002)
    assert ok, bad
    assert checker.rel_err_normwise(got, want) <= 1e-3
    # and against the unfused chain: rms_norm -> linear -> rope kernels
    nt = ctx.empty(plain((m, k), DType.F16))
    ops.rms_norm_f16(ctx, xt, gt, nt, EPS)
    y2 = ctx.empty(plain((m, n), DType.F16))
    ops.quantized_linear_q4_0_f16(ctx, nt, wt, y2)
    from mote_b200._native import lib

    # q and k of one token are contiguous [heads, hd] runs; tokens are n apart
    for tok in range(m):
        for off, heads in ((0, qh), (qh * hd, kvh)):
            p = y2.pointer + (tok * n + off) * 2
            assert lib().mote_cuda_rope_f16(p, ct.pointer + tok * hd * 2,
                                            st.pointer + tok * hd * 2, p, 1, heads, hd, hd, 0,
                                            ctx.stream) == 0
    chain = _f16(ctx, y2, (m, n))
    ok, bad = checker.within_reference_tolerance(got, chain, 0.01, 0.002)
    assert ok, bad


def test_fused_argument_rules(ctx):
    x = ctx.from_bytes(plain((1, 256), DType.F16), np.zeros(256, np.float16))
    g = ctx.from_bytes(plain((256,), DType.F16), np.ones(256, np.float16))
    w = ctx.empty(quantized((16, 256)))
    y = ctx.empty(plain((1, 16), DType.F16))
    with pytest.raises(errors.InvalidEpsilon):
        ops.q4_0_rms_norm_linear_f16(ctx, x, g, w, y, float("nan"))
    x96 = ctx.from_bytes(plain((1, 96), DType.F16), np.zeros(96, np.float16))
    g96 = ctx.from_bytes(plain((96,), DType.F16), np.ones(96, np.float16))
    w96 = ctx.empty(quantized((16, 96)))
    with pytest.raises(errors.Runtime):  # K % 256 != 0: fast path only
        ops.q4_0_rms_norm_linear_f16(ctx, x96, g96, w96, y, EPS)


@pytest.mark.parametrize("stack", [1, 3])
def test_fused_decoder_layer_matches_chain(ctx, stack):
    """The 4-kernel layer against the 8-kernel chain (same weights), for a
    stack of layers fed from the gather."""
    shape = decoder.LayerShape()
    layers = [decoder.random_layer(ctx, shape, seed=40 + i, vocab=1000) for i in range(stack)]
    rng = np.random.default_rng(3)
    attn = [rng.normal(0, 1, (1, shape.hidden)).astype(np.float16) for _ in range(stack)]
    outs = {}
    for mode in ("chain", "fused"):
        for i, layer in enumerate(layers):
            ctx.upload_numpy(layer.ids, np.array([123], np.int32))
            ctx.upload_numpy(layer.attn, attn[i])
            layer.set_position(11)
        for i, layer in enumerate(layers):
            step = layer.step if mode == "chain" else layer.step_fused
            step(None if i == 0 else layers[i - 1].out)
        ctx.sync()
        outs[mode] = _f16(ctx, layers[-1].out, (1, shape.hidden))
        outs[mode + "_qkv"] = _f16(ctx, layers[0].qkv, (1, shape.qkv))
    assert ctx.device_status() == 0
    for key in ("", "_qkv"):
        a, b = outs["fused" + key], outs["chain" + key]
        ok, bad = checker.within_reference_tolerance(a, b, 0.01, 0.002 * 4)
        assert ok, (key, bad)
        assert checker.rel_err_normwise(a, b) <= 2e-3
