"""Config 4: the non-attention ops of one Llama-style 1B decoder layer at M=1.

The GPU chain (``mote_b200.decoder.DecoderLayerQ4_0``) is compared, step by
step, with the same chain built from the CPU oracle (mote-reference
restated), rounding to f16 at the same points the GPU chain stores f16:
gather (bit-exact), RMSNorm, QKV (f32 accumulation), RoPE on q and k,
O projection, residual add + RMSNorm, gate/up + SwiGLU, down projection +
residual.  Tolerances: the reference tests' rule (abs/rel) per step, and the
north-star bound (normwise relative error <= 1e-3 against float64) on the
linear outputs.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker

pytestmark = pytest.mark.gpu

from mote_b200 import decoder  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402

VOCAB = 1000  # the gather kernel is tested at the full 128256 rows elsewhere


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def f16(ctx, t):
    return np.frombuffer(ctx.read_bytes(t), np.float16).astype(np.float32)


def q4(ctx, t):
    return np.frombuffer(ctx.read_bytes(t), np.uint8)


def test_decoder_layer_chain_matches_oracle(ctx, oracle_lib):
    ref = oracle_lib
    shape = decoder.LayerShape()
    layer = decoder.random_layer(ctx, shape, seed=4, vocab=VOCAB)
    rng = np.random.default_rng(11)
    token = int(rng.integers(0, VOCAB))
    position = 37
    attn = rng.normal(0, 1, (1, shape.hidden)).astype(np.float16)
    ctx.upload_numpy(layer.ids, np.array([token], np.int32))
    ctx.upload_numpy(layer.attn, attn)
    layer.set_position(position)
    layer.step()
    ctx.sync()
    assert ctx.device_status() == 0

    h, hd, ffn = shape.hidden, shape.head_dim, shape.ffn
    eps = shape.eps
    table = np.frombuffer(ctx.read_bytes(layer.embedding), np.float16).reshape(VOCAB, h)
    g1, g2 = f16(ctx, layer.gamma1), f16(ctx, layer.gamma2)
    w_qkv, w_o = q4(ctx, layer.w_qkv), q4(ctx, layer.w_o)
    w_g, w_u, w_d = q4(ctx, layer.w_gate), q4(ctx, layer.w_up), q4(ctx, layer.w_down)
    cos = np.frombuffer(ctx.read_bytes(layer.cos), np.float32)
    sin = np.frombuffer(ctx.read_bytes(layer.sin), np.float32)
    want_c, want_s = ref.rope_cos_sin_f64(np.array([position], np.int32), hd, 500000.0)
    assert checker.ulp_distance_f32(cos, want_c.reshape(-1)).max() <= 1
    assert checker.ulp_distance_f32(sin, want_s.reshape(-1)).max() <= 1

    def lin(x, w, n, k):
        return ref.quantized_linear_f32(x, w, ref.Q4_0, 1, n, k, threads=8)

    # 1. gather (bit-exact)
    h0 = table[token].astype(np.float32)
    # the gathered row was overwritten in place by the residual add; check h1 below
    # 2. RMSNorm
    n1 = checker.f16_round(ref.rms_norm_f32(h0, g1, h, eps))
    got_n1 = f16(ctx, layer.n1)
    assert checker.within_reference_tolerance(got_n1, n1, 3e-3, 3e-3)[0]
    # 3. QKV from the GPU's own n1 (isolates each step's error)
    qkv32 = lin(got_n1, w_qkv, shape.qkv, h)
    # 4. RoPE of q and k (bit-exact given the same f16 inputs and tables)
    qkv16 = checker.f16_round(qkv32)
    q_end, k_end = shape.q_heads * hd, (shape.q_heads + shape.kv_heads) * hd
    q_rot = ref.rope_f32(qkv16[:q_end], cos, sin, 1, shape.q_heads, hd, hd, 0)
    k_rot = ref.rope_f32(qkv16[q_end:k_end], cos, sin, 1, shape.kv_heads, hd, hd, 0)
    got_qkv = f16(ctx, layer.qkv)
    ok, bad = checker.within_reference_tolerance(got_qkv[k_end:], qkv16[k_end:], 0.01, 0.002)
    assert ok, ("v", bad)
    for got, want in ((got_qkv[:q_end], q_rot), (got_qkv[q_end:k_end], k_rot)):
        ok, bad = checker.within_reference_tolerance(got, checker.f16_round(want), 0.01, 0.002)
        assert ok, bad
    ref64 = checker.linear_f64(got_n1[None, :], checker.q4_0_dequant_np(w_qkv, shape.qkv, h))
    assert checker.rel_err_normwise(got_qkv[k_end:], ref64[0, k_end:]) <= 1e-3
    # 5. O projection of the attention stand-in
    o = checker.f16_round(lin(attn.astype(np.float32).reshape(-1), w_o, h, h))
    got_o = f16(ctx, layer.o)
    assert checker.within_reference_tolerance(got_o, o, 0.01, 0.002)[0]
    # 6. residual add + RMSNorm
    n2, h1 = ref.fused_add_rms_norm_f32(got_o, h0, g2, h, eps)
    got_n2 = f16(ctx, layer.n2)
    got_h1 = f16(ctx, layer.h)
    assert np.array_equal(got_h1, checker.f16_round(h1))
    assert checker.within_reference_tolerance(got_n2, checker.f16_round(n2), 3e-3, 3e-3)[0]
    # 7. gate/up + SwiGLU (f32 accumulators, one f16 rounding)
    gate = lin(got_n2, w_g, ffn, h)
    up = lin(got_n2, w_u, ffn, h)
    a = checker.f16_round(ref.swiglu_f64(gate, up))
    got_a = f16(ctx, layer.a)
    assert checker.within_reference_tolerance(got_a, a, 0.01, 0.002)[0]
    a64 = checker.swiglu_f64(
        checker.linear_f64(got_n2[None, :], checker.q4_0_dequant_np(w_g, ffn, h)),
        checker.linear_f64(got_n2[None, :], checker.q4_0_dequant_np(w_u, ffn, h)))
    assert checker.rel_err_normwise(got_a, a64) <= 1e-3
    # 8. down projection + residual
    d = lin(got_a, w_d, h, ffn)
    h2 = checker.f16_round(d + got_h1)
    got_h2 = f16(ctx, layer.out)
    assert checker.within_reference_tolerance(got_h2, h2, 0.01, 0.002)[0]
    h2_64 = checker.linear_f64(got_a[None, :], checker.q4_0_dequant_np(w_d, h, ffn))[0] + got_h1
    assert checker.rel_err_normwise(got_h2, h2_64) <= 1e-3


def test_decoder_layer_runs_under_graph_capture(ctx):
    """The chain is capturable (no allocation or sync inside step())."""
    torch = pytest.importorskip("torch")
    shape = decoder.LayerShape()
    layer = decoder.random_layer(ctx, shape, seed=5, vocab=VOCAB)
    ctx.upload_numpy(layer.ids, np.array([3], np.int32))
    ctx.upload_numpy(layer.attn, np.ones((1, shape.hidden), np.float16))
    layer.set_position(1)
    layer.step()
    ctx.sync()
    eager = f16(ctx, layer.out).copy()
    # capture the same step on the context stream through the CUDA runtime
    stream = torch.cuda.ExternalStream(ctx.stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        layer.step()
    graph.replay()
    torch.cuda.synchronize()
    assert np.array_equal(f16(ctx, layer.out), eager)
