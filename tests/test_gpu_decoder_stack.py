"""The persistent decoder stack (one cooperative launch for every layer)
against the four-kernel fused layer, layer by layer.

Both compute the same arithmetic -- the same staged, normalised f16
activations, exact Q4_0 products, f32 accumulation, one f16 rounding per
output -- and differ only in how K is split over warps, i.e. the order of
the f32 partial sums.  Every per-layer output (qkv with RoPE, h1, the SwiGLU
activations, out) is compared with the reference test rule (abs 0.01,
rel 0.008) and a normwise bound of 2e-3, as the fused layer is compared with
the eight-kernel chain (test_gpu_fused_layer.py); the fused layer itself is
checked against the mote-reference oracle there.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import checker

pytestmark = pytest.mark.gpu

from mote_b200 import decoder, ops  # noqa: E402
from mote_b200.context import CudaContext  # noqa: E402
from mote_b200.types import DType, plain  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    return CudaContext(0)


def _read(ctx, t, n):
    return np.frombuffer(ctx.read_bytes(t), np.float16).astype(np.float32).reshape(-1)[:n]


@pytest.mark.parametrize("stack,shape", [
    (1, decoder.LayerShape()),
    (3, decoder.LayerShape()),
    (2, decoder.LayerShape(hidden=1024, q_heads=16, kv_heads=4, head_dim=64, ffn=2816)),
    (2, decoder.LayerShape(hidden=512, q_heads=4, kv_heads=2, head_dim=128, ffn=1536)),
])
def test_stack_matches_fused_layers(ctx, stack, shape):
    layers = [decoder.random_layer(ctx, shape, seed=60 + i, vocab=500) for i in range(stack)]
    rng = np.random.default_rng(stack + shape.hidden)
    for i, layer in enumerate(layers):
        ctx.upload_numpy(layer.ids, np.array([77], np.int32))
        ctx.upload_numpy(layer.attn, rng.normal(0, 1, (1, shape.hidden)).astype(np.float16))
        layer.set_position(19 + i)
    # layer 0's input: the gathered embedding row, kept in its own buffer
    ops.embedding_gather_f16(ctx, layers[0].embedding, layers[0].ids, layers[0].h)
    h_in = ctx.from_bytes(plain((1, shape.hidden), DType.F16), ctx.read_bytes(layers[0].h))
    st = decoder.DecoderStackQ4_0(ctx, layers)
    st.run(h_in)
    ctx.sync()
    assert ctx.device_status() == 0
    got = [{k: _read(ctx, getattr(layer, k), n) for k, n in
            (("qkv", shape.qkv), ("h1", shape.hidden), ("a", shape.ffn), ("out", shape.hidden))}
           for layer in layers]
    # the fused layers, read out layer by layer (step_fused writes h1 in
    # place into its input, so each output is read before the next step)
    want = []
    for i, layer in enumerate(layers):
        hidden = None if i == 0 else layers[i - 1].out
        layer.step_fused(hidden)
        ctx.sync()
        h1_buf = layer.h if i == 0 else layers[i - 1].out
        want.append({"qkv": _read(ctx, layer.qkv, shape.qkv), "h1": _read(ctx, h1_buf, shape.hidden),
                     "a": _read(ctx, layer.a, shape.ffn), "out": _read(ctx, layer.out, shape.hidden)})
    assert ctx.device_status() == 0
    for i in range(stack):
        for key in ("qkv", "h1", "a", "out"):
            a, b = got[i][key], want[i][key]
            assert not np.isnan(a).any(), (i, key)
            ok, bad = checker.within_reference_tolerance(a, b, 0.01, 0.002 * 4)
            assert ok, (i, key, bad, a[bad], b[bad])
            assert checker.rel_err_normwise(a, b) <= 2e-3, (i, key)


def test_stack_replays_in_a_graph_and_repeats(ctx):
    """Two launches (the second inside a CUDA graph) give identical outputs:
    the barrier word is reset by every call."""
    torch = pytest.importorskip("torch")
    shape = decoder.LayerShape()
    layers = [decoder.random_layer(ctx, shape, seed=90 + i, vocab=100) for i in range(2)]
    rng = np.random.default_rng(1)
    for i, layer in enumerate(layers):
        ctx.upload_numpy(layer.attn, rng.normal(0, 1, (1, shape.hidden)).astype(np.float16))
        layer.set_position(5)
    h_in = ctx.from_bytes(plain((1, shape.hidden), DType.F16),
                          rng.normal(0, 0.5, shape.hidden).astype(np.float16))
    st = decoder.DecoderStackQ4_0(ctx, layers)
    st.run(h_in)
    ctx.sync()
    first = ctx.read_bytes(layers[-1].out)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=torch.cuda.ExternalStream(ctx.stream)):
        st.run(h_in)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert ctx.read_bytes(layers[-1].out) == first
    assert ctx.device_status() == 0
    del g
