"""Decode step of the non-attention ops of one Llama-style decoder layer.

The chain BASELINE config 4 names, built from this backend's operators and
issued on one context stream (so a caller can capture it in a CUDA graph):

    h0  = embedding[id]                         embedding_gather_f16
    n1  = rms_norm(h0) * g1                     rms_norm_f16
    qkv = n1 @ Wqkv^T                           quantized_linear_q4_0_f16  (Q4_0)
    q,k = rope(q), rope(k)  (in place)          rope_f16 x2
    o   = attn @ Wo^T                           quantized_linear_q4_0_f16
    h1  = h0 + o ; n2 = rms_norm(h1) * g2       fused_add_rms_norm_f16 (h0 buffer -> h1)
    a   = silu(n2 @ Wg^T) * (n2 @ Wu^T)         q4_0_gate_up_swiglu_f16
    h2  = h1 + a @ Wd^T                         quantized_linear_q4_0_f16_residual

``attn`` is the attention output (an input here: the layer's attention is
outside this data plane).  Shapes follow Llama-3.2-1B: hidden 2048, 32
query / 8 KV heads of 64, FFN 8192, vocab 128256.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import ops
from .context import CudaContext, Tensor
from .types import DType, RopeLayout, plain, quantized


@dataclass(frozen=True)
class LayerShape:
    hidden: int = 2048
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 64
    ffn: int = 8192
    vocab: int = 128256
    eps: float = 1e-5

    @property
    def qkv(self) -> int:
        return (self.q_heads + 2 * self.kv_heads) * self.head_dim

    def weight_bytes(self) -> int:
        """Q4_0 bytes streamed per step (QKV, O, gate, up, down)."""
        h = self.hidden
        blocks = (self.qkv * h + h * h + 2 * self.ffn * h + h * self.ffn) // 32
        return blocks * 18


class DecoderLayerQ4_0:
    """Weights and activation buffers of one layer on one context."""

    def __init__(self, ctx: CudaContext, shape: LayerShape, *, embedding: Tensor, w_qkv: Tensor,
                 w_o: Tensor, w_gate: Tensor, w_up: Tensor, w_down: Tensor, gamma1: Tensor,
                 gamma2: Tensor):
        self.ctx = ctx
        self.shape = s = shape
        self.embedding = embedding
        self.w_qkv, self.w_o, self.w_gate, self.w_up, self.w_down = w_qkv, w_o, w_gate, w_up, w_down
        self.gamma1, self.gamma2 = gamma1, gamma2
        h = s.hidden
        self.ids = ctx.empty(plain((1,), DType.I32))
        self.h = ctx.empty(plain((1, h), DType.F16))        # h0, then h1 (in place)
        self.n1 = ctx.empty(plain((1, h), DType.F16))
        self.qkv = ctx.empty(plain((1, s.qkv), DType.F16))
        self.attn = ctx.empty(plain((1, h), DType.F16))
        self.o = ctx.empty(plain((1, h), DType.F16))
        self.n2 = ctx.empty(plain((1, h), DType.F16))
        self.a = ctx.empty(plain((1, s.ffn), DType.F16))
        self.out = ctx.empty(plain((1, h), DType.F16))      # h2
        self.h1 = ctx.empty(plain((1, h), DType.F16))       # h1 of the persistent stack
        self.cos = ctx.empty(plain((1, s.head_dim // 2), DType.F32))
        self.sin = ctx.empty(plain((1, s.head_dim // 2), DType.F32))
        self.pos = ctx.empty(plain((1,), DType.I32))
        # q and k views into the qkv buffer: [1, heads, head_dim]
        qd, kd = s.q_heads * s.head_dim, s.kv_heads * s.head_dim
        self.q_view = Tensor(plain((1, s.q_heads, s.head_dim), DType.F16), self.qkv.storage, 0)
        self.k_view = Tensor(plain((1, s.kv_heads, s.head_dim), DType.F16), self.qkv.storage,
                             qd * 2)
        self._kd = kd

    def set_position(self, position: int, theta: float = 500000.0) -> None:
        """Fills the cos/sin row for ``position`` (once per decode step)."""
        import numpy as np

        self.ctx.upload_numpy(self.pos, np.array([position], np.int32))
        ops.rope_cos_sin_f32(self.ctx, self.pos, self.cos, self.sin, theta)

    def step(self, hidden: Tensor | None = None) -> None:
        """One decode step; writes ``out`` (h2) and reads ``attn``.

        Without ``hidden`` the layer input is ``embedding[ids]`` gathered into
        ``self.h`` (the first layer of a stack); with it, ``hidden`` (the
        previous layer's ``out``, [1, hidden] f16) is the input and receives
        h1 in place, as a residual stream does.
        """
        ctx, s = self.ctx, self.shape
        h = self.h if hidden is None else hidden
        if hidden is None:
            ops.embedding_gather_f16(ctx, self.embedding, self.ids, self.h, check=False)
        ops.rms_norm_f16(ctx, h, self.gamma1, self.n1, s.eps)
        ops.quantized_linear_q4_0_f16(ctx, self.n1, self.w_qkv, self.qkv)
        # RoPE in place on the q and k slices (the C ABI takes raw pointers, so
        # the zero-offset rule of the typed wrapper does not apply here).
        from ._native import lib
        from . import errors

        errors.check(lib().mote_cuda_rope_f16(self.q_view.pointer, self.cos.pointer,
                                              self.sin.pointer, self.q_view.pointer, 1, s.q_heads,
                                              s.head_dim, s.head_dim,
                                              RopeLayout.HalfSplit.value, ctx.stream), "rope q")
        errors.check(lib().mote_cuda_rope_f16(self.k_view.pointer, self.cos.pointer,
                                              self.sin.pointer, self.k_view.pointer, 1,
                                              s.kv_heads, s.head_dim, s.head_dim,
                                              RopeLayout.HalfSplit.value, ctx.stream), "rope k")
        ops.quantized_linear_q4_0_f16(ctx, self.attn, self.w_o, self.o)
        ops.fused_add_rms_norm_f16(ctx, self.o, h, self.gamma2, self.n2, s.eps)
        ops.q4_0_gate_up_swiglu_f16(ctx, self.n2, self.w_gate, self.w_up, self.a)
        ops.quantized_linear_q4_0_f16_residual(ctx, self.a, self.w_down, h, self.out)


    def step_fused(self, hidden: Tensor | None = None) -> None:
        """The same layer in four kernels (five with the gather): the norms
        run inside the activation staging of the projection that follows
        them, RoPE inside the QKV epilogue, and the two residual adds in the
        O and down projections' epilogues.

            h   (gather, or ``hidden``)
            qkv = rope(rms_norm(h) @ Wqkv^T)              q4_0_rms_norm_qkv_rope_f16
            h1  = h + attn @ Wo^T        (in place in h)  quantized_linear_q4_0_f16_residual
            a   = swiglu(rms_norm(h1) @ [Wg; Wu]^T)       q4_0_rms_norm_gate_up_swiglu_f16
            out = h1 + a @ Wd^T                           quantized_linear_q4_0_f16_residual
        """
        ctx, s = self.ctx, self.shape
        h = self.h if hidden is None else hidden
        if hidden is None:
            ops.embedding_gather_f16(ctx, self.embedding, self.ids, self.h, check=False)
        ops.q4_0_rms_norm_qkv_rope_f16(ctx, h, self.gamma1, self.w_qkv, self.cos, self.sin,
                                       self.qkv, s.q_heads, s.kv_heads, s.head_dim, s.eps)
        ops.quantized_linear_q4_0_f16_residual(ctx, self.attn, self.w_o, h, h)
        ops.q4_0_rms_norm_gate_up_swiglu_f16(ctx, h, self.gamma2, self.w_gate, self.w_up, self.a,
                                             s.eps)
        ops.quantized_linear_q4_0_f16_residual(ctx, self.a, self.w_down, h, self.out)


def random_layer(ctx: CudaContext, shape: LayerShape, seed: int = 0, vocab: int | None = None):
    """A layer with seeded N(0, 0.02) weights Q4_0-encoded on the device,
    gammas 1 + N(0, 0.1) and an N(0, 0.02) f16 embedding table."""
    import numpy as np

    from ._native import lib
    from . import errors

    rng = np.random.default_rng(seed)
    h = shape.hidden

    def q4(n, k):
        w = ctx.empty(quantized((n, k)))
        f = ctx.from_numpy(plain((n, k), DType.F32),
                           rng.normal(0, 0.02, (n, k)).astype(np.float32))
        ops.q4_0_encode_f32(ctx, f, w)
        ctx.sync()
        return w

    v = shape.vocab if vocab is None else vocab
    table = ctx.from_numpy(plain((v, h), DType.F16),
                           rng.normal(0, 0.02, (v, h)).astype(np.float16))
    g1 = ctx.from_numpy(plain((h,), DType.F16), (1 + rng.normal(0, 0.1, h)).astype(np.float16))
    g2 = ctx.from_numpy(plain((h,), DType.F16), (1 + rng.normal(0, 0.1, h)).astype(np.float16))
    layer = DecoderLayerQ4_0(ctx, shape, embedding=table, w_qkv=q4(shape.qkv, h), w_o=q4(h, h),
                             w_gate=q4(shape.ffn, h), w_up=q4(shape.ffn, h),
                             w_down=q4(h, shape.ffn), gamma1=g1, gamma2=g2)
    return layer


class DecoderStackQ4_0:
    """A stack of layers run by the persistent kernel
    (``mote_cuda_q4_0_decoder_stack_f16``): one cooperative launch for all
    layers, grid barriers in place of kernel boundaries.  Per layer it writes
    ``qkv`` (RoPE applied), ``h1`` (= h + attn @ Wo^T, its own buffer), ``a``
    (SwiGLU) and ``out``; layer 0 reads ``hidden``, layer l the previous
    layer's ``out`` -- the arithmetic of ``step_fused``."""

    def __init__(self, ctx: CudaContext, layers: list[DecoderLayerQ4_0]):
        import ctypes

        import numpy as np

        self.ctx, self.layers = ctx, layers
        s = layers[0].shape
        rows = []
        for layer in layers:
            rows.append([t.pointer for t in (layer.w_qkv, layer.w_o, layer.w_gate, layer.w_up,
                                             layer.w_down, layer.gamma1, layer.gamma2,
                                             layer.attn, layer.cos, layer.sin, layer.qkv,
                                             layer.h1, layer.a, layer.out)])
        table = np.asarray(rows, np.uint64).reshape(-1)
        self.table = ctx.from_bytes(plain((table.size * 8,), DType.U8), table.view(np.uint8))
        from ._native import lib
        from . import errors

        need = ctypes.c_uint64(0)
        errors.check(lib().mote_cuda_q4_0_decoder_stack_workspace_bytes(s.hidden,
                                                                         ctypes.byref(need)),
                     "stack workspace size")
        self.workspace = ctx.empty(plain((need.value,), DType.U8))
        self._c = ctypes

    def run(self, hidden: Tensor) -> None:
        from ._native import lib
        from . import errors

        s = self.layers[0].shape
        self.ctx.inner.select()
        errors.check(lib().mote_cuda_q4_0_decoder_stack_f16(
            self.table.pointer, len(self.layers), hidden.pointer, s.hidden, s.ffn, s.q_heads,
            s.kv_heads, s.head_dim, self._c.c_float(s.eps), self.workspace.pointer,
            self.workspace.desc.required_span_bytes, self.ctx.stream), "launch decoder stack")
