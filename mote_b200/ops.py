"""Typed operators of the CUDA backend.

Each function mirrors the validation of the HIP backend's typed wrapper
(encodings, ranks, shapes, context ownership, aliasing, launch limits) and
then calls the C ABI on the context's stream.  All launches are
asynchronous; ``CudaContext.sync`` / ``read_bytes`` wait for them.

Reference wrappers mirrored:
  quantized_linear_q4_0_f16  crates/mote-backend-hip/src/quantized_linear.rs:20-98
  rms_norm_f16               crates/mote-backend-hip/src/rms_norm.rs:20-106
  fused_add_rms_norm_f16     crates/mote-backend-hip/src/fused_add_rms_norm.rs:156-269
  rope_f16                   crates/mote-backend-hip/src/rope.rs:25-131
The remaining operators (fused RMSNorm+RoPE, SwiGLU, gate/up+SwiGLU,
embedding gather, Q4_0 encode/decode, cos/sin tables) have no reference
counterpart and follow the same conventions.
"""
from __future__ import annotations

import ctypes
import math

from . import errors
from ._native import lib
from .context import CudaContext, Tensor
from .types import DType, QuantFormat, RopeLayout, TensorDesc

U32_MAX = 0xFFFFFFFF


# ---------------------------------------------------------------- helpers --
def _plain(tensor: Tensor, name: str, expected: DType) -> None:
    enc = tensor.desc.encoding
    if enc.plain is None:
        raise errors.UnsupportedEncoding(actual=enc)
    if enc.plain is not expected:
        raise errors.DTypeMismatch(tensor=name, expected=expected, actual=enc.plain)


def _rank(tensor: Tensor, name: str, expected: int) -> None:
    if tensor.desc.rank != expected:
        raise errors.RankMismatch(tensor=name, expected=expected, actual=tensor.desc.rank)


def _rank_at_least(tensor: Tensor, name: str, minimum: int) -> None:
    if tensor.desc.rank < minimum:
        raise errors.RankTooSmall(tensor=name, minimum=minimum, actual=tensor.desc.rank)


def _q4_0_matrix(tensor: Tensor, name: str = "weights") -> None:
    enc = tensor.desc.encoding
    if enc.quantized is not QuantFormat.Q4_0:
        raise errors.UnsupportedEncoding(actual=enc)
    _rank(tensor, name, 2)


def _shape(tensor: Tensor, name: str, expected) -> None:
    if tuple(tensor.shape) != tuple(expected):
        raise errors.ShapeMismatch(tensor=name, expected=tuple(expected), actual=tensor.shape)


def _not_aliased(a: Tensor, a_name: str, b: Tensor, b_name: str) -> None:
    if a.shares_storage_with(b):
        raise errors.AliasedStorage(tensor=a_name, other=b_name)


def _epsilon(epsilon: float) -> None:
    if not math.isfinite(epsilon) or epsilon < 0.0:
        raise errors.InvalidEpsilon(epsilon=epsilon)


# ------------------------------------------------------------ Q4_0 linear --
_LINEAR_SYMBOLS = {
    (DType.F16, DType.F16): "mote_cuda_quantized_linear_q4_0_f16",
    (DType.F16, DType.F32): "mote_cuda_quantized_linear_q4_0_f16_f32out",
    (DType.F32, DType.F32): "mote_cuda_quantized_linear_q4_0_f32",
}


def quantized_linear_q4_0(context: CudaContext, input: Tensor, weights: Tensor, output: Tensor,
                          input_dtype: DType = DType.F16,
                          output_dtype: DType = DType.F16) -> None:
    """``output = input @ weights^T`` with Q4_0 weights and f32 accumulation.

    ``input`` [rows, K] and ``output`` [rows, N] are plain tensors of the
    given dtypes; ``weights`` is Q4_0 [N, K].  ``output`` must not share
    storage with either input.  Validated empty outputs return without a
    launch.
    """
    f16 = input_dtype is DType.F16 and output_dtype is DType.F16  # the common case
    symbol = _LINEAR_SYMBOLS[(DType.F16, DType.F16)] if f16 else \
        _LINEAR_SYMBOLS.get((input_dtype, output_dtype))
    if symbol is None:
        raise errors.DTypeMismatch(tensor="output", expected=DType.F16, actual=output_dtype)
    _plain(input, "input", input_dtype)
    _rank(input, "input", 2)
    _q4_0_matrix(weights)
    _plain(output, "output", output_dtype)
    _rank(output, "output", 2)
    rows, k = input.shape
    n, wk = weights.shape
    if wk != k:
        raise errors.ShapeMismatch(tensor="weights", expected=(n, k), actual=weights.shape)
    _shape(output, "output", (rows, n))
    in_s = context.storage(input)
    w_s = context.storage(weights)
    out_s = context.storage(output)
    _not_aliased(output, "output", input, "input")
    _not_aliased(output, "output", weights, "weights")
    if rows * n > U32_MAX:
        raise errors.QuantizedLinearDimensionsTooLarge(rows=rows, output_features=n,
                                                       input_features=k)
    if rows * n == 0:
        return
    context.inner.select()
    if f16:
        # the workspace entry (split-K decode, split last wave on tcgen05)
        need = context.linear_workspace_bytes(rows, n, k)
        ws_ptr, ws_bytes = context.linear_workspace(need) if need else (None, 0)
        st = lib().mote_cuda_quantized_linear_q4_0_f16_ws(
            in_s.pointer, w_s.pointer, out_s.pointer, rows, n, k, ws_ptr, ws_bytes,
            context.inner.stream)
        if st:
            errors.check(st, "launch Q4_0 linear kernel")
        return
    errors.check(getattr(lib(), symbol)(in_s.pointer, w_s.pointer, out_s.pointer, rows, n, k,
                                        context.stream), "launch Q4_0 linear kernel")


def quantized_linear_q4_0_f16(context: CudaContext, input: Tensor, weights: Tensor,
                              output: Tensor) -> None:
    """Drop-in for ``mote_backend_hip::quantized_linear_q4_0_f16``: f16 in, f16 out."""
    quantized_linear_q4_0(context, input, weights, output, DType.F16, DType.F16)


_Q8_0_SYMBOLS = {
    (DType.F16, DType.F16): "mote_cuda_quantized_linear_q8_0_f16",
    (DType.F16, DType.F32): "mote_cuda_quantized_linear_q8_0_f16_f32out",
}


def quantized_linear_q8_0(context: CudaContext, input: Tensor, weights: Tensor, output: Tensor,
                          output_dtype: DType = DType.F16) -> None:
    """``output = input @ weights^T`` with Q8_0 weights [N, K] (34-byte
    blocks: f16 scale, 32 signed bytes), f16 input, f32 accumulation and an
    f16 or f32 output -- the device counterpart of mote-reference's
    ``quantized_linear_f32`` for Q8_0.  Same validation as the Q4_0 op."""
    symbol = _Q8_0_SYMBOLS.get((DType.F16, output_dtype))
    if symbol is None:
        raise errors.DTypeMismatch(tensor="output", expected=DType.F16, actual=output_dtype)
    _plain(input, "input", DType.F16)
    _rank(input, "input", 2)
    enc = weights.desc.encoding
    if enc.quantized is not QuantFormat.Q8_0:
        raise errors.UnsupportedEncoding(actual=enc)
    _rank(weights, "weights", 2)
    _plain(output, "output", output_dtype)
    _rank(output, "output", 2)
    rows, k = input.shape
    n, wk = weights.shape
    if wk != k:
        raise errors.ShapeMismatch(tensor="weights", expected=(n, k), actual=weights.shape)
    _shape(output, "output", (rows, n))
    in_s, w_s, out_s = (context.storage(t) for t in (input, weights, output))
    _not_aliased(output, "output", input, "input")
    _not_aliased(output, "output", weights, "weights")
    if rows * n > U32_MAX:
        raise errors.QuantizedLinearDimensionsTooLarge(rows=rows, output_features=n,
                                                       input_features=k)
    if rows * n == 0:
        return
    context.inner.select()
    errors.check(getattr(lib(), symbol)(in_s.pointer, w_s.pointer, out_s.pointer, rows, n, k,
                                        context.stream), "launch Q8_0 linear kernel")


_KQUANT_SYMBOLS = {
    (QuantFormat.Q4_K, DType.F16): "mote_cuda_quantized_linear_q4_k_f16",
    (QuantFormat.Q4_K, DType.F32): "mote_cuda_quantized_linear_q4_k_f16_f32out",
    (QuantFormat.Q6_K, DType.F16): "mote_cuda_quantized_linear_q6_k_f16",
}


def quantized_linear_kquant(context: CudaContext, input: Tensor, weights: Tensor, output: Tensor,
                            output_dtype: DType = DType.F16) -> None:
    """``output = input @ weights^T`` with K-quant weights [N, K] (ggml Q4_K,
    144-byte super-blocks, or Q6_K, 210 bytes, per 256 elements), f16 input,
    f32 accumulation.  Q4_K writes f16 or f32, Q6_K f16.  mote-reference has
    no K-quant linear (it rejects the formats, quantized.rs:152-157); the
    checks are the Q4_0 op's, with K a multiple of 256."""
    enc = weights.desc.encoding
    fmt = enc.quantized
    if fmt not in (QuantFormat.Q4_K, QuantFormat.Q6_K):
        raise errors.UnsupportedEncoding(actual=enc)
    symbol = _KQUANT_SYMBOLS.get((fmt, output_dtype))
    if symbol is None:
        raise errors.DTypeMismatch(tensor="output", expected=DType.F16, actual=output_dtype)
    _plain(input, "input", DType.F16)
    _rank(input, "input", 2)
    _rank(weights, "weights", 2)
    _plain(output, "output", output_dtype)
    _rank(output, "output", 2)
    rows, k = input.shape
    n, wk = weights.shape
    if wk != k:
        raise errors.ShapeMismatch(tensor="weights", expected=(n, k), actual=weights.shape)
    _shape(output, "output", (rows, n))
    in_s, w_s, out_s = (context.storage(t) for t in (input, weights, output))
    _not_aliased(output, "output", input, "input")
    _not_aliased(output, "output", weights, "weights")
    if rows * n > U32_MAX:
        raise errors.QuantizedLinearDimensionsTooLarge(rows=rows, output_features=n,
                                                       input_features=k)
    if rows * n == 0:
        return
    context.inner.select()
    errors.check(getattr(lib(), symbol)(in_s.pointer, w_s.pointer, out_s.pointer, rows, n, k,
                                        context.stream), "launch K-quant linear kernel")


def kquant_decode_f32(context: CudaContext, weights: Tensor, output: Tensor) -> None:
    """Decodes a Q4_K / Q6_K matrix [N, K] into f32 values [N, K]."""
    enc = weights.desc.encoding
    fmt = enc.quantized
    if fmt not in (QuantFormat.Q4_K, QuantFormat.Q6_K):
        raise errors.UnsupportedEncoding(actual=enc)
    _rank(weights, "weights", 2)
    _plain(output, "output", DType.F32)
    _shape(output, "output", weights.shape)
    w_s, out_s = context.storage(weights), context.storage(output)
    n, k = weights.shape
    if n * k == 0:
        return
    context.inner.select()
    code = 2 if fmt is QuantFormat.Q4_K else 3
    errors.check(lib().mote_cuda_kquant_dequantize_f32(code, w_s.pointer, out_s.pointer, n, k,
                                                       context.stream), "decode K-quant matrix")


def matmul_f16_f32(context: CudaContext, lhs: Tensor, rhs: Tensor, output: Tensor) -> None:
    """``output[m, n] = lhs[m, k] @ rhs[k, n]``: row-major f16 inputs, f32
    accumulation and output, through cuBLASLt (the HIP backend's
    ``matmul_f16_f32``, crates/mote-backend-hip/src/matmul.rs:11-113, same
    checks).  The first call of a new (m, n, k) tunes and caches an
    algorithm, synchronizing the stream: make it before any graph capture."""
    for t, name, dt in ((lhs, "lhs", DType.F16), (rhs, "rhs", DType.F16),
                        (output, "output", DType.F32)):
        _plain(t, name, dt)
        _rank(t, name, 2)
    m, k = lhs.shape
    rk, n = rhs.shape
    if rk != k:
        raise errors.ShapeMismatch(tensor="rhs", expected=(k, n), actual=rhs.shape)
    _shape(output, "output", (m, n))
    if m * n == 0:
        return
    if max(m, n, k) > 0x7FFFFFFFFFFFFFFF:
        raise errors.MatmulDimensionsTooLarge(m=m, n=n, k=k)
    l_s, r_s, o_s = (context.storage(t) for t in (lhs, rhs, output))
    handle, ws, ws_bytes = context.blas()
    context.inner.select()
    st = lib().mote_cuda_blaslt_matmul_f16_f32(handle, m, n, k, l_s.pointer, r_s.pointer,
                                                o_s.pointer, ws, ws_bytes, context.stream)
    if st != 0:
        msg = lib().mote_cuda_blaslt_last_error(handle)
        raise errors.BlasLt(operation="matmul", status=int(st),
                            message=(msg or b"").decode(errors="replace"))


def quantized_linear_q4_0_f32(context: CudaContext, input: Tensor, weights: Tensor,
                              output: Tensor) -> None:
    """f32 in, f32 out (device counterpart of ``quantized_linear_f32``)."""
    quantized_linear_q4_0(context, input, weights, output, DType.F32, DType.F32)


def quantized_linear_q4_0_f16_residual(context: CudaContext, input: Tensor, weights: Tensor,
                                       residual: Tensor, output: Tensor) -> None:
    """``output = input @ weights^T + residual`` (f16, one rounding).

    ``output`` may be ``residual`` (in-place residual update) but must not
    share storage with ``input`` or ``weights``.
    """
    _plain(input, "input", DType.F16)
    _rank(input, "input", 2)
    _q4_0_matrix(weights)
    _plain(residual, "residual", DType.F16)
    _plain(output, "output", DType.F16)
    rows, k = input.shape
    n, wk = weights.shape
    if wk != k:
        raise errors.ShapeMismatch(tensor="weights", expected=(n, k), actual=weights.shape)
    _shape(output, "output", (rows, n))
    _shape(residual, "residual", (rows, n))
    in_s, w_s, r_s, out_s = (context.storage(t) for t in (input, weights, residual, output))
    _not_aliased(output, "output", input, "input")
    _not_aliased(output, "output", weights, "weights")
    if rows * n > U32_MAX:
        raise errors.QuantizedLinearDimensionsTooLarge(rows=rows, output_features=n,
                                                       input_features=k)
    if rows * n == 0:
        return
    context.inner.select()
    errors.check(lib().mote_cuda_quantized_linear_q4_0_f16_residual(
        in_s.pointer, w_s.pointer, r_s.pointer, out_s.pointer, rows, n, k, context.stream),
        "launch Q4_0 linear + residual kernel")


def q4_0_gate_up_swiglu_f16(context: CudaContext, input: Tensor, gate: Tensor, up: Tensor,
                            output: Tensor) -> None:
    """``output = silu(input @ gate^T) * (input @ up^T)`` in one kernel."""
    _plain(input, "input", DType.F16)
    _rank(input, "input", 2)
    _q4_0_matrix(gate, "gate")
    _q4_0_matrix(up, "up")
    _plain(output, "output", DType.F16)
    _rank(output, "output", 2)
    rows, k = input.shape
    f = gate.shape[0]
    _shape(gate, "gate", (f, k))
    _shape(up, "up", (f, k))
    _shape(output, "output", (rows, f))
    in_s, g_s, u_s, out_s = (context.storage(t) for t in (input, gate, up, output))
    for other, name in ((input, "input"), (gate, "gate"), (up, "up")):
        _not_aliased(output, "output", other, name)
    if rows * f > U32_MAX:
        raise errors.QuantizedLinearDimensionsTooLarge(rows=rows, output_features=f,
                                                       input_features=k)
    if rows * f == 0:
        return
    context.inner.select()
    errors.check(lib().mote_cuda_q4_0_gate_up_swiglu_f16(
        in_s.pointer, g_s.pointer, u_s.pointer, out_s.pointer, rows, f, k, context.stream),
        "launch gate/up SwiGLU kernel")


# ------------------------------------------------- decoder-layer fusions --
def _norm_gamma(gamma: Tensor, k: int) -> None:
    _plain(gamma, "gamma", DType.F16)
    _shape(gamma, "gamma", (k,))


def q4_0_rms_norm_linear_f16(context: CudaContext, input: Tensor, gamma: Tensor, weights: Tensor,
                             output: Tensor, epsilon: float) -> None:
    """``output = rms_norm(input) * gamma @ weights^T`` (norm fused into the
    projection's activation staging; f16 in, f16 out)."""
    _plain(input, "input", DType.F16)
    _rank(input, "input", 2)
    _q4_0_matrix(weights)
    _plain(output, "output", DType.F16)
    _epsilon(epsilon)
    rows, k = input.shape
    n = weights.shape[0]
    _shape(weights, "weights", (n, k))
    _shape(output, "output", (rows, n))
    _norm_gamma(gamma, k)
    in_s, g_s, w_s, out_s = (context.storage(t) for t in (input, gamma, weights, output))
    for other, name in ((input, "input"), (weights, "weights"), (gamma, "gamma")):
        _not_aliased(output, "output", other, name)
    if rows * n > U32_MAX:
        raise errors.QuantizedLinearDimensionsTooLarge(rows=rows, output_features=n,
                                                       input_features=k)
    if rows * n == 0:
        return
    context.inner.select()
    errors.check(lib().mote_cuda_q4_0_rms_norm_linear_f16(
        in_s.pointer, g_s.pointer, w_s.pointer, out_s.pointer, rows, n, k,
        ctypes.c_float(epsilon), context.stream), "launch RMSNorm + Q4_0 linear kernel")


def q4_0_rms_norm_gate_up_swiglu_f16(context: CudaContext, input: Tensor, gamma: Tensor,
                                     gate: Tensor, up: Tensor, output: Tensor,
                                     epsilon: float) -> None:
    """``output = silu(x_n @ gate^T) * (x_n @ up^T)``, x_n = rms_norm(input) * gamma."""
    _plain(input, "input", DType.F16)
    _rank(input, "input", 2)
    _q4_0_matrix(gate, "gate")
    _q4_0_matrix(up, "up")
    _plain(output, "output", DType.F16)
    _epsilon(epsilon)
    rows, k = input.shape
    f = gate.shape[0]
    _shape(gate, "gate", (f, k))
    _shape(up, "up", (f, k))
    _shape(output, "output", (rows, f))
    _norm_gamma(gamma, k)
    in_s, gm_s, g_s, u_s, out_s = (context.storage(t) for t in (input, gamma, gate, up, output))
    for other, name in ((input, "input"), (gate, "gate"), (up, "up"), (gamma, "gamma")):
        _not_aliased(output, "output", other, name)
    if rows * f > U32_MAX:
        raise errors.QuantizedLinearDimensionsTooLarge(rows=rows, output_features=f,
                                                       input_features=k)
    if rows * f == 0:
        return
    context.inner.select()
    errors.check(lib().mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16(
        in_s.pointer, gm_s.pointer, g_s.pointer, u_s.pointer, out_s.pointer, rows, f, k,
        ctypes.c_float(epsilon), context.stream), "launch RMSNorm + gate/up SwiGLU kernel")


def q4_0_rms_norm_qkv_rope_f16(context: CudaContext, input: Tensor, gamma: Tensor,
                               weights: Tensor, cos: Tensor, sin: Tensor, output: Tensor,
                               q_heads: int, kv_heads: int, head_dim: int,
                               epsilon: float) -> None:
    """QKV projection of ``rms_norm(input) * gamma`` with RoPE (HalfSplit)
    applied to the q and k heads before the f16 rounding.  ``output`` is
    ``[rows, (q_heads + 2 kv_heads) * head_dim]``; cos/sin ``[rows, head_dim/2]``."""
    _plain(input, "input", DType.F16)
    _rank(input, "input", 2)
    _q4_0_matrix(weights)
    _plain(output, "output", DType.F16)
    _plain(cos, "cos", DType.F32)
    _plain(sin, "sin", DType.F32)
    _epsilon(epsilon)
    rows, k = input.shape
    n = (q_heads + 2 * kv_heads) * head_dim
    _shape(weights, "weights", (n, k))
    _shape(output, "output", (rows, n))
    _shape(cos, "cos", (rows, head_dim // 2))
    _shape(sin, "sin", (rows, head_dim // 2))
    _norm_gamma(gamma, k)
    ptrs = [context.storage(t).pointer for t in (input, gamma, weights, cos, sin, output)]
    for other, name in ((input, "input"), (weights, "weights"), (gamma, "gamma"), (cos, "cos"),
                        (sin, "sin")):
        _not_aliased(output, "output", other, name)
    if rows * n == 0:
        return
    context.inner.select()
    errors.check(lib().mote_cuda_q4_0_rms_norm_qkv_rope_f16(
        *ptrs, rows, q_heads, kv_heads, head_dim, k, ctypes.c_float(epsilon), context.stream),
        "launch RMSNorm + QKV + RoPE kernel")


def q4_0_encode_f32(context: CudaContext, input: Tensor, weights: Tensor) -> None:
    """Quantizes f32 [N, K] into Q4_0 [N, K] (ggml reference rule)."""
    _plain(input, "input", DType.F32)
    _rank(input, "input", 2)
    _q4_0_matrix(weights)
    _shape(weights, "weights", input.shape)
    in_s, w_s = context.storage(input), context.storage(weights)
    context.inner.select()
    errors.check(lib().mote_cuda_q4_0_encode_f32(in_s.pointer, w_s.pointer, input.shape[0],
                                                 input.shape[1], context.stream),
                 "launch Q4_0 encode kernel")


def q4_0_decode_f32(context: CudaContext, weights: Tensor, output: Tensor) -> None:
    """Dequantizes Q4_0 [N, K] into f32 [N, K] (bit-exact)."""
    _q4_0_matrix(weights)
    _plain(output, "output", DType.F32)
    _shape(output, "output", weights.shape)
    w_s, o_s = context.storage(weights), context.storage(output)
    context.inner.select()
    errors.check(lib().mote_cuda_q4_0_decode_f32(w_s.pointer, o_s.pointer, weights.shape[0],
                                                 weights.shape[1], context.stream),
                 "launch Q4_0 decode kernel")


# ----------------------------------------------------------------- norms --
def _rows_hidden(input: Tensor, weight: Tensor):
    _rank_at_least(input, "input", 1)
    _rank(weight, "weight", 1)
    hidden = input.shape[-1]
    if weight.shape[0] != hidden:
        raise errors.ShapeMismatch(tensor="weight", expected=(hidden,), actual=weight.shape)
    return hidden


def rms_norm_f16(context: CudaContext, input: Tensor, weight: Tensor, output: Tensor,
                 epsilon: float) -> None:
    """Row RMSNorm over the last dimension; f16 tensors, f32 math."""
    for t, name in ((input, "input"), (weight, "weight"), (output, "output")):
        _plain(t, name, DType.F16)
    hidden = _rows_hidden(input, weight)
    _shape(output, "output", input.shape)
    _epsilon(epsilon)
    in_s, w_s, out_s = (context.storage(t) for t in (input, weight, output))
    numel = input.desc.numel
    if numel == 0:
        return
    rows = numel // hidden
    if rows > U32_MAX:
        raise errors.RmsNormDimensionsTooLarge(rows=rows, hidden=hidden)
    context.inner.select()
    errors.check(lib().mote_cuda_rms_norm_f16(in_s.pointer, w_s.pointer, out_s.pointer, rows,
                                              hidden, ctypes.c_float(epsilon), context.stream),
                 "launch RMSNorm kernel")


def fused_add_rms_norm_f16(context: CudaContext, input: Tensor, residual: Tensor, weight: Tensor,
                           output: Tensor, epsilon: float) -> None:
    """``residual <- f16(input + residual)``; ``output = rms_norm(input + residual)``."""
    for t, name in ((input, "input"), (residual, "residual"), (weight, "weight"),
                    (output, "output")):
        _plain(t, name, DType.F16)
    hidden = _rows_hidden(input, weight)
    _shape(residual, "residual", input.shape)
    _shape(output, "output", input.shape)
    _epsilon(epsilon)
    in_s, r_s, w_s, out_s = (context.storage(t) for t in (input, residual, weight, output))
    _not_aliased(output, "output", residual, "residual")
    _not_aliased(weight, "weight", output, "output")
    _not_aliased(weight, "weight", residual, "residual")
    numel = input.desc.numel
    if numel == 0:
        return
    rows = numel // hidden
    if rows > U32_MAX:
        raise errors.FusedAddRmsNormDimensionsTooLarge(rows=rows, hidden=hidden)
    context.inner.select()
    errors.check(lib().mote_cuda_fused_add_rms_norm_f16(
        in_s.pointer, r_s.pointer, w_s.pointer, out_s.pointer, rows, hidden,
        ctypes.c_float(epsilon), context.stream), "launch fused add + RMSNorm kernel")


# ------------------------------------------------------------------ RoPE --
def _rope_geometry(input: Tensor, cos: Tensor, sin: Tensor, output: Tensor, rotary_dim: int):
    _plain(input, "input", DType.F16)
    _plain(cos, "cos", DType.F32)
    _plain(sin, "sin", DType.F32)
    _plain(output, "output", DType.F16)
    _rank_at_least(input, "input", 2)
    *lead, heads, head_dim = input.shape
    if rotary_dim % 2 or rotary_dim > head_dim:
        raise errors.InvalidRotaryDim(rotary_dim=rotary_dim, head_dim=head_dim)
    _shape(output, "output", input.shape)
    cache = tuple(lead) + (rotary_dim // 2,)
    _shape(cos, "cos", cache)
    _shape(sin, "sin", cache)
    return math.prod(lead), heads, head_dim


def rope_f16(context: CudaContext, input: Tensor, cos: Tensor, sin: Tensor, output: Tensor,
             rotary_dim: int, layout: RopeLayout) -> None:
    """Rotary embedding of ``[..., heads, head_dim]`` vectors; in-place allowed."""
    tokens, heads, head_dim = _rope_geometry(input, cos, sin, output, rotary_dim)
    in_s, c_s, s_s, out_s = (context.storage(t) for t in (input, cos, sin, output))
    if input.desc.numel == 0:
        return
    if tokens * heads > U32_MAX:
        raise errors.RopeDimensionsTooLarge(tokens=tokens, heads=heads, head_dim=head_dim,
                                            rotary_dim=rotary_dim)
    context.inner.select()
    errors.check(lib().mote_cuda_rope_f16(in_s.pointer, c_s.pointer, s_s.pointer, out_s.pointer,
                                          tokens, heads, head_dim, rotary_dim, layout.value,
                                          context.stream), "launch RoPE kernel")


def rms_norm_rope_f16(context: CudaContext, x: Tensor, gamma: Tensor, x_out: Tensor, q: Tensor,
                      q_out: Tensor, k: Tensor, k_out: Tensor, cos: Tensor, sin: Tensor,
                      epsilon: float, layout: RopeLayout = RopeLayout.HalfSplit) -> None:
    """One launch: ``x_out = rms_norm(x) * gamma``, ``q_out/k_out = rope(q/k)``.

    ``x`` is [tokens, hidden]; ``q`` [tokens, q_heads, head_dim] and ``k``
    [tokens, kv_heads, head_dim] rotate over the whole head
    (rotary_dim == head_dim) with the per-token cos/sin rows.
    """
    for t, name in ((x, "x"), (gamma, "gamma"), (x_out, "x_out")):
        _plain(t, name, DType.F16)
    _rank(x, "x", 2)
    hidden = _rows_hidden(x, gamma)
    _shape(x_out, "x_out", x.shape)
    _epsilon(epsilon)
    _rank(q, "q", 3)
    _rank(k, "k", 3)
    tokens = x.shape[0]
    head_dim = q.shape[2]
    _shape(q, "q", (tokens, q.shape[1], head_dim))
    _shape(k, "k", (tokens, k.shape[1], head_dim))
    _rope_geometry(q, cos, sin, q_out, head_dim)
    _rope_geometry(k, cos, sin, k_out, head_dim)
    ptrs = [context.storage(t).pointer for t in (x, gamma, x_out, q, q_out, k, k_out, cos, sin)]
    if tokens == 0:
        return
    context.inner.select()
    errors.check(lib().mote_cuda_rms_norm_rope_f16(*ptrs, tokens, hidden, q.shape[1], k.shape[1],
                                                   head_dim, layout.value,
                                                   ctypes.c_float(epsilon), context.stream),
                 "launch fused RMSNorm + RoPE kernel")


def rope_cos_sin_f32(context: CudaContext, positions: Tensor, cos: Tensor, sin: Tensor,
                     theta: float = 10000.0) -> None:
    """Fills ``cos``/``sin`` [tokens, rotary_dim/2] for int32 ``positions`` [tokens]."""
    _plain(positions, "positions", DType.I32)
    _rank(positions, "positions", 1)
    _plain(cos, "cos", DType.F32)
    _plain(sin, "sin", DType.F32)
    tokens = positions.shape[0]
    _rank(cos, "cos", 2)
    _shape(cos, "cos", (tokens, cos.shape[1]))
    _shape(sin, "sin", cos.shape)
    p, c, s = (context.storage(t).pointer for t in (positions, cos, sin))
    context.inner.select()
    errors.check(lib().mote_cuda_rope_cos_sin_f32(p, c, s, tokens, 2 * cos.shape[1],
                                                  ctypes.c_double(theta), context.stream),
                 "launch RoPE table kernel")


# ---------------------------------------------------------- SwiGLU, gather --
def swiglu_f16(context: CudaContext, gate: Tensor, up: Tensor, output: Tensor) -> None:
    """``output = silu(gate) * up`` elementwise (f16, f32 math)."""
    for t, name in ((gate, "gate"), (up, "up"), (output, "output")):
        _plain(t, name, DType.F16)
    _shape(up, "up", gate.shape)
    _shape(output, "output", gate.shape)
    g, u, o = (context.storage(t).pointer for t in (gate, up, output))
    n = gate.desc.numel
    if n == 0:
        return
    context.inner.select()
    errors.check(lib().mote_cuda_swiglu_f16(g, u, o, n, context.stream), "launch SwiGLU kernel")


class _Flag:
    def __init__(self, context: CudaContext):
        from .types import plain

        self.tensor = context.empty(plain((1,), DType.I32))


def embedding_gather_f16(context: CudaContext, table: Tensor, ids: Tensor, output: Tensor,
                         check: bool = True) -> None:
    """``output[t] = table[ids[t]]`` (bit-exact).

    Ids outside ``[0, vocab)`` give a zero row.  With ``check`` the call
    synchronizes and raises :class:`errors.IndexOutOfRange` if any id was
    out of range; without it the launch stays asynchronous.
    """
    _plain(table, "table", DType.F16)
    _rank(table, "table", 2)
    _plain(ids, "ids", DType.I32)
    _rank(ids, "ids", 1)
    _plain(output, "output", DType.F16)
    vocab, hidden = table.shape
    _shape(output, "output", (ids.shape[0], hidden))
    t, i, o = (context.storage(x).pointer for x in (table, ids, output))
    _not_aliased(output, "output", table, "table")
    tokens = ids.shape[0]
    if tokens == 0 or hidden == 0:
        return
    flag = getattr(context, "_gather_flag", None)
    if flag is None:
        flag = context._gather_flag = _Flag(context)
    fptr = flag.tensor.pointer
    context.inner.select()
    errors.check(lib().mote_cuda_memset_async(fptr, 0, 4, context.stream), "clear gather flag")
    errors.check(lib().mote_cuda_embedding_gather_f16(t, i, o, tokens, vocab, hidden, fptr,
                                                      context.stream),
                 "launch embedding gather kernel")
    if check:
        import numpy as np

        value = int(np.frombuffer(context.read_bytes(flag.tensor), np.uint32)[0])
        if value:
            raise errors.IndexOutOfRange(vocab=vocab)


# --------------------------------------------------------------- attention --
def kv_cache_append_f16(context: CudaContext, k_new: Tensor, v_new: Tensor, k_cache: Tensor,
                        v_cache: Tensor, slots: Tensor, check: bool = True) -> None:
    """Writes ``k_new[t]``/``v_new[t]`` ([tokens, kv_heads, head_dim] f16)
    into cache row ``slots[t]`` of ``k_cache``/``v_cache`` ([rows, kv_heads,
    head_dim] f16).  Slots outside the cache are skipped; with ``check`` the
    call synchronizes and raises :class:`errors.IndexOutOfRange` for them.
    No reference counterpart (the reference lists KV-cache operations as
    planned, docs/roadmap.md:60)."""
    for t, name in ((k_new, "k_new"), (v_new, "v_new"), (k_cache, "k_cache"),
                    (v_cache, "v_cache")):
        _plain(t, name, DType.F16)
        _rank(t, name, 3)
    _plain(slots, "slots", DType.I32)
    _rank(slots, "slots", 1)
    tokens, kvh, hd = k_new.shape
    _shape(v_new, "v_new", k_new.shape)
    rows = k_cache.shape[0]
    _shape(k_cache, "k_cache", (rows, kvh, hd))
    _shape(v_cache, "v_cache", (rows, kvh, hd))
    _shape(slots, "slots", (tokens,))
    _not_aliased(k_cache, "k_cache", v_cache, "v_cache")
    if tokens == 0:
        return
    flag = getattr(context, "_append_flag", None)
    if flag is None:
        flag = context._append_flag = _Flag(context)
    fptr = flag.tensor.pointer
    ptrs = [context.storage(t).pointer for t in (k_new, v_new, k_cache, v_cache, slots)]
    context.inner.select()
    errors.check(lib().mote_cuda_memset_async(fptr, 0, 4, context.stream), "clear append flag")
    errors.check(lib().mote_cuda_kv_cache_append_f16(*ptrs, tokens, kvh, hd, rows, fptr,
                                                     context.stream),
                 "launch KV-cache append kernel")
    if check:
        import numpy as np

        if int(np.frombuffer(context.read_bytes(flag.tensor), np.uint32)[0]):
            raise errors.IndexOutOfRange(vocab=rows)


def gqa_attention_decode_f16(context: CudaContext, q: Tensor, k_cache: Tensor, v_cache: Tensor,
                             seq_lens: Tensor, output: Tensor, seq_capacity: int, max_len: int,
                             scale: float | None = None) -> None:
    """One query token per sequence over its cached K/V (grouped-query):
    ``output[b, h] = softmax(scale * q[b, h] . K_b[:len_b, h // g]) . V_b``
    with ``g = q_heads // kv_heads``, sequence ``b`` at cache rows
    ``b * seq_capacity + position`` and ``len_b = min(seq_lens[b], max_len)``.
    ``scale`` defaults to ``1 / sqrt(head_dim)``."""
    import math

    _plain(q, "q", DType.F16)
    _rank(q, "q", 3)
    _plain(output, "output", DType.F16)
    _shape(output, "output", q.shape)
    batch, qh, hd = q.shape
    for t, name in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        _plain(t, name, DType.F16)
        _rank(t, name, 3)
    rows, kvh, hd2 = k_cache.shape
    _shape(k_cache, "k_cache", (rows, kvh, hd))
    _shape(v_cache, "v_cache", k_cache.shape)
    _plain(seq_lens, "seq_lens", DType.I32)
    _shape(seq_lens, "seq_lens", (batch,))
    if batch * seq_capacity > rows or max_len > seq_capacity:
        raise errors.ShapeMismatch(tensor="k_cache", expected=(batch * seq_capacity, kvh, hd),
                                   actual=k_cache.shape)
    _not_aliased(output, "output", q, "q")
    if batch == 0 or qh == 0:
        return
    scale = 1.0 / math.sqrt(hd) if scale is None else float(scale)
    need = ctypes.c_uint64(0)
    errors.check(lib().mote_cuda_gqa_attention_decode_workspace_bytes(
        batch, qh, kvh, hd, max_len, ctypes.byref(need)), "query attention workspace")
    ws_ptr, ws_bytes = context.attention_workspace(need.value) if need.value else (None, 0)
    ptrs = [context.storage(t).pointer for t in (q, k_cache, v_cache, seq_lens, output)]
    context.inner.select()
    errors.check(lib().mote_cuda_gqa_attention_decode_f16(
        *ptrs, batch, qh, kvh, hd, seq_capacity, max_len, ctypes.c_float(scale), ws_ptr,
        ws_bytes, context.stream), "launch GQA decode attention kernel")


def gqa_attention_prefill_f16(context: CudaContext, q: Tensor, k_cache: Tensor, v_cache: Tensor,
                              output: Tensor, start: int, row0: int = 0,
                              scale: float | None = None) -> None:
    """Causal attention of a prefill chunk on the tensor cores: ``q``
    [tokens, q_heads, 64] f16 holds the queries at positions ``start ..
    start + tokens - 1`` of one sequence whose position ``p`` is cache row
    ``row0 + p`` (the chunk's own K/V already appended);
    ``output[t, h] = softmax_{p <= start + t}(scale q[t, h] . K[p, h // g]) . V[p, h // g]``.
    ``scale`` defaults to ``1 / sqrt(head_dim)``."""
    _plain(q, "q", DType.F16)
    _rank(q, "q", 3)
    _plain(output, "output", DType.F16)
    _shape(output, "output", q.shape)
    tokens, qh, hd = q.shape
    for t, name in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        _plain(t, name, DType.F16)
        _rank(t, name, 3)
    rows, kvh, _ = k_cache.shape
    _shape(k_cache, "k_cache", (rows, kvh, hd))
    _shape(v_cache, "v_cache", k_cache.shape)
    if row0 + start + tokens > rows:
        raise errors.ShapeMismatch(tensor="k_cache", expected=(row0 + start + tokens, kvh, hd),
                                   actual=k_cache.shape)
    _not_aliased(output, "output", q, "q")
    if tokens == 0 or qh == 0:
        return
    scale = 1.0 / math.sqrt(hd) if scale is None else float(scale)
    ptrs = [context.storage(t).pointer for t in (q, k_cache, v_cache, output)]
    context.inner.select()
    errors.check(lib().mote_cuda_gqa_attention_prefill_f16(
        *ptrs, tokens, start, qh, kvh, hd, row0, rows, ctypes.c_float(scale), context.stream),
        "launch GQA prefill attention kernel")
