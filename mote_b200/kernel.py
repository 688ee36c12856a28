"""Operator surface and dispatch mirroring ``mote-kernel`` / ``mote-runtime``.

``KernelKey``, ``KernelArgs``, ``KernelImpl``, ``KernelRegistry`` and
``Runtime`` follow crates/mote-kernel/src/lib.rs:7-56 and
crates/mote-runtime/src/lib.rs:10-38: a registry maps a semantic key to a
list of implementations and ``resolve`` returns the most recently registered
one whose ``supports(device, key)`` is true.

:func:`register_cuda_kernels` registers this backend's C-ABI entry points as
``KernelImpl``s.  ``KernelArgs.opaque`` carries exactly the C argument list
of the entry point as unsigned machine words (pointers, dimensions, the
stream handle); ``f32`` / ``f64`` scalars travel as their IEEE bit patterns.
That is how a Rust ``KernelImpl::launch`` would forward ``&[usize]`` to the
``extern "C"`` function.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field
from typing import Protocol

from ._native import lib
from .types import DType


@dataclass(frozen=True)
class KernelKey:
    op: str
    dtype: DType | None = None
    shape_class: str | None = None


@dataclass(frozen=True)
class KernelArgs:
    opaque: tuple[int, ...] = ()


class KernelError(Exception):
    pass


class Unsupported(KernelError):
    def __init__(self):
        super().__init__("kernel is not supported on this device")


class Launch(KernelError):
    def __init__(self, message: str):
        super().__init__(f"kernel launch failed: {message}")


class KernelImpl(Protocol):
    def name(self) -> str: ...

    def supports(self, device, key: KernelKey) -> bool: ...

    def launch(self, device, args: KernelArgs) -> None: ...


@dataclass
class KernelRegistry:
    entries: dict[KernelKey, list[KernelImpl]] = field(default_factory=dict)

    def register(self, key: KernelKey, kernel: KernelImpl) -> None:
        self.entries.setdefault(key, []).append(kernel)

    def resolve(self, key: KernelKey, device) -> KernelImpl | None:
        """Later registrations take precedence (mote-kernel/src/lib.rs:43-55)."""
        for kernel in reversed(self.entries.get(key, [])):
            if kernel.supports(device, key):
                return kernel
        return None


class Runtime:
    def __init__(self):
        self._kernels = KernelRegistry()

    def kernels(self) -> KernelRegistry:
        return self._kernels

    def kernels_mut(self) -> KernelRegistry:
        return self._kernels

    def resolve(self, key: KernelKey, device) -> KernelImpl | None:
        return self._kernels.resolve(key, device)


def f32_bits(value: float) -> int:
    return struct.unpack("<I", struct.pack("<f", value))[0]


def f64_bits(value: float) -> int:
    return struct.unpack("<Q", struct.pack("<d", value))[0]


# Per C entry point, the kind of each argument: p = pointer, u = u64,
# w = u32, f = f32 (bits), d = f64 (bits).
_ARG_KINDS = {
    "mote_cuda_quantized_linear_q4_0_f16": "pppuuup",
    "mote_cuda_quantized_linear_q4_0_f16_f32out": "pppuuup",
    "mote_cuda_quantized_linear_q4_0_f32": "pppuuup",
    "mote_cuda_quantized_linear_q8_0_f16": "pppuuup",
    "mote_cuda_quantized_linear_q8_0_f16_f32out": "pppuuup",
    "mote_cuda_quantized_linear_q4_k_f16": "pppuuup",
    "mote_cuda_quantized_linear_q4_k_f16_f32out": "pppuuup",
    "mote_cuda_quantized_linear_q6_k_f16": "pppuuup",
    "mote_cuda_q4_0_gate_up_swiglu_f16": "ppppuuup",
    "mote_cuda_quantized_linear_q4_0_f16_residual": "ppppuuup",
    "mote_cuda_quantized_linear_q4_0_f16_ws": "pppuuupup",
    "mote_cuda_quantized_linear_q4_0_f16_noalloc": "pppuuup",
    "mote_cuda_q4_0_rms_norm_linear_f16": "ppppuuufp",
    "mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16": "pppppuuufp",
    "mote_cuda_q4_0_rms_norm_qkv_rope_f16": "ppppppuuuuufp",
    "mote_cuda_rms_norm_f16": "pppuufp",
    "mote_cuda_fused_add_rms_norm_f16": "ppppuufp",
    "mote_cuda_rope_f16": "ppppuuuuwp",
    "mote_cuda_rms_norm_rope_f16": "pppppppppuuuuuwfp",
    "mote_cuda_swiglu_f16": "pppup",
    "mote_cuda_embedding_gather_f16": "pppuuupp",
    "mote_cuda_q4_0_decode_f32": "ppuup",
    "mote_cuda_q4_0_encode_f32": "ppuup",
    "mote_cuda_rope_cos_sin_f32": "pppuudp",
    "mote_cuda_kv_cache_append_f16": "pppppuuuupp",
    "mote_cuda_gqa_attention_decode_f16": "pppppuuuuuufpup",
    "mote_cuda_gqa_attention_prefill_f16": "ppppuuuuuuufp",
    "mote_cuda_q4_0_decoder_stack_f16": "pwpuuuuufpup",
}

# (op, dtype) -> entry point
CUDA_KERNELS = {
    ("quantized_linear_q4_0", DType.F16): "mote_cuda_quantized_linear_q4_0_f16",
    ("quantized_linear_q4_0_f32out", DType.F16): "mote_cuda_quantized_linear_q4_0_f16_f32out",
    ("quantized_linear_q4_0", DType.F32): "mote_cuda_quantized_linear_q4_0_f32",
    ("quantized_linear_q8_0", DType.F16): "mote_cuda_quantized_linear_q8_0_f16",
    ("quantized_linear_q8_0_f32out", DType.F16): "mote_cuda_quantized_linear_q8_0_f16_f32out",
    ("quantized_linear_q4_k", DType.F16): "mote_cuda_quantized_linear_q4_k_f16",
    ("quantized_linear_q4_k_f32out", DType.F16): "mote_cuda_quantized_linear_q4_k_f16_f32out",
    ("quantized_linear_q6_k", DType.F16): "mote_cuda_quantized_linear_q6_k_f16",
    ("gate_up_swiglu_q4_0", DType.F16): "mote_cuda_q4_0_gate_up_swiglu_f16",
    ("quantized_linear_q4_0_residual", DType.F16): "mote_cuda_quantized_linear_q4_0_f16_residual",
    ("quantized_linear_q4_0_ws", DType.F16): "mote_cuda_quantized_linear_q4_0_f16_ws",
    ("quantized_linear_q4_0_noalloc", DType.F16): "mote_cuda_quantized_linear_q4_0_f16_noalloc",
    ("rms_norm_linear_q4_0", DType.F16): "mote_cuda_q4_0_rms_norm_linear_f16",
    ("rms_norm_gate_up_swiglu_q4_0", DType.F16): "mote_cuda_q4_0_rms_norm_gate_up_swiglu_f16",
    ("rms_norm_qkv_rope_q4_0", DType.F16): "mote_cuda_q4_0_rms_norm_qkv_rope_f16",
    ("rms_norm", DType.F16): "mote_cuda_rms_norm_f16",
    ("fused_add_rms_norm", DType.F16): "mote_cuda_fused_add_rms_norm_f16",
    ("rope", DType.F16): "mote_cuda_rope_f16",
    ("rms_norm_rope", DType.F16): "mote_cuda_rms_norm_rope_f16",
    ("swiglu", DType.F16): "mote_cuda_swiglu_f16",
    ("embedding_gather", DType.F16): "mote_cuda_embedding_gather_f16",
    ("q4_0_decode", DType.F32): "mote_cuda_q4_0_decode_f32",
    ("q4_0_encode", DType.F32): "mote_cuda_q4_0_encode_f32",
    ("rope_cos_sin", DType.F32): "mote_cuda_rope_cos_sin_f32",
    ("kv_cache_append", DType.F16): "mote_cuda_kv_cache_append_f16",
    ("gqa_attention_decode", DType.F16): "mote_cuda_gqa_attention_decode_f16",
    ("gqa_attention_prefill", DType.F16): "mote_cuda_gqa_attention_prefill_f16",
    ("decoder_stack_q4_0", DType.F16): "mote_cuda_q4_0_decoder_stack_f16",
}


class CudaKernel:
    """A ``KernelImpl`` forwarding opaque words to one C entry point."""

    def __init__(self, op: str, dtype: DType, symbol: str):
        self._op = op
        self._dtype = dtype
        self.symbol = symbol
        self.kinds = _ARG_KINDS[symbol]

    def name(self) -> str:
        return self.symbol

    def supports(self, device, key: KernelKey) -> bool:
        return getattr(device, "backend", None) == "cuda" and key.op == self._op and \
            key.dtype in (None, self._dtype)

    def launch(self, device, args: KernelArgs) -> None:
        if len(args.opaque) != len(self.kinds):
            raise Launch(f"{self.symbol} takes {len(self.kinds)} words, got {len(args.opaque)}")
        values = []
        for kind, word in zip(self.kinds, args.opaque):
            if kind == "f":
                values.append(ctypes.c_float(struct.unpack("<f", struct.pack("<I", word))[0]))
            elif kind == "d":
                values.append(ctypes.c_double(struct.unpack("<d", struct.pack("<Q", word))[0]))
            else:
                values.append(word)
        st = lib().mote_cuda_set_device(int(device.ordinal))
        if st == 0:
            st = getattr(lib(), self.symbol)(*values)
        if st != 0:
            from ._native import status_string

            raise Launch(f"{self.symbol}: status {st} ({status_string(st)})")


def register_cuda_kernels(registry: KernelRegistry) -> None:
    """Registers every CUDA entry point under its semantic key."""
    for (op, dtype), symbol in CUDA_KERNELS.items():
        registry.register(KernelKey(op, dtype), CudaKernel(op, dtype, symbol))
