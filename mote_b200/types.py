"""Tensor metadata mirroring ``mote-types`` (crates/mote-types/src).

Only what the CUDA data plane's wrappers validate is mirrored: dtypes,
quantization formats and their block geometry, encodings, the RoPE pairing
selector, shapes, layouts and the byte-span / alignment rules of
``TensorDesc`` (crates/mote-types/src/tensor_desc.rs:52-151).
"""
from __future__ import annotations

import enum
import math
from dataclasses import dataclass, field
from functools import cached_property


class DType(enum.Enum):
    """crates/mote-types/src/lib.rs (DType): size and alignment in bytes."""

    F32 = ("f32", 4)
    F16 = ("f16", 2)
    BF16 = ("bf16", 2)
    I32 = ("i32", 4)
    I8 = ("i8", 1)
    U8 = ("u8", 1)

    @property
    def size_bytes(self) -> int:
        return self.value[1]

    @property
    def alignment_bytes(self) -> int:
        return self.value[1]


class QuantFormat(enum.Enum):
    """crates/mote-types/src/lib.rs:39-74 (ggml-common.h block ABI)."""

    Q8_0 = ("q8_0", 32, 34, 2)
    Q4_0 = ("q4_0", 32, 18, 2)
    Q4_K = ("q4_k", 256, 144, 4)
    Q6_K = ("q6_k", 256, 210, 2)

    @property
    def block_elements(self) -> int:
        return self.value[1]

    @property
    def block_bytes(self) -> int:
        return self.value[2]

    @property
    def alignment_bytes(self) -> int:
        return self.value[3]


@dataclass(frozen=True)
class Encoding:
    """``Encoding::Plain(DType)`` or ``Encoding::Quantized(QuantFormat)``."""

    plain: DType | None = None
    quantized: QuantFormat | None = None

    @staticmethod
    def Plain(dtype: DType) -> "Encoding":
        return Encoding(plain=dtype)

    @staticmethod
    def Quantized(fmt: QuantFormat) -> "Encoding":
        return Encoding(quantized=fmt)

    def __repr__(self) -> str:
        return f"Plain({self.plain.name})" if self.plain else f"Quantized({self.quantized.name})"


class RopeLayout(enum.Enum):
    """crates/mote-types/src/lib.rs:82-89; values are the ABI selectors."""

    HalfSplit = 0
    Interleaved = 1


class TensorDescError(ValueError):
    pass


@dataclass(frozen=True)
class Layout:
    """``Layout::Contiguous`` (strides None) or ``Layout::Strided``."""

    strides: tuple[int, ...] | None = None

    @staticmethod
    def contiguous() -> "Layout":
        return Layout(None)


@dataclass(frozen=True)
class TensorDesc:
    # Immutable, so the derived figures below are computed once per
    # descriptor (cached in the instance dictionary, outside the fields that
    # equality and hashing compare).
    shape: tuple[int, ...]
    encoding: Encoding
    layout: Layout = field(default_factory=Layout.contiguous)

    def __post_init__(self):
        object.__setattr__(self, "shape", tuple(int(d) for d in self.shape))
        if self.encoding.quantized is not None:
            fmt = self.encoding.quantized
            if self.layout.strides is not None:
                raise TensorDescError("UnsupportedQuantizedStrides")
            if not self.shape:
                raise TensorDescError(f"QuantizedScalarShape {fmt}")
            if self.shape[-1] % fmt.block_elements:
                raise TensorDescError(
                    f"QuantizedRowMisaligned {fmt} {self.shape[-1]} {fmt.block_elements}")
        if self.layout.strides is not None and len(self.layout.strides) != len(self.shape):
            raise TensorDescError("RankMismatch")

    @cached_property
    def rank(self) -> int:
        return len(self.shape)

    @cached_property
    def numel(self) -> int:
        return math.prod(self.shape)

    @cached_property
    def is_contiguous(self) -> bool:
        if self.layout.strides is None or 0 in self.shape:
            return True
        expected = 1
        for dim, stride in zip(reversed(self.shape), reversed(self.layout.strides)):
            if dim != 1 and stride != expected:
                return False
            expected *= dim
        return True

    @cached_property
    def required_span_bytes(self) -> int:
        """tensor_desc.rs:59-101: plain = span * size; quantized = rows * blocks * bytes."""
        if self.encoding.quantized is not None:
            fmt = self.encoding.quantized
            if self.numel == 0:
                return 0
            rows = self.numel // self.shape[-1]
            return rows * (self.shape[-1] // fmt.block_elements) * fmt.block_bytes
        if self.numel == 0:
            return 0
        if self.layout.strides is None:
            span = self.numel
        else:
            span = 1 + sum((d - 1) * s for d, s in zip(self.shape, self.layout.strides))
        return span * self.encoding.plain.size_bytes

    @cached_property
    def required_alignment(self) -> int:
        if self.encoding.quantized is not None:
            return self.encoding.quantized.alignment_bytes
        return self.encoding.plain.alignment_bytes


def plain(shape, dtype: DType) -> TensorDesc:
    return TensorDesc(tuple(shape), Encoding.Plain(dtype))


def quantized(shape, fmt: QuantFormat = QuantFormat.Q4_0) -> TensorDesc:
    return TensorDesc(tuple(shape), Encoding.Quantized(fmt))
