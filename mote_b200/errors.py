"""Error taxonomy mirroring ``HipError`` (crates/mote-backend-hip/src/error.rs:6-131).

Each variant is a subclass of :class:`CudaError` carrying the variant's
fields as attributes, so callers can match on the class the way the Rust
tests match on the enum variant.
"""
from __future__ import annotations


class CudaError(Exception):
    """Base class; ``fields`` holds the variant's named fields."""

    def __init__(self, **fields):
        self.fields = fields
        for k, v in fields.items():
            setattr(self, k, v)
        super().__init__(f"{type(self).__name__}({', '.join(f'{k}={v!r}' for k, v in fields.items())})")


class Runtime(CudaError):
    """A CUDA runtime call or kernel launch returned a non-zero status."""


class DeviceUnavailable(CudaError):
    pass


class DeviceOrdinalTooLarge(CudaError):
    pass


class ByteLengthMismatch(CudaError):
    pass


class UnsupportedEncoding(CudaError):
    pass


class UnsupportedLayout(CudaError):
    pass


class DeviceMismatch(CudaError):
    pass


class UnsupportedByteOffset(CudaError):
    pass


class WrongStorage(CudaError):
    pass


class AliasedStorage(CudaError):
    pass


class DTypeMismatch(CudaError):
    pass


class ShapeMismatch(CudaError):
    pass


class RankMismatch(CudaError):
    pass


class RankTooSmall(CudaError):
    pass


class QuantizedLinearDimensionsTooLarge(CudaError):
    pass


class RmsNormDimensionsTooLarge(CudaError):
    pass


class FusedAddRmsNormDimensionsTooLarge(CudaError):
    pass


class RopeDimensionsTooLarge(CudaError):
    pass


class InvalidRotaryDim(CudaError):
    pass


class InvalidEpsilon(CudaError):
    pass


class BlasLt(CudaError):
    """``HipError::BlasLt`` (error.rs:14-19): the dense-matmul library call
    failed; ``message`` is the context's last-error text."""


class MatmulDimensionsTooLarge(CudaError):
    """``HipError::MatmulDimensionsTooLarge`` (error.rs:79-80)."""


class IndexOutOfRange(CudaError):
    """An embedding id was outside [0, vocab) (no reference counterpart)."""


class DeviceWaitTimeout(CudaError):
    """A bounded device-side wait expired (no reference counterpart)."""


def check(status: int, operation: str) -> None:
    """``check_hip`` (error.rs:125-131): non-zero status -> Runtime error."""
    if status != 0:
        from ._native import status_string

        raise Runtime(operation=operation, status=int(status), message=status_string(status))
