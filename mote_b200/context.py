"""Device context, storage and tensors of the CUDA backend.

Mirrors ``HipContext`` / ``HipStorage`` (crates/mote-backend-hip/src/
context.rs:13-206, storage.rs:8-96) and ``mote_core::Tensor``
(crates/mote-core/src/tensor.rs:5-117): a context owns one stream on one
device plus every allocation made through it; tensors are a descriptor, a
shared storage handle and a byte offset; the typed ops accept only
contiguous, zero-offset tensors whose storage belongs to the context they
are given.
"""
from __future__ import annotations

import ctypes
import itertools
import threading
from dataclasses import dataclass

import numpy as np

from . import errors
from ._native import lib
from .types import TensorDesc

STORAGE_ALIGNMENT = 256  # cudaMalloc guarantees 256-byte alignment (storage.rs:89-91)


@dataclass(frozen=True)
class Device:
    """``mote_types::Device`` (crates/mote-types/src/device.rs:9-31)."""

    backend: str
    ordinal: int


@dataclass(frozen=True)
class MemoryInfo:
    free_bytes: int
    total_bytes: int


class _ContextInner:
    def __init__(self, ordinal: int):
        self.ordinal = ordinal
        self.device = Device("cuda", ordinal)
        stream = ctypes.c_void_p()
        errors.check(lib().mote_cuda_set_device(ordinal), "select device")
        errors.check(lib().mote_cuda_stream_create(ctypes.byref(stream)), "create stream")
        self.stream = stream.value
        self.copy_stream = None  # created by the first overlapped download
        self.copy_event = None
        self._lock = threading.Lock()

    def select(self) -> None:
        errors.check(lib().mote_cuda_set_device(self.ordinal), "select device")

    def copy_channel(self) -> tuple[int, int]:
        """The copy stream and the event that orders it after the compute
        stream, created on first use."""
        if self.copy_stream is None:
            self.select()
            stream, event = ctypes.c_void_p(), ctypes.c_void_p()
            errors.check(lib().mote_cuda_stream_create(ctypes.byref(stream)),
                         "create copy stream")
            errors.check(lib().mote_cuda_event_create(ctypes.byref(event)), "create event")
            self.copy_stream, self.copy_event = stream.value, event.value
        return self.copy_stream, self.copy_event

    def close(self) -> None:
        if self.copy_stream:
            lib().mote_cuda_set_device(self.ordinal)
            lib().mote_cuda_stream_synchronize(self.copy_stream)
            lib().mote_cuda_event_destroy(self.copy_event)
            lib().mote_cuda_stream_destroy(self.copy_stream)
            self.copy_stream = self.copy_event = None
        if self.stream:
            lib().mote_cuda_set_device(self.ordinal)
            lib().mote_cuda_stream_synchronize(self.stream)
            state = getattr(self, "blas_state", None)
            if state is not None:
                lib().mote_cuda_blaslt_destroy(state[0])
                self.blas_state = None
            lib().mote_cuda_stream_destroy(self.stream)
            self.stream = None

    def __del__(self):  # pragma: no cover - best effort at interpreter exit
        try:
            self.close()
        except Exception:
            pass


_storage_ids = itertools.count(1)


class CudaStorage:
    """One device allocation owned by a context (``HipStorage``)."""

    def __init__(self, context: "_ContextInner", size_bytes: int, initial: bytes | None = None):
        self.context = context
        self.size_bytes = int(size_bytes)
        self.id = next(_storage_ids)
        self.alignment = STORAGE_ALIGNMENT
        context.select()
        ptr = ctypes.c_void_p()
        errors.check(lib().mote_cuda_malloc(ctypes.byref(ptr), max(self.size_bytes, 1)),
                     "allocate device storage")
        self.pointer = ptr.value
        if initial is not None and len(initial):
            buf = np.frombuffer(initial, np.uint8) if not isinstance(initial, np.ndarray) \
                else np.ascontiguousarray(initial).view(np.uint8).reshape(-1)
            st = lib().mote_cuda_memcpy_host_to_device(self.pointer, buf.ctypes.data, buf.nbytes)
            if st != 0:
                lib().mote_cuda_free(self.pointer)
                self.pointer = None
                errors.check(st, "upload device storage")

    def read_bytes(self) -> bytes:
        if self.size_bytes == 0:
            return b""
        self.context.select()
        errors.check(lib().mote_cuda_stream_synchronize(self.context.stream),
                     "synchronize before readback")
        out = np.empty(self.size_bytes, np.uint8)
        errors.check(lib().mote_cuda_memcpy_device_to_host(out.ctypes.data, self.pointer,
                                                           self.size_bytes), "read device storage")
        return out.tobytes()

    def __del__(self):  # pragma: no cover
        try:
            if self.pointer:
                lib().mote_cuda_set_device(self.context.ordinal)
                lib().mote_cuda_free(self.pointer)
                self.pointer = None
        except Exception:
            pass


class TensorError(ValueError):
    pass


class Tensor:
    """``mote_core::Tensor``: descriptor + shared storage + byte offset."""

    def __init__(self, desc: TensorDesc, storage: CudaStorage, byte_offset: int = 0):
        span = desc.required_span_bytes
        if byte_offset > storage.size_bytes:
            raise TensorError(f"OffsetOutOfBounds {byte_offset} > {storage.size_bytes}")
        if byte_offset + span > storage.size_bytes:
            raise TensorError(f"StorageTooSmall [{byte_offset}, {byte_offset + span}) > "
                              f"{storage.size_bytes}")
        if span and (storage.alignment < desc.required_alignment or
                     byte_offset % desc.required_alignment):
            raise TensorError("Misaligned")
        self.desc = desc
        self.storage = storage
        self.byte_offset = int(byte_offset)

    @property
    def device(self) -> Device:
        return self.storage.context.device

    @property
    def shape(self) -> tuple[int, ...]:
        return self.desc.shape

    @property
    def pointer(self) -> int:
        return self.storage.pointer + self.byte_offset

    def shares_storage_with(self, other: "Tensor") -> bool:
        return self.storage is other.storage

    def __repr__(self) -> str:
        return f"Tensor({self.desc.shape}, {self.desc.encoding!r}, storage={self.storage.id})"


class CudaContext:
    """``HipContext``: one device, one stream, owned allocations."""

    def __init__(self, ordinal: int = 0):
        if ordinal < 0 or ordinal > 0x7FFFFFFF:
            raise errors.DeviceOrdinalTooLarge(ordinal=ordinal)
        count = ctypes.c_int(0)
        errors.check(lib().mote_cuda_get_device_count(ctypes.byref(count)), "enumerate devices")
        if ordinal >= count.value:
            raise errors.DeviceUnavailable(ordinal=ordinal, available=count.value)
        self.inner = _ContextInner(ordinal)

    # -- identity ---------------------------------------------------------
    @property
    def device(self) -> Device:
        return self.inner.device

    @property
    def stream(self) -> int:
        """The raw cudaStream_t handle every op of this context runs on."""
        return self.inner.stream

    # -- allocation -------------------------------------------------------
    def _validate_desc(self, desc: TensorDesc) -> None:
        if not desc.is_contiguous:
            raise errors.UnsupportedLayout(actual=desc.layout)

    def empty(self, desc: TensorDesc) -> Tensor:
        self._validate_desc(desc)
        return Tensor(desc, CudaStorage(self.inner, desc.required_span_bytes), 0)

    def from_bytes(self, desc: TensorDesc, data) -> Tensor:
        self._validate_desc(desc)
        buf = np.ascontiguousarray(data).view(np.uint8).reshape(-1) \
            if isinstance(data, np.ndarray) else np.frombuffer(bytes(data), np.uint8)
        expected = desc.required_span_bytes
        if buf.nbytes != expected:
            raise errors.ByteLengthMismatch(expected=expected, actual=buf.nbytes)
        return Tensor(desc, CudaStorage(self.inner, expected, buf), 0)

    def from_numpy(self, desc: TensorDesc, array: np.ndarray) -> Tensor:
        return self.from_bytes(desc, np.ascontiguousarray(array))

    def upload_numpy(self, tensor: Tensor, array: np.ndarray) -> None:
        """Synchronous host-to-device copy into an existing tensor."""
        buf = np.ascontiguousarray(array).view(np.uint8).reshape(-1)
        if buf.nbytes != tensor.desc.required_span_bytes:
            raise errors.ByteLengthMismatch(expected=tensor.desc.required_span_bytes,
                                            actual=buf.nbytes)
        self.sync()
        errors.check(lib().mote_cuda_memcpy_host_to_device(tensor.pointer, buf.ctypes.data,
                                                           buf.nbytes), "upload")

    # the dense-matmul library context and its workspace (context.rs:11, 42:
    # 32 MiB, as the HIP backend), made on first use
    BLAS_WORKSPACE_BYTES = 32 * 1024 * 1024

    def blas(self) -> tuple[int, int, int]:
        """(cuBLASLt context, workspace pointer, workspace bytes)."""
        state = getattr(self.inner, "blas_state", None)
        if state is None:
            self.inner.select()
            handle = ctypes.c_void_p()
            st = lib().mote_cuda_blaslt_create(ctypes.byref(handle))
            if st != 0:
                raise errors.BlasLt(operation="create", status=int(st),
                                    message="cuBLASLt could not be started")
            ws = CudaStorage(self.inner, self.BLAS_WORKSPACE_BYTES)
            state = self.inner.blas_state = (handle.value, ws)
        return state[0], state[1].pointer, state[1].size_bytes

    def linear_workspace_bytes(self, rows: int, n: int, k: int) -> int:
        """mote_cuda_q4_0_linear_workspace_bytes for a shape, memoised (it
        depends only on the shape and this context's device)."""
        cache = self.__dict__.setdefault("_ws_need", {})
        key = (rows, n, k)
        need = cache.get(key)
        if need is None:
            out = ctypes.c_uint64(0)
            errors.check(lib().mote_cuda_q4_0_linear_workspace_bytes(rows, n, k,
                                                                     ctypes.byref(out)),
                         "query linear workspace")
            need = cache[key] = out.value
        return need

    def linear_workspace(self, nbytes: int) -> tuple[int, int]:
        """A zeroed device workspace of at least ``nbytes`` owned by this
        context (for the split-K linear), grown on demand.  The kernels leave
        it zeroed; growing synchronizes the stream, so the first call of a
        new, larger shape must come before any CUDA-graph capture."""
        ws = getattr(self, "_workspace", None)
        if ws is None or ws.size_bytes < nbytes:
            self.sync()
            size = max(int(nbytes), 1 << 20)
            ws = CudaStorage(self.inner, size, np.zeros(size, np.uint8))
            self._workspace = ws
        return ws.pointer, ws.size_bytes

    def attention_workspace(self, nbytes: int) -> tuple[int, int]:
        """A device workspace of at least ``nbytes`` for the attention
        kernels' split partials (contents need no initialisation; separate
        from the linear's zeroed workspace), grown on demand with a stream
        synchronisation."""
        ws = getattr(self, "_attn_workspace", None)
        if ws is None or ws.size_bytes < nbytes:
            self.sync()
            ws = CudaStorage(self.inner, max(int(nbytes), 1 << 20))
            self._attn_workspace = ws
        return ws.pointer, ws.size_bytes

    def read_bytes(self, tensor: Tensor) -> bytes:
        storage = self.storage(tensor)
        return storage.read_bytes()[: tensor.desc.required_span_bytes]

    def read_numpy(self, tensor: Tensor, dtype) -> np.ndarray:
        return np.frombuffer(self.read_bytes(tensor), dtype=dtype).reshape(tensor.shape) \
            if tensor.desc.encoding.plain is not None else np.frombuffer(self.read_bytes(tensor),
                                                                          np.uint8)

    def sync(self) -> None:
        """Waits for the compute stream and, if overlapped downloads were
        issued, the copy stream."""
        self.inner.select()
        errors.check(lib().mote_cuda_stream_synchronize(self.stream), "synchronize stream")
        if self.inner.copy_stream is not None:
            errors.check(lib().mote_cuda_stream_synchronize(self.inner.copy_stream),
                         "synchronize copy stream")

    def memory_info(self) -> MemoryInfo:
        self.inner.select()
        free, total = ctypes.c_size_t(), ctypes.c_size_t()
        errors.check(lib().mote_cuda_mem_get_info(ctypes.byref(free), ctypes.byref(total)),
                     "query device memory info")
        return MemoryInfo(free.value, total.value)

    def device_status(self, clear: bool = True) -> int:
        """Reads the device status word (bounded-wait timeouts, bad indices)."""
        self.inner.select()
        st = ctypes.c_uint(0)
        errors.check(lib().mote_cuda_device_status(ctypes.byref(st), int(clear)),
                     "read device status")
        return st.value

    # -- host transfers on the context stream -----------------------------
    def upload_async(self, tensor: Tensor, host: "PinnedBuffer", nbytes: int | None = None):
        n = tensor.desc.required_span_bytes if nbytes is None else nbytes
        errors.check(lib().mote_cuda_memcpy_host_to_device_async(
            tensor.pointer, host.pointer, n, self.stream), "upload (async)")

    def download_async(self, host: "PinnedBuffer", tensor: Tensor, nbytes: int | None = None):
        n = tensor.desc.required_span_bytes if nbytes is None else nbytes
        errors.check(lib().mote_cuda_memcpy_device_to_host_async(
            host.pointer, tensor.pointer, n, self.stream), "download (async)")

    def download_overlapped(self, host: "PinnedBuffer", tensor: Tensor,
                            nbytes: int | None = None):
        """Device-to-host copy on the context's copy stream, ordered after
        everything issued so far on the compute stream, so the kernels issued
        after it run while it copies.  ``tensor`` must not be written again,
        nor ``host`` read, before ``sync()`` (which waits for both streams)."""
        n = tensor.desc.required_span_bytes if nbytes is None else nbytes
        copy_stream, event = self.inner.copy_channel()
        errors.check(lib().mote_cuda_event_record(event, self.stream), "record event")
        errors.check(lib().mote_cuda_stream_wait_event(copy_stream, event), "order copy stream")
        errors.check(lib().mote_cuda_memcpy_device_to_host_async(
            host.pointer, tensor.pointer, n, copy_stream), "download (overlapped)")

    # -- ownership check used by every op (context.rs:150-176) --------------
    def storage(self, tensor: Tensor) -> CudaStorage:
        st = tensor.storage
        if (st.__class__ is CudaStorage and st.context is self.inner and tensor.byte_offset == 0
                and tensor.desc.is_contiguous):
            return st  # every check below passes (same context implies same device)
        if tensor.device != self.device:
            raise errors.DeviceMismatch(expected=self.device, actual=tensor.device)
        if tensor.byte_offset != 0:
            raise errors.UnsupportedByteOffset(byte_offset=tensor.byte_offset)
        if not tensor.desc.is_contiguous:
            raise errors.UnsupportedLayout(actual=tensor.desc.layout)
        if not isinstance(tensor.storage, CudaStorage) or tensor.storage.context is not self.inner:
            raise errors.WrongStorage()
        return tensor.storage


class PinnedBuffer:
    """Page-locked host memory (cudaHostAlloc) viewed as a numpy array."""

    def __init__(self, nbytes: int):
        ptr = ctypes.c_void_p()
        errors.check(lib().mote_cuda_host_alloc(ctypes.byref(ptr), max(int(nbytes), 1)),
                     "allocate pinned host memory")
        self.pointer = ptr.value
        self.nbytes = int(nbytes)
        raw = (ctypes.c_uint8 * max(self.nbytes, 1)).from_address(self.pointer)
        self.array = np.frombuffer(raw, np.uint8)[: self.nbytes]

    def view(self, dtype) -> np.ndarray:
        return self.array.view(dtype)

    def __del__(self):  # pragma: no cover
        try:
            if self.pointer:
                lib().mote_cuda_host_free(self.pointer)
                self.pointer = None
        except Exception:
            pass
