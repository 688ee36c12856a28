"""GGUF weight files: a memory-mapped reader and the upload of its tensors to
device storage, for the encodings this data plane runs.

GGUF is the file format of llama.cpp / ggml, and the on-disk format Mote's
roadmap names next (docs/roadmap.md:26-27, 88-90).  Versions 2 and 3,
little-endian:

* header: magic ``GGUF``, u32 version, u64 tensor count, u64 metadata count;
* metadata: key (u64 byte length + UTF-8), u32 value type, value -- scalars
  of 1, 2, 4 or 8 bytes, bool, string, or an array (u32 element type, u64
  count, elements; arrays may nest);
* tensor infos: name, u32 dimension count, u64 ``ne`` per dimension
  (``ne[0]`` is the row length, the innermost axis), u32 ggml type, u64
  offset into the data section;
* the data section starts at the first multiple of ``general.alignment``
  (default 32) after the infos; every tensor starts at an aligned offset.

The file is mapped read-only; a tensor's bytes stay a view of the mapping
until :func:`load_tensor` copies them to the device.  Shapes are reported
outermost first (numpy order), so a ggml ``[K, N]`` weight is ``(N, K)`` --
the ``[output_features, input_features]`` shape the linear ops take.
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .types import DType, QuantFormat, TensorDesc, plain, quantized

MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32
MAX_DIMS = 4

# metadata value types
_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 10: "<Q", 11: "<q",
            12: "<d"}
_BOOL, _STRING, _ARRAY = 7, 8, 9

# ggml tensor types: name, elements per block, bytes per block
GGML_TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20),
    6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144),
    13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292),
    24: ("I8", 1, 1), 25: ("I16", 1, 2), 26: ("I32", 1, 4), 27: ("I64", 1, 8),
    28: ("F64", 1, 8), 30: ("BF16", 1, 2),
}

# the ggml types that map onto an encoding the ops take
_ENCODINGS = {
    0: ("plain", DType.F32), 1: ("plain", DType.F16), 30: ("plain", DType.BF16),
    2: ("quantized", QuantFormat.Q4_0), 8: ("quantized", QuantFormat.Q8_0),
    12: ("quantized", QuantFormat.Q4_K), 14: ("quantized", QuantFormat.Q6_K),
}


class GGUFError(ValueError):
    """A file that is not GGUF, is truncated, or holds an inconsistent tensor."""


@dataclass(frozen=True)
class GGUFTensorInfo:
    name: str
    shape: tuple[int, ...]   # outermost first; shape[-1] is ggml's ne[0]
    ggml_type: int
    offset: int              # absolute byte offset in the file
    nbytes: int | None       # None for ggml types this reader has no size for

    @property
    def type_name(self) -> str:
        return GGML_TYPES.get(self.ggml_type, (f"type{self.ggml_type}",))[0]


class _Cursor:
    def __init__(self, buf, size: int):
        self.buf = buf
        self.size = size
        self.pos = 0

    def take(self, n: int) -> bytes:
        if n < 0 or self.pos + n > self.size:
            raise GGUFError(f"truncated file: {n} bytes wanted at offset {self.pos} of {self.size}")
        out = self.buf[self.pos:self.pos + n]
        self.pos += n
        return bytes(out)

    def unpack(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        return self.take(self.unpack("<Q")).decode("utf-8", errors="replace")

    def value(self, vtype: int, depth: int = 0):
        if vtype in _SCALARS:
            return self.unpack(_SCALARS[vtype])
        if vtype == _BOOL:
            return self.take(1) != b"\x00"
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            if depth > 8:
                raise GGUFError("metadata arrays nested too deeply")
            etype = self.unpack("<I")
            count = self.unpack("<Q")
            if etype in _SCALARS and count:
                width = struct.calcsize(_SCALARS[etype])
                raw = self.take(width * count)
                return np.frombuffer(raw, np.dtype(_SCALARS[etype])).tolist()
            if count > self.size:
                raise GGUFError(f"array of {count} elements in a {self.size}-byte file")
            return [self.value(etype, depth + 1) for _ in range(count)]
        raise GGUFError(f"unknown metadata value type {vtype} at offset {self.pos}")


class GGUFFile:
    """A GGUF file mapped read-only.

    ``metadata`` maps keys to Python values; ``tensors`` maps names to
    :class:`GGUFTensorInfo` in file order.  Use as a context manager or call
    :meth:`close`; views from :meth:`tensor_bytes` must not outlive it."""

    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        self._file = open(self.path, "rb")
        size = os.fstat(self._file.fileno()).st_size
        if size < 24:
            self._file.close()
            raise GGUFError(f"{self.path}: {size} bytes is too short for a GGUF header")
        self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            self._parse(size)
        except Exception:
            self.close()
            raise

    def _parse(self, size: int) -> None:
        cur = _Cursor(self._map, size)
        if cur.take(4) != MAGIC:
            raise GGUFError(f"{self.path}: not a GGUF file (bad magic)")
        self.version = cur.unpack("<I")
        if self.version not in (2, 3):
            raise GGUFError(f"{self.path}: GGUF version {self.version} is not supported")
        n_tensors = cur.unpack("<Q")
        n_kv = cur.unpack("<Q")
        if n_tensors > size or n_kv > size:
            raise GGUFError(f"{self.path}: counts exceed the file size")
        self.metadata: dict[str, object] = {}
        for _ in range(n_kv):
            key = cur.string()
            self.metadata[key] = cur.value(cur.unpack("<I"))
        self.alignment = int(self.metadata.get("general.alignment", DEFAULT_ALIGNMENT))
        if self.alignment <= 0 or self.alignment & (self.alignment - 1):
            raise GGUFError(f"general.alignment {self.alignment} is not a power of two")
        raw = []
        for _ in range(n_tensors):
            name = cur.string()
            n_dims = cur.unpack("<I")
            if n_dims == 0 or n_dims > MAX_DIMS:
                raise GGUFError(f"tensor {name!r}: {n_dims} dimensions")
            ne = [cur.unpack("<Q") for _ in range(n_dims)]
            raw.append((name, ne, cur.unpack("<I"), cur.unpack("<Q")))
        self.data_offset = -(-cur.pos // self.alignment) * self.alignment
        self.tensors: dict[str, GGUFTensorInfo] = {}
        for name, ne, gtype, rel in raw:
            if name in self.tensors:
                raise GGUFError(f"tensor {name!r} appears twice")
            if rel % self.alignment:
                raise GGUFError(f"tensor {name!r}: offset {rel} is not aligned to "
                                f"{self.alignment}")
            nbytes = None
            if gtype in GGML_TYPES:
                _, be, bb = GGML_TYPES[gtype]
                if ne[0] % be:
                    raise GGUFError(f"tensor {name!r}: row length {ne[0]} is not a multiple "
                                    f"of the {be}-element block")
                count = 1
                for d in ne:
                    count *= d
                nbytes = count // be * bb
                if self.data_offset + rel + nbytes > size:
                    raise GGUFError(f"tensor {name!r}: data runs past the end of the file")
            self.tensors[name] = GGUFTensorInfo(name, tuple(reversed(ne)), gtype,
                                                self.data_offset + rel, nbytes)

    # -- access ---------------------------------------------------------------
    def tensor_bytes(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the mapping."""
        info = self._info(name)
        if info.nbytes is None:
            raise GGUFError(f"tensor {name!r}: ggml type {info.ggml_type} has no known size")
        return np.frombuffer(self._map, np.uint8, info.nbytes, info.offset)

    def descriptor(self, name: str) -> TensorDesc:
        """The data-plane descriptor of a tensor (outermost-first shape)."""
        info = self._info(name)
        enc = _ENCODINGS.get(info.ggml_type)
        if enc is None:
            raise GGUFError(f"tensor {name!r}: ggml type {info.type_name} has no encoding here "
                            f"(F32, F16, BF16, Q4_0, Q8_0, Q4_K, Q6_K)")
        kind, what = enc
        return plain(info.shape, what) if kind == "plain" else quantized(info.shape, what)

    def _info(self, name: str) -> GGUFTensorInfo:
        try:
            return self.tensors[name]
        except KeyError:
            raise GGUFError(f"no tensor {name!r} in {self.path}") from None

    def close(self) -> None:
        m, self._map = getattr(self, "_map", None), None
        if m is not None:
            try:
                m.close()
            except BufferError:  # a view is still alive; the mapping goes with it
                pass
        f = getattr(self, "_file", None)
        if f is not None:
            f.close()

    def __enter__(self) -> "GGUFFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def load_tensor(context, gguf: GGUFFile, name: str):
    """Copies one tensor from the mapping into a new device tensor of
    ``context`` (the descriptor from :meth:`GGUFFile.descriptor`)."""
    desc = gguf.descriptor(name)
    return context.from_bytes(desc, gguf.tensor_bytes(name))


def load_tensors(context, gguf: GGUFFile, names=None) -> dict:
    """Loads every tensor with an encoding here (or ``names``) to the device."""
    if names is None:
        names = [n for n, t in gguf.tensors.items() if t.ggml_type in _ENCODINGS]
    return {n: load_tensor(context, gguf, n) for n in names}
