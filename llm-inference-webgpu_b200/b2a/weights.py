"""Safetensors checkpoints over libb2a.so: the host mirror of Safetensors
(src/core/safetensors.js:23-199). Opening validates the header against the
file with the reference's checks and messages; tensors are read on demand.
A checkpoint loads into a device model with `Model.load_safetensors`.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from . import _lib
from ._lib import check, load


class TensorInfo:
    """TensorInfo (safetensors.js:23-34): name, dtype, shape, byteLength, numel."""

    def __init__(self, name: str, dtype: str, shape: tuple, byte_length: int):
        self.name, self.dtype, self.shape, self.byteLength = name, dtype, shape, byte_length

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


class Safetensors:
    """Safetensors.open(source) (safetensors.js:56-123): `Safetensors.open(path)` reads a
    file, `Safetensors.fromBytes(data)` a memory image. Errors raise b2a.B2AError with the
    reference's messages."""

    def __init__(self, handle):
        self._lib = load()
        self.handle = handle

    @classmethod
    def open(cls, path: str) -> "Safetensors":
        h = ctypes.c_void_p()
        check(load().b2a_safetensors_open(str(path).encode(), ctypes.byref(h)))
        return cls(h)

    @classmethod
    def fromBytes(cls, data) -> "Safetensors":
        buf = bytes(data)
        h = ctypes.c_void_p()
        check(load().b2a_safetensors_open_memory(buf, len(buf), ctypes.byref(h)))
        return cls(h)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.b2a_safetensors_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def size(self) -> int:
        return self._lib.b2a_safetensors_count(self.handle)

    def names(self) -> list:
        return [self._lib.b2a_safetensors_name(self.handle, i).decode() for i in range(self.size)]

    def has(self, name: str) -> bool:
        return name in self.names()

    @property
    def metadata(self):
        m = self._lib.b2a_safetensors_metadata(self.handle)
        return None if m is None else json.loads(m.decode())

    def info(self, name: str) -> TensorInfo:
        dt = ctypes.create_string_buffer(16)
        shape = (ctypes.c_int64 * 16)()
        nd = ctypes.c_int()
        nb = ctypes.c_int64()
        check(self._lib.b2a_safetensors_info(self.handle, name.encode(), dt, shape, 16, ctypes.byref(nd),
                                             ctypes.byref(nb)))
        return TensorInfo(name, dt.value.decode(), tuple(shape[i] for i in range(nd.value)), nb.value)

    def readRaw(self, name: str) -> bytes:
        t = self.info(name)
        out = ctypes.create_string_buffer(max(1, t.byteLength))
        check(self._lib.b2a_safetensors_read_raw(self.handle, name.encode(), out, t.byteLength))
        return out.raw[:t.byteLength]

    def readF32(self, name: str) -> np.ndarray:
        t = self.info(name)
        out = np.empty(t.numel, np.float32)
        check(self._lib.b2a_safetensors_read_f32(self.handle, name.encode(), out.ctypes.data if out.size else None,
                                                 out.size))
        return out.reshape(t.shape)


def write_safetensors(tensors: dict, metadata: dict | None = None) -> bytes:
    """A safetensors image of {name: numpy array} (for tests and tools): u64 header length,
    the JSON header, then the tensors back to back in the given order."""
    dt = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.float64): "F64",
          np.dtype(np.int8): "I8", np.dtype(np.uint8): "U8", np.dtype(np.int32): "I32"}
    header, blobs, at = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (arr, dtype) in ((k, v if isinstance(v, tuple) else (v, None)) for k, v in tensors.items()):
        a = np.ascontiguousarray(arr)
        kind = dtype or dt[a.dtype]
        raw = a.tobytes()
        header[name] = {"dtype": kind, "shape": list(a.shape), "data_offsets": [at, at + len(raw)]}
        blobs.append(raw)
        at += len(raw)
    text = json.dumps(header).encode()
    return len(text).to_bytes(8, "little") + text + b"".join(blobs)
