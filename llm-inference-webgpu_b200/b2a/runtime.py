"""Host-side objects over libb2a.so: the device context, the f64 RoPE table and
the device KV cache, mirroring the reference's GpuContext / ropeTable /
GpuKVCache (src/gpu/device.js:21, src/gpu/model.js:69-84,200-205) and KVCache
(src/cpu/cache.js:18-119).

Arrays may be numpy arrays (host memory: the call stages them to the device and
returns when the results are back) or torch CUDA tensors (device memory: the
call only enqueues work on the context's stream). All arrays of one call must
live on the same side.
"""
from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import B2A_DEVICE, B2A_HOST, DTYPES, DTYPE_SIZE, EXCHANGE_HANDLE_BYTES, check, load

try:  # torch is optional: only needed for device-pointer calls
    import torch
except Exception:  # pragma: no cover
    torch = None

_TORCH_DT = {}
if torch is not None:
    _TORCH_DT = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}
_NP_DT = {np.dtype(np.float32): "f32", np.dtype(np.float16): "f16"}


@dataclass
class _Arg:
    ptr: int
    where: int          # B2A_HOST | B2A_DEVICE
    dtype: str | None   # "f32" | "f16" | "bf16" | None (raw uint16 bits, dtype given by caller)
    nbytes: int
    keep: object


def _arg(x, dtype: str | None = None, writable: bool = False) -> _Arg | None:
    if x is None:
        return None
    if torch is not None and isinstance(x, torch.Tensor):
        if not x.is_contiguous():
            raise ValueError("tensor arguments must be contiguous")
        dt = _TORCH_DT.get(x.dtype)
        if dt is None and x.dtype in (torch.int16, torch.uint16):
            dt = dtype
        if dt is None:
            raise ValueError(f"unsupported tensor dtype {x.dtype}")
        return _Arg(x.data_ptr(), B2A_DEVICE if x.is_cuda else B2A_HOST, dt, x.numel() * x.element_size(), x)
    a = x if isinstance(x, np.ndarray) else np.asarray(x, dtype=np.float32)
    if not a.flags["C_CONTIGUOUS"]:
        if writable:
            raise ValueError("output arrays must be C-contiguous")
        a = np.ascontiguousarray(a)
    if writable and not a.flags["WRITEABLE"]:
        raise ValueError("output array is read-only")
    dt = _NP_DT.get(a.dtype)
    if dt is None:
        if a.dtype == np.uint16 and dtype in ("f16", "bf16"):
            dt = dtype
        else:
            raise ValueError(f"unsupported array dtype {a.dtype} (give uint16 bits with dtype='bf16')")
    return _Arg(a.ctypes.data, B2A_HOST, dt, a.nbytes, a)


def _where(*args: _Arg | None) -> int:
    ws = {a.where for a in args if a is not None}
    if len(ws) > 1:
        raise ValueError("mix of host and device arrays in one call")
    return ws.pop() if ws else B2A_HOST


def _same_dtype(*args: _Arg | None) -> str:
    ds = {a.dtype for a in args if a is not None}
    if len(ds) != 1:
        raise ValueError(f"inputs must share one dtype, got {sorted(d for d in ds if d)}")
    return ds.pop()


class Context:
    """One device and one stream (GpuContext, src/gpu/device.js:21). Not re-entrant."""

    def __init__(self, device: int = 0):
        self._lib = load()
        h = ctypes.c_void_p()
        check(self._lib.b2a_init(device, ctypes.byref(h)))
        self.handle = h
        self.device = device
        self._children = weakref.WeakSet()   # caches and rope tables made on this context

    def close(self) -> None:
        """Free the context, after every cache and rope table made on it."""
        if getattr(self, "handle", None):
            for child in list(self._children):
                child.close()
            self._lib.b2a_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream) -> None:
        """Enqueue on an external stream (torch.cuda.Stream, a raw handle, or None for our own)."""
        if stream is None:
            ptr = None
        elif isinstance(stream, int):
            ptr = stream
        else:
            ptr = stream.cuda_stream
        check(self._lib.b2a_set_stream(self.handle, ctypes.c_void_p(ptr)))

    def synchronize(self) -> None:
        check(self._lib.b2a_synchronize(self.handle))

    def enable_timing(self, on: bool = True) -> None:
        """Bracket every kernel launch with CUDA events (GpuContext.timed, src/gpu/device.js:301-338)."""
        check(self._lib.b2a_timing_enable(self.handle, 1 if on else 0))

    def read_timing(self) -> dict:
        """{kernel kind: (launches, total device ms)} since the last read; waits for the stream."""
        entries = (_KernelTime * 16)()
        n = ctypes.c_int()
        check(self._lib.b2a_timing_read(self.handle, entries, 16, ctypes.byref(n)))
        return {entries[i].name.decode(): (entries[i].launches, entries[i].total_ms) for i in range(n.value)}


class _KernelTime(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int), ("total_ms", ctypes.c_double)]


class RopeTable:
    """f64 cos/sin for positions 0..maxPositions-1 on the device (ropeTables, src/core/ops.js:123-136,
    kept in f64 so the rotation is the one ropeInPlace computes)."""

    def __init__(self, ctx: Context, headDim: int, theta: float, maxPositions: int):
        self.ctx = ctx
        h = ctypes.c_void_p()
        check(ctx._lib.b2a_rope_create(ctx.handle, headDim, float(theta), maxPositions, ctypes.byref(h)))
        self.handle = h
        self.headDim, self.theta, self.maxPositions = headDim, theta, maxPositions
        ctx._children.add(self)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.ctx._lib.b2a_rope_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class CacheConfig:
    """The ModelConfig fields the cache needs (src/core/config.js:67-72)."""
    numLayers: int
    numKVHeads: int
    headDim: int
    numHeads: int = 0

    @property
    def kvDim(self) -> int:
        return self.numKVHeads * self.headDim


class GpuKVCache:
    """Device KV cache for `batch` sequences (GpuKVCache src/gpu/model.js:69-84 with the
    KVCache bookkeeping of src/cpu/cache.js:18-119). Storage is head-major per
    sequence and layer, [kvHead][position][headDim] in `dtype`.

    With pageSize (a power of two >= 128) the cache is paged: the sequences share a
    pool of numPages pages of pageSize positions, taken as sequences grow and given
    back on reset (b2a_kvcache_create_paged); capacity stays the per-sequence bound.
    Every operation works on either layout."""

    def __init__(self, ctx: Context, config, capacity, batch: int = 1, dtype: str = "f32",
                 pageSize: int = 0, numPages: int = 0):
        if not isinstance(capacity, (int, np.integer)) or isinstance(capacity, bool):
            raise _lib.RangeError(_lib.B2A_ERANGE, f"cache capacity must be a positive integer, got {capacity}")
        self.ctx = ctx
        self.config = config
        self.capacity = int(capacity)
        self.batch = batch
        self.dtype = dtype
        self.pageSize = int(pageSize)
        self.numPages = int(numPages)
        h = ctypes.c_void_p()
        if self.pageSize:
            check(ctx._lib.b2a_kvcache_create_paged(ctx.handle, config.numLayers, config.numKVHeads, config.headDim,
                                                    self.capacity, batch, DTYPES[dtype], self.pageSize,
                                                    self.numPages, ctypes.byref(h)))
        else:
            check(ctx._lib.b2a_kvcache_create(ctx.handle, config.numLayers, config.numKVHeads, config.headDim,
                                              self.capacity, batch, DTYPES[dtype], ctypes.byref(h)))
        self.handle = h
        ctx._children.add(self)

    # -- pages (paged caches) --
    def pageTable(self, seq: int = 0) -> np.ndarray:
        """The pages backing sequence `seq`, in position order (empty when contiguous)."""
        n = ctypes.c_int()
        cap = (self.capacity + self.pageSize - 1) // self.pageSize if self.pageSize else 0
        out = np.zeros(max(cap, 1), np.int32)
        check(self.ctx._lib.b2a_kvcache_page_table(self.handle, seq, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                   out.size, ctypes.byref(n)))
        return out[:n.value].copy()

    @property
    def freePages(self) -> int:
        n = ctypes.c_int()
        check(self.ctx._lib.b2a_kvcache_free_pages(self.handle, ctypes.byref(n)))
        return n.value

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.ctx._lib.b2a_kvcache_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- bookkeeping (src/cpu/cache.js:37-60, 84-86, 118) --
    def lengthOf(self, seq: int = 0) -> int:
        n = ctypes.c_int()
        check(self.ctx._lib.b2a_kvcache_length(self.handle, seq, ctypes.byref(n)))
        return n.value

    @property
    def length(self) -> int:
        return self.lengthOf(0)

    @property
    def byteLength(self) -> int:
        n = ctypes.c_size_t()
        check(self.ctx._lib.b2a_kvcache_byte_length(self.handle, ctypes.byref(n)))
        return n.value

    def allocate(self, count: int, seq: int = 0) -> int:
        at = ctypes.c_int()
        check(self.ctx._lib.b2a_kvcache_allocate(self.handle, seq, count, ctypes.byref(at)))
        return at.value

    def commit(self, count: int, seq: int | None = 0) -> None:
        check(self.ctx._lib.b2a_kvcache_commit(self.handle, -1 if seq is None else seq, count))

    def setLengths(self, lengths) -> None:
        arr = np.ascontiguousarray(lengths, dtype=np.int32)
        if arr.size != self.batch:
            raise ValueError("one length per sequence")
        check(self.ctx._lib.b2a_kvcache_set_lengths(self.handle, arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))

    def reset(self, seq: int | None = None) -> None:
        check(self.ctx._lib.b2a_kvcache_reset(self.handle, -1 if seq is None else seq))

    def pools(self):
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        strides = (ctypes.c_int64 * 4)()
        check(self.ctx._lib.b2a_kvcache_pools(self.handle, ctypes.byref(k), ctypes.byref(v), strides))
        return k.value, v.value, tuple(strides)

    # -- data (src/cpu/cache.js:63-115) --
    def writeAt(self, layer: int, at: int, keys, values, count: int, seq: int = 0, dtype: str | None = None) -> None:
        k, v = _arg(keys, dtype), _arg(values, dtype)
        check(self.ctx._lib.b2a_kvcache_write_at(self.ctx.handle, self.handle, layer, seq, at, k.ptr, v.ptr,
                                                 DTYPES[_same_dtype(k, v)], count, _where(k, v)))

    def read(self, layer: int, n: int, seq: int = 0):
        """Raw head-major [numKVHeads, n, headDim] keys and values in the cache dtype
        (uint16 bits for f16/bf16)."""
        shape = (self.config.numKVHeads, n, self.config.headDim)
        npdt = np.float32 if self.dtype == "f32" else np.uint16
        k, v = np.empty(shape, npdt), np.empty(shape, npdt)
        check(self.ctx._lib.b2a_kvcache_read(self.ctx.handle, self.handle, layer, seq, n, k.ctypes.data,
                                             v.ctypes.data, B2A_HOST))
        return k, v

    def present(self, layer: int, seq: int = 0):
        """KVCache.present (src/cpu/cache.js:97-115): [numKVHeads, length, headDim]."""
        k, v = self.read(layer, self.lengthOf(seq), seq)
        return {"key": k, "value": v}

    def keysUpTo(self, layer: int, n: int, seq: int = 0) -> np.ndarray:
        """KVCache.keysUpTo (src/cpu/cache.js:75-77): position-major [n * kvDim]."""
        k, _ = self.read(layer, n, seq)
        return np.ascontiguousarray(k.transpose(1, 0, 2)).reshape(-1)

    def valuesUpTo(self, layer: int, n: int, seq: int = 0) -> np.ndarray:
        _, v = self.read(layer, n, seq)
        return np.ascontiguousarray(v.transpose(1, 0, 2)).reshape(-1)


class Exchange:
    """A split-KV exchange between `world` ranks, one GPU each (b2a_exchange_*):
    partials travel by peer stores inside the attention kernel. Every rank makes
    one, shares handle() with the others, and calls open() with all handles in
    rank order."""

    def __init__(self, ctx: Context, world: int, rank: int, batch: int, numHeads: int, numKVHeads: int,
                 numLayers: int = 1):
        self.ctx = ctx
        h = ctypes.c_void_p()
        check(ctx._lib.b2a_exchange_create_layers(ctx.handle, world, rank, batch, numLayers, numHeads, numKVHeads,
                                                  ctypes.byref(h)))
        self.numLayers = numLayers
        self.handle = h
        self.world, self.rank = world, rank
        ctx._children.add(self)

    def handle_bytes(self) -> bytes:
        buf = ctypes.create_string_buffer(EXCHANGE_HANDLE_BYTES)
        check(self.ctx._lib.b2a_exchange_handle(self.handle, buf))
        return buf.raw

    def open(self, handles: bytes) -> None:
        """handles: world * 64 bytes in rank order (this rank's slot is ignored)."""
        if len(handles) != self.world * EXCHANGE_HANDLE_BYTES:
            raise ValueError(f"expected {self.world * EXCHANGE_HANDLE_BYTES} handle bytes, got {len(handles)}")
        buf = ctypes.create_string_buffer(bytes(handles), len(handles))
        check(self.ctx._lib.b2a_exchange_open(self.handle, buf))

    def connect_local(self, peer: int, other: "Exchange") -> None:
        """Wire rank `peer` to another exchange of this process (single-GPU tests only)."""
        check(self.ctx._lib.b2a_exchange_connect_local(self.handle, peer, other.handle))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.ctx._lib.b2a_exchange_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PagePool:
    """The host page allocator of a paged cache on its own (b2a_pagepool_*): page
    tables and free pages, no device memory."""

    def __init__(self, numPages: int, pageSize: int, batch: int, capacity: int):
        self._lib = _lib.load()
        self.pageSize, self.capacity = pageSize, capacity
        h = ctypes.c_void_p()
        check(self._lib.b2a_pagepool_create(numPages, pageSize, batch, capacity, ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.b2a_pagepool_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reserve(self, seq: int, positions: int) -> None:
        check(self._lib.b2a_pagepool_reserve(self.handle, seq, positions))

    def release(self, seq: int | None = None) -> None:
        check(self._lib.b2a_pagepool_release(self.handle, -1 if seq is None else seq))

    def table(self, seq: int) -> np.ndarray:
        n = ctypes.c_int()
        out = np.zeros((self.capacity + self.pageSize - 1) // self.pageSize, np.int32)
        check(self._lib.b2a_pagepool_table(self.handle, seq, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                           out.size, ctypes.byref(n)))
        return out[:n.value].copy()

    @property
    def freePages(self) -> int:
        n = ctypes.c_int()
        check(self._lib.b2a_pagepool_free_pages(self.handle, ctypes.byref(n)))
        return n.value
