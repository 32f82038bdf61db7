"""ctypes view of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY. The oracle restates the reference engine's f32 CPU
attention path (src/core/attention.js, src/core/ops.js, src/cpu/cache.js,
src/core/dtype.js of abho7/llm-inference-webgpu) in C. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module,
and only as the checker or as the timed CPU baseline; the product path (the
b2a package and libb2a.so) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        L = _lib
        L.or_f32_to_bf16.restype = ctypes.c_uint16
        L.or_f32_to_bf16.argtypes = [ctypes.c_float]
        L.or_bf16_to_f32.restype = ctypes.c_float
        L.or_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f32_to_f16.restype = ctypes.c_uint16
        L.or_f32_to_f16.argtypes = [ctypes.c_float]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        for name, a, b in (("or_f32_to_f16_array", _f32p, _u16p), ("or_f16_to_f32_array", _u16p, _f32p),
                           ("or_f32_to_bf16_array", _f32p, _u16p), ("or_bf16_to_f32_array", _u16p, _f32p)):
            getattr(L, name).restype = None
            getattr(L, name).argtypes = [a, b, ctypes.c_size_t]
        L.or_softmax_inplace.argtypes = [_f32p, ctypes.c_int]
        L.or_rope_frequencies.argtypes = [ctypes.c_int, ctypes.c_double, _f64p]
        L.or_rope_tables.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_int, _f32p, _f32p]
        L.or_rope_tables_f64.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_int, _f64p, _f64p]
        L.or_rope_inplace.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f64p]
        L.or_kv_head_for.restype = ctypes.c_int
        L.or_kv_head_for.argtypes = [ctypes.c_int] * 3
        L.or_grouped_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 5
        L.or_expanded_attention.argtypes = [_f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 5
        L.or_kvcache_new.restype = ctypes.c_void_p
        L.or_kvcache_new.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        L.or_kvcache_free.argtypes = [ctypes.c_void_p]
        L.or_kvcache_length.restype = ctypes.c_int
        L.or_kvcache_length.argtypes = [ctypes.c_void_p]
        L.or_kvcache_capacity.restype = ctypes.c_int
        L.or_kvcache_capacity.argtypes = [ctypes.c_void_p]
        L.or_kvcache_byte_length.restype = ctypes.c_size_t
        L.or_kvcache_byte_length.argtypes = [ctypes.c_void_p]
        L.or_kvcache_allocate.restype = ctypes.c_int
        L.or_kvcache_allocate.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        L.or_kvcache_write_at.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, ctypes.c_int]
        L.or_kvcache_keys_up_to.restype = _f32p
        L.or_kvcache_keys_up_to.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_kvcache_values_up_to.restype = _f32p
        L.or_kvcache_values_up_to.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_kvcache_commit.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_kvcache_present.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.or_kvcache_reset.argtypes = [ctypes.c_void_p]
        L.or_layer_attention.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f64p]
        L.or_decode_head_major.argtypes = [_f32p, _f32p, _f32p] + [ctypes.c_int] * 5 + [_f32p]
        L.or_decode_partial.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        _f32p, _f32p, _f32p]
        L.or_lse_combine.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.or_random_array.argtypes = [_f32p, ctypes.c_size_t, ctypes.c_uint32]
        L.or_normal_array.argtypes = [_f32p, ctypes.c_size_t, ctypes.c_uint64]
        L.or_batched_decode_f16.restype = ctypes.c_int
        L.or_batched_decode_f16.argtypes = [_f32p, ctypes.c_size_t, _u16p, _u16p, ctypes.c_size_t, _i32p,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            _f32p, ctypes.c_size_t, ctypes.c_int]
        _i8p = ctypes.POINTER(ctypes.c_int8)
        L.or_quantize_int8_per_channel.restype = None
        L.or_quantize_int8_per_channel.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _i8p, _f32p]
        L.or_dequantize_int8_per_channel.restype = None
        L.or_dequantize_int8_per_channel.argtypes = [_i8p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.or_matvec.restype = None
        L.or_matvec.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.or_rmsnorm.restype = None
        L.or_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_double, ctypes.c_int, _f32p]
        L.or_silu.restype = ctypes.c_double
        L.or_silu.argtypes = [ctypes.c_double]
        L.or_swiglu_inplace.restype = None
        L.or_swiglu_inplace.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.or_argmax.restype = ctypes.c_int
        L.or_argmax.argtypes = [_f32p, ctypes.c_int]
        L.or_model_new.restype = ctypes.c_void_p
        L.or_model_new.argtypes = [ctypes.c_int] * 6 + [ctypes.c_double, ctypes.c_double, ctypes.c_int,
                                                        ctypes.c_int]
        L.or_model_free.restype = None
        L.or_model_free.argtypes = [ctypes.c_void_p]
        L.or_model_set_layer.restype = None
        L.or_model_set_layer.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p, _f32p, _i8p, _f32p, _f32p, _i8p,
                                         _f32p, _i8p, _f32p, _i8p, _f32p, _i8p, _f32p]
        L.or_model_set_embedding.restype = None
        L.or_model_set_embedding.argtypes = [ctypes.c_void_p, _i8p, _f32p, _f32p]
        L.or_model_forward.restype = ctypes.c_int
        L.or_model_forward.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, _f32p, ctypes.c_char_p,
                                       ctypes.c_size_t]
        L.or_model_length.restype = ctypes.c_int
        L.or_model_length.argtypes = [ctypes.c_void_p]
        L.or_model_reset.restype = None
        L.or_model_reset.argtypes = [ctypes.c_void_p]
        L.or_model_present.restype = None
        L.or_model_present.argtypes = [ctypes.c_void_p, ctypes.c_int, _f32p, _f32p]
    return _lib


def _p(a: np.ndarray, ctype):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- dtype (src/core/dtype.js) ------------------------------------------------

def f32_to_f16_bits(x) -> np.ndarray:
    x = f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().or_f32_to_f16_array(_p(x.reshape(-1), ctypes.c_float), _p(out.reshape(-1), ctypes.c_uint16), x.size)
    return out


def f16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().or_f16_to_f32_array(_p(b.reshape(-1), ctypes.c_uint16), _p(out.reshape(-1), ctypes.c_float), b.size)
    return out


def f32_to_bf16_bits(x) -> np.ndarray:
    x = f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().or_f32_to_bf16_array(_p(x.reshape(-1), ctypes.c_float), _p(out.reshape(-1), ctypes.c_uint16), x.size)
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().or_bf16_to_f32_array(_p(b.reshape(-1), ctypes.c_uint16), _p(out.reshape(-1), ctypes.c_float), b.size)
    return out


def to_bits(x, dtype: str) -> np.ndarray:
    """Round an f32 array to `dtype` ('f32' | 'f16' | 'bf16') as raw storage."""
    if dtype == "f32":
        return f32(x)
    if dtype == "f16":
        return f32_to_f16_bits(x)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    raise ValueError(dtype)


def from_bits(b, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return f32(b)
    if dtype == "f16":
        return f16_bits_to_f32(b)
    if dtype == "bf16":
        return bf16_bits_to_f32(b)
    raise ValueError(dtype)


def round_to(x, dtype: str) -> np.ndarray:
    """f32 -> dtype -> f32: the value a kernel with that input dtype sees."""
    return from_bits(to_bits(x, dtype), dtype)


# ---- ops (src/core/ops.js) ------------------------------------------------------

def softmax_inplace(x: np.ndarray, n: int | None = None) -> np.ndarray:
    assert x.dtype == np.float32
    lib().or_softmax_inplace(_p(x, ctypes.c_float), x.size if n is None else n)
    return x


def rope_frequencies(head_dim: int, theta: float) -> np.ndarray:
    inv = np.empty(head_dim // 2, np.float64)
    lib().or_rope_frequencies(head_dim, theta, _p(inv, ctypes.c_double))
    return inv


def rope_tables(head_dim: int, theta: float, positions: int):
    half = head_dim // 2
    c = np.empty(positions * half, np.float32)
    s = np.empty(positions * half, np.float32)
    lib().or_rope_tables(head_dim, theta, positions, _p(c, ctypes.c_float), _p(s, ctypes.c_float))
    return c, s, half


def rope_tables_f64(head_dim: int, theta: float, positions: int):
    half = head_dim // 2
    c = np.empty(positions * half, np.float64)
    s = np.empty(positions * half, np.float64)
    lib().or_rope_tables_f64(head_dim, theta, positions, _p(c, ctypes.c_double), _p(s, ctypes.c_double))
    return c, s


def rope_inplace(vec: np.ndarray, offset: int, head_dim: int, position: int, inv_freq: np.ndarray) -> np.ndarray:
    assert vec.dtype == np.float32 and inv_freq.dtype == np.float64
    lib().or_rope_inplace(_p(vec, ctypes.c_float), offset, head_dim, position, _p(inv_freq, ctypes.c_double))
    return vec


def rope_rows(x: np.ndarray, positions, head_dim: int, theta: float) -> np.ndarray:
    """Rotate every head of x [rows, heads*head_dim] at positions[row]; returns a copy."""
    x = f32(x).copy()
    rows = x.shape[0]
    flat = x.reshape(rows, -1)
    heads = flat.shape[1] // head_dim
    inv = rope_frequencies(head_dim, theta)
    for r in range(rows):
        row = np.ascontiguousarray(flat[r])
        for h in range(heads):
            rope_inplace(row, h * head_dim, head_dim, int(positions[r]), inv)
        flat[r] = row
    return flat.reshape(x.shape)


# ---- attention (src/core/attention.js) --------------------------------------------

def kv_head_for(h: int, num_heads: int, num_kv_heads: int) -> int:
    return lib().or_kv_head_for(h, num_heads, num_kv_heads)


def grouped_attention(q, keys, values, seq, past, num_heads, num_kv_heads, head_dim) -> np.ndarray:
    q, keys, values = f32(q).reshape(-1), f32(keys).reshape(-1), f32(values).reshape(-1)
    out = np.empty(seq * num_heads * head_dim, np.float32)
    scores = np.empty(max(past + seq, 1), np.float32)
    lib().or_grouped_attention(_p(q, ctypes.c_float), _p(keys, ctypes.c_float), _p(values, ctypes.c_float),
                               _p(out, ctypes.c_float), _p(scores, ctypes.c_float),
                               seq, past, num_heads, num_kv_heads, head_dim)
    return out


def expanded_attention(q, keys, values, seq, past, num_heads, num_kv_heads, head_dim) -> np.ndarray:
    q, keys, values = f32(q).reshape(-1), f32(keys).reshape(-1), f32(values).reshape(-1)
    out = np.empty(seq * num_heads * head_dim, np.float32)
    lib().or_expanded_attention(_p(q, ctypes.c_float), _p(keys, ctypes.c_float), _p(values, ctypes.c_float),
                                _p(out, ctypes.c_float), seq, past, num_heads, num_kv_heads, head_dim)
    return out


def decode_head_major(q, kcache, vcache, cap, length, num_heads, num_kv_heads, head_dim) -> np.ndarray:
    q, kcache, vcache = f32(q).reshape(-1), f32(kcache).reshape(-1), f32(vcache).reshape(-1)
    out = np.empty(num_heads * head_dim, np.float32)
    lib().or_decode_head_major(_p(q, ctypes.c_float), _p(kcache, ctypes.c_float), _p(vcache, ctypes.c_float),
                               cap, length, num_heads, num_kv_heads, head_dim, _p(out, ctypes.c_float))
    return out


def decode_partial(qh, kh, vh, p0, p1, head_dim):
    qh, kh, vh = f32(qh).reshape(-1), f32(kh).reshape(-1), f32(vh).reshape(-1)
    m = np.empty(1, np.float32)
    l = np.empty(1, np.float32)
    o = np.empty(head_dim, np.float32)
    lib().or_decode_partial(_p(qh, ctypes.c_float), _p(kh, ctypes.c_float), _p(vh, ctypes.c_float),
                            p0, p1, head_dim, _p(m, ctypes.c_float), _p(l, ctypes.c_float), _p(o, ctypes.c_float))
    return float(m[0]), float(l[0]), o


def lse_combine(m, l, o, head_dim) -> np.ndarray:
    m, l, o = f32(m).reshape(-1), f32(l).reshape(-1), f32(o).reshape(-1)
    out = np.empty(head_dim, np.float32)
    lib().or_lse_combine(_p(m, ctypes.c_float), _p(l, ctypes.c_float), _p(o, ctypes.c_float),
                         m.size, head_dim, _p(out, ctypes.c_float))
    return out


def batched_decode_f16(q, q_stride, kbits, vbits, seq_stride, lengths, batch, cap,
                       num_heads, num_kv_heads, head_dim, out_stride, threads=0):
    """CPU baseline: f16 head-major caches; returns (out, threads_used)."""
    q = f32(q).reshape(-1)
    kbits = np.ascontiguousarray(kbits, np.uint16).reshape(-1)
    vbits = np.ascontiguousarray(vbits, np.uint16).reshape(-1)
    lengths = np.ascontiguousarray(lengths, np.int32)
    out = np.zeros(batch * out_stride, np.float32)
    used = lib().or_batched_decode_f16(_p(q, ctypes.c_float), q_stride, _p(kbits, ctypes.c_uint16),
                                       _p(vbits, ctypes.c_uint16), seq_stride, _p(lengths, ctypes.c_int32),
                                       batch, cap, num_heads, num_kv_heads, head_dim,
                                       _p(out, ctypes.c_float), out_stride, threads)
    return out, used


# ---- KV cache (src/cpu/cache.js) ----------------------------------------------------

class RangeError_(ValueError):
    """The oracle's stand-in for the reference's RangeError."""


class OracleKVCache:
    """src/cpu/cache.js:18-119 through the C restatement."""

    def __init__(self, num_layers: int, kv_dim: int, capacity: int):
        err = ctypes.create_string_buffer(256)
        if not isinstance(capacity, int):
            raise RangeError_(f"cache capacity must be a positive integer, got {capacity}")
        self._c = lib().or_kvcache_new(num_layers, kv_dim, capacity, err, 256)
        if not self._c:
            raise RangeError_(err.value.decode())
        self.num_layers, self.kv_dim, self.capacity = num_layers, kv_dim, capacity

    def __del__(self):
        if getattr(self, "_c", None):
            lib().or_kvcache_free(self._c)
            self._c = None

    @property
    def length(self) -> int:
        return lib().or_kvcache_length(self._c)

    @property
    def byte_length(self) -> int:
        return lib().or_kvcache_byte_length(self._c)

    def allocate(self, count: int) -> int:
        err = ctypes.create_string_buffer(256)
        at = lib().or_kvcache_allocate(self._c, count, err, 256)
        if at < 0:
            raise RangeError_(err.value.decode())
        return at

    def write_at(self, layer, at, keys, values, count):
        k, v = f32(keys).reshape(-1), f32(values).reshape(-1)
        lib().or_kvcache_write_at(self._c, layer, at, _p(k, ctypes.c_float), _p(v, ctypes.c_float), count)

    def keys_up_to(self, layer, n) -> np.ndarray:
        p = lib().or_kvcache_keys_up_to(self._c, layer, n)
        return np.ctypeslib.as_array(p, shape=(n * self.kv_dim,)).copy()

    def values_up_to(self, layer, n) -> np.ndarray:
        p = lib().or_kvcache_values_up_to(self._c, layer, n)
        return np.ctypeslib.as_array(p, shape=(n * self.kv_dim,)).copy()

    def commit(self, count):
        lib().or_kvcache_commit(self._c, count)

    def present(self, layer, num_kv_heads, head_dim):
        n = self.length
        k = np.empty(num_kv_heads * n * head_dim, np.float32)
        v = np.empty(num_kv_heads * n * head_dim, np.float32)
        if n:
            lib().or_kvcache_present(self._c, layer, num_kv_heads, head_dim, _p(k, ctypes.c_float),
                                     _p(v, ctypes.c_float))
        return k, v

    def reset(self):
        lib().or_kvcache_reset(self._c)

    def layer_attention(self, layer, q, k, v, seq, num_heads, num_kv_heads, head_dim, theta):
        """src/cpu/model.js:103-123. Returns (out, rotated q, rotated k)."""
        q, k, v = f32(q).reshape(-1).copy(), f32(k).reshape(-1).copy(), f32(v).reshape(-1)
        out = np.empty(seq * num_heads * head_dim, np.float32)
        inv = rope_frequencies(head_dim, theta)
        lib().or_layer_attention(self._c, layer, _p(q, ctypes.c_float), _p(k, ctypes.c_float),
                                 _p(v, ctypes.c_float), _p(out, ctypes.c_float), seq, num_heads,
                                 num_kv_heads, head_dim, _p(inv, ctypes.c_double))
        return out, q, k


# ---- generators ---------------------------------------------------------------------

def quantize_int8(w, rows: int, cols: int):
    """quantizeInt8PerChannel (src/core/quantize.js:36-58): (codes int8 [rows, cols], scales f32 [rows])."""
    w = np.ascontiguousarray(f32(w).reshape(-1))
    codes = np.zeros(rows * cols, np.int8)
    scales = np.zeros(rows, np.float32)
    lib().or_quantize_int8_per_channel(_p(w, ctypes.c_float), rows, cols, _p(codes, ctypes.c_int8),
                                       _p(scales, ctypes.c_float))
    return codes.reshape(rows, cols), scales


def dequantize_int8(codes, scales, rows: int, cols: int) -> np.ndarray:
    """dequantizeInt8PerChannel (src/core/quantize.js:60-67)."""
    codes = np.ascontiguousarray(codes, np.int8).reshape(-1)
    scales = np.ascontiguousarray(f32(scales))
    out = np.zeros(rows * cols, np.float32)
    lib().or_dequantize_int8_per_channel(_p(codes, ctypes.c_int8), _p(scales, ctypes.c_float), rows, cols,
                                         _p(out, ctypes.c_float))
    return out.reshape(rows, cols)


def matvec(w, x, rows: int, cols: int, bias=None) -> np.ndarray:
    """matVec (src/core/ops.js:33-41): f64 accumulation, f32 result."""
    w = np.ascontiguousarray(f32(w).reshape(-1))
    x = np.ascontiguousarray(f32(x).reshape(-1))
    out = np.zeros(rows, np.float32)
    b = None if bias is None else np.ascontiguousarray(f32(bias).reshape(-1))
    lib().or_matvec(_p(w, ctypes.c_float), _p(x, ctypes.c_float), rows, cols,
                    None if b is None else _p(b, ctypes.c_float), _p(out, ctypes.c_float))
    return out


def quantize_test_rand(n: int, seed: int) -> np.ndarray:
    """test/quantize.test.js:10-18: LCG s = s*1664525 + 1013904223 (mod 2^32), a = s/0xffffffff*2 - 1, f32."""
    s = seed & 0xffffffff
    out = np.empty(n, np.float32)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xffffffff
        out[i] = np.float32(s / 0xffffffff * 2 - 1)
    return out


def random_array(n: int, seed: int) -> np.ndarray:
    """test/attention.test.js:60-69."""
    out = np.empty(n, np.float32)
    lib().or_random_array(_p(out, ctypes.c_float), n, seed & 0xFFFFFFFF)
    return out


def normal_array(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_normal_array(_p(out, ctypes.c_float), n, seed & 0xFFFFFFFFFFFFFFFF)
    return out


# ---- the decoder around attention (src/core/ops.js, src/cpu/model.js) -------------------

def rmsnorm(x, weight, eps: float) -> np.ndarray:
    """rmsNorm (src/core/ops.js:17-24)."""
    x = np.ascontiguousarray(f32(x).reshape(-1))
    w = np.ascontiguousarray(f32(weight).reshape(-1))
    out = np.empty_like(x)
    lib().or_rmsnorm(_p(x, ctypes.c_float), _p(w, ctypes.c_float), float(eps), x.size, _p(out, ctypes.c_float))
    return out


def silu(x: float) -> float:
    """silu (src/core/ops.js:81-83)."""
    return lib().or_silu(float(x))


def swiglu(gate, up) -> np.ndarray:
    """swigluInPlace (src/core/ops.js:88-91) on a copy of gate."""
    g = np.ascontiguousarray(f32(gate).reshape(-1)).copy()
    u = np.ascontiguousarray(f32(up).reshape(-1))
    lib().or_swiglu_inplace(_p(g, ctypes.c_float), _p(u, ctypes.c_float), g.size)
    return g


def argmax(logits) -> int:
    """The greedy pick of generate (src/cpu/model.js:181-183): first index of the largest."""
    x = np.ascontiguousarray(f32(logits).reshape(-1))
    return lib().or_argmax(_p(x, ctypes.c_float), x.size)


def synthetic_weights(hidden: int, inter: int, layers: int, heads: int, kv_heads: int, vocab: int, seed: int,
                      std: float = 0.02, norm_jitter: float = 0.0, bias_std: float = 0.0) -> dict:
    """Seeded random-init weights of the Qwen2 architecture, already int8 per output row
    (quantizeInt8PerChannel's rule, src/core/quantize.js:36-58: scale = max|w|/127, codes =
    round(w/scale)) with scales rounded to f16: N(0, std) matrices, norm gains 1 (+ N(0, norm_jitter)),
    q/k/v bias N(0, bias_std). Returns {"layers": [dict], "embedding": (codes, scales16),
    "final_norm": f32}; every scale array is float16."""
    rng = np.random.default_rng(seed)
    kv_dim = kv_heads * (hidden // heads)

    def mat(rows, cols):
        w = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std))
        peak = np.abs(w).max(axis=1).astype(np.float64)
        scale = (peak / 127.0).astype(np.float32).astype(np.float16)
        s32 = scale.astype(np.float64)
        with np.errstate(divide="ignore", invalid="ignore"):
            lv = np.where(s32[:, None] > 0, w.astype(np.float64) / s32[:, None], 0.0)
        codes = np.clip(np.sign(lv) * np.floor(np.abs(lv) + 0.5), -127, 127).astype(np.int8)
        return codes, scale

    def gain():
        g = np.ones(hidden, np.float32)
        if norm_jitter:
            g += rng.standard_normal(hidden, dtype=np.float32) * np.float32(norm_jitter)
        return g

    out = {"layers": []}
    for _ in range(layers):
        qkv, sqkv = mat(hidden + 2 * kv_dim, hidden)
        o, so = mat(hidden, hidden)
        gate, sg = mat(inter, hidden)
        up, su = mat(inter, hidden)
        down, sd = mat(hidden, inter)
        bias = (rng.standard_normal(hidden + 2 * kv_dim, dtype=np.float32) * np.float32(bias_std)
                if bias_std else np.zeros(hidden + 2 * kv_dim, np.float32))
        out["layers"].append(dict(input_norm=gain(), post_attn_norm=gain(), qkv=qkv, qkv_scales=sqkv,
                                  qkv_bias=bias, o=o, o_scales=so, gate=gate, gate_scales=sg, up=up,
                                  up_scales=su, down=down, down_scales=sd))
    out["embedding"] = mat(vocab, hidden)
    out["final_norm"] = gain()
    return out


class OracleModel:
    """ReferenceModel (src/cpu/model.js:31-231) over int8 weights, in C, with the device
    path's f16 boundaries (q/k/v after projection, the KV cache)."""

    def __init__(self, weights: dict, hidden, inter, layers, heads, kv_heads, vocab, theta, eps, capacity,
                 threads: int = 1):
        self._keep = []
        self.vocab, self.kv_heads, self.head_dim = vocab, kv_heads, hidden // heads
        self._m = lib().or_model_new(hidden, inter, layers, heads, kv_heads, vocab, theta, eps, capacity, threads)

        def keep(a, dt):
            a = np.ascontiguousarray(np.asarray(a).astype(dt))
            self._keep.append(a)
            return _p(a, ctypes.c_float if dt == np.float32 else ctypes.c_int8)

        for i, w in enumerate(weights["layers"]):
            lib().or_model_set_layer(self._m, i, keep(w["input_norm"], np.float32),
                                     keep(w["post_attn_norm"], np.float32), keep(w["qkv"], np.int8),
                                     keep(w["qkv_scales"], np.float32), keep(w["qkv_bias"], np.float32),
                                     keep(w["o"], np.int8), keep(w["o_scales"], np.float32),
                                     keep(w["gate"], np.int8), keep(w["gate_scales"], np.float32),
                                     keep(w["up"], np.int8), keep(w["up_scales"], np.float32),
                                     keep(w["down"], np.int8), keep(w["down_scales"], np.float32))
        codes, scales = weights["embedding"]
        lib().or_model_set_embedding(self._m, keep(codes, np.int8), keep(scales, np.float32),
                                     keep(weights["final_norm"], np.float32))

    def __del__(self):
        if getattr(self, "_m", None):
            lib().or_model_free(self._m)
            self._m = None

    def forward(self, tokens) -> tuple[np.ndarray, int]:
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        logits = np.empty(self.vocab, np.float32)
        err = ctypes.create_string_buffer(256)
        best = lib().or_model_forward(self._m, _p(ids, ctypes.c_int32), ids.size, _p(logits, ctypes.c_float),
                                      err, 256)
        if best < 0:
            raise RangeError_(err.value.decode())
        return logits, best

    @property
    def length(self) -> int:
        return lib().or_model_length(self._m)

    def reset(self):
        lib().or_model_reset(self._m)

    def present(self, layer: int):
        n = self.length
        k = np.empty((self.kv_heads, n, self.head_dim), np.float32)
        v = np.empty_like(k)
        lib().or_model_present(self._m, layer, _p(k, ctypes.c_float), _p(v, ctypes.c_float))
        return k, v
