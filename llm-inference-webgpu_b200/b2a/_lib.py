"""ctypes binding of libb2a.so (include/b2a.h).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

B2A_OK, B2A_EINVAL, B2A_ERANGE, B2A_EBUSY, B2A_ECUDA, B2A_ENCCL, B2A_ETIMEDOUT, B2A_ENODEV = range(8)
B2A_F32, B2A_F16, B2A_BF16 = 0, 1, 2
B2A_HOST, B2A_DEVICE = 0, 1
B2A_NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024   # include/b2a.h: the no-alloc decode's fixed array

DTYPES = {"f32": B2A_F32, "f16": B2A_F16, "bf16": B2A_BF16}
DTYPE_SIZE = {B2A_F32: 4, B2A_F16: 2, B2A_BF16: 2}

# Every symbol include/b2a.h declares, with (restype, argtypes).
_vp, _i, _d, _f32p, _i32p, _szp, _i64p = (ctypes.c_void_p, ctypes.c_int, ctypes.c_double,
                                          ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32),
                                          ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_int64))
_pp = ctypes.POINTER(ctypes.c_void_p)
_ip = ctypes.POINTER(ctypes.c_int)
SIGNATURES = {
    "b2a_last_error": (ctypes.c_char_p, []),
    "b2a_status_name": (ctypes.c_char_p, [_i]),
    "b2a_abi_version": (_i, []),
    "b2a_init": (_i, [_i, _pp]),
    "b2a_destroy": (_i, [_vp]),
    "b2a_set_stream": (_i, [_vp, _vp]),
    "b2a_synchronize": (_i, [_vp]),
    "b2a_timing_enable": (_i, [_vp, _i]),
    "b2a_timing_read": (_i, [_vp, _vp, _i, _ip]),
    "b2a_kv_head_for": (_i, [_i, _i, _i]),
    "b2a_rope_frequencies": (_i, [_i, _d, ctypes.POINTER(ctypes.c_double)]),
    "b2a_rope_tables": (_i, [_i, _d, _i, _f32p, _f32p]),
    "b2a_rope_create": (_i, [_vp, _i, _d, _i, _pp]),
    "b2a_rope_destroy": (_i, [_vp]),
    "b2a_kvcache_create": (_i, [_vp, _i, _i, _i, _i, _i, _i, _pp]),
    "b2a_kvcache_destroy": (_i, [_vp]),
    "b2a_kvcache_allocate": (_i, [_vp, _i, _i, _ip]),
    "b2a_kvcache_commit": (_i, [_vp, _i, _i]),
    "b2a_kvcache_length": (_i, [_vp, _i, _ip]),
    "b2a_kvcache_set_lengths": (_i, [_vp, _i32p]),
    "b2a_kvcache_reset": (_i, [_vp, _i]),
    "b2a_kvcache_byte_length": (_i, [_vp, _szp]),
    "b2a_kvcache_pools": (_i, [_vp, _pp, _pp, _i64p]),
    "b2a_kvcache_write_at": (_i, [_vp, _vp, _i, _i, _i, _vp, _vp, _i, _i, _i]),
    "b2a_kvcache_read": (_i, [_vp, _vp, _i, _i, _i, _vp, _vp, _i]),
    "b2a_kvcache_create_paged": (_i, [_vp, _i, _i, _i, _i, _i, _i, _i, _i, _pp]),
    "b2a_kvcache_page_table": (_i, [_vp, _i, _i32p, _i, _ip]),
    "b2a_kvcache_free_pages": (_i, [_vp, _ip]),
    "b2a_pagepool_create": (_i, [_i, _i, _i, _i, _pp]),
    "b2a_pagepool_destroy": (_i, [_vp]),
    "b2a_pagepool_reserve": (_i, [_vp, _i, _i]),
    "b2a_pagepool_release": (_i, [_vp, _i]),
    "b2a_pagepool_table": (_i, [_vp, _i, _i32p, _i, _ip]),
    "b2a_pagepool_free_pages": (_i, [_vp, _ip]),
    "b2a_append_rope": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _i, _i, _i]),
    "b2a_attention_decode": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _i, _i]),
    "b2a_attention_decode_noalloc": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _i]),
    "b2a_attention_decode_host_async": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _i]),
    "b2a_attention_prefill": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp, _i, _i]),
    "b2a_attention_prefill_batch": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp, _i, _i]),
    "b2a_grouped_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i]),
    "b2a_attention_decode_partial": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _i]),
    "b2a_attention_decode_partial_layers": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _i]),
    "b2a_lse_combine": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _i, _i]),
    "b2a_split_kv_decode_nccl": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _vp, _i,
                                      _i]),
    "b2a_quantize_int8_per_channel": (_i, [_vp, _i, _i, _vp, _vp]),
    "b2a_linear_int8": (_i, [_vp, _vp, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _vp, _vp, _i, _i]),
    "b2a_qkv_int8": (_i, [_vp, _vp, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i]),
    "b2a_exchange_create": (_i, [_vp, _i, _i, _i, _i, _i, _pp]),
    "b2a_exchange_create_layers": (_i, [_vp, _i, _i, _i, _i, _i, _i, _pp]),
    "b2a_exchange_handle": (_i, [_vp, _vp]),
    "b2a_exchange_open": (_i, [_vp, _vp]),
    "b2a_exchange_connect_local": (_i, [_vp, _i, _vp]),
    "b2a_exchange_destroy": (_i, [_vp]),
    "b2a_attention_decode_split": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i]),
    "b2a_attention_decode_split_layers": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i,
                                                _i]),
    "b2a_model_create": (_i, [_vp, _vp, _i, _pp]),
    "b2a_model_destroy": (_i, [_vp]),
    "b2a_model_load_layer": (_i, [_vp, _i, _vp, _i]),
    "b2a_model_load_embedding": (_i, [_vp, _vp, _vp, _i]),
    "b2a_model_load_final_norm": (_i, [_vp, _vp, _i]),
    "b2a_model_forward": (_i, [_vp, _vp, _i, _vp, _vp, _i]),
    "b2a_model_generate": (_i, [_vp, _vp, _i, _i, _vp, _i, _vp, _vp, _ip]),
    "b2a_model_set_decode_path": (_i, [_vp, _i]),
    "b2a_model_decode_path": (_i, [_vp, _ip]),
    "b2a_model_reset": (_i, [_vp]),
    "b2a_safetensors_open": (_i, [ctypes.c_char_p, _pp]),
    "b2a_safetensors_open_memory": (_i, [_vp, ctypes.c_size_t, _pp]),
    "b2a_safetensors_close": (_i, [_vp]),
    "b2a_safetensors_count": (_i, [_vp]),
    "b2a_safetensors_name": (ctypes.c_char_p, [_vp, _i]),
    "b2a_safetensors_metadata": (ctypes.c_char_p, [_vp]),
    "b2a_safetensors_info": (_i, [_vp, ctypes.c_char_p, ctypes.c_char_p, _i64p, _i, _ip, _i64p]),
    "b2a_safetensors_read_raw": (_i, [_vp, ctypes.c_char_p, _vp, ctypes.c_size_t]),
    "b2a_safetensors_read_f32": (_i, [_vp, ctypes.c_char_p, _vp, ctypes.c_size_t]),
    "b2a_model_load_safetensors": (_i, [_vp, _vp]),
    "b2a_model_length": (_i, [_vp, _ip]),
    "b2a_model_cache": (_i, [_vp, _pp]),
}
EXCHANGE_HANDLE_BYTES = 64

_lib = None


class B2AError(RuntimeError):
    """A failed libb2a call; `status` is the b2a_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class RangeError(B2AError, ValueError):
    """The reference's RangeError (capacity and position range checks)."""


class BusyError(B2AError):
    """A call was made while another call on the same context was running."""


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = False) -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        if not build_if_missing:
            raise RuntimeError(f"libb2a.so is not built ({path}); run `python -m b2a.build` "
                               "or __graft_entry__.build()")
        _build.build()
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return load().b2a_last_error().decode(errors="replace")


def check(status: int) -> None:
    if status == B2A_OK:
        return
    msg = last_error()
    if status == B2A_ERANGE:
        raise RangeError(status, msg)
    if status == B2A_EBUSY:
        raise BusyError(status, msg)
    name = load().b2a_status_name(status).decode()
    raise B2AError(status, f"{name}: {msg}")
