"""The allocation-free decode entry point, checked against the regular one.

Some callers of this library cannot allocate device memory while a call runs:
a server that handed the GPU's memory to its own pools at start-up (a late
cudaMalloc may fail or eat into memory it planned for), or a caller whose other
streams must not stall on the device-wide synchronization cudaMalloc/cudaFree
can cause. b2a_attention_decode_noalloc serves them from one fixed device
array. Here it runs through the C ABI on the same inputs as
b2a_attention_decode, two calls in a row with different inputs (the shared
array keeps the previous call's contents), and its outputs must agree within
the tolerance every other parity test uses. This file sorts last so that a run
stopping at the first failure has run everything else first.
"""
import ctypes

import numpy as np
import pytest

import b2a
from b2a import _lib
from helpers import ATOL, RTOL, compare

pytestmark = pytest.mark.gpu

H, KVH, D = 14, 2, 64


def _fill(cache, torch, dev, layers, batch, cap, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    for b in range(batch):
        for layer in range(layers):
            k = torch.randn(cap, KVH * D, device=dev, generator=g).half()
            v = torch.randn(cap, KVH * D, device=dev, generator=g).half()
            cache.writeAt(layer, 0, k, v, cap, seq=b)


def test_noalloc_decode_matches_decode_on_two_calls():
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    ctx = b2a.Context(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    layers, batch, cap = 3, 6, 2500
    cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), cap, batch=batch, dtype="f16")
    rope = b2a.RopeTable(ctx, D, 1e6, cap + 1)
    with torch.cuda.stream(stream):
        _fill(cache, torch, dev, layers, batch, cap, 5)
    torch.cuda.synchronize(dev)
    rng = np.random.default_rng(3)
    for call in range(2):
        lengths = rng.integers(1, cap - 1, size=batch).astype(np.int32)
        lengths[call] = 1
        cache.setLengths(lengths)
        g = torch.Generator(device=dev)
        g.manual_seed(100 + call)
        with torch.cuda.stream(stream):
            q = torch.randn(batch, layers, H, D, device=dev, generator=g).half()
            kn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
            vn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
            out_ref = torch.full((batch, layers, H, D), float("nan"), device=dev)
            out_na = torch.full((batch, layers, H, D), float("nan"), device=dev)
        torch.cuda.synchronize(dev)
        _lib.check(lib.b2a_attention_decode(ctx.handle, cache.handle, rope.handle, 0, layers, H, q.data_ptr(),
                                            kn.data_ptr(), vn.data_ptr(), _lib.B2A_F16, out_ref.data_ptr(),
                                            _lib.B2A_F32, _lib.B2A_DEVICE))
        _lib.check(lib.b2a_attention_decode_noalloc(ctx.handle, cache.handle, rope.handle, 0, layers, H,
                                                    q.data_ptr(), kn.data_ptr(), vn.data_ptr(), _lib.B2A_F16,
                                                    out_na.data_ptr(), _lib.B2A_F32))
        torch.cuda.synchronize(dev)
        ctx.synchronize()
        c = compare(out_na.cpu().numpy(), out_ref.cpu().numpy())
        assert c["finite"], f"call {call}: non-finite output"
        assert c["max_abs"] <= ATOL and c["rel"] <= RTOL, f"call {call}: {c}"
    cache.close()
    rope.close()
    ctx.close()


def test_noalloc_rejects_work_beyond_its_scratch():
    import torch

    lib = _lib.load()
    ctx = b2a.Context(0)
    layers, batch, cap = 48, 128, 64
    cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), cap, batch=batch, dtype="f16")
    rope = b2a.RopeTable(ctx, D, 1e6, cap + 1)
    dev = torch.device("cuda", 0)
    q = torch.zeros(batch, layers, H, D, device=dev, dtype=torch.float16)
    out = torch.empty(batch, layers, H, D, device=dev)
    st = lib.b2a_attention_decode_noalloc(ctx.handle, cache.handle, rope.handle, 0, layers, H, q.data_ptr(), None,
                                          None, _lib.B2A_F16, out.data_ptr(), _lib.B2A_F32)
    assert st == _lib.B2A_ERANGE
    assert "no-alloc array" in _lib.last_error()
    cache.close()
    rope.close()
    ctx.close()
