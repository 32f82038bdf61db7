"""The allocation-free decode entry point, checked against the regular one.

Some callers of this library cannot allocate device memory while a call runs:
a server that handed the GPU's memory to its own pools at start-up (a late
cudaMalloc may fail or eat into memory it planned for), or a caller whose other
streams must not stall on the device-wide synchronization cudaMalloc/cudaFree
can cause. b2a_attention_decode_noalloc serves them from one fixed device
array, made resident (with the kernels it launches) when the context is
created. Here it runs through the C ABI on the same inputs as
b2a_attention_decode, two calls in a row with different inputs (the shared
array keeps the previous call's contents), and its outputs must agree within
the tolerance every other parity test uses; sampled rows are also checked
against the CPU oracle directly. Further cases cover the CUDA-core path (f32
cache), the long-chunk planning branch, and that a call on a new, larger shape
leaves the device's free memory unchanged. This file sorts last so that a run
stopping at the first failure has run everything else first.
"""
import numpy as np
import pytest

import b2a
from b2a import _lib
from helpers import ATOL, RTOL, check_decode_rows, compare

pytestmark = pytest.mark.gpu

H, KVH, D = 14, 2, 64


def _fill(cache, torch, dev, layers, batch, cap, seed, dtype=None):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    for b in range(batch):
        for layer in range(layers):
            k = torch.randn(cap, KVH * D, device=dev, generator=g)
            v = torch.randn(cap, KVH * D, device=dev, generator=g)
            if dtype != torch.float32:
                k, v = k.half(), v.half()
            cache.writeAt(layer, 0, k, v, cap, seq=b)


def _calls(lib, ctx, cache, rope, layers, q, kn, vn, in_dt, out_ref, out_na):
    _lib.check(lib.b2a_attention_decode(ctx.handle, cache.handle, rope.handle, 0, layers, H, q.data_ptr(),
                                        kn.data_ptr(), vn.data_ptr(), in_dt, out_ref.data_ptr(), _lib.B2A_F32,
                                        _lib.B2A_DEVICE))
    _lib.check(lib.b2a_attention_decode_noalloc(ctx.handle, cache.handle, rope.handle, 0, layers, H, q.data_ptr(),
                                                kn.data_ptr(), vn.data_ptr(), in_dt, out_na.data_ptr(),
                                                _lib.B2A_F32))


def test_noalloc_decode_matches_decode_on_two_calls(oracle):
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
        _calls(lib, ctx, cache, rope, layers, q, kn, vn, _lib.B2A_F16, out_ref, out_na)
        torch.cuda.synchronize(dev)
        ctx.synchronize()
        got = out_na.cpu().numpy()
        c = compare(got, out_ref.cpu().numpy())
        assert c["finite"], f"call {call}: non-finite output"
        assert c["max_abs"] <= ATOL and c["rel"] <= RTOL, f"call {call}: {c}"
        # and directly against the oracle on a few rows (the short sequence included)
        check_decode_rows(oracle, cache, q.float().cpu().numpy(), lengths, [(call, 0), (5, 2), (3, 1)], got, "f16",
                          kn=kn.float().cpu().numpy(), what=f"no-alloc call {call}")
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


def test_noalloc_f32_cache_takes_the_cuda_core_path(oracle):
    """An f32 cache has no tensor-core path: 256-position chunks on the CUDA cores."""
    import torch

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    ctx = b2a.Context(0)
    layers, batch, cap = 2, 3, 1500
    cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), cap, batch=batch, dtype="f32")
    rope = b2a.RopeTable(ctx, D, 1e6, cap + 1)
    _fill(cache, torch, dev, layers, batch, cap, 17, dtype=torch.float32)
    lengths = np.array([1, 700, 1400], np.int32)
    cache.setLengths(lengths)
    g = torch.Generator(device=dev)
    g.manual_seed(18)
    q = torch.randn(batch, layers, H, D, device=dev, generator=g)
    kn = torch.randn(batch, layers, KVH, D, device=dev, generator=g)
    vn = torch.randn(batch, layers, KVH, D, device=dev, generator=g)
    out_ref = torch.full((batch, layers, H, D), float("nan"), device=dev)
    out_na = torch.full((batch, layers, H, D), float("nan"), device=dev)
    torch.cuda.synchronize(dev)
    _calls(lib, ctx, cache, rope, layers, q, kn, vn, _lib.B2A_F32, out_ref, out_na)
    ctx.synchronize()
    got = out_na.cpu().numpy()
    c = compare(got, out_ref.cpu().numpy())
    assert c["finite"] and c["max_abs"] <= ATOL and c["rel"] <= RTOL, c
    check_decode_rows(oracle, cache, q.cpu().numpy(), lengths, [(0, 0), (1, 1), (2, 0)], got, "f32",
                      kn=kn.cpu().numpy(), what="no-alloc f32")
    cache.close()
    rope.close()
    ctx.close()


def test_noalloc_long_chunks_when_short_ones_overflow(oracle):
    """64 sequences x 24 layers with one 8192-position context: 4096-position
    chunks would need 21504 rows x 3 chunks of partials, more than the array
    holds, so the planner takes 8192-position chunks (2 per row) instead."""
    import torch

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    ctx = b2a.Context(0)
    layers, batch, cap = 24, 64, 8200
    rows = batch * layers * H
    slots = _lib.B2A_NOALLOC_SCRATCH_BYTES // ((D + 4) * 4)
    assert rows * 3 > slots >= rows * 2
    cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), cap, batch=batch, dtype="f16")
    rope = b2a.RopeTable(ctx, D, 1e6, cap + 1)
    kp, vp, _ = cache.pools()

    class _CAI:
        def __init__(self, ptr, shape):
            self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f2", "data": (ptr, False), "version": 3}

    g = torch.Generator(device=dev)
    g.manual_seed(23)
    torch.as_tensor(_CAI(kp, (batch, layers, KVH, cap, D)), device=dev).normal_(generator=g)
    torch.as_tensor(_CAI(vp, (batch, layers, KVH, cap, D)), device=dev).normal_(generator=g)
    lengths = np.random.default_rng(24).integers(100, 1000, size=batch).astype(np.int32)
    lengths[5] = 8192
    cache.setLengths(lengths)
    q = torch.randn(batch, layers, H, D, device=dev, generator=g).half()
    kn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    vn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    out_ref = torch.full((batch, layers, H, D), float("nan"), device=dev)
    out_na = torch.full((batch, layers, H, D), float("nan"), device=dev)
    torch.cuda.synchronize(dev)
    _calls(lib, ctx, cache, rope, layers, q, kn, vn, _lib.B2A_F16, out_ref, out_na)
    ctx.synchronize()
    got = out_na.cpu().numpy()
    c = compare(got, out_ref.cpu().numpy())
    assert c["finite"] and c["max_abs"] <= ATOL and c["rel"] <= RTOL, c
    check_decode_rows(oracle, cache, q.float().cpu().numpy(), lengths, [(5, 0), (5, 23), (0, 11), (63, 7)], got,
                      "f16", kn=kn.float().cpu().numpy(), what="no-alloc long chunks")
    cache.close()
    rope.close()
    ctx.close()


def test_noalloc_allocates_nothing(oracle):
    """After one call on short contexts, a call on a new, larger shape leaves the
    device's free memory exactly as it was (no regular decode in between)."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    ctx = b2a.Context(0)
    layers, batch, cap = 4, 8, 3000
    cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), cap, batch=batch, dtype="f16")
    rope = b2a.RopeTable(ctx, D, 1e6, cap + 1)
    _fill(cache, torch, dev, layers, batch, cap, 31)
    g = torch.Generator(device=dev)
    g.manual_seed(32)
    q = torch.randn(batch, layers, H, D, device=dev, generator=g).half()
    kn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    vn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    out = torch.full((batch, layers, H, D), float("nan"), device=dev)

    def call():
        _lib.check(lib.b2a_attention_decode_noalloc(ctx.handle, cache.handle, rope.handle, 0, layers, H,
                                                    q.data_ptr(), kn.data_ptr(), vn.data_ptr(), _lib.B2A_F16,
                                                    out.data_ptr(), _lib.B2A_F32))
        ctx.synchronize()

    cache.setLengths([200] * batch)
    call()
    lengths = np.random.default_rng(33).integers(1500, cap - 1, size=batch).astype(np.int32)
    cache.setLengths(lengths)
    torch.cuda.synchronize(dev)
    free0 = torch.cuda.mem_get_info(dev)[0]
    call()
    free1 = torch.cuda.mem_get_info(dev)[0]
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes across a no-alloc call"
    check_decode_rows(oracle, cache, q.float().cpu().numpy(), lengths, [(0, 0), (7, 3)], out.cpu().numpy(), "f16",
                      what="no-alloc larger shape")
    cache.close()
    rope.close()
    ctx.close()
