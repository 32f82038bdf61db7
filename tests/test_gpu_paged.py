"""Paged KV caches (b2a_kvcache_create_paged) against contiguous ones.

A paged cache must behave exactly like the contiguous cache of the reference's
KVCache layout (src/cpu/cache.js:18-119): the same kernels run, only the row
of each position comes from the sequence's page table. So every operation is
run on a contiguous cache and on a paged cache holding the same keys and
values, with the paged cache's pages scattered over the pool (sequences grow
interleaved, in steps that do not line up with pages), and the results must be
the same bits: decode (tensor-core f16/bf16, CUDA-core f32), prefill (both
tensor-core kernels and the CUDA-core path, one sequence and a batch), the
fused appends and the raw writes and reads. One decode is also checked against
the oracle's grouped attention (src/core/attention.js:32-66) within the
attention tolerance.
"""
import numpy as np
import pytest

import b2a
from b2a import _lib
from helpers import assert_parity

pytestmark = pytest.mark.gpu

H, KVH, D, THETA = 14, 2, 64, 1e6
P = 128


@pytest.fixture(scope="module")
def ctx():
    c = b2a.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def rope(ctx):
    return b2a.RopeTable(ctx, D, THETA, 4096)


def _pair(ctx, oracle, dtype, layers, batch, cap, lens, seed, spare_pages=8):
    """A contiguous and a paged cache with the same contents at lengths `lens`."""
    cfg = b2a.CacheConfig(numLayers=layers, numKVHeads=KVH, headDim=D, numHeads=H)
    cc = b2a.GpuKVCache(ctx, cfg, cap, batch=batch, dtype=dtype)
    pages = sum(-(-L // P) for L in lens) + spare_pages
    pc = b2a.GpuKVCache(ctx, cfg, cap, batch=batch, dtype=dtype, pageSize=P, numPages=pages)
    data = {}
    for b, L in enumerate(lens):
        for layer in range(layers):
            data[b, layer] = (oracle.normal_array(L * KVH * D, seed + 10 * b + layer),
                              oracle.normal_array(L * KVH * D, seed + 5000 + 10 * b + layer))
            if L:
                cc.writeAt(layer, 0, *data[b, layer], L, seq=b)
    # the paged cache is filled in 100-position pieces, last sequence first,
    # round after round: every sequence's pages end up scattered over the pool
    done = [0] * batch
    while any(done[b] < lens[b] for b in range(batch)):
        for b in reversed(range(batch)):
            n = min(100, lens[b] - done[b])
            if n <= 0:
                continue
            for layer in range(layers):
                k, v = data[b, layer]
                sl = slice(done[b] * KVH * D, (done[b] + n) * KVH * D)
                pc.writeAt(layer, done[b], k[sl], v[sl], n, seq=b)
            done[b] += n
    cc.setLengths(lens)
    pc.setLengths(lens)
    tables = [pc.pageTable(b) for b in range(batch)]
    assert any(t.size > 1 and np.any(np.diff(t) != 1) for t in tables), tables
    return cc, pc, data


def _same_contents(cc, pc, layers, batch, n_of):
    for b in range(batch):
        for layer in range(layers):
            n = n_of(b)
            kc, vc = cc.read(layer, n, seq=b)
            kp, vp = pc.read(layer, n, seq=b)
            assert np.array_equal(kc, kp) and np.array_equal(vc, vp), (b, layer)


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_paged_decode_equals_contiguous(ctx, rope, oracle, dtype):
    layers, batch, cap = 2, 5, 1200
    lens = [0, 127, 128, 383, 1000]    # the new slot: page starts, page ends, mid-page
    cc, pc, data = _pair(ctx, oracle, dtype, layers, batch, cap, lens, 11)
    for step in range(2):
        q = oracle.normal_array(batch * layers * H * D, 70 + step).reshape(batch, layers, H, D)
        kn = oracle.normal_array(batch * layers * KVH * D, 80 + step).reshape(batch, layers, KVH, D)
        vn = oracle.normal_array(batch * layers * KVH * D, 90 + step).reshape(batch, layers, KVH, D)
        oc = np.full((batch, layers, H, D), np.nan, np.float32)
        op = np.full_like(oc, np.nan)
        b2a.attentionDecode(ctx, cc, rope, 0, q, kn, vn, oc, H, numLayers=layers)
        b2a.attentionDecode(ctx, pc, rope, 0, q, kn, vn, op, H, numLayers=layers)
        assert np.array_equal(oc, op), f"step {step}"
        if step == 0 and dtype == "f16":
            for b, L in enumerate(lens):
                for layer in range(layers):
                    qr = oracle.rope_rows(q[b, layer].reshape(1, -1), [L], D, THETA).reshape(-1)
                    kr = oracle.round_to(oracle.rope_rows(kn[b, layer].reshape(1, -1), [L], D, THETA), dtype)
                    k0, v0 = data[b, layer]
                    keys = np.concatenate([oracle.round_to(k0, dtype).reshape(L, KVH * D), kr.reshape(1, -1)])
                    vals = np.concatenate([oracle.round_to(v0, dtype).reshape(L, KVH * D),
                                           oracle.round_to(vn[b, layer], dtype).reshape(1, -1)])
                    ref = oracle.grouped_attention(qr, keys.reshape(-1), vals.reshape(-1), 1, L, H, KVH, D)
                    assert_parity(op[b, layer].reshape(-1), ref, "f32", f"paged decode seq {b} layer {layer}")
        cc.commit(1, None)
        pc.commit(1, None)
        lens = [L + 1 for L in lens]
        _same_contents(cc, pc, layers, batch, lambda b: lens[b])
    cc.close()
    pc.close()


@pytest.mark.parametrize("dtype,tiles", [("f16", "1"), ("f16", "2"), ("bf16", "1"), ("f32", "1")])
def test_paged_prefill_equals_contiguous(ctx, rope, oracle, monkeypatch, dtype, tiles):
    monkeypatch.setenv("B2A_PREFILL_TILES", tiles)
    layers, batch, cap = 1, 4, 1024
    lens = [0, 100, 300, 129]
    cc, pc, _ = _pair(ctx, oracle, dtype, layers, batch, cap, lens, 23)
    bits = lambda x: oracle.to_bits(oracle.round_to(x, "f16"), "f16")  # noqa: E731
    # one sequence: 200 tokens after 300 cached (pages 2..3 of sequence 2)
    count = 200
    q = bits(oracle.normal_array(count * H * D, 31)).reshape(count, H * D)
    k = bits(oracle.normal_array(count * KVH * D, 32)).reshape(count, KVH * D)
    v = bits(oracle.normal_array(count * KVH * D, 33)).reshape(count, KVH * D)
    oc = np.empty((count, H * D), np.float32)
    op = np.empty_like(oc)
    b2a.attentionPrefill(ctx, cc, rope, 0, q, k, v, oc, count, H, seq=2, dtype="f16", out_dtype="f32")
    b2a.attentionPrefill(ctx, pc, rope, 0, q, k, v, op, count, H, seq=2, dtype="f16", out_dtype="f32")
    assert np.array_equal(oc, op)
    # a batch: sequences 0 and 1 (lengths 0 and 100), 150 tokens each
    count, nseq = 150, 2
    q = bits(oracle.normal_array(nseq * count * H * D, 41)).reshape(nseq, count, H * D)
    k = bits(oracle.normal_array(nseq * count * KVH * D, 42)).reshape(nseq, count, KVH * D)
    v = bits(oracle.normal_array(nseq * count * KVH * D, 43)).reshape(nseq, count, KVH * D)
    oc = np.empty((nseq, count, H * D), np.float32)
    op = np.empty_like(oc)
    b2a.attentionPrefillBatch(ctx, cc, rope, 0, q, k, v, oc, count, H, 0, nseq, dtype="f16", out_dtype="f32")
    b2a.attentionPrefillBatch(ctx, pc, rope, 0, q, k, v, op, count, H, 0, nseq, dtype="f16", out_dtype="f32")
    assert np.array_equal(oc, op)
    _same_contents(cc, pc, layers, batch, lambda b: [150, 250, 500, 129][b])
    cc.close()
    pc.close()


def test_paged_append_and_raw_writes(ctx, rope, oracle):
    layers, batch, cap = 2, 3, 900
    lens = [50, 260, 0]
    cc, pc, _ = _pair(ctx, oracle, "bf16", layers, batch, cap, lens, 37)
    for b, count in [(0, 300), (1, 7), (2, 129)]:
        for layer in range(layers):
            k = oracle.normal_array(count * KVH * D, 100 + b + layer)
            v = oracle.normal_array(count * KVH * D, 200 + b + layer)
            b2a.appendRope(ctx, cc, rope, layer, k, v, count, seq=b)
            b2a.appendRope(ctx, pc, rope, layer, k, v, count, seq=b)
        cc.commit(count, b)
        pc.commit(count, b)
    # a raw write far from the sequence's length maps every page before it
    k = oracle.normal_array(20 * KVH * D, 300)
    cc.writeAt(1, 700, k, k, 20, seq=2)
    pc.writeAt(1, 700, k, k, 20, seq=2)
    assert pc.pageTable(2).size == 6
    _same_contents(cc, pc, layers, batch, lambda b: [350, 267, 720][b])
    cc.close()
    pc.close()


def test_paged_pool_exhaustion_reset_and_zero_reads(ctx, rope):
    cfg = b2a.CacheConfig(numLayers=1, numKVHeads=KVH, headDim=D, numHeads=H)
    pc = b2a.GpuKVCache(ctx, cfg, 1024, batch=2, dtype="f16", pageSize=P, numPages=3)
    assert pc.byteLength == 2 * 4 * 1 * KVH * P * D * 2   # pages + the scratch page, keys and values
    pc.setLengths([256, 128])
    assert pc.freePages == 0
    q = np.zeros((2, 1, H, D), np.float32)
    kv = np.zeros((2, 1, KVH, D), np.float32)
    out = np.zeros((2, 1, H, D), np.float32)
    with pytest.raises(b2a.RangeError, match=r"page pool exhausted: 3 of 3 pages in use; sequence 0 needs 1 more"):
        b2a.attentionDecode(ctx, pc, rope, 0, q, kv, kv, out, H)
    assert [pc.lengthOf(0), pc.lengthOf(1)] == [256, 128]
    assert [pc.pageTable(0).tolist(), pc.pageTable(1).tolist()] == [[0, 1], [2]]
    pc.reset(1)
    assert pc.freePages == 1 and pc.pageTable(1).size == 0
    k1, _ = pc.read(0, 300, seq=1)   # nothing mapped: zeros
    assert not k1.any()
    with pytest.raises(b2a.RangeError, match=r"2 of 3 pages in use; sequence 1 needs 1 more"):
        b2a.attentionDecode(ctx, pc, rope, 0, q, kv, kv, out, H)
    with pytest.raises(b2a.RangeError, match="page pool exhausted"):
        pc.allocate(300, seq=1)
    assert pc.allocate(128, seq=1) == 0 and pc.freePages == 0
    pc.reset()
    assert pc.freePages == 3
    b2a.attentionDecode(ctx, pc, rope, 0, q, kv, kv, out, H)
    assert np.isfinite(out).all()
    with pytest.raises(b2a.B2AError, match="power of two of at least 128"):
        b2a.GpuKVCache(ctx, cfg, 1024, batch=2, dtype="f16", pageSize=96, numPages=3)
    pc.close()


def test_paged_noalloc_decode_equals_contiguous(ctx, rope, oracle):
    import torch

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    layers, batch, cap = 2, 3, 800
    lens = [5, 130, 700]
    cc, pc, _ = _pair(ctx, oracle, "f16", layers, batch, cap, lens, 51)
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    q = torch.randn(batch, layers, H, D, device=dev, generator=g).half()
    kn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    vn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    outs = []
    for c in (cc, pc):
        o = torch.full((batch, layers, H, D), float("nan"), device=dev)
        torch.cuda.synchronize(dev)
        _lib.check(lib.b2a_attention_decode_noalloc(ctx.handle, c.handle, rope.handle, 0, layers, H, q.data_ptr(),
                                                    kn.data_ptr(), vn.data_ptr(), _lib.B2A_F16, o.data_ptr(),
                                                    _lib.B2A_F32))
        ctx.synchronize()
        outs.append(o.cpu().numpy())
    assert np.isfinite(outs[0]).all()
    assert np.array_equal(outs[0], outs[1])
    _same_contents(cc, pc, layers, batch, lambda b: lens[b] + 1)
    cc.close()
    pc.close()
