"""Batched prefill (b2a_attention_prefill_batch): several sequences, each at its
own cache length, in one append launch and one attention launch.

It must give what one b2a_attention_prefill call per sequence gives: the same
bits on the tensor-core paths (the same kernels, a sequence index more), the
same cache contents, and the oracle's causal attention (src/cpu/model.js:103-123)
within the attention tolerance.
"""
import numpy as np
import pytest

import b2a
from helpers import assert_parity

pytestmark = pytest.mark.gpu

H, KVH, D, THETA = 14, 2, 64, 1e6
PASTS = [0, 37, 130]


@pytest.fixture(scope="module")
def ctx():
    c = b2a.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def rope(ctx):
    return b2a.RopeTable(ctx, D, THETA, 4096)


def _cache(ctx, oracle, dtype, count):
    """4 sequences; sequences 1..3 hold PASTS[b] cached positions."""
    c = b2a.GpuKVCache(ctx, b2a.CacheConfig(numLayers=2, numKVHeads=KVH, headDim=D, numHeads=H),
                       max(PASTS) + count, batch=4, dtype=dtype)
    lens = [0] + PASTS
    hk, hv = {}, {}
    for b, L in enumerate(lens):
        if L == 0:
            continue
        kk = oracle.normal_array(L * KVH * D, 500 + b)
        vv = oracle.normal_array(L * KVH * D, 600 + b)
        c.writeAt(1, 0, kk, vv, L, seq=b)
        hk[b], hv[b] = oracle.round_to(kk, dtype), oracle.round_to(vv, dtype)
    c.setLengths(lens)
    return c, hk, hv


@pytest.mark.parametrize("cache_dtype,tiles", [("f16", "2"), ("f16", "1"), ("bf16", "1"), ("f32", "1")])
def test_batched_prefill_equals_one_call_per_sequence(ctx, rope, oracle, monkeypatch, cache_dtype, tiles):
    monkeypatch.setenv("B2A_PREFILL_TILES", tiles)
    count, nseq = 70, len(PASTS)
    q = oracle.round_to(oracle.normal_array(nseq * count * H * D, 71), "f16").reshape(nseq, count, H * D)
    k = oracle.round_to(oracle.normal_array(nseq * count * KVH * D, 72), "f16").reshape(nseq, count, KVH * D)
    v = oracle.round_to(oracle.normal_array(nseq * count * KVH * D, 73), "f16").reshape(nseq, count, KVH * D)
    bits = lambda x: oracle.to_bits(x, "f16")  # noqa: E731
    cb, hk, hv = _cache(ctx, oracle, cache_dtype, count)
    cs, _, _ = _cache(ctx, oracle, cache_dtype, count)
    ob = np.empty((nseq, count, H * D), np.float32)
    b2a.attentionPrefillBatch(ctx, cb, rope, 1, bits(q), bits(k), bits(v), ob, count, H, 1, nseq, dtype="f16",
                              out_dtype="f32")
    os_ = np.empty_like(ob)
    for i in range(nseq):
        b2a.attentionPrefill(ctx, cs, rope, 1, bits(q[i]), bits(k[i]), bits(v[i]), os_[i], count, H, seq=1 + i,
                             dtype="f16", out_dtype="f32")
    refs = []
    for i, past in enumerate(PASTS):
        # the oracle: RoPE at past..past+count-1, causal over the cached and new keys
        qr = oracle.rope_rows(q[i], range(past, past + count), D, THETA).reshape(-1)
        kr = oracle.round_to(oracle.rope_rows(k[i], range(past, past + count), D, THETA), cache_dtype)
        keys = np.concatenate([hk[1 + i].reshape(past, KVH * D), kr]) if past else kr
        vals = np.concatenate([hv[1 + i].reshape(past, KVH * D), oracle.round_to(v[i], cache_dtype)]) if past else \
            oracle.round_to(v[i], cache_dtype)
        refs.append(oracle.grouped_attention(qr, keys.reshape(-1), vals.reshape(-1), count, past, H, KVH, D))
    if cache_dtype != "f32":
        if not np.array_equal(ob, os_):
            # say which call strays from the oracle, and where, before failing
            where = []
            for i in range(nseq):
                for name, o in (("batched", ob[i]), ("single", os_[i])):
                    err = np.abs(o.reshape(count, H, D) - refs[i].reshape(count, H, D)).max(axis=2)
                    bad = np.argwhere(err > 1e-2)
                    where.append(f"seq {i} {name}: max err {err.max():.2e}, {len(bad)} bad (token, head) rows, "
                                 f"tokens {sorted(set(bad[:, 0].tolist()))[:8]}, heads {sorted(set(bad[:, 1].tolist()))}")
            for i, past in enumerate(PASTS):
                kb, vb = cb.read(1, past + count, seq=1 + i)
                ks, vs = cs.read(1, past + count, seq=1 + i)
                where.append(f"seq {i} cache: keys equal {np.array_equal(kb, ks)}, values equal {np.array_equal(vb, vs)}")
            raise AssertionError("batched and per-sequence outputs differ:\n" + "\n".join(where))
    else:   # the CUDA-core path may chunk the keys differently for one sequence and for three
        assert_parity(ob.reshape(-1), os_.reshape(-1), "f32", "batched vs single (f32 cache)")
    for i, past in enumerate(PASTS):
        kb, vb = cb.read(1, past + count, seq=1 + i)
        ks, vs = cs.read(1, past + count, seq=1 + i)
        assert np.array_equal(kb, ks) and np.array_equal(vb, vs)
        assert_parity(ob[i].reshape(-1), refs[i], "f32", f"{cache_dtype} batched prefill, sequence {i}")
    # the untouched sequence 0 and layer 0 stay as they were
    assert cb.lengthOf(0) == 0
    cb.close()
    cs.close()


def test_batched_prefill_checks_every_sequence(ctx, rope, oracle):
    c, _, _ = _cache(ctx, oracle, "f16", 8)
    q = np.zeros((3, 20, H * D), np.uint16)
    k = np.zeros((3, 20, KVH * D), np.uint16)
    o = np.zeros((3, 20, H * D), np.float32)
    with pytest.raises(b2a.RangeError, match="cannot add 20 more"):
        b2a.attentionPrefillBatch(ctx, c, rope, 1, q, k, k, o, 20, H, 1, 3, dtype="f16", out_dtype="f32")
    with pytest.raises(b2a.B2AError, match="out of range"):
        b2a.attentionPrefillBatch(ctx, c, rope, 1, q, k, k, o, 8, H, 2, 3, dtype="f16", out_dtype="f32")
    c.close()


@pytest.mark.parametrize("in_dtype", ["f16", "bf16"])
def test_batched_prefill_more_units_than_sms(ctx, rope, oracle, monkeypatch, in_dtype):
    """24 sequences of 200 new tokens at ragged cache lengths: 384 CTAs of the
    two-tile kernel (query tile, sequence, head pair), more than one wave on
    the SMs, with partial last tiles in every sequence. The result must carry
    the same bits as one call per sequence (16 CTAs each) and match the oracle;
    the 16-bit output must be the f32 output rounded."""
    monkeypatch.setenv("B2A_PREFILL_TILES", "2")
    count, nseq = 200, 24
    pasts = [(37 * i) % 301 for i in range(nseq)]
    cap = max(pasts) + count
    cfg = b2a.CacheConfig(numLayers=1, numKVHeads=KVH, headDim=D, numHeads=H)
    cb = b2a.GpuKVCache(ctx, cfg, cap, batch=nseq, dtype="f16")
    cs = b2a.GpuKVCache(ctx, cfg, cap, batch=nseq, dtype="f16")
    hk, hv = {}, {}
    for b, L in enumerate(pasts):
        if L:
            kk = oracle.normal_array(L * KVH * D, 700 + b)
            vv = oracle.normal_array(L * KVH * D, 800 + b)
            for c in (cb, cs):
                c.writeAt(0, 0, kk, vv, L, seq=b)
            hk[b], hv[b] = oracle.round_to(kk, "f16"), oracle.round_to(vv, "f16")
    cb.setLengths(pasts)
    cs.setLengths(pasts)
    q = oracle.round_to(oracle.normal_array(nseq * count * H * D, 91), in_dtype).reshape(nseq, count, H * D)
    k = oracle.round_to(oracle.normal_array(nseq * count * KVH * D, 92), in_dtype).reshape(nseq, count, KVH * D)
    v = oracle.round_to(oracle.normal_array(nseq * count * KVH * D, 93), in_dtype).reshape(nseq, count, KVH * D)
    bits = lambda x: oracle.to_bits(x, in_dtype)  # noqa: E731
    ob = np.empty((nseq, count, H * D), np.float32)
    b2a.attentionPrefillBatch(ctx, cb, rope, 0, bits(q), bits(k), bits(v), ob, count, H, 0, nseq, dtype=in_dtype,
                              out_dtype="f32")
    os_ = np.empty_like(ob)
    for i in range(nseq):
        b2a.attentionPrefill(ctx, cs, rope, 0, bits(q[i]), bits(k[i]), bits(v[i]), os_[i], count, H, seq=i,
                             dtype=in_dtype, out_dtype="f32")
    for i in range(nseq):
        assert np.array_equal(ob[i], os_[i]), f"sequence {i} (past {pasts[i]}): batched and single calls differ"
    # 16-bit output (rows past each sequence's tokens left alone): the same
    # values as the f32 output, rounded to nearest even
    cb2 = b2a.GpuKVCache(ctx, cfg, cap, batch=nseq, dtype="f16")
    for b, L in enumerate(pasts):
        if L:
            cb2.writeAt(0, 0, oracle.normal_array(L * KVH * D, 700 + b), oracle.normal_array(L * KVH * D, 800 + b), L,
                        seq=b)
    cb2.setLengths(pasts)
    o16 = np.zeros((nseq, count, H * D), np.uint16)
    b2a.attentionPrefillBatch(ctx, cb2, rope, 0, bits(q), bits(k), bits(v), o16, count, H, 0, nseq, dtype=in_dtype,
                              out_dtype="bf16")
    want = oracle.to_bits(ob.reshape(-1), "bf16").reshape(o16.shape)
    bad = np.argwhere(o16 != want)
    assert len(bad) == 0, f"bf16 output differs from the rounded f32 output at {len(bad)} places, first {bad[:4]}"
    cb2.close()
    for i in (0, 1, nseq - 1):
        past = pasts[i]
        qr = oracle.rope_rows(q[i], range(past, past + count), D, THETA).reshape(-1)
        kr = oracle.round_to(oracle.rope_rows(k[i], range(past, past + count), D, THETA), "f16")
        keys = np.concatenate([hk[i].reshape(past, KVH * D), kr]) if past else kr
        vals = np.concatenate([hv[i].reshape(past, KVH * D), oracle.round_to(v[i], "f16")]) if past else \
            oracle.round_to(v[i], "f16")
        ref = oracle.grouped_attention(qr, keys.reshape(-1), vals.reshape(-1), count, past, H, KVH, D)
        assert_parity(ob[i].reshape(-1), ref, "f32", f"{in_dtype} batched prefill over many units, sequence {i}")
    cb.close()
    cs.close()


@pytest.mark.parametrize("tiles", ["1", "2"])
def test_rotated_queries_from_unaligned_and_f32_rows(ctx, rope, oracle, monkeypatch, tiles):
    """With an f16 cache the append kernel rotates the queries for the
    tensor-core kernels: 16-byte-aligned 16-bit rows by vector loads, rows one
    element off that alignment and f32 rows by other loads. The values are the
    same bf16 numbers in all three, and the rotation rounds to f16 once either
    way, so all three must give the same output bits (and the oracle's
    attention within the tolerance)."""
    import torch
    dev = torch.device("cuda", 0)
    monkeypatch.setenv("B2A_PREFILL_TILES", tiles)
    count = 300
    cfg = b2a.CacheConfig(numLayers=1, numKVHeads=KVH, headDim=D, numHeads=H)
    q = oracle.round_to(oracle.normal_array(count * H * D, 121), "bf16").reshape(count, H * D)
    k = oracle.round_to(oracle.normal_array(count * KVH * D, 122), "bf16").reshape(count, KVH * D)
    v = oracle.round_to(oracle.normal_array(count * KVH * D, 123), "bf16").reshape(count, KVH * D)

    def dev_rows(a, tdt, offset):
        flat = torch.zeros(a.size + offset, dtype=tdt, device=dev)
        flat[offset:] = torch.as_tensor(a.reshape(-1).astype(np.float32)).to(tdt).to(dev)
        return flat[offset:].view(a.shape)

    outs = []
    for tdt, offset in ((torch.bfloat16, 0), (torch.bfloat16, 1), (torch.float32, 0)):
        c = b2a.GpuKVCache(ctx, cfg, count, batch=1, dtype="f16")
        qt, kt, vt = dev_rows(q, tdt, offset), dev_rows(k, tdt, offset), dev_rows(v, tdt, offset)
        assert (qt.data_ptr() % 16 == 0) == (offset == 0)
        out = torch.empty(count, H * D, device=dev)
        b2a.attentionPrefill(ctx, c, rope, 0, qt, kt, vt, out, count, H)
        torch.cuda.synchronize(dev)
        outs.append(out.cpu().numpy())
        c.close()
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), "unaligned 16-bit rows differ"
    assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32)), "f32 rows differ"
    qr = oracle.rope_rows(q, range(count), D, THETA).reshape(-1)
    kr = oracle.round_to(oracle.rope_rows(k, range(count), D, THETA), "f16")
    ref = oracle.grouped_attention(qr, kr.reshape(-1), oracle.round_to(v, "f16").reshape(-1), count, 0, H, KVH, D)
    assert_parity(outs[0].reshape(-1), ref, "f32", f"prefill with rotated queries, {tiles} tile(s) per CTA")
