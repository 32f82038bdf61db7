"""GPU parity: the CUDA kernels (through the C ABI) against the CPU oracle on
the same seeded inputs. Every case restates a reference test or a BASELINE
configuration; see tests/helpers.py for the tolerance."""
import numpy as np
import pytest

import b2a
from helpers import assert_parity

pytestmark = pytest.mark.gpu

H, KVH, D, THETA = 14, 2, 64, 1e6


@pytest.fixture(scope="module")
def ctx():
    c = b2a.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def rope(ctx):
    return b2a.RopeTable(ctx, D, THETA, 40000)


def cfg(layers=1):
    return b2a.CacheConfig(numLayers=layers, numKVHeads=KVH, headDim=D, numHeads=H)


# ---------------------------------------------------------------- drop-in --

@pytest.mark.parametrize("name,shape,seeds", [
    ("attn_kernels_html", (3, 5, 14, 2, 64), (31, 32, 33)),
    ("attn_prefill_s5_p0", (5, 0, 14, 2, 64), (1, 2, 3)),
    ("attn_decode_s1_p11", (1, 11, 14, 2, 64), (99, 100, 101)),
    ("attn_mixed_s3_p7", (3, 7, 14, 2, 64), (4242, 4243, 4244)),
    ("attn_mha_4_4", (4, 2, 4, 4, 8), (1, 2, 3)),
    ("attn_mqa_6_1", (4, 3, 6, 1, 8), (1, 2, 3)),
])
def test_grouped_attention_dropin_matches_golden(ctx, oracle, golden, name, shape, seeds):
    seq, past, nh, nkv, hd = shape
    total = past + seq
    q = oracle.random_array(seq * nh * hd, seeds[0])
    k = oracle.random_array(total * nkv * hd, seeds[1])
    v = oracle.random_array(total * nkv * hd, seeds[2])
    out = np.empty(seq * nh * hd, np.float32)
    b2a.groupedAttention(q, k, v, out, None, dict(seq=seq, past=past, numHeads=nh, numKVHeads=nkv, headDim=hd),
                         ctx=ctx)
    c = assert_parity(out, golden[name], "f32", name)
    # web/kernels.html:351-385 holds the WGSL kernel to 1e-5 relative; so do we.
    assert c["rel"] <= 1e-5, c


def test_dropin_first_position_returns_value(ctx, oracle):
    nh, nkv, hd = 4, 2, 8
    q = oracle.random_array(nh * hd, 21)
    k = oracle.random_array(nkv * hd, 22)
    v = oracle.random_array(nkv * hd, 23)
    out = np.empty(nh * hd, np.float32)
    b2a.groupedAttention(q, k, v, out, None, seq=1, past=0, numHeads=nh, numKVHeads=nkv, headDim=hd, ctx=ctx)
    for h in range(nh):
        g = b2a.kvHeadFor(h, nh, nkv)
        assert np.array_equal(out[h * hd:(h + 1) * hd], v[g * hd:(g + 1) * hd])


def test_dropin_is_causal(ctx, oracle):
    seq, nh, nkv, hd = 4, 4, 2, 8
    q_dim, kv_dim = nh * hd, nkv * hd
    q = oracle.random_array(seq * q_dim, 7)
    k = oracle.random_array(seq * kv_dim, 8)
    v = oracle.random_array(seq * kv_dim, 9)
    shape = dict(seq=seq, past=0, numHeads=nh, numKVHeads=nkv, headDim=hd)
    before = np.empty(seq * q_dim, np.float32)
    b2a.groupedAttention(q, k, v, before, None, shape, ctx=ctx)
    k2, v2 = k.copy(), v.copy()
    k2[(seq - 1) * kv_dim:] += np.float32(3.5)
    v2[(seq - 1) * kv_dim:] -= np.float32(2.25)
    after = np.empty(seq * q_dim, np.float32)
    b2a.groupedAttention(q, k2, v2, after, None, shape, ctx=ctx)
    assert np.array_equal(after[:(seq - 1) * q_dim], before[:(seq - 1) * q_dim])
    assert not np.array_equal(after[(seq - 1) * q_dim:], before[(seq - 1) * q_dim:])


def test_dropin_long_context(ctx, oracle):
    """More keys than one 1024-position chunk: exercises the online rescale."""
    seq, past = 2, 3000
    q = oracle.normal_array(seq * H * D, 41)
    k = oracle.normal_array((past + seq) * KVH * D, 42)
    v = oracle.normal_array((past + seq) * KVH * D, 43)
    out = np.empty(seq * H * D, np.float32)
    b2a.groupedAttention(q, k, v, out, None, seq=seq, past=past, numHeads=H, numKVHeads=KVH, headDim=D, ctx=ctx)
    ref = oracle.grouped_attention(q, k, v, seq, past, H, KVH, D)
    assert_parity(out, ref, "f32", "long context")


# ------------------------------------------------------------------- cache --

def test_cache_bookkeeping_matches_reference(ctx):
    c = b2a.GpuKVCache(ctx, b2a.CacheConfig(2, 2, 8), 3, dtype="f32")
    assert c.length == 0 and c.capacity == 3
    assert c.allocate(3) == 0
    c.commit(3)
    with pytest.raises(b2a.RangeError, match="holds 3 of 3 positions"):
        c.allocate(1)
    assert c.length == 3
    c.reset()
    assert c.length == 0 and c.allocate(3) == 0
    with pytest.raises(b2a.RangeError, match="positive integer"):
        b2a.GpuKVCache(ctx, b2a.CacheConfig(2, 2, 8), 0)


def test_cache_present_transpose(ctx):
    # test/cache.test.js:136-150 with kvDim = 2 heads x head width 8 (kernel minimum), same pattern
    c = b2a.GpuKVCache(ctx, b2a.CacheConfig(2, 2, 8), 2, dtype="f32")
    at = c.allocate(2)
    keys = np.arange(32, dtype=np.float32)
    c.writeAt(0, at, keys, keys, 2)
    c.commit(2)
    k = c.present(0)["key"]
    assert list(k.reshape(-1)) == [*range(0, 8), *range(16, 24), *range(8, 16), *range(24, 32)]


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_append_rope_is_bit_exact(ctx, rope, oracle, dtype):
    """RoPE(K) at absolute positions, rounded to the cache dtype: the stored bytes
    equal the oracle's ropeInPlace (src/core/ops.js:147-158) rounded the same way."""
    layers, cap, past, count = 2, 300, 37, 50
    c = b2a.GpuKVCache(ctx, cfg(layers), cap, dtype=dtype)
    c.setLengths([past])
    k = oracle.normal_array(count * KVH * D, 51) * np.float32(3)
    v = oracle.normal_array(count * KVH * D, 52)
    b2a.appendRope(ctx, c, rope, 1, k, v, count)
    got_k, got_v = c.read(1, past + count)
    ref_k = oracle.rope_rows(k.reshape(count, KVH * D), range(past, past + count), D, THETA)
    ref_k = oracle.to_bits(ref_k.reshape(count, KVH, D).transpose(1, 0, 2), dtype)
    ref_v = oracle.to_bits(v.reshape(count, KVH, D).transpose(1, 0, 2), dtype)
    assert np.array_equal(got_k[:, past:], ref_k)
    assert np.array_equal(got_v[:, past:], ref_v)
    assert not np.any(got_k[:, :past])   # untouched, zero-filled


# ----------------------------------------------------------- config 1 decode --

def _fill_cache(ctx, c, oracle, lengths, layers, dtype, seed):
    """Positions 0..L-1 of every sequence/layer: N(0,1) keys and values, stored as
    already-rotated cache contents (the cache holds post-RoPE keys)."""
    hk, hv = {}, {}
    for b, L in enumerate(lengths):
        for layer in range(layers):
            kk = oracle.normal_array(L * KVH * D, seed + 1000 * b + 10 * layer)
            vv = oracle.normal_array(L * KVH * D, seed + 1000 * b + 10 * layer + 1)
            c.writeAt(layer, 0, kk, vv, L, seq=b)
            hk[b, layer] = oracle.round_to(kk, dtype).reshape(L, KVH, D).transpose(1, 0, 2)
            hv[b, layer] = oracle.round_to(vv, dtype).reshape(L, KVH, D).transpose(1, 0, 2)
    c.setLengths(lengths)
    return hk, hv


def _oracle_decode(oracle, q, kn, vn, hk, hv, L, dtype):
    """src/cpu/model.js:103-123 for one token at position L over a cache holding
    hk/hv (head-major, already rounded). Returns (out [H*D], new K row, new V row)."""
    qr = oracle.rope_rows(q.reshape(1, H * D), [L], D, THETA).reshape(-1)
    kr = oracle.rope_rows(kn.reshape(1, KVH * D), [L], D, THETA).reshape(KVH, D)
    kr = oracle.round_to(kr, dtype)
    vr = oracle.round_to(vn.reshape(KVH, D), dtype)
    kc = np.concatenate([hk, kr[:, None, :]], axis=1)
    vc = np.concatenate([hv, vr[:, None, :]], axis=1)
    out = oracle.decode_head_major(qr, np.ascontiguousarray(kc), np.ascontiguousarray(vc), L + 1, L, H, KVH, D)
    return out, kr, vr


def test_config1_decode_f32(ctx, rope, oracle):
    """batch 1, 14/2 heads, D 64, cache positions 0..127, new token at 128, f32."""
    L = 128
    c = b2a.GpuKVCache(ctx, cfg(1), 256, dtype="f32")
    hk, hv = _fill_cache(ctx, c, oracle, [L], 1, "f32", 100)
    q = oracle.normal_array(H * D, 1)
    kn = oracle.normal_array(KVH * D, 2)
    vn = oracle.normal_array(KVH * D, 3)
    out = np.empty((1, 1, H, D), np.float32)
    b2a.attentionDecode(ctx, c, rope, 0, q.reshape(1, 1, H, D), kn.reshape(1, 1, KVH, D), vn.reshape(1, 1, KVH, D),
                        out, H)
    ref, kr, vr = _oracle_decode(oracle, q, kn, vn, hk[0, 0], hv[0, 0], L, "f32")
    assert_parity(out, ref, "f32", "config 1")
    gk, gv = c.read(0, L + 1)
    assert np.array_equal(gk[:, L], oracle.to_bits(kr, "f32"))
    assert np.array_equal(gv[:, L], oracle.to_bits(vr, "f32"))
    assert c.length == L   # not advanced until commit


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_batched_decode_multilayer(ctx, rope, oracle, dtype):
    """BASELINE config 3, scaled down: independent sequences of different lengths,
    several layers in one call, RoPE at each sequence's own position."""
    rng = np.random.default_rng(7)
    batch, layers = 6, 3
    lengths = [int(x) for x in rng.integers(1, 1500, size=batch)]
    lengths[0] = 1
    lengths[1] = 256
    c = b2a.GpuKVCache(ctx, cfg(layers), 1600, batch=batch, dtype=dtype)
    hk, hv = _fill_cache(ctx, c, oracle, lengths, layers, dtype, 300)
    q = oracle.round_to(oracle.normal_array(batch * layers * H * D, 5), dtype).reshape(batch, layers, H, D)
    kn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 6), dtype).reshape(batch, layers, KVH, D)
    vn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 7), dtype).reshape(batch, layers, KVH, D)
    out = np.empty((batch, layers, H, D), np.float32)
    b2a.attentionDecode(ctx, c, rope, 0, oracle.to_bits(q, dtype), oracle.to_bits(kn, dtype),
                        oracle.to_bits(vn, dtype), out, H, numLayers=layers, dtype=dtype)
    for b in range(batch):
        for layer in range(layers):
            ref, kr, vr = _oracle_decode(oracle, q[b, layer], kn[b, layer], vn[b, layer], hk[b, layer],
                                         hv[b, layer], lengths[b], dtype)
            assert_parity(out[b, layer].reshape(-1), ref, "f32", f"seq {b} layer {layer}")
            gk, gv = c.read(layer, lengths[b] + 1, seq=b)
            assert np.array_equal(gk[:, lengths[b]], oracle.to_bits(kr, dtype))
            assert np.array_equal(gv[:, lengths[b]], oracle.to_bits(vr, dtype))


@pytest.mark.parametrize("batch,length", [(8, 4000), (8, 9000), (2, 20000)])
def test_uniform_long_decode_equal_chunks(ctx, rope, oracle, batch, length):
    """BASELINE config 5 shapes, scaled down: sequences of equal length are cut
    into equal chunks that fill the resident CTAs once; up to 32 chunks per
    group are merged inside the attention kernel, more by the combine kernel."""
    c = b2a.GpuKVCache(ctx, cfg(1), length + 1, batch=batch, dtype="f16")
    hk, hv = _fill_cache(ctx, c, oracle, [length] * batch, 1, "f16", 500)
    q = oracle.round_to(oracle.normal_array(batch * H * D, 8), "f16").reshape(batch, 1, H, D)
    kn = oracle.round_to(oracle.normal_array(batch * KVH * D, 9), "f16").reshape(batch, 1, KVH, D)
    vn = oracle.round_to(oracle.normal_array(batch * KVH * D, 10), "f16").reshape(batch, 1, KVH, D)
    out = np.empty((batch, 1, H, D), np.float32)
    b2a.attentionDecode(ctx, c, rope, 0, oracle.to_bits(q, "f16"), oracle.to_bits(kn, "f16"),
                        oracle.to_bits(vn, "f16"), out, H, dtype="f16")
    for b in range(batch):
        ref, _, _ = _oracle_decode(oracle, q[b, 0], kn[b, 0], vn[b, 0], hk[b, 0], hv[b, 0], length, "f16")
        assert_parity(out[b, 0].reshape(-1), ref, "f32", f"seq {b} of {batch} x {length}")


@pytest.mark.parametrize("cache_dtype,in_dtype", [("f16", "f16"), ("f16", "f32"), ("bf16", "bf16"), ("bf16", "f32")])
def test_decode_device_inputs_aligned_and_unaligned(ctx, rope, oracle, cache_dtype, in_dtype):
    """Device-resident q / k_new / v_new. 16-byte-aligned blocks reach the tensor-core decode
    kernel's shared memory by bulk copies, and the CTA holding the new token's slot writes the
    appended row to the cache and patches it into the tile it streams; blocks one element off
    that alignment take per-element loads with the append done before the stream. Both forms
    give the same output bits and cache bytes, and both match the oracle (slots at a tile's
    last row, at a tile's first row, and in the last chunk of a many-chunk group)."""
    import torch
    dev = torch.device("cuda", 0)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[in_dtype]
    batch, layers = 3, 2
    lengths = [703, 64, 9000]
    caches, hist = [], None
    for _ in range(2):
        c = b2a.GpuKVCache(ctx, cfg(layers), 9100, batch=batch, dtype=cache_dtype)
        hist = _fill_cache(ctx, c, oracle, lengths, layers, cache_dtype, 900)
        caches.append(c)
    hk, hv = hist
    q = oracle.round_to(oracle.normal_array(batch * layers * H * D, 11), in_dtype).reshape(batch, layers, H, D)
    kn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 12), in_dtype).reshape(batch, layers, KVH, D)
    vn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 13), in_dtype).reshape(batch, layers, KVH, D)

    def dev_tensor(a, offset):
        flat = torch.zeros(a.size + offset, dtype=tdt, device=dev)
        flat[offset:] = torch.as_tensor(a.reshape(-1).astype(np.float32)).to(tdt).to(dev)
        return flat[offset:].view(a.shape)

    outs = []
    for c, off in zip(caches, (0, 1)):
        qt, kt, vt = dev_tensor(q, off), dev_tensor(kn, off), dev_tensor(vn, off)
        assert (qt.data_ptr() % 16 == 0) == (off == 0)
        out = torch.empty(batch, layers, H, D, device=dev)
        b2a.attentionDecode(ctx, c, rope, 0, qt, kt, vt, out, H, numLayers=layers)
        torch.cuda.synchronize(dev)
        outs.append(out.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    for b in range(batch):
        for layer in range(layers):
            ref, kr, vr = _oracle_decode(oracle, q[b, layer], kn[b, layer], vn[b, layer], hk[b, layer],
                                         hv[b, layer], lengths[b], cache_dtype)
            assert_parity(outs[0][b, layer].reshape(-1), ref, "f32", f"seq {b} layer {layer}")
            for c in caches:
                gk, gv = c.read(layer, lengths[b] + 1, seq=b)
                assert np.array_equal(gk[:, lengths[b]], oracle.to_bits(kr, cache_dtype))
                assert np.array_equal(gv[:, lengths[b]], oracle.to_bits(vr, cache_dtype))
    for c in caches:
        c.close()


# ---------------------------------------------------------- config 2 prefill --

@pytest.mark.parametrize("S", [8, 64, 512])
def test_config2_prefill_bf16(ctx, rope, oracle, S):
    """causal prefill, bf16 Q/K/V N(0,1), RoPE at 0..S-1, bf16 out."""
    q = oracle.round_to(oracle.normal_array(S * H * D, 11), "bf16")
    k = oracle.round_to(oracle.normal_array(S * KVH * D, 12), "bf16")
    v = oracle.round_to(oracle.normal_array(S * KVH * D, 13), "bf16")
    c = b2a.GpuKVCache(ctx, cfg(1), S, dtype="bf16")
    out = np.empty(S * H * D, np.uint16)
    b2a.attentionPrefill(ctx, c, rope, 0, oracle.to_bits(q, "bf16"), oracle.to_bits(k, "bf16"),
                         oracle.to_bits(v, "bf16"), out, S, H, dtype="bf16")
    # the oracle on the same inputs; its cache is f32, so K is rounded to bf16
    # in the cache the way the kernel stores it, before attention reads it
    qr = oracle.rope_rows(q.reshape(S, H * D), range(S), D, THETA).reshape(-1)
    kr = oracle.round_to(oracle.rope_rows(k.reshape(S, KVH * D), range(S), D, THETA), "bf16").reshape(-1)
    ref = oracle.grouped_attention(qr, kr, v, S, 0, H, KVH, D)
    got = oracle.from_bits(out, "bf16")
    assert_parity(got, ref, "bf16", f"prefill S={S}")
    gk, _ = c.read(0, S)
    assert np.array_equal(gk, oracle.to_bits(kr.reshape(S, KVH, D).transpose(1, 0, 2), "bf16"))


@pytest.mark.parametrize("cache_dtype,splits,tiles", [
    ("f16", [8], 2), ("f16", [130], 2), ("f16", [512], 2), ("f16", [2048], 2), ("f16", [300, 200, 1], 2),
    ("f16", [8], 1), ("f16", [130], 1), ("f16", [512], 1), ("f16", [300, 200, 1], 1),
    ("bf16", [8], 1), ("bf16", [130], 1), ("bf16", [1000], 1), ("bf16", [129, 257], 1),
])
def test_prefill_tensor_core(ctx, rope, oracle, monkeypatch, cache_dtype, splits, tiles):
    """Causal prefill through the tcgen05 kernels: bf16 Q/K/V,
    K/V cached as f16 (bf16 values are exact in f16) or bf16; several calls in a
    row continue one sequence (chunked prefill, past > 0). tiles: query tiles per
    CTA, forced with B2A_PREFILL_TILES (by default f16 caches take the two-head
    kernel once there are two CTAs per SM, bf16 caches the one-tile kernel)."""
    monkeypatch.setenv("B2A_PREFILL_TILES", str(tiles))
    n = sum(splits)
    q = oracle.round_to(oracle.normal_array(n * H * D, 71), "bf16").reshape(n, H * D)
    k = oracle.round_to(oracle.normal_array(n * KVH * D, 72), "bf16").reshape(n, KVH * D)
    v = oracle.round_to(oracle.normal_array(n * KVH * D, 73), "bf16").reshape(n, KVH * D)
    c = b2a.GpuKVCache(ctx, cfg(1), n, dtype=cache_dtype)
    outs = []
    t0 = 0
    for s in splits:
        c.allocate(s)
        o = np.empty(s * H * D, np.uint16)
        b2a.attentionPrefill(ctx, c, rope, 0, oracle.to_bits(q[t0:t0 + s], "bf16"),
                             oracle.to_bits(k[t0:t0 + s], "bf16"), oracle.to_bits(v[t0:t0 + s], "bf16"), o, s, H,
                             dtype="bf16")
        outs.append(oracle.from_bits(o, "bf16"))
        c.commit(s)
        t0 += s
    got = np.concatenate(outs)
    qr = oracle.rope_rows(q, range(n), D, THETA).reshape(-1)
    kr = oracle.round_to(oracle.rope_rows(k, range(n), D, THETA), cache_dtype).reshape(-1)
    ref = oracle.grouped_attention(qr, kr, oracle.round_to(v, cache_dtype), n, 0, H, KVH, D)
    assert_parity(got, ref, "bf16", f"{cache_dtype} prefill {splits}")
    gk, gv = c.read(0, n)
    assert np.array_equal(gk, oracle.to_bits(kr.reshape(n, KVH, D).transpose(1, 0, 2), cache_dtype))
    assert np.array_equal(gv, oracle.to_bits(v.reshape(n, KVH, D).transpose(1, 0, 2), cache_dtype))


@pytest.mark.parametrize("nh,nkv,in_dt,out_dt,n", [
    (2, 2, "bf16", "bf16", 300),   # group 1: one head per CTA
    (4, 2, "f16", "f16", 257),     # group 2: one full pair
    (6, 2, "f32", "f32", 200),     # group 3: a pair and a single head; f32 staging path
    (8, 1, "bf16", "f32", 129),    # one KV head, group 8
])
def test_prefill_pairs_over_group_shapes(ctx, rope, oracle, monkeypatch, nh, nkv, in_dt, out_dt, n):
    """The two-head prefill kernel pairs the query heads of each KV group (an odd
    group leaves one head alone): other group sizes, input and output dtypes."""
    monkeypatch.setenv("B2A_PREFILL_TILES", "2")
    q = oracle.normal_array(n * nh * D, 81).reshape(n, nh * D)
    k = oracle.normal_array(n * nkv * D, 82).reshape(n, nkv * D)
    v = oracle.normal_array(n * nkv * D, 83).reshape(n, nkv * D)
    if in_dt != "f32":
        q, k, v = (oracle.round_to(x, in_dt) for x in (q, k, v))
    c = b2a.GpuKVCache(ctx, b2a.CacheConfig(numLayers=1, numKVHeads=nkv, headDim=D, numHeads=nh), n, dtype="f16")
    c.allocate(n)
    wrap = (lambda x: x.astype(np.float32)) if in_dt == "f32" else (lambda x: oracle.to_bits(x, in_dt))
    o = np.empty(n * nh * D, np.float32 if out_dt == "f32" else np.uint16)
    b2a.attentionPrefill(ctx, c, rope, 0, wrap(q), wrap(k), wrap(v), o, n, nh, dtype=in_dt,
                         out_dtype=out_dt)
    got = o if out_dt == "f32" else oracle.from_bits(o, out_dt)
    qr = oracle.rope_rows(q, range(n), D, THETA).reshape(-1)
    kr = oracle.round_to(oracle.rope_rows(k, range(n), D, THETA), "f16").reshape(-1)
    ref = oracle.grouped_attention(qr, kr, oracle.round_to(v, "f16"), n, 0, nh, nkv, D)
    assert_parity(got, ref, out_dt, f"prefill pairs nh={nh} nkv={nkv} {in_dt}->{out_dt}")


@pytest.mark.parametrize("splits", [[40], [1] * 12 + [28], [17, 1, 22]])
def test_incremental_equals_full_recompute(ctx, rope, oracle, splits):
    """validate/phase2.js:83-121 on synthetic projections: prefill in one call,
    in chunks, or token by token gives the same cache bits and outputs within
    the tolerance."""
    n = sum(splits)
    q = oracle.normal_array(n * H * D, 61).reshape(n, H * D)
    k = oracle.normal_array(n * KVH * D, 62).reshape(n, KVH * D)
    v = oracle.normal_array(n * KVH * D, 63).reshape(n, KVH * D)
    c = b2a.GpuKVCache(ctx, cfg(1), n, dtype="f32")
    outs = []
    t0 = 0
    for s in splits:
        c.allocate(s)
        o = np.empty(s * H * D, np.float32)
        if s == 1:
            b2a.attentionDecode(ctx, c, rope, 0, q[t0].reshape(1, 1, H, D), k[t0].reshape(1, 1, KVH, D),
                                v[t0].reshape(1, 1, KVH, D), o.reshape(1, 1, H, D), H)
        else:
            b2a.attentionPrefill(ctx, c, rope, 0, q[t0:t0 + s], k[t0:t0 + s], v[t0:t0 + s], o, s, H)
        outs.append(o)
        c.commit(s)
        t0 += s
    got = np.concatenate(outs)
    oc = oracle.OracleKVCache(1, KVH * D, n)
    oc.allocate(n)
    ref, _, kr = oc.layer_attention(0, q, k, v, n, H, KVH, D, THETA)
    assert_parity(got, ref, "f32", f"splits {splits}")
    gk, gv = c.read(0, n)
    assert np.array_equal(gk, kr.reshape(n, KVH, D).transpose(1, 0, 2))
    assert np.array_equal(gv, v.reshape(n, KVH, D).transpose(1, 0, 2))


# ------------------------------------------------------- split-KV partials --

def test_split_kv_partials_combine_to_full_decode(ctx, rope, oracle):
    """BASELINE config 5, scaled down: the KV sequence split into parts held by
    separate caches (as separate ranks would), partials combined in order."""
    batch, L, parts = 3, 2500, 3
    dtype = "f16"
    chunk = (L + parts - 1) // parts
    kfull = [oracle.round_to(oracle.normal_array(L * KVH * D, 900 + b), dtype).reshape(L, KVH, D) for b in range(batch)]
    vfull = [oracle.round_to(oracle.normal_array(L * KVH * D, 950 + b), dtype).reshape(L, KVH, D) for b in range(batch)]
    q = oracle.round_to(oracle.normal_array(batch * H * D, 31), dtype).reshape(batch, H, D)
    kn = oracle.round_to(oracle.normal_array(batch * KVH * D, 32), dtype).reshape(batch, KVH, D)
    vn = oracle.round_to(oracle.normal_array(batch * KVH * D, 33), dtype).reshape(batch, KVH, D)
    pos = np.full(batch, L, np.int32)
    partials = np.empty((parts, batch, H, D + 4), np.float32)
    for r in range(parts):
        lo, hi = r * chunk, min(L, (r + 1) * chunk)
        last = r == parts - 1
        c = b2a.GpuKVCache(ctx, cfg(1), (hi - lo) + 1, batch=batch, dtype=dtype)
        for b in range(batch):
            c.writeAt(0, 0, oracle.to_bits(kfull[b][lo:hi], dtype), oracle.to_bits(vfull[b][lo:hi], dtype),
                      hi - lo, seq=b, dtype=dtype)
        c.setLengths([hi - lo] * batch)
        b2a.decodePartial(ctx, c, rope, 0, oracle.to_bits(q, dtype),
                          oracle.to_bits(kn, dtype) if last else None, oracle.to_bits(vn, dtype) if last else None,
                          pos, partials[r], H, dtype=dtype)
    out = np.empty((batch, H, D), np.float32)
    b2a.lseCombine(ctx, partials, parts, batch, H, D, out)
    for b in range(batch):
        ref, _, _ = _oracle_decode(oracle, q[b], kn[b], vn[b], np.ascontiguousarray(kfull[b].transpose(1, 0, 2)),
                                   np.ascontiguousarray(vfull[b].transpose(1, 0, 2)), L, dtype)
        assert_parity(out[b].reshape(-1), ref, "f32", f"split seq {b}")


def test_split_kv_nccl_call_single_rank(ctx, rope, oracle):
    """b2a_split_kv_decode_nccl through a one-rank NCCL communicator: the partials,
    the in-place ncclAllGather and the combine in one call, over two layers; two
    steps in a row (new q/k/v each), checked against the oracle, with the appended
    rows bit for bit."""
    import torch
    from b2a import dist
    dev = torch.device("cuda", 0)
    batch, L, layers = 3, 1500, 2
    c = b2a.GpuKVCache(ctx, cfg(layers), L + 1, batch=batch, dtype="f16")
    hk, hv = _fill_cache(ctx, c, oracle, [L] * batch, layers, "f16", 700)
    comm = dist.NcclComm.single(0)
    try:
        split = dist.NcclSplitKV(ctx, c, rope, 0, H, comm, num_layers=layers)
        pos = torch.full((batch,), L, dtype=torch.int32, device=dev)
        for step in range(2):
            q = oracle.round_to(oracle.normal_array(batch * layers * H * D, 40 + step), "f16")
            kn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 50 + step), "f16")
            vn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 60 + step), "f16")
            qt = torch.as_tensor(q).to(dev).half().view(batch, layers, H, D)
            kt = torch.as_tensor(kn).to(dev).half().view(batch, layers, KVH, D)
            vt = torch.as_tensor(vn).to(dev).half().view(batch, layers, KVH, D)
            out = torch.empty(batch, layers, H, D, device=dev)
            torch.cuda.synchronize(dev)
            split.step(qt, kt, vt, pos, out)
            ctx.synchronize()
            got = out.cpu().numpy()
            q4, k4, v4 = (q.reshape(batch, layers, H, D), kn.reshape(batch, layers, KVH, D),
                          vn.reshape(batch, layers, KVH, D))
            for b in range(batch):
                for layer in range(layers):
                    ref, kr, vr = _oracle_decode(oracle, q4[b, layer], k4[b, layer], v4[b, layer], hk[b, layer],
                                                 hv[b, layer], L, "f16")
                    assert_parity(got[b, layer].reshape(-1), ref, "f32", f"step {step} seq {b} layer {layer}")
                    gk, gv = c.read(layer, L + 1, seq=b)
                    assert np.array_equal(gk[:, L], oracle.to_bits(kr, "f16"))
                    assert np.array_equal(gv[:, L], oracle.to_bits(vr, "f16"))
        # argument errors come back before any device work
        with pytest.raises(b2a.B2AError):   # host arrays: the call takes device pointers only
            b2a.decodeSplitNccl(ctx, c, rope, 0, q.reshape(batch, layers, H, D), None, None, np.full(batch, L, np.int32),
                                comm, 1, 0, np.empty((batch, layers, H, D), np.float32), H, numLayers=layers,
                                dtype="f16")
        with pytest.raises(b2a.B2AError):   # a rank outside the world
            b2a.decodeSplitNccl(ctx, c, rope, 0, qt, None, None, pos, comm, 1, 1, out, H, numLayers=layers)
    finally:
        comm.close()
        c.close()


def test_split_exchange_single_rank_matches_decode(ctx, rope, oracle):
    """The in-kernel exchange path with one rank: the group partials go through
    the exchange buffer and flags of this GPU only, and the output equals the
    full decode (several steps, so both buffer parities are used)."""
    batch, L, dtype = 4, 1500, "f16"
    c = b2a.GpuKVCache(ctx, cfg(1), L + 1, batch=batch, dtype=dtype)
    hk, hv = _fill_cache(ctx, c, oracle, [L] * batch, 1, dtype, 700)
    q = oracle.round_to(oracle.normal_array(batch * H * D, 41), dtype).reshape(batch, H, D)
    kn = oracle.round_to(oracle.normal_array(batch * KVH * D, 42), dtype).reshape(batch, KVH, D)
    vn = oracle.round_to(oracle.normal_array(batch * KVH * D, 43), dtype).reshape(batch, KVH, D)
    ex = b2a.Exchange(ctx, 1, 0, batch, H, KVH)
    outs = []
    for _ in range(3):
        out = np.empty((batch, H, D), np.float32)
        b2a.decodeSplit(ctx, c, rope, 0, oracle.to_bits(q, dtype), oracle.to_bits(kn, dtype),
                        oracle.to_bits(vn, dtype), np.full(batch, L, np.int32), ex, out, H, dtype=dtype)
        outs.append(out)
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    for b in range(batch):
        ref, _, _ = _oracle_decode(oracle, q[b], kn[b], vn[b], hk[b, 0], hv[b, 0], L, dtype)
        assert_parity(outs[0][b].reshape(-1), ref, "f32", f"exchange seq {b}")
    ex.close()


def test_split_exchange_single_rank_several_layers(ctx, rope, oracle):
    """Several layers per call (b2a_attention_decode_split_layers and
    b2a_attention_decode_partial_layers): one exchange covers every (sequence,
    layer, KV head) group of the call; both paths against the oracle."""
    batch, layers, L, dtype = 3, 3, 1500, "f16"
    c = b2a.GpuKVCache(ctx, cfg(layers), L + 1, batch=batch, dtype=dtype)
    hk, hv = _fill_cache(ctx, c, oracle, [L] * batch, layers, dtype, 720)
    q = oracle.round_to(oracle.normal_array(batch * layers * H * D, 45), dtype).reshape(batch, layers, H, D)
    kn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 46), dtype).reshape(batch, layers, KVH, D)
    vn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 47), dtype).reshape(batch, layers, KVH, D)
    pos = np.full(batch, L, np.int32)
    ex = b2a.Exchange(ctx, 1, 0, batch, H, KVH, numLayers=layers)
    out = np.empty((batch, layers, H, D), np.float32)
    for _ in range(2):
        b2a.decodeSplit(ctx, c, rope, 0, oracle.to_bits(q, dtype), oracle.to_bits(kn, dtype),
                        oracle.to_bits(vn, dtype), pos, ex, out, H, dtype=dtype, numLayers=layers)
    partial = np.empty((batch, layers, H, D + 4), np.float32)
    b2a.decodePartial(ctx, c, rope, 0, oracle.to_bits(q, dtype), oracle.to_bits(kn, dtype), oracle.to_bits(vn, dtype),
                      pos, partial, H, dtype=dtype, numLayers=layers)
    comb = np.empty((batch, layers, H, D), np.float32)
    b2a.lseCombine(ctx, partial, 1, batch * layers, H, D, comb)
    for b in range(batch):
        for layer in range(layers):
            ref, _, _ = _oracle_decode(oracle, q[b, layer], kn[b, layer], vn[b, layer], hk[b, layer], hv[b, layer],
                                       L, dtype)
            assert_parity(out[b, layer].reshape(-1), ref, "f32", f"exchange seq {b} layer {layer}")
            assert_parity(comb[b, layer].reshape(-1), ref, "f32", f"partials seq {b} layer {layer}")
    with pytest.raises(b2a.B2AError):   # an exchange made for 3 layers refuses a 1-layer call
        b2a.decodeSplit(ctx, c, rope, 0, oracle.to_bits(q[:, 0], dtype), None, None, pos, ex,
                        np.empty((batch, H, D), np.float32), H, dtype=dtype)
    ex.close()


def test_split_exchange_wait_gives_up_with_error(ctx, rope, oracle):
    """A rank whose peer never arrives: rank 0 of a two-rank exchange whose
    rank 1 is a second exchange object that no kernel ever serves. The kernel's
    wait on rank 1's flag gives up after about a second, the call reports
    B2A_ETIMEDOUT, and the context keeps working."""
    import time
    batch, L, dtype = 2, 300, "f16"
    c = b2a.GpuKVCache(ctx, cfg(1), L + 1, batch=batch, dtype=dtype)
    _fill_cache(ctx, c, oracle, [L] * batch, 1, dtype, 710)
    q = oracle.to_bits(oracle.normal_array(batch * H * D, 44).reshape(batch, H, D), dtype)
    ex0 = b2a.Exchange(ctx, 2, 0, batch, H, KVH)
    ex1 = b2a.Exchange(ctx, 2, 1, batch, H, KVH)
    ex0.connect_local(1, ex1)
    out = np.empty((batch, H, D), np.float32)
    t0 = time.monotonic()
    with pytest.raises(b2a.B2AError) as err:
        b2a.decodeSplit(ctx, c, rope, 0, q, None, None, np.full(batch, L, np.int32), ex0, out, H, dtype=dtype)
    assert err.value.status == 6, err.value   # B2A_ETIMEDOUT
    assert time.monotonic() - t0 < 30
    ex0.close()
    ex1.close()
    # the context and cache still serve ordinary calls
    o2 = np.empty((batch, 1, H, D), np.float32)
    b2a.attentionDecode(ctx, c, rope, 0, q.reshape(batch, 1, H, D), None, None, o2, H, dtype=dtype)
    assert np.isfinite(o2).all()


def test_host_pipelined_decode_matches_device_path(ctx, rope, oracle):
    """The host-pointer decode splits the batch into groups whose uploads,
    kernels and downloads overlap; its output equals the device-pointer call's."""
    import torch
    batch, layers, cap = 32, 24, 700
    c = b2a.GpuKVCache(ctx, cfg(layers), cap, batch=batch, dtype="f16")
    dev = torch.device("cuda", 0)
    kp, vp, _ = c.pools()
    g = torch.Generator(device=dev)
    g.manual_seed(9)

    class _CAI:
        def __init__(self, ptr, shape):
            self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f2", "data": (ptr, False), "version": 3}

    torch.as_tensor(_CAI(kp, (batch, layers, KVH, cap, D)), device=dev).normal_(generator=g)
    torch.as_tensor(_CAI(vp, (batch, layers, KVH, cap, D)), device=dev).normal_(generator=g)
    torch.cuda.synchronize(dev)
    rng = np.random.default_rng(2)
    c.setLengths(rng.integers(1, cap - 1, size=batch).astype(np.int32))
    q = torch.randn(batch, layers, H, D, device=dev, generator=g).half()
    kn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    vn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
    out_dev = torch.empty(batch, layers, H, D, device=dev)
    b2a.attentionDecode(ctx, c, rope, 0, q, kn, vn, out_dev, H, numLayers=layers)
    ctx.synchronize()
    qh, knh, vnh = q.cpu().pin_memory(), kn.cpu().pin_memory(), vn.cpu().pin_memory()
    out_host = torch.empty(batch, layers, H, D).pin_memory()
    for _ in range(2):
        b2a.attentionDecode(ctx, c, rope, 0, qh, knh, vnh, out_host, H, numLayers=layers)
        diff = (out_host - out_dev.cpu()).abs().max().item()
        assert diff < 1e-4, diff


@pytest.mark.parametrize("layers", [24, 1])
def test_host_async_decode_matches_device_path(ctx, rope, oracle, layers):
    """Host-pointer decode calls that return before their results are back
    (b2a_attention_decode_host_async): four calls in flight with different
    inputs and output buffers, one synchronisation, then every output equals
    the device-pointer call's on the same inputs."""
    import torch
    batch, cap = 32, 700
    c = b2a.GpuKVCache(ctx, cfg(layers), cap, batch=batch, dtype="f16")
    dev = torch.device("cuda", 0)
    kp, vp, _ = c.pools()
    g = torch.Generator(device=dev)
    g.manual_seed(19)

    class _CAI:
        def __init__(self, ptr, shape):
            self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f2", "data": (ptr, False), "version": 3}

    torch.as_tensor(_CAI(kp, (batch, layers, KVH, cap, D)), device=dev).normal_(generator=g)
    torch.as_tensor(_CAI(vp, (batch, layers, KVH, cap, D)), device=dev).normal_(generator=g)
    torch.cuda.synchronize(dev)
    c.setLengths(np.random.default_rng(3).integers(1, cap - 1, size=batch).astype(np.int32))
    steps = []
    for i in range(4):
        q = torch.randn(batch, layers, H, D, device=dev, generator=g).half()
        kn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
        vn = torch.randn(batch, layers, KVH, D, device=dev, generator=g).half()
        ref = torch.empty(batch, layers, H, D, device=dev)
        b2a.attentionDecode(ctx, c, rope, 0, q, kn, vn, ref, H, numLayers=layers)
        steps.append((q.cpu().pin_memory(), kn.cpu().pin_memory(), vn.cpu().pin_memory(),
                      torch.full((batch, layers, H, D), float("nan")).pin_memory(), ref))
    ctx.synchronize()
    for qh, knh, vnh, outh, _ in steps:
        b2a.attentionDecodeAsync(ctx, c, rope, 0, qh, knh, vnh, outh, H, numLayers=layers)
    ctx.synchronize()
    for i, (_, _, _, outh, ref) in enumerate(steps):
        diff = (outh - ref.cpu()).abs().max().item()
        assert diff < 1e-4, (i, diff)
    c.close()
