"""GPU parity at the sizes bench.py measures, against the CPU oracle.

The other parity tests run scaled-down shapes; these run the benchmark's own
workloads through the same calls and check sampled rows against the oracle's
restatement of src/core/attention.js:32-66 (decode: src/cpu/model.js:103-123):

- BASELINE config 3 as bench.py builds it: 64 sequences x 24 layers, lengths
  U{256..4096} from bench.py's generator, one b2a_attention_decode call; 16
  (sequence, layer) rows including every layer's extremes of the longest and
  the shortest sequence, plus the appended key rows bit for bit.
- BASELINE config 5 on one GPU: 8 sequences x 32768 cached positions, every
  sequence checked.
- Causal prefill through the f16-cache path the benchmark times (bf16 Q/K/V,
  bf16 out) against the oracle run on an f32 cache, as the reference keeps
  it: rotated keys are NOT rounded to the cache dtype on the oracle side
  (src/cpu/cache.js:63-67, src/cpu/model.js:107-123). Config 2's S = 8, 64,
  512, 2048 are checked in full; S = 16384 (the prefill roofline point) at
  query rows of the first, middle and last tiles. The cache bytes must equal
  the oracle's rotated keys rounded to f16, bit for bit.
"""
import numpy as np
import pytest

import b2a
from helpers import assert_parity, check_decode_rows

pytestmark = pytest.mark.gpu

H, KVH, D, THETA = 14, 2, 64, 1e6


class _CAI:
    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f2", "data": (ptr, False),
                                         "version": 3}


@pytest.fixture(scope="module")
def env():
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = b2a.Context(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    yield torch, dev, ctx, stream
    ctx.close()


def test_config3_full_step(env, oracle):
    import bench
    torch, dev, ctx, stream = env
    seqs, layers, cap = bench.SEQS, bench.LAYERS, bench.CAP
    assert (seqs, layers) == (64, 24)
    lengths = bench.config3_lengths(0)
    with torch.cuda.stream(stream):
        cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), cap, batch=seqs, dtype="f16")
        rope = b2a.RopeTable(ctx, D, THETA, 32769)
        kp, vp, _ = cache.pools()
        gen = torch.Generator(device=dev)
        gen.manual_seed(4321)
        torch.as_tensor(_CAI(kp, (seqs, layers, KVH, cap, D)), device=dev).normal_(generator=gen)
        torch.as_tensor(_CAI(vp, (seqs, layers, KVH, cap, D)), device=dev).normal_(generator=gen)
        cache.setLengths(lengths)
        q = torch.randn(seqs, layers, H, D, device=dev, generator=gen).half()
        kn = torch.randn(seqs, layers, KVH, D, device=dev, generator=gen).half()
        vn = torch.randn(seqs, layers, KVH, D, device=dev, generator=gen).half()
        out = torch.full((seqs, layers, H, D), float("nan"), device=dev)
    torch.cuda.synchronize(dev)
    b2a.attentionDecode(ctx, cache, rope, 0, q, kn, vn, out, H, numLayers=layers)
    ctx.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    longest, shortest = int(np.argmax(lengths)), int(np.argmin(lengths))
    rng = np.random.default_rng(11)
    picks = [(longest, 0), (longest, layers - 1), (shortest, 0), (shortest, layers - 1)]
    while len(picks) < 16:
        p = (int(rng.integers(seqs)), int(rng.integers(layers)))
        if p not in picks:
            picks.append(p)
    check_decode_rows(oracle, cache, q.float().cpu().numpy(), lengths, picks, got, "f16",
                      kn=kn.float().cpu().numpy(), what="config 3")
    cache.close()
    rope.close()


def test_config5_full_context_one_gpu(env, oracle):
    torch, dev, ctx, stream = env
    nseq, total = 8, 32768
    with torch.cuda.stream(stream):
        cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(1, KVH, D, H), total + 1, batch=nseq, dtype="f16")
        rope = b2a.RopeTable(ctx, D, THETA, total + 1)
        kp, vp, _ = cache.pools()
        gen = torch.Generator(device=dev)
        gen.manual_seed(777)
        torch.as_tensor(_CAI(kp, (nseq, 1, KVH, total + 1, D)), device=dev).normal_(generator=gen)
        torch.as_tensor(_CAI(vp, (nseq, 1, KVH, total + 1, D)), device=dev).normal_(generator=gen)
        cache.setLengths([total] * nseq)
        q = torch.randn(nseq, 1, H, D, device=dev, generator=gen).half()
        kn = torch.randn(nseq, 1, KVH, D, device=dev, generator=gen).half()
        vn = torch.randn(nseq, 1, KVH, D, device=dev, generator=gen).half()
        out = torch.full((nseq, 1, H, D), float("nan"), device=dev)
    torch.cuda.synchronize(dev)
    b2a.attentionDecode(ctx, cache, rope, 0, q, kn, vn, out, H)
    ctx.synchronize()
    check_decode_rows(oracle, cache, q.float().cpu().numpy(), [total] * nseq, [(b, 0) for b in range(nseq)],
                      out.cpu().numpy(), "f16", kn=kn.float().cpu().numpy(), what="config 5")
    cache.close()
    rope.close()


@pytest.mark.parametrize("S,tiles", [(8, None), (64, None), (512, None), (2048, None), (2048, "2"),
                                     (16384, None)])
def test_prefill_f16_cache_against_f32_cache_oracle(env, oracle, monkeypatch, S, tiles):
    torch, dev, ctx, stream = env
    if tiles is not None:
        monkeypatch.setenv("B2A_PREFILL_TILES", tiles)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5000 + S)
    with torch.cuda.stream(stream):
        cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(1, KVH, D, H), S, batch=1, dtype="f16")
        rope = b2a.RopeTable(ctx, D, THETA, S)
        q = torch.randn(S, H, D, device=dev, generator=gen).bfloat16()
        k = torch.randn(S, KVH, D, device=dev, generator=gen).bfloat16()
        v = torch.randn(S, KVH, D, device=dev, generator=gen).bfloat16()
        o = torch.empty(S, H, D, device=dev, dtype=torch.bfloat16)
    torch.cuda.synchronize(dev)
    b2a.attentionPrefill(ctx, cache, rope, 0, q, k, v, o, S, H)
    ctx.synchronize()
    got = o.float().cpu().numpy().reshape(S, H * D)
    qn = q.float().cpu().numpy().reshape(S, H * D)
    kn = k.float().cpu().numpy().reshape(S, KVH * D)
    vn = v.float().cpu().numpy().reshape(S, KVH * D)
    kr = oracle.rope_rows(kn, range(S), D, THETA)       # f32, as the reference's cache holds it
    gk, gv = cache.read(0, S)
    assert np.array_equal(gk, oracle.to_bits(kr.reshape(S, KVH, D).transpose(1, 0, 2), "f16"))
    assert np.array_equal(gv, oracle.to_bits(vn.reshape(S, KVH, D).transpose(1, 0, 2), "f16"))
    if S <= 2048:
        qr = oracle.rope_rows(qn, range(S), D, THETA)
        ref = oracle.grouped_attention(qr, kr, vn, S, 0, H, KVH, D)
        assert_parity(got.reshape(-1), ref, "bf16", f"prefill S={S} tiles={tiles}")
    else:
        rows = [0, 1, 63, 127, 128, 129, S // 2 - 1, S // 2, S // 2 + 1, S - 129, S - 128, S - 2, S - 1]
        rng = np.random.default_rng(S)
        rows += [int(x) for x in rng.integers(0, S, size=7)]
        for t in rows:
            qr = oracle.rope_rows(qn[t:t + 1], [t], D, THETA)
            ref = oracle.grouped_attention(qr, kr[:t + 1], vn[:t + 1], 1, t, H, KVH, D)
            assert_parity(got[t], ref, "bf16", f"prefill S={S} row {t}")
    cache.close()
    rope.close()
