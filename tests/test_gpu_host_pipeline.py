"""The host-pointer decode path against the device-pointer one.

b2a_attention_decode with host arrays uploads q and the new keys/values,
runs the attention and downloads the outputs in groups so the copies overlap
the kernels: with several layers, groups of whole layers for every sequence,
moved by strided 2D copies into dense per-group staging. Here a 24-layer call
large enough to make several groups must give what the same call on device
tensors gives (one launch; the chunking differs, so within the attention
tolerance), append the same cache bytes, and match the oracle's grouped
attention (src/core/attention.js:32-66) on a sample of rows.
"""
import numpy as np
import pytest

import b2a
from helpers import assert_parity

pytestmark = pytest.mark.gpu

H, KVH, D, THETA = 14, 2, 64, 1e6


def test_layer_grouped_host_decode_matches_device_decode(oracle):
    import torch

    dev = torch.device("cuda", 0)
    ctx = b2a.Context(0)
    rope = b2a.RopeTable(ctx, D, THETA, 1024)
    # 64 sequences x 24 layers: ~9 MB of transfers, three layer groups
    layers, batch, cap = 24, 64, 400
    rng = np.random.default_rng(5)
    lens = rng.integers(1, 350, size=batch).astype(np.int32)
    cfg = b2a.CacheConfig(numLayers=layers, numKVHeads=KVH, headDim=D, numHeads=H)
    caches = [b2a.GpuKVCache(ctx, cfg, cap, batch=batch, dtype="f16") for _ in range(2)]
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    keys = torch.randn(batch, layers, cap, KVH * D, device=dev, generator=g).half()
    vals = torch.randn(batch, layers, cap, KVH * D, device=dev, generator=g).half()
    for c in caches:
        for b in range(batch):
            for layer in range(layers):
                c.writeAt(layer, 0, keys[b, layer], vals[b, layer], cap, seq=b)
        c.setLengths(lens)
    q = oracle.round_to(oracle.normal_array(batch * layers * H * D, 21), "f16").reshape(batch, layers, H, D)
    kn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 22), "f16").reshape(batch, layers, KVH, D)
    vn = oracle.round_to(oracle.normal_array(batch * layers * KVH * D, 23), "f16").reshape(batch, layers, KVH, D)
    bits = lambda x: oracle.to_bits(x, "f16")  # noqa: E731
    out_host = np.full((batch, layers, H, D), np.nan, np.float32)
    b2a.attentionDecode(ctx, caches[0], rope, 0, bits(q), bits(kn), bits(vn), out_host, H, numLayers=layers,
                        dtype="f16")
    tq, tk, tv = (torch.from_numpy(bits(x).astype(np.int16)).to(dev) for x in (q, kn, vn))
    out_dev = torch.full((batch, layers, H, D), float("nan"), device=dev)
    torch.cuda.synchronize(dev)
    b2a.attentionDecode(ctx, caches[1], rope, 0, tq, tk, tv, out_dev, H, numLayers=layers, dtype="f16")
    ctx.synchronize()
    out_dev = out_dev.cpu().numpy()
    assert np.isfinite(out_host).all()
    assert_parity(out_host.reshape(-1), out_dev.reshape(-1), "f32", "host-path vs device-path decode")
    for b in range(0, batch, 9):
        for layer in (0, 7, 23):
            kh, vh = caches[0].read(layer, int(lens[b]) + 1, seq=b)
            kd, vd = caches[1].read(layer, int(lens[b]) + 1, seq=b)
            assert np.array_equal(kh, kd) and np.array_equal(vh, vd), (b, layer)
            L = int(lens[b])
            ck = oracle.from_bits(kh, "f16").transpose(1, 0, 2).reshape(L + 1, KVH * D)
            cv = oracle.from_bits(vh, "f16").transpose(1, 0, 2).reshape(L + 1, KVH * D)
            qr = oracle.rope_rows(q[b, layer].reshape(1, -1), [L], D, THETA).reshape(-1)
            ref = oracle.grouped_attention(qr, ck.reshape(-1), cv.reshape(-1), 1, L, H, KVH, D)
            assert_parity(out_host[b, layer].reshape(-1), ref, "f32", f"host decode seq {b} layer {layer}")
    for c in caches:
        c.close()
    rope.close()
    ctx.close()
