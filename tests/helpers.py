"""Parity helpers shared by the GPU tests.

Tolerance (from the hot path's specification): outputs within max abs error
2e-3 and max relative error 1e-2 of the reference's f32 CPU attention run on
the same inputs rounded to the kernel's input dtype. "Relative error" is the
reference's own definition, max|a-b| / max|b| (web/kernels.html:56-66,
test/model.test.js:64-75). For f16/bf16 outputs the output's own rounding
(half an ulp of the output format at the reference value) is excluded from the
absolute error: no kernel can return a bf16 closer than that. KV-cache bytes
are compared bit for bit.
"""
from __future__ import annotations

import numpy as np

ATOL = 2e-3
RTOL = 1e-2


def half_ulp(ref: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return np.zeros_like(ref, dtype=np.float64)
    mant = {"f16": 10, "bf16": 7}[dtype]
    a = np.abs(ref).astype(np.float64)
    e = np.floor(np.log2(np.maximum(a, 1e-30)))
    if dtype == "f16":
        e = np.maximum(e, -14)
    return np.ldexp(1.0, (e - mant).astype(np.int64)) / 2


def compare(got, ref, out_dtype: str = "f32") -> dict:
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    diff = np.abs(got - ref)
    beyond = np.maximum(diff - half_ulp(ref, out_dtype), 0.0)
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    return {
        "max_abs": float(diff.max()) if diff.size else 0.0,
        "max_abs_beyond_rounding": float(beyond.max()) if beyond.size else 0.0,
        "rel": float(diff.max() / scale) if scale > 0 else 0.0,
        "finite": bool(np.all(np.isfinite(got))),
    }


def assert_parity(got, ref, out_dtype: str = "f32", what: str = "") -> dict:
    c = compare(got, ref, out_dtype)
    assert c["finite"], f"{what}: non-finite output"
    assert c["max_abs_beyond_rounding"] <= ATOL, f"{what}: {c}"
    assert c["rel"] <= RTOL, f"{what}: {c}"
    return c


def check_decode_rows(oracle, cache, q, lengths, picks, out, cache_dtype: str, theta: float = 1e6,
                      kn=None, what: str = "") -> list:
    """Decode outputs of (sequence, layer) rows against the oracle's decode
    (src/cpu/model.js:103-123: RoPE(q) at position L, attention over the L
    cached positions plus the appended one). The cache contents, including the
    appended row at position L, are read back from the device, so a call may
    fill its cache on the GPU; when `kn` (the new keys, [batch][layers][kv
    heads][64], unrotated) is given, the appended key row must also equal the
    oracle's RoPE(k) rounded to the cache dtype, bit for bit. q and out are
    float arrays [batch][layers][heads][64]. Returns the comparisons."""
    heads, hd = q.shape[2], q.shape[3]
    kvh = cache.config.numKVHeads
    res = []
    for b, layer in picks:
        L = int(lengths[b])
        kb, vb = cache.read(layer, L + 1, seq=b)
        kc = oracle.from_bits(kb, cache_dtype)
        vc = oracle.from_bits(vb, cache_dtype)
        qr = oracle.rope_rows(np.asarray(q[b, layer], np.float32).reshape(1, heads * hd), [L], hd, theta)
        ref = oracle.decode_head_major(qr.reshape(-1), np.ascontiguousarray(kc), np.ascontiguousarray(vc), L + 1, L,
                                       heads, kvh, hd)
        res.append(assert_parity(np.asarray(out[b, layer]).reshape(-1), ref, "f32", f"{what} seq {b} layer {layer}"))
        if kn is not None:
            kr = oracle.rope_rows(np.asarray(kn[b, layer], np.float32).reshape(1, kvh * hd), [L], hd, theta)
            want = oracle.to_bits(kr.reshape(kvh, hd), cache_dtype)
            assert np.array_equal(kb[:, L], want), f"{what} seq {b} layer {layer}: appended key bits differ"
    return res
