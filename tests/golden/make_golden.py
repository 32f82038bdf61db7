"""Generate the committed golden fixtures for the attention hot path.

This is an independent, line-by-line Python transliteration of the reference's
JavaScript (abho7/llm-inference-webgpu):

  src/core/attention.js:32-66   groupedAttention
  src/core/ops.js:66-78         softmaxInPlace
  src/core/ops.js:99-104        ropeFrequencies
  src/core/ops.js:123-136       ropeTables
  src/core/ops.js:147-158       ropeInPlace
  src/core/dtype.js:23-35,81-113  f32 -> bf16 / f16 rounding
  test/attention.test.js:60-69  the seeded LCG the reference tests use

JS semantics map one to one onto Python: a JS number and a Python float are
both IEEE f64, and a Float32Array store is a round-to-nearest-even to f32
(`_f32` below). It shares no code with the C oracle (oracle/attn_ref.c), so the
C restatement is checked against it. The inputs are the reference's own test
cases (test/attention.test.js, web/kernels.html), same seeds and shapes.

Run:  python tests/golden/make_golden.py   (writes tests/golden/golden.npz)
"""
from __future__ import annotations

import math
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _f32(x: float) -> float:
    """A Float32Array store: round an f64 to the nearest f32 (ties to even)."""
    return struct.unpack("<f", struct.pack("<f", x))[0]


def random_array(n: int, seed: int) -> list[float]:
    """test/attention.test.js:60-69 (also web/kernels.html:41-49)."""
    state = seed & 0xFFFFFFFF
    out = []
    for _ in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out.append(_f32((state / 0xFFFFFFFF) * 2 - 1))
    return out


def softmax_inplace(x: list[float], n: int) -> None:
    """src/core/ops.js:66-78."""
    mx = -math.inf
    for i in range(n):
        if x[i] > mx:
            mx = x[i]
    total = 0.0
    for i in range(n):
        e = math.exp(x[i] - mx)
        x[i] = _f32(e)
        total += e
    inv = 1 / total
    for i in range(n):
        x[i] = _f32(x[i] * inv)


def grouped_attention(q, keys, values, seq, past, num_heads, num_kv_heads, head_dim):
    """src/core/attention.js:32-66."""
    group = num_heads / num_kv_heads
    q_dim = num_heads * head_dim
    kv_dim = num_kv_heads * head_dim
    scale = 1 / math.sqrt(head_dim)
    out = [0.0] * (seq * q_dim)
    scores = [0.0] * (past + seq)
    for h in range(num_heads):
        kv_base = math.floor(h / group) * head_dim
        for t in range(seq):
            q_base = t * q_dim + h * head_dim
            up_to = past + t
            for s in range(up_to + 1):
                k_base = s * kv_dim + kv_base
                dot = 0.0
                for i in range(head_dim):
                    dot += q[q_base + i] * keys[k_base + i]
                scores[s] = _f32(dot * scale)
            softmax_inplace(scores, up_to + 1)
            out_base = t * q_dim + h * head_dim
            for s in range(up_to + 1):
                w = scores[s]
                v_base = s * kv_dim + kv_base
                for i in range(head_dim):
                    out[out_base + i] = _f32(out[out_base + i] + w * values[v_base + i])
    return out


def rope_frequencies(head_dim: int, theta: float) -> list[float]:
    """src/core/ops.js:99-104."""
    return [math.pow(theta, (-2 * j) / head_dim) for j in range(head_dim >> 1)]


def rope_tables(head_dim: int, theta: float, positions: int):
    """src/core/ops.js:123-136."""
    half = head_dim >> 1
    inv = rope_frequencies(head_dim, theta)
    cos_t, sin_t = [], []
    for p in range(positions):
        for j in range(half):
            angle = p * inv[j]
            cos_t.append(_f32(math.cos(angle)))
            sin_t.append(_f32(math.sin(angle)))
    return cos_t, sin_t


def rope_inplace(vec, offset, head_dim, position, inv_freq) -> None:
    """src/core/ops.js:147-158."""
    half = head_dim >> 1
    for j in range(half):
        angle = position * inv_freq[j]
        c = math.cos(angle)
        s = math.sin(angle)
        lo = vec[offset + j]
        hi = vec[offset + j + half]
        vec[offset + j] = _f32(lo * c - hi * s)
        vec[offset + j + half] = _f32(hi * c + lo * s)


def rope_via_table(vec, offset, head_dim, position, cos_t, sin_t) -> None:
    """The table rotation the WGSL ROPE kernel performs (src/gpu/kernels.js:360-389),
    evaluated with JS f64 arithmetic as test/ops.test.js:281-292 does."""
    half = head_dim >> 1
    for j in range(half):
        c = cos_t[position * half + j]
        s = sin_t[position * half + j]
        lo = vec[offset + j]
        hi = vec[offset + j + half]
        vec[offset + j] = _f32(lo * c - hi * s)
        vec[offset + j + half] = _f32(hi * c + lo * s)


def _bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def f32_to_bf16(x: float) -> int:
    """src/core/dtype.js:23-35."""
    u = _bits(x)
    if (u & 0x7F800000) == 0x7F800000 and (u & 0x007FFFFF) != 0:
        return ((u >> 16) | 0x0040) & 0xFFFF
    lsb = (u >> 16) & 1
    return ((u + 0x7FFF + lsb) >> 16) & 0xFFFF


def f32_to_f16(x: float) -> int:
    """src/core/dtype.js:81-113."""
    u = _bits(x)
    sign = (u >> 16) & 0x8000
    exp = (u >> 23) & 0xFF
    mant = u & 0x7FFFFF
    if exp == 0xFF:
        return sign | 0x7C00 | (((mant >> 13) | 0x200) if mant != 0 else 0)
    e = exp - 127 + 15
    if e >= 0x1F:
        return sign | 0x7C00
    if e <= 0:
        if e < -10:
            return sign
        m = mant | 0x800000
        shift = 14 - e
        half = 1 << (shift - 1)
        lsb = (m >> shift) & 1
        return sign | ((m + half - 1 + lsb) >> shift)
    lsb = (mant >> 13) & 1
    rounded = mant + 0x0FFF + lsb
    return sign | ((e << 10) + (rounded >> 13))


def attention_case(seq, past, num_heads, num_kv_heads, head_dim, seeds):
    total = past + seq
    q = random_array(seq * num_heads * head_dim, seeds[0])
    k = random_array(total * num_kv_heads * head_dim, seeds[1])
    v = random_array(total * num_kv_heads * head_dim, seeds[2])
    out = grouped_attention(q, k, v, seq, past, num_heads, num_kv_heads, head_dim)
    return np.array(out, np.float32)


def main() -> None:
    fx: dict[str, np.ndarray] = {}

    # web/kernels.html:351-385 -- the attention parity case (seq 3, past 5, 14/2, D 64, seeds 31/32/33).
    fx["attn_kernels_html"] = attention_case(3, 5, 14, 2, 64, (31, 32, 33))
    # test/attention.test.js:102-129 -- run(shape, seed) uses seeds seed, seed+1, seed+2.
    fx["attn_prefill_s5_p0"] = attention_case(5, 0, 14, 2, 64, (1, 2, 3))
    fx["attn_decode_s1_p11"] = attention_case(1, 11, 14, 2, 64, (99, 100, 101))
    fx["attn_mixed_s3_p7"] = attention_case(3, 7, 14, 2, 64, (4242, 4243, 4244))
    fx["attn_mha_4_4"] = attention_case(4, 2, 4, 4, 8, (1, 2, 3))
    fx["attn_mqa_6_1"] = attention_case(4, 3, 6, 1, 8, (1, 2, 3))

    # web/kernels.html:315-349 -- RoPE 6 rows x 14 heads x 64 from position 3, theta 1e6, seed 21.
    rows, heads, hd, theta, base = 6, 14, 64, 1e6, 3
    v = random_array(rows * heads * hd, 21)
    inv = rope_frequencies(hd, theta)
    direct = list(v)
    for r in range(rows):
        for h in range(heads):
            rope_inplace(direct, r * heads * hd + h * hd, hd, base + r, inv)
    cos_t, sin_t = rope_tables(hd, theta, base + rows)
    table = list(v)
    for r in range(rows):
        for h in range(heads):
            rope_via_table(table, r * heads * hd + h * hd, hd, base + r, cos_t, sin_t)
    fx["rope_input"] = np.array(v, np.float32)
    fx["rope_direct"] = np.array(direct, np.float32)
    fx["rope_table"] = np.array(table, np.float32)
    fx["rope_inv_freq"] = np.array(inv, np.float64)

    # test/ops.test.js:263-304 -- table at D=64, theta=1e6, 40 positions.
    c40, s40 = rope_tables(64, 1e6, 40)
    fx["rope_cos_64_1e6_40"] = np.array(c40, np.float32)
    fx["rope_sin_64_1e6_40"] = np.array(s40, np.float32)

    # RoPE of a head at large positions (BASELINE config 5 reaches 32768).
    big = random_array(64, 77)
    out_big = []
    for p in (1000, 4096, 32768):
        vec = list(big)
        rope_inplace(vec, 0, 64, p, inv)
        out_big.extend(vec)
    fx["rope_big_input"] = np.array(big, np.float32)
    fx["rope_big_positions"] = np.array([1000, 4096, 32768], np.int32)
    fx["rope_big_out"] = np.array(out_big, np.float32)

    # Rounding probes for src/core/dtype.js (values between representable ones).
    probes = random_array(4096, 555)
    probes = [p * 70000.0 if i % 3 == 0 else (p * 1e-5 if i % 3 == 1 else p) for i, p in enumerate(probes)]
    probes = [_f32(p) for p in probes]
    fx["dtype_probes"] = np.array(probes, np.float32)
    fx["dtype_probes_f16"] = np.array([f32_to_f16(p) for p in probes], np.uint16)
    fx["dtype_probes_bf16"] = np.array([f32_to_bf16(p) for p in probes], np.uint16)

    # softmax of the reference tests' vectors (test/ops.test.js:104-151).
    sm = [1.0, 2.0, 3.0, 4.0]
    softmax_inplace(sm, 4)
    fx["softmax_1234"] = np.array(sm, np.float32)

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **fx)
    print(f"wrote {path}: {', '.join(sorted(fx))}")


if __name__ == "__main__":
    main()
