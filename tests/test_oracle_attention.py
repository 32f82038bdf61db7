"""The reference's attention tests (test/attention.test.js), restated against the
C oracle, plus the golden fixtures from tests/golden/make_golden.py."""
import numpy as np
import pytest

QWEN = dict(num_heads=14, num_kv_heads=2, head_dim=64)


def run(o, seq, past, num_heads, num_kv_heads, head_dim, seed=1):
    """test/attention.test.js:71-81."""
    total = past + seq
    q = o.random_array(seq * num_heads * head_dim, seed)
    k = o.random_array(total * num_kv_heads * head_dim, seed + 1)
    v = o.random_array(total * num_kv_heads * head_dim, seed + 2)
    mine = o.grouped_attention(q, k, v, seq, past, num_heads, num_kv_heads, head_dim)
    ref = o.expanded_attention(q, k, v, seq, past, num_heads, num_kv_heads, head_dim)
    return mine, ref


def test_mapping_is_blocked_not_interleaved(oracle):
    # test/attention.test.js:85-94
    mapping = [oracle.kv_head_for(h, 14, 2) for h in range(14)]
    assert mapping == [0] * 7 + [1] * 7
    assert mapping != [h % 2 for h in range(14)]


def test_mapping_covers_every_kv_head_evenly(oracle):
    # test/attention.test.js:96-100
    counts = [0, 0]
    for h in range(14):
        counts[oracle.kv_head_for(h, 14, 2)] += 1
    assert counts == [7, 7]


@pytest.mark.parametrize("shape,seed", [
    (dict(seq=5, past=0, **QWEN), 1),            # :102-106
    (dict(seq=1, past=11, **QWEN), 99),          # :108-111
    (dict(seq=3, past=7, **QWEN), 4242),         # :113-116
    (dict(seq=4, past=2, num_heads=4, num_kv_heads=4, head_dim=8), 1),   # :118-123
    (dict(seq=4, past=3, num_heads=6, num_kv_heads=1, head_dim=8), 1),   # :125-129
])
def test_grouped_equals_expanded_exactly(oracle, shape, seed):
    mine, ref = run(oracle, seed=seed, **shape)
    assert np.array_equal(mine, ref)


def test_attention_is_causal(oracle):
    # test/attention.test.js:131-168
    seq, past, nh, nkv, hd = 4, 0, 4, 2, 8
    q_dim, kv_dim, total = nh * hd, nkv * hd, seq
    q = oracle.random_array(seq * q_dim, 7)
    k = oracle.random_array(total * kv_dim, 8)
    v = oracle.random_array(total * kv_dim, 9)
    before = oracle.grouped_attention(q, k, v, seq, past, nh, nkv, hd)
    k2, v2 = k.copy(), v.copy()
    k2[(total - 1) * kv_dim:] += np.float32(3.5)
    v2[(total - 1) * kv_dim:] -= np.float32(2.25)
    after = oracle.grouped_attention(q, k2, v2, seq, past, nh, nkv, hd)
    assert np.array_equal(after[: (seq - 1) * q_dim], before[: (seq - 1) * q_dim])
    assert not np.array_equal(after[(seq - 1) * q_dim:], before[(seq - 1) * q_dim:])


def test_first_position_returns_its_value(oracle):
    # test/attention.test.js:170-191
    nh, nkv, hd = 4, 2, 8
    q = oracle.random_array(nh * hd, 21)
    k = oracle.random_array(nkv * hd, 22)
    v = oracle.random_array(nkv * hd, 23)
    out = oracle.grouped_attention(q, k, v, 1, 0, nh, nkv, hd)
    for h in range(nh):
        g = oracle.kv_head_for(h, nh, nkv)
        assert np.array_equal(out[h * hd:(h + 1) * hd], v[g * hd:(g + 1) * hd])


def test_output_is_convex_combination(oracle):
    # test/attention.test.js:193-224
    seq, nh, nkv, hd = 6, 4, 2, 8
    q_dim, kv_dim = nh * hd, nkv * hd
    q = oracle.random_array(seq * q_dim, 31)
    k = oracle.random_array(seq * kv_dim, 32)
    v = oracle.random_array(seq * kv_dim, 33)
    out = oracle.grouped_attention(q, k, v, seq, 0, nh, nkv, hd).reshape(seq, nh, hd)
    vv = v.reshape(seq, nkv, hd)
    for h in range(nh):
        g = oracle.kv_head_for(h, nh, nkv)
        for t in range(seq):
            lo = vv[: t + 1, g].min(axis=0)
            hi = vv[: t + 1, g].max(axis=0)
            assert np.all(out[t, h] >= lo - 1e-6) and np.all(out[t, h] <= hi + 1e-6)


@pytest.mark.parametrize("name,shape,seeds", [
    ("attn_kernels_html", (3, 5, 14, 2, 64), (31, 32, 33)),     # web/kernels.html:351-385
    ("attn_prefill_s5_p0", (5, 0, 14, 2, 64), (1, 2, 3)),
    ("attn_decode_s1_p11", (1, 11, 14, 2, 64), (99, 100, 101)),
    ("attn_mixed_s3_p7", (3, 7, 14, 2, 64), (4242, 4243, 4244)),
    ("attn_mha_4_4", (4, 2, 4, 4, 8), (1, 2, 3)),
    ("attn_mqa_6_1", (4, 3, 6, 1, 8), (1, 2, 3)),
])
def test_oracle_matches_golden_transliteration(oracle, golden, name, shape, seeds):
    """The C oracle equals the independent Python transliteration of the JS bit for bit."""
    seq, past, nh, nkv, hd = shape
    total = past + seq
    q = oracle.random_array(seq * nh * hd, seeds[0])
    k = oracle.random_array(total * nkv * hd, seeds[1])
    v = oracle.random_array(total * nkv * hd, seeds[2])
    out = oracle.grouped_attention(q, k, v, seq, past, nh, nkv, hd)
    ref = golden[name]
    # glibc exp and the transliteration's math.exp are the same function, so the
    # two restatements agree exactly; the reference's own bound would be 1e-5.
    assert np.array_equal(out, ref), float(np.abs(out - ref).max())


def test_split_kv_combine_equals_full(oracle):
    """The split-KV decomposition the CUDA decode uses, restated on the CPU:
    partial (m, l, o) per chunk + LSE combine == one softmax over everything."""
    hd, n = 64, 777
    q = oracle.normal_array(hd, 5)
    k = oracle.normal_array(n * hd, 6)
    v = oracle.normal_array(n * hd, 7)
    full = oracle.grouped_attention(q, k, v, 1, n - 1, 1, 1, hd)
    cuts = [0, 100, 101, 400, 777]
    parts = [oracle.decode_partial(q, k, v, a, b, hd) for a, b in zip(cuts, cuts[1:])]
    m = np.array([p[0] for p in parts], np.float32)
    l = np.array([p[1] for p in parts], np.float32)
    o = np.stack([p[2] for p in parts])
    got = oracle.lse_combine(m, l, o, hd)
    assert np.abs(got - full).max() < 1e-5
