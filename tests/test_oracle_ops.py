"""The reference's softmax and RoPE tests (test/ops.test.js:104-316, web/kernels.html:315-349)
restated against the C oracle."""
import math

import numpy as np


def close(a, b, tol):
    return abs(a - b) <= tol


def test_softmax_produces_distribution(oracle):
    x = np.array([1, 2, 3, 4], np.float32)
    oracle.softmax_inplace(x)
    assert all(0 < v < 1 for v in x)
    assert close(float(np.float64(x).sum()), 1.0, 1e-6)
    assert x[3] > x[2] > x[1]


def test_softmax_invariant_to_constant(oracle):
    a = np.array([1, 2, 3], np.float32)
    b = np.array([101, 102, 103], np.float32)
    oracle.softmax_inplace(a)
    oracle.softmax_inplace(b)
    assert np.all(np.abs(a - b) <= 1e-6)


def test_softmax_survives_overflow_range(oracle):
    x = np.array([800, 801, 802], np.float32)
    oracle.softmax_inplace(x)
    assert np.all(np.isfinite(x))
    assert close(float(np.float64(x).sum()), 1.0, 1e-6)


def test_softmax_prefix_leaves_rest_alone(oracle):
    x = np.array([1, 1, 999, 999], np.float32)
    oracle.softmax_inplace(x, 2)
    assert close(x[0], 0.5, 1e-6) and close(x[1], 0.5, 1e-6)
    assert x[2] == 999


def test_one_element_softmax_is_exactly_one(oracle):
    x = np.array([-12345], np.float32)
    oracle.softmax_inplace(x, 1)
    assert x[0] == 1.0


def test_softmax_golden(oracle, golden):
    x = np.array([1, 2, 3, 4], np.float32)
    oracle.softmax_inplace(x)
    assert np.array_equal(x, golden["softmax_1234"])


def test_rope_frequencies_decay(oracle):
    inv = oracle.rope_frequencies(8, 10000)
    assert inv.size == 4 and close(inv[0], 1, 1e-12)
    assert all(inv[j] < inv[j - 1] for j in range(1, 4))
    assert close(inv[1], math.pow(10000, -2 / 8), 1e-12)


def test_rope_preserves_pair_length(oracle):
    hd = 8
    inv = oracle.rope_frequencies(hd, 10000)
    v = np.arange(1, 9, dtype=np.float32)
    before = v.copy()
    oracle.rope_inplace(v, 0, hd, 37, inv)
    for j in range(4):
        assert close(math.hypot(v[j], v[j + 4]), math.hypot(before[j], before[j + 4]), 1e-5)


def test_rope_is_half_split(oracle):
    hd = 8
    inv = oracle.rope_frequencies(hd, 10000)
    v = np.zeros(hd, np.float32)
    v[0] = 1
    oracle.rope_inplace(v, 0, hd, 1, inv)
    assert close(v[0], math.cos(1), 1e-6)
    assert close(v[4], math.sin(1), 1e-6)
    assert close(v[1], 0, 1e-12)


def test_rope_at_zero_is_identity(oracle):
    inv = oracle.rope_frequencies(8, 10000)
    v = np.arange(1, 9, dtype=np.float32)
    before = v.copy()
    oracle.rope_inplace(v, 0, 8, 0, inv)
    assert np.array_equal(v, before)


def test_rope_relative_position(oracle):
    hd, theta = 16, 1e6
    inv = oracle.rope_frequencies(hd, theta)
    q0 = np.array([math.sin(i * 1.7) for i in range(hd)], np.float32)
    k0 = np.array([math.cos(i * 0.9) for i in range(hd)], np.float32)

    def dot_at(m, n):
        q, k = q0.copy(), k0.copy()
        oracle.rope_inplace(q, 0, hd, m, inv)
        oracle.rope_inplace(k, 0, hd, n, inv)
        return float(np.dot(q.astype(np.float64), k.astype(np.float64)))

    for m, n in [(0, 0), (5, 2), (100, 97), (1000, 997)]:
        assert close(dot_at(m, n), dot_at(m - n, 0), 1e-4)
    assert abs(dot_at(5, 2) - dot_at(5, 1)) > 1e-3


def test_rope_offset_slice(oracle):
    inv = oracle.rope_frequencies(4, 10000)
    buf = np.array([9, 9, 9, 9, 1, 0, 0, 0, 7, 7, 7, 7], np.float32)
    oracle.rope_inplace(buf, 4, 4, 1, inv)
    assert list(buf[:4]) == [9, 9, 9, 9] and list(buf[8:]) == [7, 7, 7, 7]
    assert close(buf[4], math.cos(1), 1e-6)


def test_rope_table_equals_direct(oracle):
    # test/ops.test.js:263-304
    hd, theta, positions, heads = 64, 1e6, 40, 3
    cos_t, sin_t, half = oracle.rope_tables(hd, theta, positions)
    inv = oracle.rope_frequencies(hd, theta)
    assert half == 32 and cos_t.size == positions * half
    for position in (0, 1, 7, 39):
        direct = np.array([math.sin(i * 0.3) + 0.1 for i in range(heads * hd)], np.float32)
        via = direct.copy()
        for h in range(heads):
            oracle.rope_inplace(direct, h * hd, hd, position, inv)
        for h in range(heads):
            base = h * hd
            for j in range(half):
                c = float(cos_t[position * half + j])
                s = float(sin_t[position * half + j])
                lo, hi = float(via[base + j]), float(via[base + j + half])
                via[base + j] = np.float32(lo * c - hi * s)
                via[base + j + half] = np.float32(hi * c + lo * s)
        assert np.all(np.abs(via - direct) <= 1e-6)


def test_rope_table_identity_and_bounds(oracle):
    cos_t, sin_t, half = oracle.rope_tables(64, 1e6, 2048)
    assert np.all(cos_t[:half] == 1) and np.all(sin_t[:half] == 0)
    assert np.all(np.abs(cos_t) <= 1.0000001) and np.all(np.abs(sin_t) <= 1.0000001)


def test_rope_matches_golden(oracle, golden):
    # web/kernels.html:315-349: 6 rows x 14 heads x 64 from position 3, theta 1e6, seed 21.
    rows, heads, hd, theta, base = 6, 14, 64, 1e6, 3
    v = oracle.random_array(rows * heads * hd, 21)
    assert np.array_equal(v, golden["rope_input"])
    inv = oracle.rope_frequencies(hd, theta)
    assert np.array_equal(inv, golden["rope_inv_freq"])
    direct = v.copy()
    for r in range(rows):
        for h in range(heads):
            oracle.rope_inplace(direct, r * heads * hd + h * hd, hd, base + r, inv)
    assert np.array_equal(direct, golden["rope_direct"])
    # The reference's bound for its table kernel against this is 1e-5 (relative to max).
    rel = np.abs(golden["rope_table"] - direct).max() / np.abs(direct).max()
    assert rel <= 1e-5


def test_rope_tables_golden(oracle, golden):
    c, s, _ = oracle.rope_tables(64, 1e6, 40)
    assert np.array_equal(c, golden["rope_cos_64_1e6_40"])
    assert np.array_equal(s, golden["rope_sin_64_1e6_40"])


def test_rope_large_positions_golden(oracle, golden):
    inv = oracle.rope_frequencies(64, 1e6)
    base = golden["rope_big_input"]
    got = []
    for p in golden["rope_big_positions"]:
        v = base.copy()
        oracle.rope_inplace(v, 0, 64, int(p), inv)
        got.append(v)
    assert np.array_equal(np.concatenate(got), golden["rope_big_out"])


def test_f64_table_is_the_direct_angle(oracle):
    """The device's f64 table holds exactly the cos/sin ropeInPlace evaluates."""
    c64, s64 = oracle.rope_tables_f64(64, 1e6, 50)
    inv = oracle.rope_frequencies(64, 1e6)
    for p in (0, 1, 49):
        for j in range(32):
            assert c64[p * 32 + j] == math.cos(p * inv[j])
            assert s64[p * 32 + j] == math.sin(p * inv[j])
