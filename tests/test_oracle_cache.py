"""The reference's KV-cache tests (test/cache.test.js:40-161) restated against
the C oracle, plus the incremental == full-recompute gate (validate/phase2.js:83-121,
test/cache.test.js:172-207) on synthetic Q/K/V instead of the absent weights."""
import numpy as np
import pytest

TINY_LAYERS, KV = 2, 4   # test/cache.test.js:19-34: kvDim = 2 kv heads * 2 head width


def filled(value, count=KV):
    return np.array([value + i / 100 for i in range(count)], np.float32)


def test_new_cache_is_empty(oracle):
    c = oracle.OracleKVCache(TINY_LAYERS, KV, 10)
    assert c.length == 0 and c.capacity == 10
    assert c.byte_length == 2 * 10 * KV * 4 * 2


@pytest.mark.parametrize("cap", [0, -1, 1.5])
def test_rejects_bad_capacity(oracle, cap):
    with pytest.raises(ValueError, match="positive integer"):
        oracle.OracleKVCache(TINY_LAYERS, KV, cap)


def test_length_advances_only_on_commit(oracle):
    c = oracle.OracleKVCache(TINY_LAYERS, KV, 4)
    at = c.allocate(1)
    assert at == 0
    c.write_at(0, at, filled(1), filled(2), 1)
    assert c.length == 0
    c.commit(1)
    assert c.length == 1


def test_allocate_refuses_overflow(oracle):
    c = oracle.OracleKVCache(TINY_LAYERS, KV, 3)
    c.allocate(3)
    c.commit(3)
    with pytest.raises(ValueError, match="holds 3 of 3 positions"):
        c.allocate(1)
    assert c.length == 3


def test_appends_land_consecutively(oracle):
    c = oracle.OracleKVCache(TINY_LAYERS, KV, 4)
    for step in range(3):
        at = c.allocate(1)
        assert at == step
        c.write_at(0, at, filled(10 * step), filled(100 * step), 1)
        c.write_at(1, at, filled(20 * step), filled(200 * step), 1)
        c.commit(1)
    keys = c.keys_up_to(0, 3)
    for step in range(3):
        for i in range(KV):
            assert keys[step * KV + i] == np.float32(10 * step + i / 100)
    assert c.keys_up_to(1, 3)[KV] != keys[KV]


def test_bulk_write_equals_one_by_one(oracle):
    bulk = oracle.OracleKVCache(TINY_LAYERS, KV, 4)
    single = oracle.OracleKVCache(TINY_LAYERS, KV, 4)
    keys = np.array([i * 1.5 for i in range(3 * KV)], np.float32)
    values = np.array([-i for i in range(3 * KV)], np.float32)
    at = bulk.allocate(3)
    bulk.write_at(0, at, keys, values, 3)
    bulk.write_at(1, at, keys, values, 3)
    bulk.commit(3)
    for t in range(3):
        w = single.allocate(1)
        single.write_at(0, w, keys[t * KV:(t + 1) * KV], values[t * KV:(t + 1) * KV], 1)
        single.write_at(1, w, keys[t * KV:(t + 1) * KV], values[t * KV:(t + 1) * KV], 1)
        single.commit(1)
    assert np.array_equal(bulk.keys_up_to(0, 3), single.keys_up_to(0, 3))
    assert np.array_equal(bulk.values_up_to(1, 3), single.values_up_to(1, 3))


def test_present_transpose(oracle):
    c = oracle.OracleKVCache(TINY_LAYERS, KV, 2)
    at = c.allocate(2)
    keys = np.array([0, 1, 2, 3, 10, 11, 12, 13], np.float32)
    c.write_at(0, at, keys, keys, 2)
    c.commit(2)
    k, _ = c.present(0, 2, 2)
    assert list(k) == [0, 1, 10, 11, 2, 3, 12, 13]


def test_reset_keeps_allocation(oracle):
    c = oracle.OracleKVCache(TINY_LAYERS, KV, 4)
    c.write_at(0, c.allocate(2), filled(1, 2 * KV), filled(2, 2 * KV), 2)
    c.commit(2)
    c.reset()
    assert c.length == 0 and c.capacity == 4 and c.allocate(4) == 0


@pytest.mark.parametrize("splits", [[1] * 9, [5, 1, 1, 1, 1], [2, 4, 3]])
def test_incremental_equals_full_recompute(oracle, splits):
    """validate/phase2.js:83-121 on synthetic projections: every split of one
    sequence gives the same outputs and the same present() bits."""
    nh, nkv, hd, theta, layers = 14, 2, 64, 1e6, 2
    n = sum(splits)
    q = oracle.normal_array(n * nh * hd, 11).reshape(n, nh * hd)
    k = oracle.normal_array(n * nkv * hd, 12).reshape(n, nkv * hd)
    v = oracle.normal_array(n * nkv * hd, 13).reshape(n, nkv * hd)

    def run(parts):
        c = oracle.OracleKVCache(layers, nkv * hd, n)
        outs = []
        t0 = 0
        for s in parts:
            c.allocate(s)
            for layer in range(layers):
                out, _, _ = c.layer_attention(layer, q[t0:t0 + s], k[t0:t0 + s], v[t0:t0 + s],
                                              s, nh, nkv, hd, theta)
                if layer == layers - 1:
                    outs.append(out)
            c.commit(s)
            t0 += s
        return np.concatenate(outs), c.present(0, nkv, hd), c.present(1, nkv, hd)

    full = run([n])
    inc = run(splits)
    assert np.array_equal(full[0], inc[0])
    for a, b in zip(full[1] + full[2], inc[1] + inc[2]):
        assert np.array_equal(a, b)
