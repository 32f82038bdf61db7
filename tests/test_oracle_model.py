"""The oracle's restatement of the decoder around attention (no GPU).

Known answers from the reference's own tests (test/ops.test.js:15-58 for
rmsNorm, :155-170 for silu / swiglu, test/model.test.js:146-157 for the greedy
pick and :179-186 for the errors), the phase-2 property the reference states at
src/cpu/model.js:17-21 (incremental decode equals full recomputation bit for
bit), and an independent numpy transliteration of ReferenceModel.forward
(src/cpu/model.js:55-161) on a tiny configuration.
"""
import math

import numpy as np
import pytest

from oracle import oracle as o


def close(a, b, tol):
    assert abs(a - b) <= tol, f"{a} vs {b} (tolerance {tol})"


# ---------------------------------------------------------------- rmsNorm --

def test_rmsnorm_unit_rms_with_unit_gain():
    out = o.rmsnorm([1, -2, 3, -4, 5], np.ones(5), 0)
    close(math.sqrt(float(np.sum(out.astype(np.float64) ** 2)) / 5), 1, 1e-6)


def test_rmsnorm_applies_gain_per_channel():
    out = o.rmsnorm([3, 4], [2, 10], 0)
    rms = math.sqrt(25 / 2)
    close(out[0], 3 / rms * 2, 1e-6)
    close(out[1], 4 / rms * 10, 1e-6)


def test_rmsnorm_epsilon_inside_the_root():
    out = o.rmsnorm([1e-4, 1e-4], [1, 1], 1e-6)
    close(out[0], np.float32(1e-4) / math.sqrt(1e-8 + 1e-6), 1e-9)
    assert abs(out[0] - 1e-4 / (math.sqrt(1e-8) + 1e-6)) > 0.5


def test_rmsnorm_scale_equivariant_only_through_gain():
    a = o.rmsnorm([1, 2, 3, 4], np.ones(4), 0)
    b = o.rmsnorm([2, 4, 6, 8], np.ones(4), 0)
    for i in range(4):
        close(a[i], b[i], 1e-6)


# ----------------------------------------------------------- silu, swiglu --

def test_silu_known_points():
    close(o.silu(0), 0, 1e-12)
    close(o.silu(1), 1 / (1 + math.exp(-1)), 1e-12)
    close(o.silu(-1), -1 / (1 + math.exp(1)), 1e-12)
    assert -0.279 < o.silu(-1.2784) < -0.278


def test_swiglu_multiplies_gate_by_up():
    g = o.swiglu([1, -1, 0], [2, 3, 5])
    close(g[0], o.silu(1) * 2, 1e-6)
    close(g[1], o.silu(-1) * 3, 1e-6)
    close(g[2], 0, 1e-12)


# ---------------------------------------------------------------- argmax --

def test_argmax_takes_the_first_maximum():
    assert o.argmax([0.5, 2.0, -1.0, 2.0]) == 1
    assert o.argmax([3.0, 3.0]) == 0
    assert o.argmax([-np.inf, -np.inf]) == 0
    assert o.argmax([np.nan, 5.0, 6.0]) == 0      # nothing compares greater than NaN
    assert o.argmax([1.0, np.nan, 2.0]) == 2      # a NaN never wins


# ------------------------------------------------------------ the decoder --

TINY = dict(hidden=128, inter=256, layers=2, heads=2, kv_heads=1, vocab=300)


def _tiny(seed=3, capacity=64, threads=1):
    c = TINY
    w = o.synthetic_weights(c["hidden"], c["inter"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], seed,
                            norm_jitter=0.1, bias_std=0.1)
    m = o.OracleModel(w, c["hidden"], c["inter"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], 1e6, 1e-6,
                      capacity, threads)
    return w, m


def _numpy_forward(w, tokens, c, theta=1e6, eps=1e-6):
    """An independent transliteration of ReferenceModel.forward over a fresh cache
    (f64 reductions, f32 stores, q/k/v and the cache rounded to f16)."""
    H, I, heads, kvh = c["hidden"], c["inter"], c["heads"], c["kv_heads"]
    D = H // heads
    kv = kvh * D
    f16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)  # noqa: E731

    def deq(codes, scales):
        return (codes.astype(np.float64) * scales.astype(np.float32).astype(np.float64)[:, None]).astype(np.float32)

    def mv(codes, scales, x, bias=None):
        acc = deq(codes, scales).astype(np.float64) @ np.asarray(x, np.float64)
        if bias is not None:
            acc = acc + bias.astype(np.float64)
        return acc.astype(np.float32)

    def norm(x, g):
        x64 = x.astype(np.float64)
        scale = 1.0 / math.sqrt(float(np.sum(x64 * x64)) / x.size + eps)
        return (x64 * scale * g.astype(np.float64)).astype(np.float32)

    inv = np.array([theta ** (-(2 * j) / D) for j in range(D // 2)], np.float64)

    def rope(vec, pos):
        out = vec.copy()
        for j in range(D // 2):
            a = pos * inv[j]
            cs, sn = math.cos(a), math.sin(a)
            lo, hi = float(vec[j]), float(vec[j + D // 2])
            out[j] = np.float32(lo * cs - hi * sn)
            out[j + D // 2] = np.float32(hi * cs + lo * sn)
        return out

    codes, scales = w["embedding"]
    T = len(tokens)
    x = np.stack([deq(codes[t:t + 1], scales[t:t + 1])[0] for t in tokens])
    for lw in w["layers"]:
        q = np.zeros((T, H), np.float32)
        ks = np.zeros((T, kv), np.float32)
        vs = np.zeros((T, kv), np.float32)
        for t in range(T):
            y = mv(lw["qkv"], lw["qkv_scales"], norm(x[t], lw["input_norm"]), lw["qkv_bias"])
            qt, kt, vt = f16(y[:H]), f16(y[H:H + kv]), f16(y[H + kv:])
            q[t] = np.concatenate([rope(qt[h * D:(h + 1) * D], t) for h in range(heads)])
            ks[t] = f16(np.concatenate([rope(kt[h * D:(h + 1) * D], t) for h in range(kvh)]))
            vs[t] = vt
        att = np.zeros((T, H), np.float32)
        for h in range(heads):
            g = h // (heads // kvh)
            for t in range(T):
                s = np.array([np.float32(float(np.dot(q[t, h * D:(h + 1) * D].astype(np.float64),
                                                      ks[u, g * D:(g + 1) * D].astype(np.float64))) / math.sqrt(D))
                              for u in range(t + 1)], np.float32)
                e = np.exp(s.astype(np.float64) - float(s.max())).astype(np.float32)
                p = (e.astype(np.float64) * (1.0 / float(np.sum(e.astype(np.float64))))).astype(np.float32)
                att[t, h * D:(h + 1) * D] = (p.astype(np.float64) @ vs[:t + 1, g * D:(g + 1) * D].astype(np.float64))
        for t in range(T):
            x[t] = x[t] + mv(lw["o"], lw["o_scales"], att[t])
            nx = norm(x[t], lw["post_attn_norm"])
            gt = mv(lw["gate"], lw["gate_scales"], nx).astype(np.float64)
            up = mv(lw["up"], lw["up_scales"], nx).astype(np.float64)
            h_ = (gt / (1.0 + np.exp(-gt)) * up).astype(np.float32)
            x[t] = x[t] + mv(lw["down"], lw["down_scales"], h_)
    nl = norm(x[-1], w["final_norm"])
    return mv(codes, scales, nl)


def test_forward_matches_an_independent_transliteration():
    w, m = _tiny()
    tokens = [5, 77, 3, 299, 0, 150, 42]
    logits, best = m.forward(tokens)
    ref = _numpy_forward(w, tokens, TINY)
    rel = np.abs(logits - ref).max() / np.abs(ref).max()
    assert rel < 1e-5, rel
    assert best == int(np.argmax(ref))


def test_incremental_decode_equals_full_recompute_bit_for_bit():
    # src/cpu/model.js:17-21: one attention implementation, so both orders agree exactly
    w, inc = _tiny()
    _, full = _tiny()
    prompt = [1, 2, 3, 250, 17]
    _, t0 = inc.forward(prompt)
    l1, t1 = inc.forward([t0])
    l2, t2 = inc.forward([t1])
    lf, tf = full.forward(prompt + [t0, t1])
    assert np.array_equal(l2, lf) and t2 == tf
    for layer in range(TINY["layers"]):
        ki, vi = inc.present(layer)
        kf, vf = full.present(layer)
        assert np.array_equal(ki, kf) and np.array_equal(vi, vf)


def test_threads_do_not_change_the_result():
    w, one = _tiny(threads=1)
    _, many = _tiny(threads=4)
    tokens = [9, 8, 7, 6]
    a, _ = one.forward(tokens)
    b, _ = many.forward(tokens)
    assert np.array_equal(a, b)


def test_cache_keeps_f16_rounded_rotated_keys():
    w, m = _tiny()
    m.forward([4, 5, 6])
    k, v = m.present(0)
    assert k.shape == (1, 3, 64)
    assert np.array_equal(k, k.astype(np.float16).astype(np.float32))
    assert np.array_equal(v, v.astype(np.float16).astype(np.float32))


def test_rejects_out_of_vocabulary_and_empty():
    _, m = _tiny()
    with pytest.raises(o.RangeError_, match="outside the vocabulary"):
        m.forward([TINY["vocab"]])
    with pytest.raises(o.RangeError_, match="outside the vocabulary"):
        m.forward([-1])
    with pytest.raises(o.RangeError_, match="at least one token"):
        m.forward([])
    assert m.length == 0


def test_full_cache_is_a_range_error():
    _, m = _tiny(capacity=4)
    m.forward([1, 2, 3])
    with pytest.raises(o.RangeError_, match="cannot add 2"):
        m.forward([1, 2])
