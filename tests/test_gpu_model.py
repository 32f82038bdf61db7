"""The decoder around attention on the GPU (b2a_model_*) against the oracle's
ReferenceModel restatement (src/cpu/model.js:55-187) on the same int8 weights.

The comparison surface is the reference's own (test/model.test.js:63-157):
the worst absolute logit error relative to the largest logit, the per-layer
present keys and values, the greedy pick, and the errors for bad token ids.
Tolerances: logits 1e-3 relative (worstRelative), present K/V within the
attention path's 2e-3 absolute / 1e-2 relative bound. The pick must be equal
wherever the oracle's best two logits are further apart than the observed
logit error, so a near tie cannot fail the test and a real defect cannot pass.
"""
import numpy as np
import pytest

import b2a
from oracle import oracle as o

pytestmark = pytest.mark.gpu

QWEN2 = dict(hidden=896, inter=4864, layers=2, heads=14, kv_heads=2, vocab=4096)
SMALL = dict(hidden=256, inter=512, layers=3, heads=4, kv_heads=2, vocab=1000)
LOGIT_REL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = b2a.Context(0)
    yield c
    c.close()


def _config(c, max_positions=4096):
    return b2a.ModelConfig(dict(model_type="qwen2", hidden_size=c["hidden"], intermediate_size=c["inter"],
                                num_hidden_layers=c["layers"], num_attention_heads=c["heads"],
                                num_key_value_heads=c["kv_heads"], vocab_size=c["vocab"],
                                max_position_embeddings=max_positions, rope_theta=1e6, rms_norm_eps=1e-6,
                                tie_word_embeddings=True))


def _weights(c, seed):
    return o.synthetic_weights(c["hidden"], c["inter"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], seed,
                               norm_jitter=0.1, bias_std=0.1)


def _gpu_model(ctx, c, w, capacity=256):
    m = b2a.Model(ctx, _config(c), capacity, scale_dtype="f16")
    for i, lw in enumerate(w["layers"]):
        m.load_layer(i, lw)
    m.load_embedding(*w["embedding"])
    m.load_final_norm(w["final_norm"])
    return m


def _oracle_model(c, w, capacity=256, threads=8):
    return o.OracleModel(w, c["hidden"], c["inter"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], 1e6, 1e-6,
                         capacity, threads)


def worst_relative(mine, theirs):
    diff = np.abs(mine.astype(np.float64) - theirs.astype(np.float64))
    scale = np.abs(theirs).max()
    return float(diff.max() / scale) if scale > 0 else 0.0, float(diff.max())


def margin(logits):
    top = np.sort(logits.astype(np.float64))[-2:]
    return float(top[1] - top[0])


def check_pick(gpu_token, ref_logits, err_abs):
    if margin(ref_logits) > 2 * err_abs:
        assert gpu_token == o.argmax(ref_logits)


@pytest.mark.parametrize("path", ["persistent", "layered"])
@pytest.mark.parametrize("shape", ["qwen2", "small"])
def test_prefill_then_decode_matches_oracle(ctx, shape, path):
    c = QWEN2 if shape == "qwen2" else SMALL
    w = _weights(c, 11)
    gm, om = _gpu_model(ctx, c, w), _oracle_model(c, w)
    gm.decode_path = path
    rng = np.random.default_rng(5)
    tokens = rng.integers(0, c["vocab"], 37).tolist()
    out = gm.forward(tokens)
    ref, ref_best = om.forward(tokens)
    rel, err = worst_relative(out["logits"], ref)
    assert rel <= LOGIT_REL, f"prefill logits {rel:.2e} relative"
    check_pick(out["token"], ref, err)
    assert out["token"] == o.argmax(out["logits"])
    # decode steps, each fed the oracle's own pick so both walk the same sequence
    nxt = ref_best
    for step in range(6):
        out = gm.forward([nxt])
        ref, ref_best = om.forward([nxt])
        rel, err = worst_relative(out["logits"], ref)
        assert rel <= LOGIT_REL, f"decode step {step} logits {rel:.2e} relative"
        check_pick(out["token"], ref, err)
        nxt = ref_best
    assert gm.length == om.length == 43
    for layer in range(c["layers"]):
        p = gm.present(layer)
        rk, rv = om.present(layer)
        gk = o.from_bits(p["key"], "f16")
        gv = o.from_bits(p["value"], "f16")
        for g, r, what in ((gk, rk, "key"), (gv, rv, "value")):
            d = np.abs(g - r)
            assert (d <= 2e-3 + 1e-2 * np.abs(r)).all(), f"layer {layer} {what}: max abs {d.max():.3g}"
    gm.close()


def test_incremental_decode_agrees_with_full_recompute(ctx):
    c = QWEN2
    w = _weights(c, 12)
    inc, full = _gpu_model(ctx, c, w), _gpu_model(ctx, c, w)
    prompt = np.random.default_rng(6).integers(0, c["vocab"], 20).tolist()
    t0 = inc.forward(prompt)["token"]
    t1 = inc.forward([t0])["token"]
    last = inc.forward([t1])
    ref = full.forward(prompt + [t0, t1])
    rel, _ = worst_relative(last["logits"], ref["logits"])
    assert rel <= LOGIT_REL
    for layer in range(c["layers"]):
        a, b_ = inc.present(layer), full.present(layer)
        ka, kb = o.from_bits(a["key"], "f16"), o.from_bits(b_["key"], "f16")
        assert np.abs(ka - kb).max() <= 2e-3
    inc.close()
    full.close()


def test_generate_is_greedy_on_device(ctx):
    c = QWEN2
    w = _weights(c, 13)
    gm, om = _gpu_model(ctx, c, w), _oracle_model(c, w)
    prompt = np.random.default_rng(7).integers(0, c["vocab"], 9).tolist()
    steps = list(gm.generate(prompt, maxTokens=12))
    assert [s["step"] for s in steps] == list(range(12))
    assert [s["context"] for s in steps] == [9 + i for i in range(12)]
    assert gm.length == 9 + 11
    # teacher-forced through the oracle along the GPU's own tokens
    ref, _ = om.forward(prompt)
    for s in steps:
        err = np.abs(ref).max() * LOGIT_REL
        check_pick(s["token"], ref, err)
        assert abs(s["logit"] - ref[s["token"]]) <= 2 * err
        if s["step"] < 11:
            ref, _ = om.forward([s["token"]])
    # a second run starts from an empty cache and repeats itself exactly
    again = [s["token"] for s in gm.generate(prompt, maxTokens=12)]
    assert again == [s["token"] for s in steps]
    gm.close()


def test_generate_stops_after_a_stop_token(ctx):
    c = SMALL
    w = _weights(c, 14)
    gm = _gpu_model(ctx, c, w)
    prompt = [1, 2, 3]
    toks, _ = gm.generate_all(prompt, maxTokens=8)
    stop = int(toks[3])
    first = int(np.flatnonzero(toks == stop)[0])
    cut, _ = gm.generate_all(prompt, maxTokens=8, stopTokens=[stop])
    assert cut.tolist() == toks[:first + 1].tolist()
    gm.close()


def test_errors_match_the_reference(ctx):
    c = SMALL
    w = _weights(c, 15)
    gm = _gpu_model(ctx, c, w, capacity=16)
    with pytest.raises(b2a.RangeError, match="outside the vocabulary"):
        gm.forward([c["vocab"]])
    with pytest.raises(b2a.RangeError, match="outside the vocabulary"):
        gm.forward([-1])
    with pytest.raises(b2a.B2AError, match="at least one token"):
        gm.forward([])
    assert gm.length == 0
    gm.forward(list(range(10)))
    with pytest.raises(b2a.RangeError, match="cannot add 7"):
        gm.forward(list(range(7)))
    with pytest.raises(b2a.RangeError):
        gm.generate_all(list(range(10)), maxTokens=8)
    gm.reset()
    assert gm.length == 0
    fresh = b2a.Model(ctx, _config(c), 16)
    with pytest.raises(b2a.B2AError, match="not loaded"):
        fresh.forward([1])
    fresh.close()
    gm.close()


def test_device_token_outside_vocabulary_reports_at_sync(ctx):
    torch = pytest.importorskip("torch")
    c = SMALL
    w = _weights(c, 16)
    gm = _gpu_model(ctx, c, w)
    toks = torch.tensor([1, c["vocab"] + 5], dtype=torch.int32, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    gm.forward_device(toks, next_token=nxt)
    with pytest.raises(b2a.RangeError, match="outside the vocabulary"):
        ctx.synchronize()
    gm.close()


def test_config4_full_size_prefill_and_decode(ctx):
    """BASELINE config 4's shapes: 24 layers, vocab 151936, N(0, 0.02) weights."""
    c = dict(hidden=896, inter=4864, layers=24, heads=14, kv_heads=2, vocab=151936)
    w = o.synthetic_weights(c["hidden"], c["inter"], c["layers"], c["heads"], c["kv_heads"], c["vocab"], 4)
    gm = _gpu_model(ctx, c, w, capacity=64)
    om = _oracle_model(c, w, capacity=64, threads=16)
    prompt = np.random.default_rng(8).integers(0, c["vocab"], 6).tolist()
    out = gm.forward(prompt)
    ref, best = om.forward(prompt)
    rel, err = worst_relative(out["logits"], ref)
    assert rel <= LOGIT_REL
    check_pick(out["token"], ref, err)
    for _ in range(2):
        out = gm.forward([best])
        ref, best = om.forward([best])
        rel, err = worst_relative(out["logits"], ref)
        assert rel <= LOGIT_REL
        check_pick(out["token"], ref, err)
    gm.close()


def test_decode_paths_agree_over_a_long_context(ctx):
    """The one-kernel step and the per-layer launches walk the same 300-token
    sequence (the step kernel's attention splits into several chunks there)."""
    c = QWEN2
    w = _weights(c, 17)
    a, b = _gpu_model(ctx, c, w, capacity=512), _gpu_model(ctx, c, w, capacity=512)
    assert a.decode_path == "persistent"
    b.decode_path = "layered"
    prompt = np.random.default_rng(9).integers(0, c["vocab"], 290).tolist()
    ra, rb = a.forward(prompt), b.forward(prompt)
    assert np.array_equal(ra["logits"], rb["logits"])        # the same prefill path
    nxt = ra["token"]
    for _ in range(12):
        ra, rb = a.forward([nxt]), b.forward([nxt])
        rel, err = worst_relative(ra["logits"], rb["logits"])
        assert rel <= LOGIT_REL
        check_pick(ra["token"], rb["logits"], err)
        nxt = rb["token"]
    for layer in range(c["layers"]):
        ka = o.from_bits(a.present(layer)["key"], "f16")
        kb = o.from_bits(b.present(layer)["key"], "f16")
        assert np.abs(ka - kb).max() <= 2e-3
    a.close()
    b.close()
