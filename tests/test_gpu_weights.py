"""A Qwen2 checkpoint through Model.load_safetensors (b2a_model_load_safetensors).

A small Qwen2-shaped checkpoint in bfloat16 (as the real one is stored) is
written with the reference's tensor names. Loaded through the library, the
model must equal one loaded tensor by tensor with the same int8 codes
(quantizeInt8PerChannel, src/core/quantize.js:36-58, of the widened bf16
values; scales rounded to f16) bit for bit, and match the oracle's
ReferenceModel restatement on those weights within the model tests'
tolerance. A checkpoint that disagrees with the config is refused with the
reference's message (config.checkAgainst, src/core/config.js:125-150).
"""
import numpy as np
import pytest

import b2a
from oracle import oracle as o

pytestmark = pytest.mark.gpu

C = dict(hidden=256, inter=512, layers=2, heads=4, kv_heads=2, vocab=1000)


def _config():
    return b2a.ModelConfig(dict(model_type="qwen2", hidden_size=C["hidden"], intermediate_size=C["inter"],
                                num_hidden_layers=C["layers"], num_attention_heads=C["heads"],
                                num_key_value_heads=C["kv_heads"], vocab_size=C["vocab"],
                                max_position_embeddings=512, rope_theta=1e6, rms_norm_eps=1e-6,
                                tie_word_embeddings=True))


def _bf16(rng, shape, std, mean=0.0):
    w = (rng.standard_normal(shape) * std + mean).astype(np.float32)
    return o.f32_to_bf16_bits(w).reshape(shape)


def _checkpoint(seed=3):
    rng = np.random.default_rng(seed)
    cfg = _config()
    t = {}
    for name, shape in cfg.expectedTensors().items():
        if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            t[name] = (_bf16(rng, shape, 0.1, 1.0), "BF16")
        elif name.endswith(".bias"):
            t[name] = (_bf16(rng, shape, 0.1), "BF16")
        else:
            t[name] = (_bf16(rng, shape, 0.02), "BF16")
    return t


def _widen(bits):
    return o.bf16_bits_to_f32(bits)


def _quant(bits):
    w = _widen(bits)
    codes, scales = o.quantize_int8(w, w.shape[0], w.shape[1])
    return codes, scales.astype(np.float16)


def _layer_arrays(t, i):
    p = f"model.layers.{i}."
    q, sq = _quant(t[p + "self_attn.q_proj.weight"][0])
    k, sk = _quant(t[p + "self_attn.k_proj.weight"][0])
    v, sv = _quant(t[p + "self_attn.v_proj.weight"][0])
    oo, so = _quant(t[p + "self_attn.o_proj.weight"][0])
    g, sg = _quant(t[p + "mlp.gate_proj.weight"][0])
    u, su = _quant(t[p + "mlp.up_proj.weight"][0])
    d, sd = _quant(t[p + "mlp.down_proj.weight"][0])
    bias = np.concatenate([_widen(t[p + f"self_attn.{x}_proj.bias"][0]) for x in "qkv"])
    return dict(input_norm=_widen(t[p + "input_layernorm.weight"][0]),
                post_attn_norm=_widen(t[p + "post_attention_layernorm.weight"][0]),
                qkv=np.concatenate([q, k, v]), qkv_scales=np.concatenate([sq, sk, sv]), qkv_bias=bias,
                o=oo, o_scales=so, gate=g, gate_scales=sg, up=u, up_scales=su, down=d, down_scales=sd)


@pytest.fixture(scope="module")
def ctx():
    c = b2a.Context(0)
    yield c
    c.close()


def test_checkpoint_loads_as_the_quantized_tensors(ctx, tmp_path):
    t = _checkpoint()
    path = tmp_path / "qwen2-small.safetensors"
    path.write_bytes(b2a.write_safetensors(t, {"format": "pt"}))
    st = b2a.Safetensors.open(str(path))
    a = b2a.Model(ctx, _config(), 128)
    a.load_safetensors(st)
    st.close()
    layers = [_layer_arrays(t, i) for i in range(C["layers"])]
    emb = _quant(t["model.embed_tokens.weight"][0])
    fin = _widen(t["model.norm.weight"][0])
    b = b2a.Model(ctx, _config(), 128)
    for i, lw in enumerate(layers):
        b.load_layer(i, lw)
    b.load_embedding(*emb)
    b.load_final_norm(fin)
    oracle_w = {"layers": layers, "embedding": emb, "final_norm": fin}
    om = o.OracleModel(oracle_w, C["hidden"], C["inter"], C["layers"], C["heads"], C["kv_heads"], C["vocab"],
                       1e6, 1e-6, 128, 8)
    prompt = np.random.default_rng(1).integers(0, C["vocab"], 11).tolist()
    ra, rb = a.forward(prompt), b.forward(prompt)
    ref, best = om.forward(prompt)
    assert np.array_equal(ra["logits"], rb["logits"])
    assert np.abs(ra["logits"] - ref).max() / np.abs(ref).max() <= 1e-3
    for _ in range(3):
        ra, rb = a.forward([best]), b.forward([best])
        ref, best = om.forward([best])
        assert np.array_equal(ra["logits"], rb["logits"])
        assert np.abs(ra["logits"] - ref).max() / np.abs(ref).max() <= 1e-3
    a.close()
    b.close()


def test_checkpoint_that_disagrees_with_the_config_is_refused(ctx):
    t = _checkpoint(4)
    m = b2a.Model(ctx, _config(), 64)
    missing = {k: v for k, v in t.items() if k != "model.norm.weight"}
    with pytest.raises(b2a.B2AError, match=r"weights do not match config \(1 problem\):\s+missing model.norm.weight"):
        m.load_safetensors(b2a.Safetensors.fromBytes(b2a.write_safetensors(missing)))
    extra = dict(t)
    extra["lm_head.weight"] = t["model.embed_tokens.weight"]
    with pytest.raises(b2a.B2AError, match="unexpected tensor lm_head.weight"):
        m.load_safetensors(b2a.Safetensors.fromBytes(b2a.write_safetensors(extra)))
    wrong = dict(t)
    wrong["model.layers.1.mlp.up_proj.weight"] = (t["model.layers.1.mlp.up_proj.weight"][0][:8], "BF16")
    with pytest.raises(b2a.B2AError, match=r"up_proj.weight: expected shape \[512,256\], file has \[8,256\]"):
        m.load_safetensors(b2a.Safetensors.fromBytes(b2a.write_safetensors(wrong)))
    m.close()
