"""The Qwen2 decoder around the attention path, on the device: the host mirror
of ReferenceModel (src/cpu/model.js:31-231) and ModelConfig
(src/core/config.js:16-80) over libb2a.so's b2a_model_* entry points.

Weights are int8 with one scale per output row (the reference's symmetric
per-channel scheme, src/core/quantize.js:36-58; scales in f16 or f32). The
model owns a one-sequence f16 KV cache, so forward() continues from whatever
the previous calls left in it, like forward(tokenIds, {cache}) with a cache
that persists; reset() empties it, and generate() always starts from empty.
There is no CPU fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import B2A_DEVICE, B2A_F16, B2A_F32, B2A_HOST, check
from .runtime import Context

try:
    import torch
except Exception:  # pragma: no cover
    torch = None


class _ModelConfigC(ctypes.Structure):
    _fields_ = [("hidden_size", ctypes.c_int), ("intermediate_size", ctypes.c_int), ("num_layers", ctypes.c_int),
                ("num_heads", ctypes.c_int), ("num_kv_heads", ctypes.c_int), ("vocab_size", ctypes.c_int),
                ("max_positions", ctypes.c_int), ("rope_theta", ctypes.c_double),
                ("rms_norm_eps", ctypes.c_double), ("scale_dtype", ctypes.c_int)]


class _LayerWeightsC(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input_norm", "post_attn_norm", "qkv", "qkv_scales", "qkv_bias", "o", "o_scales", "gate", "gate_scales",
        "up", "up_scales", "down", "down_scales")]


_REQUIRED = ("hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
             "vocab_size", "max_position_embeddings", "rope_theta", "rms_norm_eps")


class ModelConfig:
    """ModelConfig (src/core/config.js:16-80) from a config.json dictionary."""

    def __init__(self, raw: dict):
        for key in _REQUIRED:
            v = raw.get(key)
            if isinstance(v, bool) or not isinstance(v, (int, float)) or not np.isfinite(v):
                raise ValueError(f"config: {key} must be a finite number, got {v!r}")
        self.modelType = raw.get("model_type", "qwen2")
        if self.modelType != "qwen2":
            raise ValueError(f"config: only qwen2 is implemented, got {self.modelType!r}")
        if raw.get("hidden_act", "silu") != "silu":
            raise ValueError(f"config: only the silu/SwiGLU MLP is implemented, got {raw.get('hidden_act')}")
        if raw.get("use_sliding_window") is True:
            raise ValueError("config: sliding-window attention is not implemented")
        self.hiddenSize = int(raw["hidden_size"])
        self.intermediateSize = int(raw["intermediate_size"])
        self.numLayers = int(raw["num_hidden_layers"])
        self.numHeads = int(raw["num_attention_heads"])
        self.numKVHeads = int(raw["num_key_value_heads"])
        self.vocabSize = int(raw["vocab_size"])
        self.maxPositionEmbeddings = int(raw["max_position_embeddings"])
        self.ropeTheta = float(raw["rope_theta"])
        self.rmsNormEps = float(raw["rms_norm_eps"])
        self.tieWordEmbeddings = raw.get("tie_word_embeddings") is True
        if not self.tieWordEmbeddings:
            raise ValueError("config: only tied embeddings are implemented (the output projection is the "
                             "embedding)")
        if self.hiddenSize % self.numHeads:
            raise ValueError(f"config: hidden_size {self.hiddenSize} is not divisible by "
                             f"num_attention_heads {self.numHeads}")
        if self.numHeads % self.numKVHeads:
            raise ValueError(f"config: num_attention_heads {self.numHeads} is not divisible by "
                             f"num_key_value_heads {self.numKVHeads}, so the query heads cannot be grouped "
                             "evenly over the key/value heads")
        self.headDim = self.hiddenSize // self.numHeads
        self.kvGroupSize = self.numHeads // self.numKVHeads
        self.kvDim = self.numKVHeads * self.headDim

    def expectedTensors(self) -> dict:
        """config.expectedTensors (src/core/config.js:88-121): every tensor the
        architecture requires, name -> shape."""
        d, kv = self.hiddenSize, self.kvDim
        shapes = {"model.embed_tokens.weight": (self.vocabSize, d), "model.norm.weight": (d,)}
        for i in range(self.numLayers):
            p = f"model.layers.{i}."
            shapes[p + "input_layernorm.weight"] = (d,)
            shapes[p + "post_attention_layernorm.weight"] = (d,)
            shapes[p + "self_attn.q_proj.weight"] = (d, d)
            shapes[p + "self_attn.q_proj.bias"] = (d,)
            shapes[p + "self_attn.k_proj.weight"] = (kv, d)
            shapes[p + "self_attn.k_proj.bias"] = (kv,)
            shapes[p + "self_attn.v_proj.weight"] = (kv, d)
            shapes[p + "self_attn.v_proj.bias"] = (kv,)
            shapes[p + "self_attn.o_proj.weight"] = (d, d)
            shapes[p + "mlp.gate_proj.weight"] = (self.intermediateSize, d)
            shapes[p + "mlp.up_proj.weight"] = (self.intermediateSize, d)
            shapes[p + "mlp.down_proj.weight"] = (d, self.intermediateSize)
        if not self.tieWordEmbeddings:
            shapes["lm_head.weight"] = (self.vocabSize, d)
        return shapes

    def parameterCount(self) -> int:
        """config.parameterCount (src/core/config.js:153-159)."""
        total = 0
        for shape in self.expectedTensors().values():
            n = 1
            for v in shape:
                n *= v
            total += n
        return total

    @staticmethod
    def qwen25_05b(**over) -> "ModelConfig":
        """Qwen2.5-0.5B's architecture."""
        raw = dict(model_type="qwen2", hidden_size=896, intermediate_size=4864, num_hidden_layers=24,
                   num_attention_heads=14, num_key_value_heads=2, vocab_size=151936, max_position_embeddings=32768,
                   rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=True, hidden_act="silu")
        raw.update(over)
        return ModelConfig(raw)


def _ptr(x, where_expected=None):
    """(pointer, where, keepalive) of a numpy array or torch tensor."""
    if x is None:
        return None, None, None
    if torch is not None and isinstance(x, torch.Tensor):
        if not x.is_contiguous():
            raise ValueError("tensor arguments must be contiguous")
        return x.data_ptr(), (B2A_DEVICE if x.is_cuda else B2A_HOST), x
    a = np.ascontiguousarray(x)
    return a.ctypes.data, B2A_HOST, a


class Model:
    """A Qwen2 decoder on the device with int8 weights (ReferenceModel,
    src/cpu/model.js:31-231; GpuModel.forward, src/gpu/model.js:227-400)."""

    def __init__(self, ctx: Context, config: ModelConfig, capacity: int, scale_dtype: str = "f16"):
        if not isinstance(capacity, (int, np.integer)) or isinstance(capacity, bool):
            raise _lib.RangeError(_lib.B2A_ERANGE, f"cache capacity must be a positive integer, got {capacity}")
        self.ctx = ctx
        self.config = config
        self.capacity = int(capacity)
        if scale_dtype not in ("f16", "f32"):
            raise ValueError("scales are f16 or f32")
        self.scale_dtype = scale_dtype
        self._np_scale = np.float16 if scale_dtype == "f16" else np.float32
        c = _ModelConfigC(config.hiddenSize, config.intermediateSize, config.numLayers, config.numHeads,
                          config.numKVHeads, config.vocabSize, config.maxPositionEmbeddings, config.ropeTheta,
                          config.rmsNormEps, B2A_F16 if scale_dtype == "f16" else B2A_F32)
        h = ctypes.c_void_p()
        check(ctx._lib.b2a_model_create(ctx.handle, ctypes.byref(c), self.capacity, ctypes.byref(h)))
        self.handle = h
        ctx._children.add(self)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.ctx._lib.b2a_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights ---------------------------------------------------------------
    def _scales(self, s):
        if torch is not None and isinstance(s, torch.Tensor):
            return s
        return np.ascontiguousarray(np.asarray(s, dtype=self._np_scale))

    def load_layer(self, layer: int, w: dict) -> None:
        """w: input_norm, post_attn_norm [hidden] f32; qkv [hidden+2kvDim, hidden] int8 with qkv_scales and
        qkv_bias (f32); o, gate, up, down int8 with their *_scales (one per output row)."""
        keep, where = [], set()
        fields = {}
        for name, _ in _LayerWeightsC._fields_:
            x = w[name]
            if name.endswith("scales"):
                x = self._scales(x)
            elif name in ("input_norm", "post_attn_norm", "qkv_bias") and not (
                    torch is not None and isinstance(x, torch.Tensor)):
                x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
            elif not (torch is not None and isinstance(x, torch.Tensor)):
                x = np.ascontiguousarray(np.asarray(x, dtype=np.int8))
            p, wh, k = _ptr(x)
            keep.append(k)
            where.add(wh)
            fields[name] = p
        if len(where) != 1:
            raise ValueError("mix of host and device arrays in one call")
        s = _LayerWeightsC(**fields)
        check(self.ctx._lib.b2a_model_load_layer(self.handle, layer, ctypes.byref(s), where.pop()))

    def load_embedding(self, codes, scales) -> None:
        """The tied embedding: int8 codes [vocab, hidden] and one scale per row."""
        if not (torch is not None and isinstance(codes, torch.Tensor)):
            codes = np.ascontiguousarray(np.asarray(codes, dtype=np.int8))
        scales = self._scales(scales)
        pc, wc, kc = _ptr(codes)
        ps, ws, ks = _ptr(scales)
        if wc != ws:
            raise ValueError("mix of host and device arrays in one call")
        check(self.ctx._lib.b2a_model_load_embedding(self.handle, ctypes.c_void_p(pc), ctypes.c_void_p(ps), wc))

    def load_safetensors(self, st) -> None:
        """The weights of a Qwen2 checkpoint (b2a.weights.Safetensors): checked against the
        config (config.checkAgainst, src/core/config.js:125-150), quantized to int8 per output
        row and uploaded."""
        check(self.ctx._lib.b2a_model_load_safetensors(self.handle, st.handle))

    def load_final_norm(self, weight) -> None:
        if not (torch is not None and isinstance(weight, torch.Tensor)):
            weight = np.ascontiguousarray(np.asarray(weight, dtype=np.float32))
        p, wh, k = _ptr(weight)
        check(self.ctx._lib.b2a_model_load_final_norm(self.handle, ctypes.c_void_p(p), wh))

    # ---- running -----------------------------------------------------------------
    @property
    def length(self) -> int:
        n = ctypes.c_int()
        check(self.ctx._lib.b2a_model_length(self.handle, ctypes.byref(n)))
        return n.value

    def reset(self) -> None:
        check(self.ctx._lib.b2a_model_reset(self.handle))

    @property
    def decode_path(self) -> str:
        """"persistent" (one kernel per token) or "layered" (per-layer launches)."""
        n = ctypes.c_int()
        check(self.ctx._lib.b2a_model_decode_path(self.handle, ctypes.byref(n)))
        return "persistent" if n.value == 1 else "layered"

    @decode_path.setter
    def decode_path(self, path: str) -> None:
        check(self.ctx._lib.b2a_model_set_decode_path(self.handle, {"layered": 0, "persistent": 1}[path]))

    def forward(self, tokenIds, logits: bool = True) -> dict:
        """forward(tokenIds, {cache}) (src/cpu/model.js:55-161) on the model's cache: the
        last position's logits [vocab] f32 and the greedy pick (first index of the largest)."""
        ids = np.ascontiguousarray(np.asarray(tokenIds, dtype=np.int64))
        if ids.ndim != 1:
            raise ValueError("tokenIds must be one-dimensional")
        if ids.size and (ids.min() < -2**31 or ids.max() >= 2**31):
            raise _lib.RangeError(_lib.B2A_ERANGE, "token outside the vocabulary")
        ids32 = ids.astype(np.int32)
        out = np.empty(self.config.vocabSize, np.float32) if logits else None
        nxt = np.zeros(1, np.int32)
        check(self.ctx._lib.b2a_model_forward(self.handle, ids32.ctypes.data if ids32.size else None, ids32.size,
                                              out.ctypes.data if out is not None else None, nxt.ctypes.data,
                                              B2A_HOST))
        return {"logits": out, "token": int(nxt[0])}

    def forward_device(self, tokens, logits=None, next_token=None) -> None:
        """forward() with device tensors (int32 tokens, f32 logits, int32 next_token); enqueues only."""
        check(self.ctx._lib.b2a_model_forward(self.handle, ctypes.c_void_p(tokens.data_ptr()), tokens.numel(),
                                              ctypes.c_void_p(logits.data_ptr()) if logits is not None else None,
                                              ctypes.c_void_p(next_token.data_ptr()) if next_token is not None
                                              else None, B2A_DEVICE))

    def generate_all(self, promptIds, maxTokens: int = 32, stopTokens=()) -> tuple[np.ndarray, np.ndarray]:
        """Greedy generation on the device from an empty cache: (tokens, their logits)."""
        ids = np.ascontiguousarray(np.asarray(promptIds, dtype=np.int32))
        stop = np.ascontiguousarray(np.asarray(list(stopTokens), dtype=np.int32))
        toks = np.zeros(max(int(maxTokens), 1), np.int32)
        best = np.zeros(max(int(maxTokens), 1), np.float32)
        n = ctypes.c_int()
        check(self.ctx._lib.b2a_model_generate(self.handle, ids.ctypes.data if ids.size else None, ids.size,
                                               int(maxTokens), stop.ctypes.data if stop.size else None, stop.size,
                                               toks.ctypes.data, best.ctypes.data, ctypes.byref(n)))
        return toks[:n.value], best[:n.value]

    def generate(self, promptIds, maxTokens: int = 32, stopTokens=()):
        """ReferenceModel.generate (src/cpu/model.js:165-186): yields {token, logit, step, context}."""
        toks, best = self.generate_all(promptIds, maxTokens, stopTokens)
        n_prompt = len(promptIds)
        for step, (t, l) in enumerate(zip(toks.tolist(), best.tolist())):
            yield {"token": t, "logit": l, "step": step, "context": n_prompt + step}

    def present(self, layer: int):
        """The cache's keys and values of `layer` for the committed positions
        (KVCache.present, src/cpu/cache.js:97-115): f16 bits [numKVHeads, length, 64]."""
        h = ctypes.c_void_p()
        check(self.ctx._lib.b2a_model_cache(self.handle, ctypes.byref(h)))
        n = self.length
        shape = (self.config.numKVHeads, n, self.config.headDim)
        k, v = np.empty(shape, np.uint16), np.empty(shape, np.uint16)
        check(self.ctx._lib.b2a_kvcache_read(self.ctx.handle, h, layer, 0, n, k.ctypes.data, v.ctypes.data,
                                             B2A_HOST))
        return {"key": k, "value": v}
