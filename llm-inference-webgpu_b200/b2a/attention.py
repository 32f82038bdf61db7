"""The attention operator API, mirroring the reference's names and arguments:

  groupedAttention(q, keys, values, out, scores, {seq, past, numHeads, numKVHeads, headDim})
                                    src/core/attention.js:32-66
  kvHeadFor(queryHead, numHeads, numKVHeads)      src/core/attention.js:74-76
  ropeFrequencies(headDim, theta)                 src/core/ops.js:99-104
  ropeTables(headDim, theta, positions)           src/core/ops.js:123-136

plus the fused device operators that replace the GPU backend's rope-q / rope-k /
KV append / ATTENTION sequence (src/gpu/model.js:323-346): appendRope,
attentionDecode, attentionPrefill, decodePartial and lseCombine. Every one runs
the CUDA kernels in libb2a.so.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import DTYPES, check, load
from .runtime import Context, GpuKVCache, RopeTable, _arg, _same_dtype, _where

_default_ctx: Context | None = None


def default_context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context(0)
    return _default_ctx


def kvHeadFor(queryHead: int, numHeads: int, numKVHeads: int) -> int:
    r = load().b2a_kv_head_for(queryHead, numHeads, numKVHeads)
    if r < 0:
        raise ValueError(f"query head {queryHead} does not map onto {numKVHeads} KV heads of {numHeads}")
    return r


def ropeFrequencies(headDim: int, theta: float) -> np.ndarray:
    inv = np.empty(headDim // 2, np.float64)
    check(load().b2a_rope_frequencies(headDim, float(theta), inv.ctypes.data_as(ctypes.POINTER(ctypes.c_double))))
    return inv


def ropeTables(headDim: int, theta: float, positions: int) -> dict:
    half = headDim >> 1
    c = np.empty(positions * half, np.float32)
    s = np.empty(positions * half, np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    check(load().b2a_rope_tables(headDim, float(theta), positions, c.ctypes.data_as(fp), s.ctypes.data_as(fp)))
    return {"cos": c, "sin": s, "half": half}


def groupedAttention(q, keys, values, out, scores=None, shape: dict | None = None, ctx: Context | None = None,
                     **kw):
    """src/core/attention.js:32-66 on the GPU. q [seq, numHeads*headDim] (already rotated),
    keys/values [past+seq, numKVHeads*headDim], out overwritten and returned. f32."""
    sh = dict(shape or {}, **kw)
    ctx = ctx or default_context()
    qa, ka, va, oa = _arg(q), _arg(keys), _arg(values), _arg(out, writable=True)
    if {a.dtype for a in (qa, ka, va, oa)} != {"f32"}:
        raise ValueError("groupedAttention takes f32 arrays, as the reference does")
    check(load().b2a_grouped_attention(ctx.handle, qa.ptr, ka.ptr, va.ptr, oa.ptr, None, sh["seq"], sh["past"],
                                       sh["numHeads"], sh["numKVHeads"], sh["headDim"], _where(qa, ka, va, oa)))
    return out


def appendRope(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, k, v, count: int, seq: int = 0,
               dtype: str | None = None) -> None:
    """RoPE on every KV head of k at absolute positions L..L+count-1 (L = the sequence's
    length), rounded to the cache dtype, and stored with v (src/cpu/model.js:103-116)."""
    ka, va = _arg(k, dtype), _arg(v, dtype)
    check(load().b2a_append_rope(ctx.handle, cache.handle, rope.handle, layer, seq, ka.ptr, va.ptr,
                                 DTYPES[_same_dtype(ka, va)], count, _where(ka, va)))


def attentionDecode(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, q, k_new, v_new, out,
                    numHeads: int, numLayers: int = 1, dtype: str | None = None,
                    out_dtype: str | None = None) -> None:
    """One new token for every sequence of the cache, over layers [layer, layer+numLayers).
    q [batch, numLayers, numHeads, headDim]; k_new/v_new [batch, numLayers, numKVHeads, headDim]
    or None; out [batch, numLayers, numHeads, headDim]."""
    qa, ka, va = _arg(q, dtype), _arg(k_new, dtype), _arg(v_new, dtype)
    oa = _arg(out, out_dtype or dtype, writable=True)
    in_dt = _same_dtype(qa, ka, va)
    check(load().b2a_attention_decode(ctx.handle, cache.handle, rope.handle, layer, numLayers, numHeads, qa.ptr,
                                      ka.ptr if ka else None, va.ptr if va else None, DTYPES[in_dt], oa.ptr,
                                      DTYPES[oa.dtype], _where(qa, ka, va, oa)))


def attentionDecodeAsync(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, q, k_new, v_new, out,
                         numHeads: int, numLayers: int = 1, dtype: str | None = None,
                         out_dtype: str | None = None) -> None:
    """attentionDecode on host arrays (pinned torch tensors keep the copies
    asynchronous) that returns once the work is enqueued
    (b2a_attention_decode_host_async): consecutive calls overlap on the GPU.
    The caller must keep q/k_new/v_new unchanged and not read `out` until
    ctx.synchronize()."""
    qa, ka, va = _arg(q, dtype), _arg(k_new, dtype), _arg(v_new, dtype)
    oa = _arg(out, out_dtype or dtype, writable=True)
    in_dt = _same_dtype(qa, ka, va)
    if _where(qa, ka, va, oa) != _lib.B2A_HOST:
        raise ValueError("attentionDecodeAsync takes host arrays")
    check(load().b2a_attention_decode_host_async(ctx.handle, cache.handle, rope.handle, layer, numLayers, numHeads,
                                                 qa.ptr, ka.ptr if ka else None, va.ptr if va else None,
                                                 DTYPES[in_dt], oa.ptr, DTYPES[oa.dtype]))


def attentionPrefill(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, q, k, v, out, count: int,
                     numHeads: int, seq: int = 0, dtype: str | None = None, out_dtype: str | None = None) -> None:
    """Causal attention of `count` new tokens of one sequence over past+count positions,
    with RoPE(q), RoPE(k) and the K/V append fused (src/cpu/model.js:103-123)."""
    qa, ka, va = _arg(q, dtype), _arg(k, dtype), _arg(v, dtype)
    oa = _arg(out, out_dtype or dtype, writable=True)
    in_dt = _same_dtype(qa, ka, va)
    check(load().b2a_attention_prefill(ctx.handle, cache.handle, rope.handle, layer, seq, numHeads, qa.ptr, ka.ptr,
                                       va.ptr, DTYPES[in_dt], count, oa.ptr, DTYPES[oa.dtype], _where(qa, ka, va, oa)))


def attentionPrefillBatch(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, q, k, v, out, count: int,
                          numHeads: int, seqBegin: int, numSeqs: int, dtype: str | None = None,
                          out_dtype: str | None = None) -> None:
    """attentionPrefill for numSeqs sequences in one call (b2a_attention_prefill_batch): q/out
    [numSeqs, count, numHeads, headDim], k/v [numSeqs, count, numKVHeads, headDim], each sequence
    at its own cache length."""
    qa, ka, va = _arg(q, dtype), _arg(k, dtype), _arg(v, dtype)
    oa = _arg(out, out_dtype or dtype, writable=True)
    in_dt = _same_dtype(qa, ka, va)
    check(load().b2a_attention_prefill_batch(ctx.handle, cache.handle, rope.handle, layer, seqBegin, numSeqs,
                                             numHeads, qa.ptr, ka.ptr, va.ptr, DTYPES[in_dt], count, oa.ptr,
                                             DTYPES[oa.dtype], _where(qa, ka, va, oa)))


def _positions(ctx: Context, q_positions, where: int):
    """The per-sequence absolute positions as int32 where the call's data lives."""
    if where == _lib.B2A_HOST:
        pos = np.ascontiguousarray(q_positions, dtype=np.int32)
        return pos.ctypes.data, pos
    import torch
    pos = q_positions if isinstance(q_positions, torch.Tensor) else torch.as_tensor(
        np.asarray(q_positions, np.int32), device=f"cuda:{ctx.device}")
    pos = pos.to(torch.int32).contiguous()
    return pos.data_ptr(), pos


def decodePartial(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, q, k_new, v_new, q_positions,
                  partial, numHeads: int, dtype: str | None = None, numLayers: int = 1) -> None:
    """Split-KV partial over this cache's positions (see b2a_attention_decode_partial;
    numLayers > 1: b2a_attention_decode_partial_layers over layers [layer, layer+numLayers)).
    partial [batch, numHeads, headDim+4] f32 ([batch, numLayers, numHeads, headDim+4])."""
    qa, ka, va, pa = _arg(q, dtype), _arg(k_new, dtype), _arg(v_new, dtype), _arg(partial, writable=True)
    in_dt = _same_dtype(qa, ka, va)
    where = _where(qa, ka, va, pa)
    pos_ptr, keep = _positions(ctx, q_positions, where)
    check(load().b2a_attention_decode_partial_layers(ctx.handle, cache.handle, rope.handle, layer, numLayers,
                                                     numHeads, qa.ptr, ka.ptr if ka else None,
                                                     va.ptr if va else None, DTYPES[in_dt], pos_ptr, pa.ptr, where))
    del keep


def decodeSplit(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, q, k_new, v_new, q_positions,
                exchange, out, numHeads: int, dtype: str | None = None, out_dtype: str | None = None,
                numLayers: int = 1) -> None:
    """One split-KV decode step with the cross-rank exchange inside the kernel
    (b2a_attention_decode_split_layers over layers [layer, layer+numLayers)): this
    rank's positions, then every rank's partials combined in rank order into
    out [batch, numHeads, headDim] ([batch, numLayers, numHeads, headDim])."""
    qa, ka, va = _arg(q, dtype), _arg(k_new, dtype), _arg(v_new, dtype)
    oa = _arg(out, out_dtype, writable=True)
    in_dt = _same_dtype(qa, ka, va)
    where = _where(qa, ka, va, oa)
    pos_ptr, keep = _positions(ctx, q_positions, where)
    check(load().b2a_attention_decode_split_layers(ctx.handle, cache.handle, rope.handle, layer, numLayers, numHeads,
                                                   qa.ptr, ka.ptr if ka else None, va.ptr if va else None,
                                                   DTYPES[in_dt], pos_ptr, exchange.handle, oa.ptr, DTYPES[oa.dtype],
                                                   where))
    del keep


def decodeSplitNccl(ctx: Context, cache: GpuKVCache, rope: RopeTable, layer: int, q, k_new, v_new, q_positions,
                    comm, world: int, rank: int, out, numHeads: int, dtype: str | None = None,
                    out_dtype: str | None = None, numLayers: int = 1) -> None:
    """One split-KV decode step over NCCL (b2a_split_kv_decode_nccl): this rank's
    partials, an in-place ncclAllGather through `comm` (an ncclComm_t, as an int
    address or an object with a `.value`), the combine in rank order into out
    [batch, numLayers, numHeads, headDim]. Device tensors only; k_new/v_new are
    used by rank world - 1 only."""
    qa, ka, va = _arg(q, dtype), _arg(k_new, dtype), _arg(v_new, dtype)
    oa = _arg(out, out_dtype, writable=True)
    in_dt = _same_dtype(qa, ka, va)
    where = _where(qa, ka, va, oa)
    pos_ptr, keep = _positions(ctx, q_positions, where)
    handle = getattr(comm, "value", comm)
    check(load().b2a_split_kv_decode_nccl(ctx.handle, cache.handle, rope.handle, layer, numLayers, numHeads, qa.ptr,
                                          ka.ptr if ka else None, va.ptr if va else None, DTYPES[in_dt], pos_ptr,
                                          handle, world, rank, oa.ptr, DTYPES[oa.dtype], where))
    del keep


def lseCombine(ctx: Context, partials, numParts: int, batch: int, numHeads: int, headDim: int, out,
               out_dtype: str | None = None) -> None:
    """Merge [numParts, batch, numHeads, headDim+4] partials in ascending part order."""
    pa, oa = _arg(partials), _arg(out, out_dtype, writable=True)
    check(load().b2a_lse_combine(ctx.handle, pa.ptr, numParts, batch, numHeads, headDim, oa.ptr, DTYPES[oa.dtype],
                                 _where(pa, oa)))


# ------------------------------------------------------------- projections --

def quantizeInt8PerChannel(W, rows: int, cols: int) -> dict:
    """quantizeInt8PerChannel (src/core/quantize.js:36-58), on the host:
    {'q': int8 [rows, cols], 'scales': f32 [rows], 'rows', 'cols', 'scheme'}."""
    w = np.ascontiguousarray(np.asarray(W, np.float32).reshape(-1))
    if w.size != rows * cols:
        raise ValueError(f"expected {rows * cols} weights, got {w.size}")
    q = np.zeros(rows * cols, np.int8)
    scales = np.zeros(rows, np.float32)
    check(load().b2a_quantize_int8_per_channel(w.ctypes.data, rows, cols, q.ctypes.data, scales.ctypes.data))
    return {"q": q.reshape(rows, cols), "scales": scales, "rows": rows, "cols": cols, "scheme": "int8-per-channel"}


def linearInt8(ctx: Context, codes, scales, bias, x, out, rows: int, cols: int, tokens: int, residual=None,
               x_dtype: str | None = None, out_dtype: str | None = None, scale_dtype: str | None = None) -> None:
    """out[t] = residual[t] + scales * (codes @ x[t]) + bias (matVec, src/core/ops.js:33-41, with int8
    per-row weights); codes int8 [rows, cols], x [tokens, cols], out [tokens, rows]. 16-bit arrays
    given as uint16 bits name their dtype ("f16"/"bf16")."""
    ca, sa, ba = _arg_i8(codes), _arg(scales, scale_dtype), _arg(bias)
    xa = _arg(x, x_dtype)
    oa = _arg(out, out_dtype, writable=True)
    ra = _arg(residual, out_dtype)
    where = _where(ca, sa, ba, xa, oa, ra)
    check(load().b2a_linear_int8(ctx.handle, ca.ptr, sa.ptr, DTYPES[sa.dtype], ba.ptr if ba else None,
                                 DTYPES[ba.dtype] if ba else 0, xa.ptr, DTYPES[xa.dtype], rows, cols, tokens,
                                 ra.ptr if ra else None, oa.ptr, DTYPES[oa.dtype], where))


def qkvInt8(ctx: Context, codes, scales, bias, x, q_out, k_out, v_out, hidden: int, q_rows: int, kv_rows: int,
            tokens: int, x_dtype: str | None = None, out_dtype: str | None = None,
            scale_dtype: str | None = None) -> None:
    """The q/k/v projections of src/cpu/model.js:98-101 in one launch: codes hold the q, k and v rows
    (q_rows, kv_rows, kv_rows); q_out [tokens, q_rows], k_out/v_out [tokens, kv_rows]."""
    ca, sa, ba = _arg_i8(codes), _arg(scales, scale_dtype), _arg(bias)
    xa = _arg(x, x_dtype)
    qa = _arg(q_out, out_dtype, writable=True)
    ka = _arg(k_out, out_dtype, writable=True)
    va = _arg(v_out, out_dtype, writable=True)
    where = _where(ca, sa, ba, xa, qa, ka, va)
    check(load().b2a_qkv_int8(ctx.handle, ca.ptr, sa.ptr, DTYPES[sa.dtype], ba.ptr if ba else None,
                              DTYPES[ba.dtype] if ba else 0, xa.ptr, DTYPES[xa.dtype], hidden, q_rows, kv_rows, tokens,
                              qa.ptr, ka.ptr, va.ptr, DTYPES[_same_dtype(qa, ka, va)], where))


def _arg_i8(x):
    """int8 codes: a numpy int8 array (host) or a torch int8 CUDA tensor (device)."""
    from .runtime import _Arg, torch as _torch
    if _torch is not None and isinstance(x, _torch.Tensor):
        if x.dtype != _torch.int8 or not x.is_contiguous():
            raise ValueError("codes must be a contiguous int8 tensor")
        return _Arg(x.data_ptr(), _lib.B2A_DEVICE if x.is_cuda else _lib.B2A_HOST, "i8", x.numel(), x)
    a = np.ascontiguousarray(x, np.int8)
    return _Arg(a.ctypes.data, _lib.B2A_HOST, "i8", a.nbytes, a)
