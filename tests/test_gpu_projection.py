"""GPU parity of the int8 projections either side of attention (csrc/k_linear.cu)
against the oracle: quantizeInt8PerChannel + dequantize + matVec in f64
(src/core/quantize.js:36-67, src/core/ops.js:33-41), token by token."""
import numpy as np
import pytest

import b2a
from helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = b2a.Context(0)
    yield c
    c.close()


def _weights(oracle, rows, cols, seed, scale_dtype):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    q, s = oracle.quantize_int8(W, rows, cols)
    if scale_dtype == "f16":   # BASELINE config 4 stores the row scales as f16
        s_used = oracle.round_to(s, "f16")
        s_arg = oracle.to_bits(s_used, "f16")
    else:
        s_used, s_arg = s, s
    return q, s_used, s_arg


def _reference(oracle, q, s, x, bias, rows, cols, residual=None):
    Wd = oracle.dequantize_int8(q, s, rows, cols)
    out = np.stack([oracle.matvec(Wd, x[t], rows, cols, bias) for t in range(x.shape[0])])
    if residual is not None:
        out = (out.astype(np.float64) + residual).astype(np.float32)
    return out


@pytest.mark.parametrize("rows,cols,tokens,x_dt,out_dt,scale_dt,with_bias,with_res", [
    (896, 896, 1, "f32", "f32", "f32", False, True),     # o_proj of one decode token, residual add
    (896, 896, 7, "f16", "f32", "f16", False, False),
    (200, 112, 33, "bf16", "f32", "f32", True, False),   # ragged rows and tokens
    (4864, 896, 5, "f32", "f16", "f16", False, False),   # MLP-sized rows
    (896, 4864, 3, "f32", "f32", "f32", True, False),    # more columns than one staged pass
])
def test_linear_int8_matches_matvec(ctx, oracle, rows, cols, tokens, x_dt, out_dt, scale_dt, with_bias, with_res):
    q, s_used, s_arg = _weights(oracle, rows, cols, rows + cols, scale_dt)
    rng = np.random.default_rng(11)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    if x_dt != "f32":
        x = oracle.round_to(x, x_dt)
    bias = (rng.standard_normal(rows) * 0.1).astype(np.float32) if with_bias else None
    res = rng.standard_normal((tokens, rows)).astype(np.float32) if with_res else None
    out = np.empty((tokens, rows), np.float32 if out_dt == "f32" else np.uint16)
    x_arg = x if x_dt == "f32" else oracle.to_bits(x, x_dt)
    b2a.linearInt8(ctx, q, s_arg, bias, x_arg, out, rows, cols, tokens, residual=res,
                   x_dtype=x_dt if x_dt != "f32" else None, out_dtype=out_dt if out_dt != "f32" else None,
                   scale_dtype=scale_dt if scale_dt != "f32" else None)
    got = out if out_dt == "f32" else oracle.from_bits(out, out_dt)
    ref = _reference(oracle, q, s_used, x, bias, rows, cols, res)
    assert_parity(got.reshape(-1), ref.reshape(-1), out_dt, f"linear {rows}x{cols} t{tokens}")


@pytest.mark.parametrize("tokens", [1, 7, 64])
def test_qkv_int8_splits_q_k_v(ctx, oracle, tokens):
    """Qwen2.5-0.5B's fused projection: 896 -> q 896, k 128, v 128 with bias,
    f16 scales, f16 outputs as the attention call takes them."""
    hidden, qr, kvr = 896, 896, 128
    rows = qr + 2 * kvr
    q, s_used, s_arg = _weights(oracle, rows, hidden, 77, "f16")
    rng = np.random.default_rng(12)
    bias = (rng.standard_normal(rows) * 0.1).astype(np.float32)
    x = rng.standard_normal((tokens, hidden)).astype(np.float32)
    qo = np.empty((tokens, qr), np.uint16)
    ko = np.empty((tokens, kvr), np.uint16)
    vo = np.empty((tokens, kvr), np.uint16)
    b2a.qkvInt8(ctx, q, s_arg, bias, x, qo, ko, vo, hidden, qr, kvr, tokens, out_dtype="f16", scale_dtype="f16")
    ref = _reference(oracle, q, s_used, x, bias, rows, hidden)
    assert_parity(oracle.from_bits(qo, "f16").reshape(-1), ref[:, :qr].reshape(-1), "f16", "q")
    assert_parity(oracle.from_bits(ko, "f16").reshape(-1), ref[:, qr:qr + kvr].reshape(-1), "f16", "k")
    assert_parity(oracle.from_bits(vo, "f16").reshape(-1), ref[:, qr + kvr:].reshape(-1), "f16", "v")


def test_linear_rejects_bad_shapes(ctx, oracle):
    q = np.zeros((4, 20), np.int8)
    with pytest.raises(b2a.B2AError, match="multiple of 16"):
        b2a.linearInt8(ctx, q, np.ones(4, np.float32), None, np.zeros((1, 20), np.float32), np.zeros((1, 4), np.float32),
                       4, 20, 1)


def test_attention_block_composes(ctx, oracle):
    """One decode step of a Qwen2.5 attention block through the library, as
    src/cpu/model.js:98-128 runs it: fused q/k/v projection (int8, bias) ->
    RoPE + append + attention over the cache -> o_proj with the residual add.
    The oracle chains matVec, ropeInPlace, writeAt, groupedAttention and matVec
    on the same inputs (q/k/v rounded to f16, the dtype handed between kernels)."""
    from test_gpu_parity import H, KVH, D, THETA, _fill_cache, _oracle_decode, cfg
    batch, hidden = 3, 896
    lengths = [37, 200, 513]
    rope = b2a.RopeTable(ctx, D, THETA, 1024)
    c = b2a.GpuKVCache(ctx, cfg(1), 600, batch=batch, dtype="f16")
    hk, hv = _fill_cache(ctx, c, oracle, lengths, 1, "f16", 900)
    rows = H * D + 2 * KVH * D
    wq, sq, sq_arg = _weights(oracle, rows, hidden, 5, "f16")
    wo, so, so_arg = _weights(oracle, hidden, H * D, 6, "f16")
    rng = np.random.default_rng(13)
    bias = (rng.standard_normal(rows) * 0.1).astype(np.float32)
    x = rng.standard_normal((batch, hidden)).astype(np.float32)
    qo = np.empty((batch, H * D), np.uint16)
    ko = np.empty((batch, KVH * D), np.uint16)
    vo = np.empty((batch, KVH * D), np.uint16)
    b2a.qkvInt8(ctx, wq, sq_arg, bias, x, qo, ko, vo, hidden, H * D, KVH * D, batch, out_dtype="f16", scale_dtype="f16")
    att = np.empty((batch, 1, H, D), np.float32)
    b2a.attentionDecode(ctx, c, rope, 0, qo.reshape(batch, 1, H, D), ko.reshape(batch, 1, KVH, D),
                        vo.reshape(batch, 1, KVH, D), att, H, dtype="f16")
    xo = np.empty((batch, hidden), np.float32)
    b2a.linearInt8(ctx, wo, so_arg, None, att.reshape(batch, H * D), xo, hidden, H * D, batch, residual=x,
                   scale_dtype="f16")
    Wqkv = oracle.dequantize_int8(wq, sq, rows, hidden)
    Wo = oracle.dequantize_int8(wo, so, hidden, H * D)
    for b in range(batch):
        qkv = oracle.round_to(oracle.matvec(Wqkv, x[b], rows, hidden, bias), "f16")
        ref_att, _, _ = _oracle_decode(oracle, qkv[:H * D], qkv[H * D:H * D + KVH * D], qkv[H * D + KVH * D:],
                                       hk[b, 0], hv[b, 0], lengths[b], "f16")
        ref_x = (oracle.matvec(Wo, ref_att, hidden, H * D).astype(np.float64) + x[b]).astype(np.float32)
        assert_parity(xo[b], ref_x, "f32", f"attention block seq {b}")
    rope.close()
