"""The reference's dtype tests (test/dtype.test.js) restated against the oracle,
and checked against numpy's own f16 (an independent implementation)."""
import numpy as np


def test_bf16_widening_is_the_shift(oracle):
    b = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.bf16_bits_to_f32(b).view(np.uint32)
    assert np.array_equal(got, b.astype(np.uint32) << 16)


def test_bf16_round_trips(oracle):
    b = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    nan = ((b & 0x7F80) == 0x7F80) & ((b & 0x007F) != 0)
    back = oracle.f32_to_bf16_bits(oracle.bf16_bits_to_f32(b))
    assert np.array_equal(back[~nan], b[~nan])


def test_bf16_rounds_to_nearest_even(oracle):
    x = np.array([0x3F808000, 0x3F818000, 0x3F808001], np.uint32).view(np.float32)
    assert list(oracle.f32_to_bf16_bits(x)) == [0x3F80, 0x3F82, 0x3F81]


def test_bf16_saturates_to_infinity(oracle):
    x = np.array([0x7F7FFFFF, 0xFF7FFFFF], np.uint32).view(np.float32)
    assert list(oracle.f32_to_bf16_bits(x)) == [0x7F80, 0xFF80]
    assert list(oracle.f32_to_bf16_bits(np.array([np.inf, -np.inf], np.float32))) == [0x7F80, 0xFF80]


def test_bf16_preserves_nan(oracle):
    for pattern in (0x7F81, 0x7FC0, 0x7FFF, 0xFFC1):
        w = oracle.bf16_bits_to_f32(np.array([pattern], np.uint16))
        assert np.isnan(w[0])
        n = int(oracle.f32_to_bf16_bits(w)[0])
        assert (n & 0x7F80) == 0x7F80 and (n & 0x007F) != 0 and (n >> 15) == (pattern >> 15)


def test_f16_widening_matches_numpy(oracle):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.f16_bits_to_f32(h)
    ref = h.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.all(np.isnan(got[nan]))
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f16_narrowing_matches_numpy_between_values(oracle):
    h = np.arange(0, 65535, dtype=np.uint32).astype(np.uint16)
    lo = h.view(np.float16).astype(np.float64)
    hi = (h + 1).astype(np.uint16).view(np.float16).astype(np.float64)
    ok = np.isfinite(lo) & np.isfinite(hi)
    probes = np.concatenate([lo[ok] + (hi[ok] - lo[ok]) / 2, lo[ok] + (hi[ok] - lo[ok]) * 0.25,
                             lo[ok] + (hi[ok] - lo[ok]) * 0.75]).astype(np.float32)
    got = oracle.f32_to_f16_bits(probes)
    ref = probes.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, ref)


def test_dtype_golden_probes(oracle, golden):
    p = golden["dtype_probes"]
    assert np.array_equal(oracle.f32_to_f16_bits(p), golden["dtype_probes_f16"])
    assert np.array_equal(oracle.f32_to_bf16_bits(p), golden["dtype_probes_bf16"])
