"""The projections either side of attention, on CPU: the oracle's matVec and
int8 per-channel quantization against the reference's own tests
(test/ops.test.js:59-82, test/quantize.test.js:20-104), and the library's host
quantizer (b2a_quantize_int8_per_channel, no device needed) against the oracle
bit for bit."""
import numpy as np

import b2a


def test_matvec_known_answers(oracle):
    W = np.array([1, 2, 3, 4, 5, 6], np.float32)
    x = np.array([1, 0, -1], np.float32)
    assert list(oracle.matvec(W, x, 2, 3)) == [-2, -2]                      # ops.test.js:61-66
    assert list(oracle.matvec(W, x, 2, 3, np.array([10, 100], np.float32))) == [8, 98]   # :68-73
    W4 = np.array([1, 2, 3, 4, 5, 6, 7, 8], np.float32)
    assert list(oracle.matvec(W4, np.array([1, 10], np.float32), 4, 2)) == [21, 43, 65, 87]   # :75-82


def test_int8_codes_stay_in_symmetric_grid(oracle):
    q, _ = oracle.quantize_int8(oracle.quantize_test_rand(4 * 64, 1), 4, 64)   # quantize.test.js:22-28
    assert q.min() >= -127 and q.max() <= 127


def test_int8_row_peak_lands_on_the_grid_top(oracle):
    W = np.array([1, -2, 0.5, 0, 0.1, 0.05, -0.1, 0], np.float32)            # quantize.test.js:30-42
    q, s = oracle.quantize_int8(W, 2, 4)
    assert q[0, 1] == -127
    assert s[0] == np.float32(2 / 127)
    assert np.abs(q[1]).max() == 127


def test_int8_scales_are_per_row(oracle):
    cols = 32                                                                # quantize.test.js:44-59
    W = np.zeros(2 * cols, np.float32)
    W[:cols] = (100 * np.sin(np.arange(cols))).astype(np.float32)
    W[cols:] = (0.001 * np.cos(np.arange(cols))).astype(np.float32)
    q, s = oracle.quantize_int8(W, 2, cols)
    back = oracle.dequantize_int8(q, s, 2, cols)
    quiet, quiet_back = W[cols:], back[1]
    assert np.linalg.norm(quiet - quiet_back) / np.linalg.norm(quiet) < 0.01


def test_int8_zero_and_zero_rows(oracle):
    W = np.array([0, 1, -1, 0, 0.5, 0], np.float32)                          # quantize.test.js:61-67
    q, s = oracle.quantize_int8(W, 2, 3)
    back = oracle.dequantize_int8(q, s, 2, 3).reshape(-1)
    assert back[0] == 0 and back[3] == 0 and back[5] == 0
    W = np.array([0, 0, 0, 0, 1, 2, 3, 4], np.float32)                       # :69-76
    q, s = oracle.quantize_int8(W, 2, 4)
    assert s[0] == 0
    back = oracle.dequantize_int8(q, s, 2, 4).reshape(-1)
    assert np.all(back[:4] == 0) and np.isfinite(back[7])


def test_int8_error_within_half_a_step(oracle):
    rows, cols = 6, 128                                                      # quantize.test.js:78-94
    W = oracle.quantize_test_rand(rows * cols, 7).reshape(rows, cols)
    q, s = oracle.quantize_int8(W, rows, cols)
    back = oracle.dequantize_int8(q, s, rows, cols)
    for r in range(rows):
        assert np.all(np.abs(back[r].astype(np.float64) - W[r]) <= s[r] / 2 * 1.0001)


def test_int8_negation_negates_codes(oracle):
    W = oracle.quantize_test_rand(3 * 16, 11)                                # quantize.test.js:96-104
    a, _ = oracle.quantize_int8(W, 3, 16)
    b, _ = oracle.quantize_int8(-W, 3, 16)
    assert np.array_equal(b, -a)


def test_library_quantizer_matches_oracle(oracle):
    rng = np.random.default_rng(5)
    cases = [(oracle.quantize_test_rand(6 * 128, 7), 6, 128),
             (np.array([0, 0, 0, 0, 1, 2, 3, 4], np.float32), 2, 4),
             ((rng.standard_normal(1152 * 896) * 0.02).astype(np.float32), 1152, 896)]
    for W, rows, cols in cases:
        got = b2a.quantizeInt8PerChannel(W, rows, cols)
        q, s = oracle.quantize_int8(W, rows, cols)
        assert np.array_equal(got["q"], q) and np.array_equal(got["scales"], s)
