"""Parity helpers shared by the GPU tests.

Tolerance (from the hot path's specification): outputs within max abs error
2e-3 and max relative error 1e-2 of the reference's f32 CPU attention run on
the same inputs rounded to the kernel's input dtype. "Relative error" is the
reference's own definition, max|a-b| / max|b| (web/kernels.html:56-66,
test/model.test.js:64-75). For f16/bf16 outputs the output's own rounding
(half an ulp of the output format at the reference value) is excluded from the
absolute error: no kernel can return a bf16 closer than that. KV-cache bytes
are compared bit for bit.
"""
from __future__ import annotations

import numpy as np

ATOL = 2e-3
RTOL = 1e-2


def half_ulp(ref: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return np.zeros_like(ref, dtype=np.float64)
    mant = {"f16": 10, "bf16": 7}[dtype]
    a = np.abs(ref).astype(np.float64)
    e = np.floor(np.log2(np.maximum(a, 1e-30)))
    if dtype == "f16":
        e = np.maximum(e, -14)
    return np.ldexp(1.0, (e - mant).astype(np.int64)) / 2


def compare(got, ref, out_dtype: str = "f32") -> dict:
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    diff = np.abs(got - ref)
    beyond = np.maximum(diff - half_ulp(ref, out_dtype), 0.0)
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    return {
        "max_abs": float(diff.max()) if diff.size else 0.0,
        "max_abs_beyond_rounding": float(beyond.max()) if beyond.size else 0.0,
        "rel": float(diff.max() / scale) if scale > 0 else 0.0,
        "finite": bool(np.all(np.isfinite(got))),
    }


def assert_parity(got, ref, out_dtype: str = "f32", what: str = "") -> dict:
    c = compare(got, ref, out_dtype)
    assert c["finite"], f"{what}: non-finite output"
    assert c["max_abs_beyond_rounding"] <= ATOL, f"{what}: {c}"
    assert c["rel"] <= RTOL, f"{what}: {c}"
    return c
