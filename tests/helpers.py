"""Seeded synthetic inputs and comparison helpers shared by the tests."""

from __future__ import annotations

import numpy as np

# fp16 outputs: |gpu - oracle| <= ATOL + RTOL * |oracle|.  RTOL is one fp16 ulp
# (2^-10 relative); ATOL 2^-11 covers results near zero.  The oracle sums the
# exact E4M3 products in float64; the GPU accumulates in fp32, so the
# matmul-output rounding to fp16 can land one ulp away when the exact value is
# near a rounding midpoint.  Same bound as the reference's fp16 kernel test
# (cpp/tests/kernel_gpu.cpp:95-108, 169).
RTOL = 2.0**-10
ATOL = 2.0**-11


def halves(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return (rng.standard_normal(shape) * std).astype(np.float16)


def as_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint16)


def as_f16(bits: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16)


def compare_halves(actual_bits: np.ndarray, expected_bits: np.ndarray, atol=ATOL, rtol=RTOL):
    """Returns (max_abs, max_rel, worst excess over the bound, mismatching count)."""
    a = as_f16(actual_bits).astype(np.float64)
    e = as_f16(expected_bits).astype(np.float64)
    assert np.isfinite(a).all(), "non-finite output"
    err = np.abs(a - e)
    bound = atol + rtol * np.abs(e)
    rel = err / np.maximum(np.abs(e), 2.0**-14)
    return float(err.max(initial=0)), float(rel.max(initial=0)), float((err - bound).max(initial=-1)), int(
        (actual_bits != expected_bits).sum())
