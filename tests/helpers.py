"""Seeded synthetic inputs and comparison helpers shared by the tests."""

from __future__ import annotations

import numpy as np

# fp16 outputs: |gpu - oracle| <= ATOL + RTOL * |oracle| + K 2^-24 sum|x w| s_x s_w.
# RTOL is one fp16 ulp (2^-10 relative) and ATOL 2^-11 covers results near
# zero -- the reference's own bound for its fp16 kernels
# (cpp/tests/kernel_gpu.cpp:95-108, 169).  The last term is the fp32 summation
# error bound of a K-term dot product: the oracle sums the exact E4M3 products
# in float64, the tensor cores accumulate in fp32 in their own order, so where
# the products cancel the fp16 rounding can move by more than one ulp.  GELU
# outputs use 2 * RTOL: a one-ulp move of the matmul output edge propagates
# through the fp16-edge GELU chain to at most two ulps.
RTOL = 2.0**-10
ATOL = 2.0**-11


def halves(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return (rng.standard_normal(shape) * std).astype(np.float16)


def as_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint16)


def as_f16(bits: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16)


def accumulation_bound(oracle, xq, wq, act_scale, w_scale, k, gain=1.0):
    """Per-output bound of fp32 summation error: K * 2^-24 * sum_k |x_k w_k| * s_x * s_w[n]
    (the classic gamma_K bound of a K-term fp32 dot product; the oracle's sum is exact).
    `gain` carries it through GELU (|GELU'| <= 1.13)."""
    xa = np.abs(oracle.e4m3_to_float(xq).astype(np.float64))
    wa = np.abs(oracle.e4m3_to_float(wq).astype(np.float64))
    mag = (xa @ wa.T) * (np.float64(act_scale) * np.asarray(w_scale, np.float64))
    return gain * k * 2.0**-24 * mag


def compare_halves(actual_bits: np.ndarray, expected_bits: np.ndarray, atol=ATOL, rtol=RTOL, extra=0.0):
    """Returns (max_abs, max_rel, worst excess over the bound, mismatching count).
    Bound: atol + rtol * |ref| + extra (per element)."""
    a = as_f16(actual_bits).astype(np.float64)
    e = as_f16(expected_bits).astype(np.float64)
    assert np.isfinite(a).all(), "non-finite output"
    err = np.abs(a - e)
    bound = atol + rtol * np.abs(e) + extra
    rel = err / np.maximum(np.abs(e), 2.0**-14)
    return float(err.max(initial=0)), float(rel.max(initial=0)), float((err - bound).max(initial=-1)), int(
        (actual_bits != expected_bits).sum())
