"""The oracle's Q/DQ linear against an independent numpy float64 evaluation of
the same graph (cpp/src/network_graph.cpp:124-183)."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import halves


def numpy_linear(xq, wq, act_scale, w_scale, bias, gelu, oracle):
    x = oracle.e4m3_to_float(xq).astype(np.float64)
    w = oracle.e4m3_to_float(wq).astype(np.float64)
    acc = x @ w.T  # exact: every partial sum fits in binary64
    y = (acc * (np.float64(act_scale) * w_scale.astype(np.float64))).astype(np.float16)
    if bias is not None:
        y = (y.astype(np.float64) + bias.astype(np.float64)).astype(np.float16)
    if gelu:
        y = oracle.halves(oracle.gelu_fp16(y))
    return y.view(np.uint16)


@pytest.mark.parametrize("m,n,k", [(1, 16, 16), (7, 48, 64), (33, 80, 1280), (5, 32, 5120)])
@pytest.mark.parametrize("gelu", [False, True])
def test_linear_matches_numpy(oracle, m, n, k, gelu):
    rng = np.random.default_rng(m * 1000 + n + k)
    x = halves(rng, (m, k))
    w = halves(rng, (n, k), 0.02)
    b = halves(rng, (n,), 0.02)
    s = np.float32(oracle.amax(x)) / np.float32(448)
    ws = oracle.weight_scales(w)
    xq, wq = oracle.quantize(x, s), oracle.quantize_rows(w, ws)
    y, codes = oracle.fp8_linear(xq, wq, s, ws, b, gelu=gelu, next_scale=np.float32(0.01))
    np.testing.assert_array_equal(y, numpy_linear(xq, wq, s, ws, b, gelu, oracle))
    np.testing.assert_array_equal(codes, oracle.quantize(y, np.float32(0.01)))
    y1, _ = oracle.fp8_linear(xq, wq, s, ws, None, threads=1)
    np.testing.assert_array_equal(y1, numpy_linear(xq, wq, s, ws, None, False, oracle))


def test_dequantized_codes_round_trip(oracle):
    # Q then DQ (half(code * scale)) is within half an E4M3 step of x.
    rng = np.random.default_rng(3)
    x = halves(rng, (4096,))
    s = np.float32(oracle.amax(x)) / np.float32(448)
    dq = oracle.e4m3_to_float(oracle.quantize(x, s)).astype(np.float64) * s
    err = np.abs(dq - x.astype(np.float64))
    step = np.maximum(np.abs(x.astype(np.float64)), 2.0**-6 * s) * 2.0**-3
    assert np.all(err <= step * 0.5 + 1e-12)
