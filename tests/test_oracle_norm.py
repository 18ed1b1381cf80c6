"""The oracle's LayerNorm producer (cpp/src/network_graph.cpp:160-166 and the
residual add of :285-287) against torch's float64 layer_norm: the exactly
rounded fp16 output the graph's fp32 normalization approximates."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import halves


@pytest.mark.parametrize("rows,cols,residual", [(4, 1280, False), (3, 1280, True), (2, 512, True), (5, 8, False)])
def test_layer_norm_matches_torch_float64(oracle, rows, cols, residual):
    import torch

    rng = np.random.default_rng(rows * cols)
    x = halves(rng, (rows, cols))
    r = halves(rng, (rows, cols)) if residual else None
    gamma = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    total, y, codes = oracle.layer_norm(x, gamma, beta, 1e-5, residual=r, code_scale=0.01)
    s = x if r is None else (x.astype(np.float32) + r.astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(total, s.view(np.uint16))
    want = torch.nn.functional.layer_norm(torch.from_numpy(s.astype(np.float64)), (cols,),
                                          torch.from_numpy(gamma.astype(np.float64)),
                                          torch.from_numpy(beta.astype(np.float64)), 1e-5)
    np.testing.assert_array_equal(y, want.numpy().astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(codes, oracle.quantize(y, np.float32(0.01)))


def test_layer_norm_constant_row_gives_beta(oracle):
    """Zero variance: (s - mean) = 0, so y = half(beta) whatever epsilon is."""
    x = np.full((2, 64), np.float16(3.5))
    beta = np.linspace(-1, 1, 64).astype(np.float32)
    _, y, _ = oracle.layer_norm(x, np.ones(64, np.float32), beta, 1e-5)
    np.testing.assert_array_equal(y, np.broadcast_to(beta.astype(np.float16).view(np.uint16), (2, 64)))
