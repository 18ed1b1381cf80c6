"""The oracle's E4M3 quantizer and fp16 conversions, pinned against the
hand-written E4M3 edge table and torch's float8_e4m3fn cast (which rounds to
nearest even but does not saturate: inputs are clamped to +-448 first)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).parent / "golden"
ALL_HALVES = np.arange(65536, dtype=np.uint32).astype(np.uint16)


def test_edge_table(oracle):
    for e in json.loads((GOLDEN / "e4m3_edges.json").read_text()):
        got = oracle.quantize(np.array([e["x_bits"]], np.uint16), e["scale"])[0]
        assert got == e["code"], e["why"]
        assert oracle.e4m3_to_float(np.array([e["code"]], np.uint8))[0] == np.float32(e["code_value"])


def torch_codes(q: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(q.astype(np.float32)).clamp(-448, 448)
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


@pytest.mark.parametrize("scale", [1.0, 0.011, 1 / 448, 3.7, 2.0**-10, 0.002232142857, 123.25])
def test_every_half_against_torch(oracle, scale):
    codes = oracle.quantize(ALL_HALVES, scale)
    x = ALL_HALVES.view(np.float16).astype(np.float32)
    q = x / np.float32(scale)  # IEEE fp32 quotient, as the Q layer computes it
    finite = np.isfinite(q)
    np.testing.assert_array_equal(codes[finite], torch_codes(q[finite]))
    nan = np.isnan(x)
    assert np.all(codes[nan] & 0x7F == 0x7F)  # NaN stays NaN
    inf = np.isinf(q) & ~nan
    np.testing.assert_array_equal(codes[inf], np.where(q[inf] > 0, 0x7E, 0xFE))


def test_decode_table_matches_torch(oracle):
    codes = np.arange(256, dtype=np.uint8)
    ours = oracle.e4m3_to_float(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    same = ~np.isnan(theirs)
    np.testing.assert_array_equal(ours[same], theirs[same])
    assert np.isnan(ours[~same]).all() and set(codes[~same]) == {0x7F, 0xFF}


def test_random_floats_against_torch(oracle):
    rng = np.random.default_rng(11)
    v = np.concatenate([rng.standard_normal(200000) * s for s in (1e-3, 1.0, 100.0, 1e4)]).astype(np.float32)
    np.testing.assert_array_equal(oracle.e4m3_from_float(v), torch_codes(v))


def test_half_rounding_matches_numpy(oracle):
    rng = np.random.default_rng(12)
    v = np.concatenate([
        rng.standard_normal(100000) * 10.0 ** rng.integers(-9, 5, 100000),
        [65504.0, 65519.99, 65520.0, 70000.0, -65520.0, 2.0**-25, 2.0**-24 * 1.5, 2.0**-24 * 0.5,
         1.0 + 2.0**-11, 1.0 + 3 * 2.0**-11, np.inf, -np.inf, 0.0, -0.0],
    ])
    np.testing.assert_array_equal(oracle.half_from_double(v), v.astype(np.float16).view(np.uint16))


def test_amax_and_weight_scales(oracle):
    x = np.array([1.0, -3.5, np.nan, 2.0], np.float16)
    assert oracle.amax(x) == 3.5
    # The toy checkpoint of python/tests/test_fp8_graph.py:150 (values (arange+1)/100):
    # the graph's weight scale is max(|W[n,:]|)/448 per output row
    # (test_fp8_graph.py:207-211).
    for shape in ((4, 4), (8, 4), (4, 8)):
        w = ((np.arange(np.prod(shape), dtype=np.float32).reshape(shape) + 1) / 100).astype(np.float16)
        expected = np.max(np.abs(w.astype(np.float32)), axis=1) / np.float32(448)
        np.testing.assert_array_equal(oracle.weight_scales(w), expected.astype(np.float32))
    zero = np.zeros((3, 16), np.float16)
    np.testing.assert_array_equal(oracle.weight_scales(zero), np.ones(3, np.float32))
