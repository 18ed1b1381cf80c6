"""The torch CPU restatement used as the timed CPU baseline (oracle/torch_qdq.py)
agrees with the C oracle: identical E4M3 codes and weight scales, the Q/DQ
linear within the fp32-summation bound, and the fp16-edge GELU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import accumulation_bound, compare_halves, halves
from oracle import torch_qdq


@pytest.fixture(scope="module")
def data():
    rng = np.random.default_rng(17)
    x = halves(rng, (64, 256))
    w = halves(rng, (96, 256), 0.02)
    w[3] = 0  # a zero row takes scale 1
    b = halves(rng, (96,), 0.02)
    return x, w, b


def test_codes_and_scales_match_oracle(oracle, data):
    x, w, _ = data
    s = np.float32(oracle.amax(x)) / np.float32(448)
    np.testing.assert_array_equal(torch_qdq.quantize(torch.from_numpy(x), float(s)).view(torch.uint8).numpy(),
                                  oracle.quantize(x, s))
    np.testing.assert_array_equal(torch_qdq.weight_scales(torch.from_numpy(w)).numpy(), oracle.weight_scales(w))
    wq, ws = torch_qdq.prepare_weight(torch.from_numpy(w))
    np.testing.assert_array_equal(torch.from_numpy(oracle.e4m3_to_float(oracle.quantize_rows(w, ws.numpy()))),
                                  wq)


@pytest.mark.parametrize("gelu", [False, True])
def test_linear_matches_oracle(oracle, data, gelu):
    x, w, b = data
    s = np.float32(oracle.amax(x)) / np.float32(448)
    xq = oracle.quantize(x, s)
    ws = oracle.weight_scales(w)
    wq = oracle.quantize_rows(w, ws)
    want, _ = oracle.fp8_linear(xq, wq, s, ws, b, gelu=gelu)
    got = torch_qdq.linear(torch_qdq.quantize(torch.from_numpy(x), float(s)),
                           torch_qdq.prepare_weight(torch.from_numpy(w)), float(s), torch.from_numpy(b), gelu=gelu)
    extra = accumulation_bound(oracle, xq, wq, s, ws, 256, gain=1.13 if gelu else 1.0)
    assert compare_halves(got.numpy().view(np.uint16), want, rtol=2.0**-9 if gelu else 2.0**-10,
                          extra=extra)[2] <= 0


def test_gelu_fp16_matches_oracle(oracle):
    every = np.arange(65536, dtype=np.uint16)
    finite = (every & 0x7C00) != 0x7C00
    got = torch_qdq.gelu_fp16(torch.from_numpy(every.view(np.float16)[finite].copy())).numpy().view(np.uint16)
    want = oracle.gelu_fp16(every[finite])
    # torch's float erf and the oracle's binary64 erf round to the same fp16 nearly everywhere
    assert (got == want).mean() > 0.999
