"""E4M3 quantization and scale kernels on the GPU: bit-exact against the oracle
and the hand-written edge table."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"
ALL_HALVES = np.arange(65536, dtype=np.uint32).astype(np.uint16)


def test_edge_table_on_gpu(cuda, fp8):
    import torch

    for e in json.loads((GOLDEN / "e4m3_edges.json").read_text()):
        x = torch.from_numpy(np.full(16, e["x_bits"], np.uint16).view(np.float16)).to(cuda)
        got = fp8.quantize(x, e["scale"]).cpu().numpy()
        assert np.all(got == e["code"]), (e["why"], got[0])


@pytest.mark.parametrize("scale", [1.0, 0.011, 1 / 448, 3.7, 2.0**-10, 123.25])
def test_every_half_bit_exact(cuda, fp8, oracle, scale):
    import torch

    x = torch.from_numpy(ALL_HALVES.view(np.float16).copy()).to(cuda)
    got = fp8.quantize(x, scale).cpu().numpy()
    want = oracle.quantize(ALL_HALVES, scale)
    nan = np.isnan(ALL_HALVES.view(np.float16))
    np.testing.assert_array_equal(got[~nan], want[~nan])
    assert np.all(got[nan] & 0x7F == 0x7F)
    # Scales in [2^-110, 128] take the magnitude quotient, which also keeps a
    # NaN's sign as the oracle does.
    np.testing.assert_array_equal(got, want)
    # scale read from device memory gives the same codes
    s = torch.tensor([scale], dtype=torch.float32, device=cuda)
    np.testing.assert_array_equal(fp8.quantize(x, s).cpu().numpy(), got)


def test_random_scales_every_half(cuda, fp8, oracle):
    """The division-free quotient equals IEEE fp32 division for every fp16 input."""
    import torch

    rng = np.random.default_rng(21)
    x = torch.from_numpy(ALL_HALVES.view(np.float16).copy()).to(cuda)
    nan = np.isnan(ALL_HALVES.view(np.float16))
    scales = list(np.exp2(rng.uniform(-20, 10, 96)).astype(np.float32))
    # significands next to 2 and to 1: the reciprocal's rounding error is largest there
    scales += [np.float32(np.nextafter(np.float32(2.0), np.float32(0)) * 2.0**e) for e in (-12, -3, 0, 5)]
    scales += [np.float32(np.nextafter(np.float32(1.0), np.float32(2)) * 2.0**e) for e in (-9, 0, 7)]
    scales += [np.float32(1 / 448), np.float32(3.0), np.float32(0.1), np.float32(2.0**-125), np.float32(2.0**125)]
    for scale in scales:
        got = fp8.quantize(x, float(scale)).cpu().numpy()
        np.testing.assert_array_equal(got[~nan], oracle.quantize(ALL_HALVES, scale)[~nan], err_msg=str(scale))


@pytest.mark.parametrize("count", [1, 15, 16, 17, 1023, 4099, 1500 * 1280])
def test_ragged_sizes_and_guard_band(cuda, fp8, oracle, count):
    import torch

    rng = np.random.default_rng(count)
    x = (rng.standard_normal(count) * 3).astype(np.float16)
    out = torch.full((count + 128,), 0xA5, dtype=torch.uint8, device=cuda)
    fp8.quantize(torch.from_numpy(x).to(cuda), 0.02, out=out[:count])
    got = out.cpu().numpy()
    np.testing.assert_array_equal(got[:count], oracle.quantize(x, 0.02))
    assert np.all(got[count:] == 0xA5), "quantize wrote past its output"


def test_weight_prep_bit_exact(cuda, fp8, oracle):
    import torch

    rng = np.random.default_rng(9)
    for rows, cols in ((3, 16), (5120, 1280), (1280, 5120), (7, 4112)):
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
        w[rows // 2] = 0  # an all-zero row maps to scale 1 (network_graph.cpp:146-147)
        wd = torch.from_numpy(w).to(cuda)
        scales = fp8.weight_scales(wd)
        want = oracle.weight_scales(w)
        np.testing.assert_array_equal(scales.cpu().numpy(), want)
        assert want[rows // 2] == 1.0
        np.testing.assert_array_equal(fp8.quantize_rows(wd, scales).cpu().numpy(), oracle.quantize_rows(w, want))


def test_gelu_every_half_matches_oracle(cuda, fp8, oracle):
    import torch

    x = torch.from_numpy(ALL_HALVES.view(np.float16).copy()).to(cuda)
    got = fp8.fp16_gelu(x).cpu().numpy().view(np.uint16)
    want = oracle.gelu_fp16(ALL_HALVES)
    nan = np.isnan(want.view(np.float16))
    assert np.all(np.isnan(got[nan].view(np.float16)))
    mismatch = np.nonzero(got[~nan] != want[~nan])[0]
    assert mismatch.size == 0, [(hex(ALL_HALVES[~nan][i]), hex(got[~nan][i]), hex(want[~nan][i]))
                                for i in mismatch[:10]]
