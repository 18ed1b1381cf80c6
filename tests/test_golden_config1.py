"""Config 1 (one encoder fc1 Q/DQ linear) against its committed golden fixture
(tests/golden/config1_fc1.npz, written by tests/golden/make_config1.py).

CPU: the oracle regenerates the fixture's scales, code digests and sampled
output rows bit for bit, and torch's own float8_e4m3fn cast agrees with the
activation codes.  GPU: the library's quantize + tcgen05 linear reproduces the
codes bit for bit and the sampled output rows within the linear's bound."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from helpers import RTOL, accumulation_bound, compare_halves

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_config1  # noqa: E402

FIXTURE = HERE / "golden" / "config1_fc1.npz"


@pytest.fixture(scope="module")
def golden():
    with np.load(FIXTURE) as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="module")
def data():
    return make_config1.inputs()


def test_fixture_shape(golden):
    assert tuple(golden["shape"]) == (make_config1.M, make_config1.K, make_config1.N)
    assert golden["y_rows"].shape == (len(golden["rows"]), make_config1.N)


def test_oracle_reproduces_scales_and_codes(golden, data, oracle):
    x, w, _ = data
    s = np.float32(oracle.amax(x)) / np.float32(448)
    assert s == golden["act_scale"][0]
    ws = oracle.weight_scales(w)
    np.testing.assert_array_equal(ws, golden["w_scales"])
    xq = oracle.quantize(x, s)
    assert make_config1.digest(xq) == str(golden["x_codes_sha256"])
    assert make_config1.digest(oracle.quantize_rows(w, ws)) == str(golden["w_codes_sha256"])
    np.testing.assert_array_equal(xq[golden["rows"]], golden["x_codes_rows"])


def test_torch_cast_agrees_with_activation_codes(golden, data):
    # An independent E4M3 rounding: torch's cast (no saturation, hence the clamp).
    import torch

    x, _, _ = data
    s = golden["act_scale"][0]
    q = (torch.from_numpy(x).float() / float(s)).clamp(-448, 448).to(torch.float8_e4m3fn)
    rows = golden["rows"]
    np.testing.assert_array_equal(q.view(torch.uint8).numpy()[rows], golden["x_codes_rows"])


def test_oracle_reproduces_output_rows(golden, data, oracle):
    x, w, b = data
    s = golden["act_scale"][0]
    ws = golden["w_scales"]
    rows = golden["rows"]
    xq = oracle.quantize(x[rows], s)
    wq = oracle.quantize_rows(w, ws)
    y, _ = oracle.fp8_linear(xq, wq, s, ws, b, gelu=True)
    np.testing.assert_array_equal(y, golden["y_rows"])


@pytest.mark.gpu
def test_gpu_config1_matches_golden(cuda, fp8, oracle, native, golden, data):
    import torch

    x, w, b = data
    xd, wd, bd = (torch.from_numpy(a).to(cuda) for a in (x, w, b))
    scale, _ = fp8.dynamic_scale(xd)
    qw = fp8.QuantizedWeight.from_half(wd, bd)
    xq = fp8.quantize(xd, scale)
    y, _ = fp8.linear(xq, qw.codes, qw.scales, scale, bias=bd, gelu=True)
    torch.cuda.synchronize()
    assert scale.item() == golden["act_scale"][0]
    np.testing.assert_array_equal(qw.scales.cpu().numpy(), golden["w_scales"])
    assert make_config1.digest(xq.cpu().numpy()) == str(golden["x_codes_sha256"])
    assert make_config1.digest(qw.codes.cpu().numpy()) == str(golden["w_codes_sha256"])
    rows = golden["rows"]
    got = y.cpu().numpy().view(np.uint16)[rows]
    extra = accumulation_bound(oracle, golden["x_codes_rows"], qw.codes.cpu().numpy(), golden["act_scale"][0],
                               golden["w_scales"], make_config1.K, gain=1.13)
    max_abs, max_rel, excess, mismatches = compare_halves(got, golden["y_rows"], rtol=2 * RTOL, extra=extra)
    print(f"config1 golden rows: max_abs={max_abs:.3g} max_rel={max_rel:.3g} mismatch={mismatches}/{got.size}")
    assert excess <= 0
    assert native.device_error() == 0
