"""LayerNorm producer on the GPU (cpp/src/network_graph.cpp:160-166 with the
residual add of :285-287) against the CPU oracle: the fp16 residual sum bit for
bit, the fp16 LayerNorm output within one fp16 ulp of the exactly rounded value
(fp32 statistics), and the E4M3 codes bit for bit against Q of the GPU's own
fp16 output."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import halves

pytestmark = pytest.mark.gpu


def _ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """|a - b| in units of the fp16 spacing at b."""
    a = a_bits.view(np.float16).astype(np.float64)
    b = b_bits.view(np.float16).astype(np.float64)
    return np.abs(a - b) / np.spacing(np.abs(b_bits.view(np.float16))).astype(np.float64)


def _inputs(rng, rows, cols, residual):
    x = halves(rng, (rows, cols))
    r = halves(rng, (rows, cols)) if residual else None
    gamma = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    return x, r, gamma, beta


@pytest.mark.parametrize("rows,cols", [(1, 1280), (7, 1280), (1500, 1280), (33, 512), (5, 4096), (3, 8),
                                       (100, 1288), (9, 2048)])
@pytest.mark.parametrize("residual", [False, True])
def test_layer_norm_matches_oracle(cuda, fp8, oracle, native, rows, cols, residual):
    import torch

    rng = np.random.default_rng(rows + cols + residual)
    x, r, gamma, beta = _inputs(rng, rows, cols, residual)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    total, y, codes = fp8.layer_norm(dev(x), dev(gamma), dev(beta), 1e-5, residual=dev(r) if residual else None,
                                     code_scale=0.011, want_sum=True)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    s_ref, y_ref, _ = oracle.layer_norm(x, gamma, beta, 1e-5, residual=r)
    np.testing.assert_array_equal(total.cpu().numpy().view(np.uint16), s_ref)
    y_bits = y.cpu().numpy().view(np.uint16)
    dist = _ulp_distance(y_bits, y_ref)
    assert dist.max() <= 1.0, float(dist.max())
    assert (y_bits == y_ref).mean() >= 0.99
    np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(y_bits, np.float32(0.011)))


def test_layer_norm_outputs_are_independent(cuda, fp8, oracle):
    """Codes only (no fp16 output: the round trip a separate quantize makes is
    skipped), sum only, and a device-resident code scale give the same bits."""
    import torch

    rng = np.random.default_rng(5)
    x, r, gamma, beta = _inputs(rng, 257, 1280, True)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    xd, rd, gd, bd = dev(x), dev(r), dev(gamma), dev(beta)
    full_sum, full_y, full_codes = fp8.layer_norm(xd, gd, bd, residual=rd, code_scale=0.02, want_sum=True)
    _, none_y, codes_only = fp8.layer_norm(xd, gd, bd, residual=rd, code_scale=0.02, want_y=False)
    sum_only, _, _ = fp8.layer_norm(xd, gd, bd, residual=rd, want_y=False, want_sum=True)
    scale = torch.tensor([0.02], dtype=torch.float32, device=cuda)
    _, _, dyn_codes = fp8.layer_norm(xd, gd, bd, residual=rd, code_scale=scale, want_y=False)
    torch.cuda.synchronize()
    assert none_y is None
    np.testing.assert_array_equal(codes_only.cpu().numpy(), full_codes.cpu().numpy())
    np.testing.assert_array_equal(dyn_codes.cpu().numpy(), full_codes.cpu().numpy())
    np.testing.assert_array_equal(sum_only.cpu().numpy(), full_sum.cpu().numpy())


def test_layer_norm_constant_rows_give_beta(cuda, fp8):
    """Zero variance: every output equals half(beta)."""
    import torch

    cols = 1280
    x = torch.full((4, cols), 2.5, dtype=torch.float16, device=cuda)
    gamma = torch.ones(cols, dtype=torch.float32, device=cuda)
    beta = torch.linspace(-1, 1, cols, dtype=torch.float32, device=cuda)
    _, y, _ = fp8.layer_norm(x, gamma, beta)
    torch.cuda.synchronize()
    want = beta.half().expand(4, cols)
    assert torch.equal(y, want)


def test_layer_norm_feeds_the_linear(cuda, fp8, oracle, native):
    """LayerNorm codes go straight into the FP8 linear: the result equals the
    linear on Q(LayerNorm output) from separate kernels."""
    import torch

    rng = np.random.default_rng(8)
    x, r, gamma, beta = _inputs(rng, 640, 1280, True)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    w = dev(halves(rng, (3840, 1280), 0.02))
    q = fp8.QuantizedWeight.from_half(w, dev(halves(rng, (3840,), 0.02)))
    _, y, codes = fp8.layer_norm(dev(x), dev(gamma), dev(beta), residual=dev(r), code_scale=0.01)
    fused, _ = fp8.linear(codes, q.codes, q.scales, 0.01, bias=q.bias)
    separate, _ = fp8.linear(fp8.quantize(y, 0.01), q.codes, q.scales, 0.01, bias=q.bias)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    assert torch.equal(fused, separate)
