"""FP8 Q/DQ linear on the GPU against the CPU oracle (bit-exact codes, fp16
outputs within helpers.ATOL/RTOL).  Semantics: cpp/src/network_graph.cpp:115-183."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import ATOL, RTOL, as_bits, compare_halves, halves

pytestmark = pytest.mark.gpu


def _to_dev(torch, a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _prepare(torch, fp8, oracle, device, m, n, k, seed, x_std=1.0, w_std=0.02):
    rng = np.random.default_rng(seed)
    x = halves(rng, (m, k), x_std)
    w = halves(rng, (n, k), w_std)
    b = halves(rng, (n,), 0.02)
    act_scale = np.float32(oracle.amax(x)) / np.float32(448)
    xd = _to_dev(torch, x, device)
    wd = _to_dev(torch, w, device)
    bd = _to_dev(torch, b, device)
    # Weight prep on the GPU must equal the oracle bit for bit.
    ws = fp8.weight_scales(wd)
    ws_ref = oracle.weight_scales(w)
    np.testing.assert_array_equal(ws.cpu().numpy().view(np.uint32), ws_ref.view(np.uint32))
    wq = fp8.quantize_rows(wd, ws)
    wq_ref = oracle.quantize_rows(w, ws_ref)
    np.testing.assert_array_equal(wq.cpu().numpy(), wq_ref)
    xq = fp8.quantize(xd, float(act_scale))
    xq_ref = oracle.quantize(x, act_scale)
    np.testing.assert_array_equal(xq.cpu().numpy(), xq_ref)
    return dict(x=x, w=w, b=b, act_scale=act_scale, xq=xq, wq=wq, ws=ws, bd=bd, xq_ref=xq_ref,
                wq_ref=wq_ref, ws_ref=ws_ref)


CASES = [
    # (m, n, k): GEMM tiles, ragged M/N/K tails, and the small-M path
    (128, 256, 128),
    (129, 384, 256),
    (256, 512, 1280),
    (300, 1280, 640),
    (1500, 512, 1280),
    (200, 272, 5120),
    (1, 5120, 1280),
    (7, 1280, 1280),
    (20, 3840, 1280),
    (32, 1280, 5120),
]


@pytest.mark.parametrize("m,n,k", CASES)
@pytest.mark.parametrize("gelu", [False, True])
def test_linear_matches_oracle(cuda, fp8, oracle, native, m, n, k, gelu):
    import torch

    d = _prepare(torch, fp8, oracle, cuda, m, n, k, seed=1000 + m + n + k)
    next_scale = np.float32(0.011)
    y, codes = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], gelu=gelu,
                          next_scale=float(next_scale))
    torch.cuda.synchronize()
    assert native.device_error() == 0
    y_ref, codes_ref = oracle.fp8_linear(d["xq_ref"], d["wq_ref"], d["act_scale"], d["ws_ref"], d["b"],
                                         gelu=gelu, next_scale=next_scale)
    y_bits = y.cpu().numpy().view(np.uint16)
    # GELU outputs: a one-ulp difference of the matmul output edge (fp32 vs
    # exact accumulation) moves the fp16-edge GELU chain by at most two ulps.
    rtol = 2 * RTOL if gelu else RTOL
    max_abs, max_rel, excess, mismatches = compare_halves(y_bits, y_ref, rtol=rtol)
    print(f"m={m} n={n} k={k} gelu={gelu}: max_abs={max_abs:.3g} max_rel={max_rel:.3g} "
          f"mismatch={mismatches}/{y_bits.size}")
    assert excess <= 0, f"fp16 output outside {ATOL}+{rtol}*|ref| (max_abs {max_abs})"
    assert mismatches <= max(8, y_bits.size // 500)
    if gelu:
        # The fused epilogue equals the oracle's GELU applied to the GPU's own
        # pre-activation (same GEMM without GELU), bit for bit.
        pre, _ = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"])
        np.testing.assert_array_equal(y_bits, oracle.gelu_fp16(pre.cpu().numpy().view(np.uint16)))
    # Codes of the fused next-linear quantize are bit-exact wherever the fp16
    # value matches, and equal the oracle's Q of the GPU's own fp16 value.
    got = codes.cpu().numpy()
    same = y_bits == y_ref
    np.testing.assert_array_equal(got[same], codes_ref[same])
    np.testing.assert_array_equal(got, oracle.quantize(y_bits, next_scale))


def test_linear_without_bias_and_codes_only(cuda, fp8, oracle):
    import torch

    m, n, k = 384, 768, 512
    d = _prepare(torch, fp8, oracle, cuda, m, n, k, seed=7)
    _, codes = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), want_y=False, next_scale=0.02)
    y, _ = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]))
    y_ref, _ = oracle.fp8_linear(d["xq_ref"], d["wq_ref"], d["act_scale"], d["ws_ref"], None)
    y_bits = y.cpu().numpy().view(np.uint16)
    assert compare_halves(y_bits, y_ref)[2] <= 0
    np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(y_bits, np.float32(0.02)))


def test_dynamic_scale_matches_oracle(cuda, fp8, oracle):
    import torch

    rng = np.random.default_rng(3)
    for count in (1, 17, 4096, 1500 * 1280 + 3):
        x = halves(rng, (count,), 1.0)
        scale, amax = fp8.dynamic_scale(torch.from_numpy(x).to(cuda))
        expected_amax = np.float32(oracle.amax(x))
        assert amax.item() == expected_amax
        assert scale.item() == np.float32(expected_amax / np.float32(448))
    zero = torch.zeros(100, dtype=torch.float16, device=cuda)
    scale, amax = fp8.dynamic_scale(zero)
    assert amax.item() == 0.0 and scale.item() == 1.0
