"""FP8 Q/DQ linear on the GPU against the CPU oracle (bit-exact codes, fp16
outputs within helpers.ATOL/RTOL).  Semantics: cpp/src/network_graph.cpp:115-183."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import ATOL, RTOL, accumulation_bound, compare_halves, halves

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
    # small-M split-K cluster sizes 1, 2 and 4 (many 128-row blocks)
    (3, 40960, 256),
    (9, 20480, 640),
    (20, 10240, 1280),
    # CTA-pair tiles (M >= 512): a last pair tile whose second CTA holds only
    # padding rows, ragged N, and both tile widths
    (600, 272, 1280),
    (1024, 3840, 1280),
    (777, 1280, 5120),
    # many tiles per persistent CTA (accumulator buffers reused): 1-CTA and pairs
    (511, 20480, 128),
    (2560, 8192, 128),
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
    extra = accumulation_bound(oracle, d["xq_ref"], d["wq_ref"], d["act_scale"], d["ws_ref"], k,
                               gain=1.13 if gelu else 1.0)
    max_abs, max_rel, excess, mismatches = compare_halves(y_bits, y_ref, rtol=rtol, extra=extra)
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


@pytest.mark.parametrize("next_scale", [128.0, 2.0**-110, 200.0, 2.0**-115])
def test_fused_codes_at_quotient_limits(cuda, fp8, oracle, native, next_scale):
    """The fused next-linear codes at the limits of the magnitude quotient
    (128 and 2^-110) and beyond them, where the general quotient runs."""
    import torch

    d = _prepare(torch, fp8, oracle, cuda, 300, 1280, 640, seed=77)
    for gelu in (False, True):
        y, codes = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], gelu=gelu,
                              next_scale=next_scale)
        torch.cuda.synchronize()
        y_bits = y.cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(y_bits, np.float32(next_scale)))
    assert native.device_error() == 0


@pytest.mark.parametrize("next_scale", [0.02, 128.0, 200.0, 2.0**-115])
def test_gelu_codes_table_every_half(cuda, fp8, oracle, native, next_scale):
    """GELU with E4M3 codes as the only output reads the codes from a per-launch
    table indexed by the fp16 pre-activation.  With zero weights the
    pre-activation is +0 + bias, so a bias holding all 65,536 fp16 bit patterns
    checks every table entry against the oracle."""
    import torch

    m, n, k = 128, 65536, 16
    xq = torch.zeros((m, k), dtype=torch.uint8, device=cuda)
    wq = torch.zeros((n, k), dtype=torch.uint8, device=cuda)
    ws = torch.ones(n, dtype=torch.float32, device=cuda)
    b = torch.from_numpy(np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).copy()).to(cuda)
    pre, _ = fp8.linear(xq, wq, ws, 1.0, bias=b)
    _, codes = fp8.linear(xq, wq, ws, 1.0, bias=b, gelu=True, want_y=False, next_scale=next_scale)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    pre_bits = pre.cpu().numpy().view(np.uint16)[0]
    got = codes.cpu().numpy()
    assert np.all(got == got[0])  # every row sees the same pre-activations
    want = oracle.quantize(oracle.gelu_fp16(pre_bits), np.float32(next_scale))
    nan = np.isnan(oracle.gelu_fp16(pre_bits).view(np.float16))
    np.testing.assert_array_equal(got[0][~nan], want[~nan])
    assert np.all(got[0][nan] & 0x7F == 0x7F)


@pytest.mark.parametrize("m,n,k", [(300, 1280, 640), (777, 1280, 5120), (1500, 5120, 1280)])
def test_gelu_codes_table_matches_direct_path(cuda, fp8, oracle, native, m, n, k):
    """Codes-only GELU (table) equals the codes of the GELU + fp16 output path
    (computed directly) bit for bit, on 1-CTA and CTA-pair tiles."""
    import torch

    d = _prepare(torch, fp8, oracle, cuda, m, n, k, seed=91)
    for next_scale in (0.011, 300.0):
        _, direct = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], gelu=True,
                               next_scale=next_scale)
        _, table = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], gelu=True,
                              want_y=False, next_scale=next_scale)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(table.cpu().numpy(), direct.cpu().numpy())
    assert native.device_error() == 0


@pytest.mark.parametrize("m,n,k,rows", [
    # 1-CTA tiles: 40 x 4 = 160 tiles on 148 persistent CTAs (a partial second wave)
    (5120, 1024, 256, (0, 5120)),
    # CTA pairs (K >= 4096): 20 x 4 = 80 pair tiles on 74 pairs; rows 3328-3839 hold
    # M-tiles 13 and 14 (the latter in the partial second wave)
    (5120, 1024, 4096, (3328, 3840)),
])
def test_partial_second_wave(cuda, fp8, oracle, native, m, n, k, rows):
    """A launch with slightly more tiles than persistent CTAs (one CTA takes two
    tiles, the rest one) matches the oracle, with 1-CTA tiles and CTA pairs."""
    import torch

    d = _prepare(torch, fp8, oracle, cuda, m, n, k, seed=m + n + k)
    y, codes = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], next_scale=0.011)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    r0, r1 = rows
    xq_rows = d["xq_ref"][r0:r1]
    y_ref, _ = oracle.fp8_linear(xq_rows, d["wq_ref"], d["act_scale"], d["ws_ref"], d["b"])
    y_bits = y.cpu().numpy().view(np.uint16)[r0:r1]
    extra = accumulation_bound(oracle, xq_rows, d["wq_ref"], d["act_scale"], d["ws_ref"], k)
    max_abs, max_rel, excess, mismatches = compare_halves(y_bits, y_ref, extra=extra)
    assert excess <= 0, f"max_abs {max_abs}"
    np.testing.assert_array_equal(codes.cpu().numpy()[r0:r1], oracle.quantize(y_bits, np.float32(0.011)))


def test_linear_without_bias_and_codes_only(cuda, fp8, oracle):
    import torch

    m, n, k = 384, 768, 512
    d = _prepare(torch, fp8, oracle, cuda, m, n, k, seed=7)
    _, codes = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), want_y=False, next_scale=0.02)
    y, _ = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]))
    y_ref, _ = oracle.fp8_linear(d["xq_ref"], d["wq_ref"], d["act_scale"], d["ws_ref"], None)
    y_bits = y.cpu().numpy().view(np.uint16)
    extra = accumulation_bound(oracle, d["xq_ref"], d["wq_ref"], d["act_scale"], d["ws_ref"], k)
    assert compare_halves(y_bits, y_ref, extra=extra)[2] <= 0
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


def test_config1_fc1_full_size(cuda, fp8, oracle, native):
    """X [1500,1280] ~N(0,1), W [5120,1280] ~N(0,0.02), b ~N(0,0.02),
    dynamic act scale amax(X)/448, per-row weight scales, fc1 + bias + GELU, fp16 out."""
    import torch

    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1500, 1280, generator=gen).half()
    w = (torch.randn(5120, 1280, generator=gen) * 0.02).half()
    b = (torch.randn(5120, generator=gen) * 0.02).half()
    xd, wd, bd = x.to(cuda), w.to(cuda), b.to(cuda)
    scale, amax = fp8.dynamic_scale(xd)
    qw = fp8.QuantizedWeight.from_half(wd, bd)
    xq = fp8.quantize(xd, scale)
    y, _ = fp8.linear(xq, qw.codes, qw.scales, scale, bias=bd, gelu=True)
    xn, wn, bn = x.numpy(), w.numpy(), b.numpy()
    s = np.float32(oracle.amax(xn)) / np.float32(448)
    assert scale.item() == s
    ws = oracle.weight_scales(wn)
    xq_ref, wq_ref = oracle.quantize(xn, s), oracle.quantize_rows(wn, ws)
    np.testing.assert_array_equal(xq.cpu().numpy(), xq_ref)
    np.testing.assert_array_equal(qw.codes.cpu().numpy(), wq_ref)
    y_ref, _ = oracle.fp8_linear(xq_ref, wq_ref, s, ws, bn, gelu=True)
    y_bits = y.cpu().numpy().view(np.uint16)
    extra = accumulation_bound(oracle, xq_ref, wq_ref, s, ws, 1280, gain=1.13)
    max_abs, max_rel, excess, mismatches = compare_halves(y_bits, y_ref, rtol=2 * RTOL, extra=extra)
    print(f"config1: max_abs={max_abs:.3g} max_rel={max_rel:.3g} mismatch={mismatches}/{y_bits.size}")
    assert excess <= 0 and mismatches <= y_bits.size // 500
    assert native.device_error() == 0


def test_config2_layer_set_rows_and_fusion(cuda, fp8, oracle, native):
    """BASELINE config 2 shapes at M=12000: every linear checked on a row sample
    against the oracle; the fc1 -> fc2 fused codes equal Q of the unfused fc1."""
    import torch

    m = 12000
    rng = np.random.default_rng(2024)
    rows = np.sort(rng.choice(m, 96, replace=False))
    for name, k, n, gelu in (("qkv", 1280, 3840, False), ("out", 1280, 1280, False),
                             ("fc1", 1280, 5120, True), ("fc2", 5120, 1280, False)):
        x = halves(rng, (m, k))
        w = halves(rng, (n, k), 0.02)
        b = halves(rng, (n,), 0.02)
        s = np.float32(oracle.amax(x)) / np.float32(448)
        qw = fp8.QuantizedWeight.from_half(torch.from_numpy(w).to(cuda), torch.from_numpy(b).to(cuda))
        xq = fp8.quantize(torch.from_numpy(x).to(cuda), float(s))
        y, codes = fp8.linear(xq, qw.codes, qw.scales, float(s), bias=qw.bias, gelu=gelu,
                              next_scale=0.0123 if gelu else None)
        ws = oracle.weight_scales(w)
        xq_rows = oracle.quantize(x[rows], s)
        np.testing.assert_array_equal(xq.cpu().numpy()[rows], xq_rows)
        y_ref, _ = oracle.fp8_linear(xq_rows, oracle.quantize_rows(w, ws), s, ws, b, gelu=gelu)
        y_bits = y.cpu().numpy().view(np.uint16)
        assert np.isfinite(y.float().cpu().numpy()).all()
        extra = accumulation_bound(oracle, xq_rows, oracle.quantize_rows(w, ws), s, ws, k, gain=1.13 if gelu else 1.0)
        max_abs, max_rel, excess, mismatches = compare_halves(y_bits[rows], y_ref, rtol=2 * RTOL if gelu else RTOL,
                                                              extra=extra)
        print(f"{name}: max_abs={max_abs:.3g} mismatch={mismatches}/{y_ref.size}")
        assert excess <= 0
        if gelu:
            np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(y_bits, np.float32(0.0123)))
    torch.cuda.synchronize()
    assert native.device_error() == 0


@pytest.mark.parametrize("m,n,k", [(1, 51866, 1280), (20, 51866, 1280), (20, 1280, 1280), (32, 5120, 640), (5, 1000, 1288)])
def test_fp16_linear_small_m_matches_oracle(cuda, fp8, native, m, n, k):
    """The decoder's fp16 logits MatMul: fp16 x fp16 -> fp32 accumulate -> fp16."""
    import torch

    rng = np.random.default_rng(m * 7 + n + k)
    x = halves(rng, (m, k))
    w = halves(rng, (n, k), 0.02)
    b = halves(rng, (n,), 0.02)
    y = fp8.fp16_linear(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), torch.from_numpy(b).to(cuda))
    torch.cuda.synchronize()
    assert native.device_error() == 0
    exact = x.astype(np.float64) @ w.astype(np.float64).T  # fp16 x fp16 products are exact in binary64
    want = (exact.astype(np.float16).astype(np.float64) + b.astype(np.float64)).astype(np.float16)
    got = y.cpu().numpy()
    mag = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T
    bound = ATOL + RTOL * np.abs(want.astype(np.float64)) + k * 2.0**-24 * mag
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= bound), float((err - bound).max())


@pytest.mark.parametrize("m,n,k,gelu", [(20, 3840, 1280, False), (20, 5120, 1280, True), (7, 1280, 5120, False),
                                        (32, 1008, 1296, False)])
def test_skinny_packed_weights_match_row_major(cuda, fp8, native, m, n, k, gelu):
    """The pre-swizzled tile layout gives bit-identical results to row-major weights."""
    import torch

    rng = np.random.default_rng(m + n + k)
    w = torch.from_numpy(halves(rng, (n, k), 0.02)).to(cuda)
    b = torch.from_numpy(halves(rng, (n,), 0.02)).to(cuda)
    q = fp8.QuantizedWeight.from_half(w, b)
    packed = fp8.pack_skinny(q.codes)
    assert packed.numel() == ((n + 127) // 128) * ((k + 127) // 128) * 16384
    xq = fp8.quantize(torch.from_numpy(halves(rng, (m, k))).to(cuda), 0.01)
    y0, c0 = fp8.linear(xq, q.codes, q.scales, 0.01, bias=b, gelu=gelu, next_scale=0.02)
    y1, c1 = fp8.linear(xq, q.codes, q.scales, 0.01, bias=b, gelu=gelu, next_scale=0.02, w_packed=packed)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y0.cpu().numpy().view(np.uint16), y1.cpu().numpy().view(np.uint16))
    np.testing.assert_array_equal(c0.cpu().numpy(), c1.cpu().numpy())
    x16 = torch.from_numpy(halves(rng, (m, k))).to(cuda)
    l0 = fp8.fp16_linear(x16, w, b)
    l1 = fp8.fp16_linear(x16, w, b, w_packed=fp8.pack_skinny(w))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(l0.cpu().numpy().view(np.uint16), l1.cpu().numpy().view(np.uint16))
    assert native.device_error() == 0


def test_packed_layout_rejected_for_large_m(cuda, fp8, native):
    import torch

    q = fp8.QuantizedWeight.from_half(torch.zeros(256, 256, dtype=torch.float16, device=cuda))
    xq = torch.zeros(64, 256, dtype=torch.uint8, device=cuda)
    with pytest.raises(native.NativeError):
        fp8.linear(xq, q.codes, q.scales, 0.01, w_packed=fp8.pack_skinny(q.codes))


@pytest.mark.parametrize("m,n,k", [(7, 256, 128), (200, 1280, 1280), (777, 1280, 5120), (1500, 1280, 1280),
                                   (2560, 3840, 1280)])
def test_residual_add_in_epilogue(cuda, fp8, oracle, native, m, n, k):
    """y = linear + residual from the epilogue equals the linear alone followed by
    one fp16 rounding of the exact sum, bit for bit: single and paired tiles, both
    tile widths, ragged M, a small m (which takes the large-m kernel), and the
    in-place form (out is the residual).  The linear alone is the same kernel with
    a residual of -0, which leaves every fp16 value (and -0) unchanged; for m > 32
    it equals the plain linear bit for bit."""
    import torch

    d = _prepare(torch, fp8, oracle, cuda, m, n, k, seed=m + n + k)
    rng = np.random.default_rng(m * 7 + 1)
    residual = halves(rng, (m, n), 1.0)
    rd = _to_dev(torch, residual, cuda)
    neg_zero = torch.full((m, n), -0.0, dtype=torch.float16, device=cuda)
    alone, _ = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], residual=neg_zero)
    plain, _ = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"])
    fused, _ = fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], residual=rd)
    inplace = rd.clone()
    fp8.linear(d["xq"], d["wq"], d["ws"], float(d["act_scale"]), bias=d["bd"], residual=inplace, out=inplace)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    if m > 32:
        np.testing.assert_array_equal(alone.cpu().numpy().view(np.uint16), plain.cpu().numpy().view(np.uint16))
    a = alone.cpu().numpy().astype(np.float64)
    want = (a + residual.view(np.float16).astype(np.float64)).astype(np.float16)
    np.testing.assert_array_equal(fused.cpu().numpy().view(np.uint16), want.view(np.uint16))
    np.testing.assert_array_equal(inplace.cpu().numpy().view(np.uint16), want.view(np.uint16))
