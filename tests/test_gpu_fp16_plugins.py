"""The reference's fp16 projection plugins rebuilt for sm_100a, called through
the plugin enqueue of the C ABI, against the reference's own seeded test data
and expected values (tests/golden/fp16_plugins.npz from
cpp/tests/kernel_reference.hpp) and the oracle.  Tolerance and exact cases
follow cpp/tests/kernel_gpu.cpp:95-202: |d| <= atol + 2^-10 |ref| with atol
2^-11 (fc1) / 2^-12 (qkv); exact for zero input, the qkv basis vector and the
fc1 cancellation sentinels; 128-element output guard bands."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from test_capi_contract import create, digest_field

pytestmark = pytest.mark.gpu
GOLDEN = np.load(Path(__file__).parent / "golden" / "fp16_plugins.npz")
GUARD = 0xD7B0  # half_bits(-123)
WIDTH = 1280


def full_case(oracle, fc1: bool):
    """The reference's x/bias and first 32 weight rows, remaining rows seeded here."""
    name = "fc1" if fc1 else "qkv"
    rows = 5120 if fc1 else 3840
    keep = int(GOLDEN[f"{name}_expected_rows"][0])
    rng = np.random.default_rng(3318)
    w = (rng.standard_normal((rows, WIDTH)) / np.sqrt(WIDTH)).astype(np.float16).view(np.uint16)
    w[:keep] = GOLDEN[f"{name}_w"]
    x = GOLDEN[f"{name}_x"].copy()
    if fc1:
        b = rng.uniform(-0.5, 0.5, rows).astype(np.float16).view(np.uint16)
        b[:keep] = GOLDEN["fc1_bias"]
        vb = None
    else:
        b, vb = GOLDEN["qkv_bias"].copy(), GOLDEN["qkv_v_bias"].copy()
    return x, w, b, vb, GOLDEN[f"{name}_expected"][:keep].astype(np.float16).view(np.uint16), keep


def run_plugin(native, lib, torch, device, fc1, x, w, b, vb):
    T = native.TensorDesc.of
    rows = w.shape[0]
    name, version = ("LffwFp16Fc1", b"1") if fc1 else ("LffwFp16Qkv", b"2")
    plugin = create(native, lib, name, version, [digest_field(native)])
    assert plugin
    try:
        tensors = [torch.from_numpy(a.view(np.float16).copy()).to(device) for a in ([x, w, b] + ([] if fc1 else [vb]))]
        out = torch.from_numpy(np.full(rows + 128, GUARD, np.uint16).view(np.float16)).to(device)
        descs = [T((1, 1, WIDTH)), T((rows, WIDTH)), T((b.size,))] + ([] if fc1 else [T((WIDTH,))])
        ins = (native.TensorDesc * len(descs))(*descs)
        od = T((1, 1, rows))
        ptrs = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
        outs = (ctypes.c_void_p * 1)(out.data_ptr())
        stream = torch.cuda.current_stream().cuda_stream
        assert lib.lffw_plugin_enqueue(plugin, ins, ctypes.byref(od), ptrs, outs, None, stream) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        assert np.all(got[rows:] == GUARD), "projection overwrote output guard"
        return got[:rows]
    finally:
        lib.lffw_plugin_destroy(plugin)


def check(got, want, atol, exact=False):
    g = got.view(np.float16).astype(np.float64)
    e = want.view(np.float16).astype(np.float64)
    assert np.isfinite(g).all()
    if exact:
        np.testing.assert_array_equal(got, want)
    else:
        err = np.abs(g - e)
        assert np.all(err <= atol + 2.0**-10 * np.abs(e)), float(err.max())


@pytest.mark.parametrize("fc1", [True, False])
def test_projection_matches_reference_and_oracle(cuda, native, oracle, fc1):
    import torch

    lib = native.library()
    atol = 2.0**-11 if fc1 else 2.0**-12
    x, w, b, vb, ref_rows, keep = full_case(oracle, fc1)

    def expected():
        return oracle.fp16_fc1(x, w, b) if fc1 else oracle.fp16_qkv(x, w, b, vb)

    got = run_plugin(native, lib, torch, cuda, fc1, x, w, b, vb)
    check(got[:keep], ref_rows, atol)  # the reference's own expected values
    check(got, expected(), atol)
    x = (x.view(np.float16) * -1).astype(np.float16).view(np.uint16)  # negated input
    check(run_plugin(native, lib, torch, cuda, fc1, x, w, b, vb), expected(), atol)
    x = np.zeros(WIDTH, np.uint16)  # bias alone, incl. Q/K/V order and the unbiased K rows: exact
    check(run_plugin(native, lib, torch, cuda, fc1, x, w, b, vb), expected(), atol, exact=True)
    x[731] = 0x3C00  # basis vector e731: exact for qkv
    check(run_plugin(native, lib, torch, cuda, fc1, x, w, b, vb), expected(), atol, exact=not fc1)


def test_fc1_cancellation_sentinels_are_exact(cuda, native, oracle):
    # cpp/tests/kernel_gpu.cpp:190-200: a single final half rounding is wrong here.
    import torch

    lib = native.library()
    sentinels = [.0001, .0002, .0003, .0004, .0005, .0006, .001, .0015]
    x = np.zeros(WIDTH, np.uint16)
    x[0] = x[1] = 0x3C00
    w = np.zeros((5120, WIDTH), np.uint16)
    w[:, 0] = 0x3C00
    w[:, 1] = np.array([sentinels[r % 8] for r in range(5120)], np.float16).view(np.uint16)
    b = np.full(5120, 0xBC00, np.uint16)  # -1
    got = run_plugin(native, lib, torch, cuda, True, x, w, b, None)
    np.testing.assert_array_equal(got, oracle.fp16_fc1(x, w, b))


def test_bias_plugin_counts_and_guard(cuda, native, oracle):
    import torch

    lib = native.library()
    T = native.TensorDesc.of
    spec = [digest_field(native), ("bias", ctypes.c_uint16, native.FIELD_FLOAT16, [0xB600])]  # -0.375
    plugin = create(native, lib, "LffwFp16Bias", b"1", spec)
    try:
        for count in (1, 127, 128, 129, 4097):
            x = np.array([np.sin(i * .17) * 5 for i in range(count)], np.float16)
            xd = torch.from_numpy(x).to(cuda)
            out = torch.from_numpy(np.full(count + 128, GUARD, np.uint16).view(np.float16)).to(cuda)
            ins = (native.TensorDesc * 1)(T((count,)))
            od = T((count,))
            rc = lib.lffw_plugin_enqueue(plugin, ins, ctypes.byref(od), (ctypes.c_void_p * 1)(xd.data_ptr()),
                                         (ctypes.c_void_p * 1)(out.data_ptr()), None,
                                         torch.cuda.current_stream().cuda_stream)
            assert rc == 0
            got = out.cpu().numpy().view(np.uint16)
            assert np.all(got[count:] == GUARD)
            np.testing.assert_array_equal(got[:count], oracle.fp16_bias(x, 0xB600))
    finally:
        lib.lffw_plugin_destroy(plugin)


def test_fp8_linear_plugin_with_half_input(cuda, native, oracle, fp8):
    """LffwFp8Linear: fp16 activations in, Q into the workspace, fused linear out."""
    import torch

    from test_capi_contract import fp8_spec

    lib = native.library()
    T = native.TensorDesc.of
    rng = np.random.default_rng(77)
    rows, k, n = 300, 1280, 512
    x = rng.standard_normal((rows, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    b = (rng.standard_normal(n) * 0.02).astype(np.float16)
    act = float(np.float32(oracle.amax(x)) / np.float32(448))
    qw = fp8.QuantizedWeight.from_half(torch.from_numpy(w).to(cuda), torch.from_numpy(b).to(cuda))
    plugin = create(native, lib, "LffwFp8Linear", b"1", fp8_spec(native, act=act, epi=1))
    try:
        xd = torch.from_numpy(x).to(cuda)
        out = torch.empty((rows, n), dtype=torch.float16, device=cuda)
        descs = (native.TensorDesc * 4)(T((rows, k)), T((n, k), native.DT_FP8), T((n,), native.DT_FLOAT), T((n,)))
        ws_bytes = lib.lffw_plugin_workspace_size(plugin, descs, 4)
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
        ptrs = (ctypes.c_void_p * 4)(xd.data_ptr(), qw.codes.data_ptr(), qw.scales.data_ptr(), qw.bias.data_ptr())
        od = T((rows, n))
        assert lib.lffw_plugin_enqueue(plugin, descs, ctypes.byref(od), ptrs, (ctypes.c_void_p * 1)(out.data_ptr()),
                                       workspace.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        xq = oracle.quantize(x, np.float32(act))
        ws = oracle.weight_scales(w)
        want, _ = oracle.fp8_linear(xq, oracle.quantize_rows(w, ws), np.float32(act), ws, b, gelu=True)
        got = out.cpu().numpy()
        e = want.view(np.float16).astype(np.float64)
        assert np.all(np.abs(got.astype(np.float64) - e) <= 2.0**-11 + 2.0**-9 * np.abs(e))
    finally:
        lib.lffw_plugin_destroy(plugin)


@pytest.mark.parametrize("fc1", [True, False])
def test_reference_kernels_on_this_box(cuda, fp8, oracle, fc1):
    """The reference's own cpp/kernels.cu, compiled for sm_100a (oracle/_ref), on its
    seeded test data beside ours: both within the reference's tolerance of its CPU
    model, and bit-identical to each other and to the oracle's restatement of the
    kernel's fp32 summation order (same fp16 products, same fold order, same edges)."""
    import torch

    kernels = oracle.reference_kernels()
    if kernels is None:
        pytest.skip("oracle/_ref not built (reference tree not mounted when building)")
    qkv_launch, fc1_launch = kernels
    x, w, b, vb, expected, keep = full_case(oracle, fc1)
    t = lambda a: torch.from_numpy(a.view(np.float16).copy()).to(cuda)
    xd, wd, bd = t(x), t(w), t(b)
    rows = w.shape[0]
    ref_out = torch.empty(rows, dtype=torch.float16, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    if fc1:
        assert fc1_launch(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), ref_out.data_ptr(), stream) == 0
        ours = fp8.fp16_fc1(xd.view(1, -1), wd, bd)
    else:
        vbd = t(vb)
        assert qkv_launch(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), vbd.data_ptr(), ref_out.data_ptr(), stream) == 0
        ours = fp8.fp16_qkv(xd.view(1, -1), wd, bd, vbd)
    torch.cuda.synchronize()
    theirs = ref_out.cpu().numpy().view(np.uint16)
    mine = ours.reshape(-1).cpu().numpy().view(np.uint16)
    atol = 2.0**-11 if fc1 else 2.0**-12
    check(theirs[:keep], expected, atol)
    check(mine[:keep], expected, atol)
    print(f"{'fc1' if fc1 else 'qkv'}: identical to the reference kernel {np.mean(theirs == mine):.4f}")
    np.testing.assert_array_equal(mine, theirs)
    kernel_order = oracle.fp16_fc1_kernel_order(x, w, b) if fc1 else oracle.fp16_qkv_kernel_order(x, w, b, vb)
    np.testing.assert_array_equal(theirs, kernel_order)


@pytest.mark.parametrize("width", [8, 120, 128, 136, 384, 504, 512, 640, 768, 1024, 1280, 2048, 2056, 4096, 4104])
def test_projection_widths_match_kernel_order(cuda, fp8, oracle, width):
    """Every width class of the slab kernel (DEPTH 128 ... 4096, ragged last
    column group, several CTAs per SM for narrow rows) is bit-identical to the
    oracle's restatement of the reference kernel's order; widths above 4096 take
    the row-per-warp kernel (sequential per-lane order) and meet the plugins'
    tolerance.  fc1 with a row count that leaves a short last CTA."""
    import torch

    rng = np.random.default_rng(width)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.float16).copy()).to(cuda)
    x = rng.standard_normal(width).astype(np.float16).view(np.uint16)
    for fc1, rows in ((True, 997), (False, 3 * width)):
        w = (rng.standard_normal((rows, width)) / np.sqrt(width)).astype(np.float16).view(np.uint16)
        b = rng.uniform(-0.5, 0.5, rows if fc1 else width).astype(np.float16).view(np.uint16)
        vb = rng.uniform(-0.5, 0.5, width).astype(np.float16).view(np.uint16)
        if fc1:
            got = fp8.fp16_fc1(t(x).view(1, -1), t(w), t(b))
            want = oracle.fp16_fc1_kernel_order(x, w, b)
            model = oracle.fp16_fc1(x, w, b)
        else:
            got = fp8.fp16_qkv(t(x).view(1, -1), t(w), t(b), t(vb))
            want = oracle.fp16_qkv_kernel_order(x, w, b, vb)
            model = oracle.fp16_qkv(x, w, b, vb)
        got = got.reshape(-1).cpu().numpy().view(np.uint16)
        if width <= 4096:
            np.testing.assert_array_equal(got, want)
        check(got, model, 2.0**-11 if fc1 else 2.0**-12)


@pytest.mark.parametrize("width", [1024, 1280])
def test_projection_signed_zero_follows_kernel_order(cuda, fp8, oracle, width):
    """x = -0 and w = 1 make every product -0.  With DEPTH = width (1024) the
    fold keeps -0, so fc1 with bias -0 gives -0; with 1280 the +0 padding of
    DEPTH 2048 turns the sum into +0, as in the reference kernel.  (The binary64
    CPU model starts from +0 and gives +0 for both.)"""
    import torch

    t = lambda a: torch.from_numpy(a.view(np.float16).copy()).to(cuda)
    x = np.full(width, 0x8000, np.uint16)
    w = np.full((300, width), 0x3C00, np.uint16)
    b = np.full(300, 0x8000, np.uint16)
    got = fp8.fp16_fc1(t(x).view(1, -1), t(w), t(b)).cpu().numpy().view(np.uint16)
    want = oracle.fp16_fc1_kernel_order(x, w, b)
    np.testing.assert_array_equal(got, want)
    assert np.all(want == (0x8000 if width == 1024 else 0x0000))
