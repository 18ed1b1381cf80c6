"""lffw_fp8_linear_half_static: the allocation-free FP8 linear on fp16
activations.  It serves callers that cannot allocate the codes buffer the
two-call path (lffw_fp8_quantize into caller memory, then lffw_fp8_linear)
needs -- e.g. a streaming thread that must not call cudaMalloc because it can
synchronize the device, or a plugin host with a fixed workspace.  Its output
must equal that two-call path's, call after call, although every call reuses
the same buffer inside the library.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process (the first
call on the device is the one that looks up the buffer's address)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _static_entry(native):
    fn = native.library().lffw_fp8_linear_half_static
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    fn.argtypes = [vp, i64, i64, i64, ctypes.c_float, vp, vp, vp, ctypes.c_int32, vp, vp]
    fn.restype = ctypes.c_int32
    return fn


def _two_call_path(fp8, x, qw, act_scale, gelu):
    codes = fp8.quantize(x, act_scale)
    y, _ = fp8.linear(codes, qw.codes, qw.scales, act_scale, bias=qw.bias, gelu=gelu)
    return y


@pytest.mark.parametrize("m,n,k,gelu", [(1500, 5120, 1280, True), (20, 1280, 1280, False), (777, 1280, 5120, False)])
def test_static_scratch_linear_matches_two_call_path_twice(cuda, fp8, native, m, n, k, gelu):
    import torch

    fn = _static_entry(native)
    rng = np.random.default_rng(m + n + k)
    w = torch.from_numpy((rng.standard_normal((n, k)) * 0.02).astype(np.float16)).to(cuda)
    b = torch.from_numpy((rng.standard_normal(n) * 0.02).astype(np.float16)).to(cuda)
    qw = fp8.QuantizedWeight.from_half(w, b)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # the second call must not see the first call's buffer contents
        x = torch.from_numpy((rng.standard_normal((m, k)) * (1 + call)).astype(np.float16)).to(cuda)
        act_scale = float(np.float32(x.abs().max().float().item()) / np.float32(448))
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device=cuda)
        status = fn(x.data_ptr(), m, n, k, act_scale, qw.codes.data_ptr(), qw.scales.data_ptr(), b.data_ptr(),
                    native.EPILOGUE_GELU if gelu else native.EPILOGUE_NONE, y.data_ptr(), stream)
        assert status == native.SUCCESS, native.status_string(status)
        expected = _two_call_path(fp8, x, qw, act_scale, gelu)
        torch.cuda.synchronize()
        # Same kernels on the same codes: identical bits, well inside the tests' tolerance.
        np.testing.assert_array_equal(y.cpu().numpy().view(np.uint16), expected.cpu().numpy().view(np.uint16))
    assert native.device_error() == 0


def test_static_scratch_rejects_oversized_input(cuda, native):
    fn = _static_entry(native)
    limit = 8 << 20  # LFFW_STATIC_SCRATCH_BYTES
    k = 1280
    m = limit // k + 1
    status = fn(0x1000, m, 1280, k, 0.01, 0x2000, 0x3000, None, 0, 0x4000, None)
    assert status == 121  # LFFW_SCRATCH_TOO_SMALL, checked before any launch
    assert "scratch" in native.status_string(status)
