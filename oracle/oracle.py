"""numpy front end of the C oracle (liblffw_oracle.so).  TEST INFRASTRUCTURE ONLY.

Each function restates the reference arithmetic cited in lffw_oracle.h:
E4M3 quantization per TensorRT's Q (cpp/src/network_graph.cpp:115-123), the
Q/DQ linear (network_graph.cpp:124-159), GELU with fp16 edges
(network_graph.cpp:168-180), and the fp16 projection plugins
(cpp/tests/kernel_reference.hpp:20-50).  Halves are numpy uint16 bit patterns
(or float16 arrays), E4M3 codes are uint8.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liblffw_oracle.so"
REF_LIBRARY = HERE / "_ref" / "libref_fp16.so"

_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_lib = None


def build() -> None:
    subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        L = ctypes.CDLL(str(LIBRARY))
        L.oracle_e4m3_from_floats.argtypes = [_f32p, ctypes.c_size_t, _u8p]
        L.oracle_e4m3_to_floats.argtypes = [_u8p, ctypes.c_size_t, _f32p]
        L.oracle_halves_from_doubles.argtypes = [_f64p, ctypes.c_size_t, _u16p]
        L.oracle_gelu_fp16_array.argtypes = [_u16p, ctypes.c_size_t, _u16p]
        L.oracle_quantize.argtypes = [_u16p, ctypes.c_size_t, ctypes.c_float, _u8p]
        L.oracle_quantize_rows.argtypes = [_u16p, ctypes.c_int64, ctypes.c_int64, _f32p, _u8p]
        L.oracle_amax.argtypes = [_u16p, ctypes.c_size_t]
        L.oracle_amax.restype = ctypes.c_float
        L.oracle_weight_scales.argtypes = [_u16p, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.oracle_fp8_linear.argtypes = [
            _u8p, _u8p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _f32p,
            _u16p, ctypes.c_int, _u16p, ctypes.c_float, _u8p, ctypes.c_int,
        ]
        L.oracle_fp16_fc1.argtypes = [_u16p, _u16p, _u16p, _u16p, ctypes.c_int64, ctypes.c_int64]
        L.oracle_fp16_qkv.argtypes = [_u16p, _u16p, _u16p, _u16p, _u16p, ctypes.c_int64]
        L.oracle_fp16_bias.argtypes = [_u16p, ctypes.c_uint16, _u16p, ctypes.c_int64]
        L.oracle_fp16_fc1_kernel_order.argtypes = [_u16p, _u16p, _u16p, _u16p, ctypes.c_int64, ctypes.c_int64]
        L.oracle_fp16_qkv_kernel_order.argtypes = [_u16p, _u16p, _u16p, _u16p, _u16p, ctypes.c_int64]
        L.oracle_threads.restype = ctypes.c_int
        L.oracle_layer_norm.argtypes = [
            _u16p, _u16p, ctypes.c_int64, ctypes.c_int64, _f32p, _f32p, ctypes.c_float, _u16p, _u16p,
            ctypes.c_float, _u8p,
        ]
        L.oracle_cross_attention.argtypes = [
            _u16p, _u16p, _u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p,
            ctypes.c_float, _u8p,
        ]
        L.oracle_self_attention.argtypes = [
            _u16p, _u16p, _u16p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, _u16p, ctypes.c_float, _u8p,
        ]
        L.oracle_erf_fp16.argtypes = [ctypes.c_uint16]
        L.oracle_erf_fp16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _ptr(array: np.ndarray | None, kind):
    if array is None:
        return None
    assert array.flags["C_CONTIGUOUS"]
    return array.ctypes.data_as(kind)


def bits16(a) -> np.ndarray:
    """float16 array (or uint16 bit patterns) -> contiguous uint16 bit patterns."""
    a = np.asarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    return np.ascontiguousarray(a, dtype=np.uint16)


def halves(bits: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16)


def e4m3_from_float(values) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(v.shape, np.uint8)
    lib().oracle_e4m3_from_floats(_ptr(v, _f32p), v.size, _ptr(out, _u8p))
    return out


def e4m3_to_float(codes) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(c.shape, np.float32)
    lib().oracle_e4m3_to_floats(_ptr(c, _u8p), c.size, _ptr(out, _f32p))
    return out


def half_from_double(values) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float64)
    out = np.empty(v.shape, np.uint16)
    lib().oracle_halves_from_doubles(_ptr(v, _f64p), v.size, _ptr(out, _u16p))
    return out


def gelu_fp16(x) -> np.ndarray:
    b = bits16(x)
    out = np.empty(b.shape, np.uint16)
    lib().oracle_gelu_fp16_array(_ptr(b, _u16p), b.size, _ptr(out, _u16p))
    return out


def erf_fp16(x) -> np.ndarray:
    b = bits16(x)
    f = lib().oracle_erf_fp16
    return np.array([f(int(v)) for v in b.ravel()], np.uint16).reshape(b.shape)


def quantize(x, scale: float) -> np.ndarray:
    """codes = E4M3_rne_sat(fp32(x / scale)) for fp16 x and one fp32 scale."""
    b = bits16(x)
    out = np.empty(b.shape, np.uint8)
    lib().oracle_quantize(_ptr(b, _u16p), b.size, float(np.float32(scale)), _ptr(out, _u8p))
    return out


def layer_norm(x, gamma, beta, eps: float = 1e-5, residual=None, code_scale=None):
    """(sum, y, codes): s = half(x + residual) (or x), y = half(LN(s) * gamma + beta)
    with binary64 statistics, codes = Q(y / code_scale) (None without a scale);
    cpp/src/network_graph.cpp:160-166, 285-287."""
    b = bits16(x)
    rows, cols = b.shape
    r = bits16(residual) if residual is not None else None
    g = np.ascontiguousarray(gamma, dtype=np.float32)
    be = np.ascontiguousarray(beta, dtype=np.float32)
    assert g.shape == (cols,) and be.shape == (cols,)
    s = np.empty(b.shape, np.uint16)
    y = np.empty(b.shape, np.uint16)
    codes = np.empty(b.shape, np.uint8) if code_scale is not None else None
    lib().oracle_layer_norm(_ptr(b, _u16p), _ptr(r, _u16p), rows, cols, _ptr(g, _f32p), _ptr(be, _f32p),
                            float(np.float32(eps)), _ptr(s, _u16p), _ptr(y, _u16p),
                            float(np.float32(code_scale)) if code_scale is not None else 1.0,
                            _ptr(codes, _u8p))
    return s, y, codes


def cross_attention(q, k, v, queries: int, code_scale=None):
    """(out, codes) of the decoder cross-attention (network_graph.cpp:235-244, 401-404):
    q [streams * queries, heads * dim], k/v [streams, heads, keys, dim] fp16."""
    qb, kb, vb = bits16(q), bits16(k), bits16(v)
    streams, heads, keys, dim = kb.shape
    assert vb.shape == kb.shape and qb.shape == (streams * queries, heads * dim)
    out = np.empty(qb.shape, np.uint16)
    codes = np.empty(qb.shape, np.uint8) if code_scale is not None else None
    lib().oracle_cross_attention(_ptr(qb, _u16p), _ptr(kb, _u16p), _ptr(vb, _u16p), streams, queries, heads, dim,
                                 keys, _ptr(out, _u16p),
                                 float(np.float32(code_scale)) if code_scale is not None else 1.0, _ptr(codes, _u8p))
    return out, codes


def self_attention(qkv, streams: int, heads: int, code_scale=None):
    """(out, codes) of the encoder self-attention (network_graph.cpp:235-247) on a fused
    QKV projection output [streams * tokens, 3 * heads * 64] (q | k | v columns)."""
    b = bits16(qkv)
    rows, cols = b.shape
    width = cols // 3
    dim = width // heads
    tokens = rows // streams
    out = np.empty((rows, width), np.uint16)
    codes = np.empty((rows, width), np.uint8) if code_scale is not None else None
    base = b.ctypes.data
    u16 = np.dtype(np.uint16).itemsize
    ptr = lambda off: ctypes.cast(base + off * u16, _u16p)
    lib().oracle_self_attention(ptr(0), ptr(width), ptr(2 * width), cols, cols, cols, streams, tokens, heads, dim,
                                _ptr(out, _u16p), float(np.float32(code_scale)) if code_scale is not None else 1.0,
                                _ptr(codes, _u8p))
    return out, codes


def mel_frames(mel) -> np.ndarray:
    """half(mel) (network_graph.cpp:257) as fp16 bits [streams, frames + 2, mels],
    time-major, with zero rows 0 and frames + 1: the padded convolution input."""
    m = np.asarray(mel, np.float32)
    streams, mels, frames = m.shape
    out = np.zeros((streams, frames + 2, mels), np.uint16)
    out[:, 1:frames + 1, :] = m.astype(np.float16).view(np.uint16).transpose(0, 2, 1)
    return out


def conv1d_gelu(frames, weight, bias, stride: int, positions=None):
    """One encoder convolution (network_graph.cpp:259-275: kernel 3, padding 1, the
    given stride, bias) followed by GELU with fp16 edges and, with `positions`, the
    fp16 positional add of :280-282.

    frames: fp16 bits [streams, frames_in + 2, c_in] (row r = input frame r - 1,
    rows 0 and frames_in + 1 zero); weight: fp16 [c_out, c_in, 3] (the checkpoint's
    conv1d layout); bias fp16 [c_out]; positions fp16 [frames_out, c_out].
    The sum of fp16 products plus the bias is accumulated in binary64 (each product
    is exact; the sum's error is below K 2^-53 of the sum of magnitudes) and
    rounded to fp16 once.  Returns (pre-GELU, GELU, output) fp16 bit arrays
    [streams, frames_out, c_out]; output is the GELU without positions."""
    x = halves(bits16(frames)).astype(np.float64)
    w = halves(bits16(weight)).astype(np.float64)
    b = halves(bits16(bias)).astype(np.float64)
    streams, rows, c_in = x.shape
    frames_in = rows - 2
    frames_out = frames_in // stride
    acc = np.zeros((streams, frames_out, w.shape[0]), np.float64)
    for j in range(3):
        taps = x[:, j: j + stride * (frames_out - 1) + 1: stride, :]  # padded row stride * t + j
        acc += taps @ w[:, :, j].T
    pre = half_from_double(acc + b)
    act = gelu_fp16(pre)
    if positions is None:
        return pre, act, act
    pos = halves(bits16(positions)).astype(np.float64)
    out = half_from_double(halves(act).astype(np.float64) + pos[None, :frames_out, :])
    return pre, act, out


def quantize_rows(w, scales) -> np.ndarray:
    b = bits16(w)
    s = np.ascontiguousarray(scales, dtype=np.float32)
    rows, cols = b.shape
    assert s.shape == (rows,)
    out = np.empty(b.shape, np.uint8)
    lib().oracle_quantize_rows(_ptr(b, _u16p), rows, cols, _ptr(s, _f32p), _ptr(out, _u8p))
    return out


def amax(x) -> float:
    b = bits16(x)
    return float(lib().oracle_amax(_ptr(b, _u16p), b.size))


def weight_scales(w) -> np.ndarray:
    b = bits16(w)
    rows, cols = b.shape
    out = np.empty(rows, np.float32)
    lib().oracle_weight_scales(_ptr(b, _u16p), rows, cols, _ptr(out, _f32p))
    return out


def fp8_linear(xq, wq, act_scale: float, w_scale, bias=None, *, gelu: bool = False,
               next_scale: float | None = None, want_y: bool = True, threads: int = 0):
    """The Q/DQ linear on E4M3 codes.  Returns (y uint16 [m,n] or None, codes or None)."""
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    wq = np.ascontiguousarray(wq, dtype=np.uint8)
    m, k = xq.shape
    n, k2 = wq.shape
    assert k == k2
    ws = np.ascontiguousarray(w_scale, dtype=np.float32)
    b = None if bias is None else bits16(bias)
    y = np.empty((m, n), np.uint16) if want_y else None
    codes = np.empty((m, n), np.uint8) if next_scale is not None else None
    lib().oracle_fp8_linear(
        _ptr(xq, _u8p), _ptr(wq, _u8p), m, n, k, float(np.float32(act_scale)), _ptr(ws, _f32p),
        _ptr(b, _u16p), int(gelu), _ptr(y, _u16p),
        float(np.float32(next_scale)) if next_scale is not None else 0.0, _ptr(codes, _u8p),
        int(threads),
    )
    return y, codes


def fp16_fc1(x, w, bias) -> np.ndarray:
    xb, wb, bb = bits16(x), bits16(w), bits16(bias)
    rows, width = wb.shape
    out = np.empty(rows, np.uint16)
    lib().oracle_fp16_fc1(_ptr(xb, _u16p), _ptr(wb, _u16p), _ptr(bb, _u16p), _ptr(out, _u16p), rows, width)
    return out


def fp16_qkv(x, w, q_bias, v_bias) -> np.ndarray:
    xb, wb, qb, vb = bits16(x), bits16(w), bits16(q_bias), bits16(v_bias)
    width = xb.size
    out = np.empty(3 * width, np.uint16)
    lib().oracle_fp16_qkv(_ptr(xb, _u16p), _ptr(wb, _u16p), _ptr(qb, _u16p), _ptr(vb, _u16p),
                          _ptr(out, _u16p), width)
    return out


def fp16_fc1_kernel_order(x, w, bias) -> np.ndarray:
    """fp16_fc1 with the reference kernel's fp32 summation order (cpp/kernels.cu:27-49)."""
    xb, wb, bb = bits16(x), bits16(w), bits16(bias)
    rows, width = wb.shape
    out = np.empty(rows, np.uint16)
    if lib().oracle_fp16_fc1_kernel_order(_ptr(xb, _u16p), _ptr(wb, _u16p), _ptr(bb, _u16p), _ptr(out, _u16p),
                                          rows, width) != 0:
        raise MemoryError("oracle_fp16_fc1_kernel_order")
    return out


def fp16_qkv_kernel_order(x, w, q_bias, v_bias) -> np.ndarray:
    """fp16_qkv with the reference kernel's fp32 summation order (cpp/kernels.cu:27-49)."""
    xb, wb, qb, vb = bits16(x), bits16(w), bits16(q_bias), bits16(v_bias)
    width = xb.size
    out = np.empty(3 * width, np.uint16)
    if lib().oracle_fp16_qkv_kernel_order(_ptr(xb, _u16p), _ptr(wb, _u16p), _ptr(qb, _u16p), _ptr(vb, _u16p),
                                          _ptr(out, _u16p), width) != 0:
        raise MemoryError("oracle_fp16_qkv_kernel_order")
    return out


def fp16_bias(x, bias_bits: int) -> np.ndarray:
    xb = bits16(x)
    out = np.empty(xb.shape, np.uint16)
    lib().oracle_fp16_bias(_ptr(xb, _u16p), int(bias_bits), _ptr(out, _u16p), xb.size)
    return out


def threads() -> int:
    return int(lib().oracle_threads())


# ---- the reference's own CPU model (oracle/_ref, built only where the
# reference tree is mounted) --------------------------------------------------

def reference_available() -> bool:
    return REF_LIBRARY.exists()


def reference_projection(fc1: bool):
    """(x, weight, bias, v_bias, expected) of the reference's seeded plugin test."""
    L = ctypes.CDLL(str(REF_LIBRARY))
    L.ref_fp16_projection.argtypes = [ctypes.c_int, _u16p, _u16p, _u16p, _u16p, _f64p]
    L.ref_fp16_projection.restype = ctypes.c_int
    width = 1280
    rows = 5120 if fc1 else 3840
    x = np.empty(width, np.uint16)
    w = np.empty(rows * width, np.uint16)
    b = np.empty(rows if fc1 else width, np.uint16)
    vb = np.empty(width, np.uint16)
    expected = np.empty(rows, np.float64)
    got = L.ref_fp16_projection(int(fc1), _ptr(x, _u16p), _ptr(w, _u16p), _ptr(b, _u16p),
                                _ptr(vb, _u16p), _ptr(expected, _f64p))
    assert got == rows
    return x, w.reshape(rows, width), b, (None if fc1 else vb), expected


def reference_gelu(dot: float, bias: float) -> float:
    L = ctypes.CDLL(str(REF_LIBRARY))
    L.ref_gelu.argtypes = [ctypes.c_double, ctypes.c_double]
    L.ref_gelu.restype = ctypes.c_double
    return float(L.ref_gelu(dot, bias))


# ---- the reference's own fp16 projection kernels (oracle/_ref, built for sm_100a
# only where the reference tree is mounted): the same-box baseline ----------------

REF_KERNELS = HERE / "_ref" / "libref_fp16_kernels.so"


def reference_kernels():
    """(qkv_launch, fc1_launch) ctypes functions launching cpp/kernels.cu's qkv_fp16 and
    fc1_fp16 with the plugins' geometry, or None when oracle/_ref was not built."""
    if not REF_KERNELS.exists():
        return None
    L = ctypes.CDLL(str(REF_KERNELS))
    vp = ctypes.c_void_p
    L.ref_qkv_fp16_launch.argtypes = [vp, vp, vp, vp, vp, vp]
    L.ref_qkv_fp16_launch.restype = ctypes.c_int
    L.ref_fc1_fp16_launch.argtypes = [vp, vp, vp, vp, vp]
    L.ref_fc1_fp16_launch.restype = ctypes.c_int
    return L.ref_qkv_fp16_launch, L.ref_fc1_fp16_launch
