"""ctypes binding of liblffw_b200.so (the C ABI in include/lffw_fp8.h).

The library is built in-tree by build.py.  There is no fallback: if it is
missing, every entry point raises, so a test or benchmark can never pass on a
CPU or library substitute.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liblffw_b200.so"
HEADER = HERE.parent / "include" / "lffw_fp8.h"

SUCCESS = 0
INVALID_ARGUMENT = 1
ABI_MISMATCH = 2
OUT_OF_MEMORY = 3
INTERNAL_ERROR = 4
CUDA_ERROR = 6
UNSUPPORTED_PRECISION = 9
DEVICE_TIMEOUT = 120

EPILOGUE_NONE = 0
EPILOGUE_GELU = 1
WEIGHTS_ROW_MAJOR = 0
WEIGHTS_SKINNY_TILES = 1

DT_FLOAT, DT_HALF, DT_INT8, DT_INT32, DT_FP8 = 0, 1, 2, 3, 6
FORMAT_LINEAR, FORMAT_CHW2 = 0, 1
FIELD_FLOAT16, FIELD_FLOAT32, FIELD_FLOAT64, FIELD_INT8, FIELD_INT16, FIELD_INT32, FIELD_CHAR = range(7)
PHASE_BUILD, PHASE_RUNTIME = 0, 1


class NativeError(RuntimeError):
    """A C ABI call returned a non-success lffw_status."""

    def __init__(self, status: int, what: str):
        super().__init__(f"{what}: {status_string(status)} (status {status})")
        self.status = status


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_size_t),
        ("m", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("x_codes", ctypes.c_void_p),
        ("act_scale", ctypes.c_float),
        ("act_scale_ptr", ctypes.c_void_p),
        ("w_codes", ctypes.c_void_p),
        ("w_scales", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("epilogue", ctypes.c_int32),
        ("y", ctypes.c_void_p),
        ("next_scale", ctypes.c_float),
        ("next_codes", ctypes.c_void_p),
        ("w_layout", ctypes.c_int32),
        ("residual", ctypes.c_void_p),
    ]


class LayerNormArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_size_t),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("x", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("sum_out", ctypes.c_void_p),
        ("gamma", ctypes.c_void_p),
        ("beta", ctypes.c_void_p),
        ("epsilon", ctypes.c_float),
        ("y", ctypes.c_void_p),
        ("code_scale", ctypes.c_float),
        ("code_scale_ptr", ctypes.c_void_p),
        ("codes", ctypes.c_void_p),
    ]


class CrossAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_size_t),
        ("streams", ctypes.c_int32),
        ("queries", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("keys", ctypes.c_int32),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("code_scale", ctypes.c_float),
        ("code_scale_ptr", ctypes.c_void_p),
        ("out_codes", ctypes.c_void_p),
    ]


class SelfAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_size_t),
        ("streams", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("q_ld", ctypes.c_int64),
        ("k_ld", ctypes.c_int64),
        ("v_ld", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("code_scale", ctypes.c_float),
        ("code_scale_ptr", ctypes.c_void_p),
        ("out_codes", ctypes.c_void_p),
    ]


class Conv1dArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_size_t),
        ("streams", ctypes.c_int32),
        ("frames_in", ctypes.c_int32),
        ("c_in", ctypes.c_int32),
        ("c_out", ctypes.c_int32),
        ("stride", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("y_rows", ctypes.c_int32),
        ("y_row0", ctypes.c_int32),
    ]


class HeadsLinearArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_size_t),
        ("streams", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("x_codes", ctypes.c_void_p),
        ("act_scale", ctypes.c_float),
        ("act_scale_ptr", ctypes.c_void_p),
        ("w_codes", ctypes.c_void_p),
        ("w_scales", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("y_streams", ctypes.c_int32),
    ]


class DecoderSelfAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_size_t),
        ("streams", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("qkv", ctypes.c_void_p),
        ("qkv_ld", ctypes.c_int64),
        ("cache_k", ctypes.c_void_p),
        ("cache_v", ctypes.c_void_p),
        ("lengths", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("code_scale", ctypes.c_float),
        ("out_codes", ctypes.c_void_p),
    ]


class PluginField(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("data", ctypes.c_void_p),
        ("type", ctypes.c_int32),
        ("length", ctypes.c_int32),
    ]


class TensorDesc(ctypes.Structure):
    _fields_ = [
        ("nb_dims", ctypes.c_int32),
        ("dims", ctypes.c_int64 * 8),
        ("type", ctypes.c_int32),
        ("format", ctypes.c_int32),
    ]

    @classmethod
    def of(cls, shape, dtype: int = DT_HALF, fmt: int = FORMAT_LINEAR) -> "TensorDesc":
        d = cls()
        d.nb_dims = len(shape)
        for i, v in enumerate(shape):
            d.dims[i] = int(v)
        d.type = dtype
        d.format = fmt
        return d

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(int(self.dims[i]) for i in range(self.nb_dims))


_lib: ctypes.CDLL | None = None
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


def library() -> ctypes.CDLL:
    """Load liblffw_b200.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise FileNotFoundError(
            f"{LIBRARY} is missing: build it with "
            "`python listenflow-fastest-whisper_b200/build.py` (nvcc, sm_100a)"
        )
    L = ctypes.CDLL(str(LIBRARY))
    sig = {
        "lffw_fp8_linear": ([ctypes.POINTER(LinearArgs), _vp], _i32),
        "lffw_fp8_quantize": ([_vp, _i64, ctypes.c_float, _vp, _vp, _vp], _i32),
        "lffw_layer_norm": ([ctypes.POINTER(LayerNormArgs), _vp], _i32),
        "lffw_cross_attention": ([ctypes.POINTER(CrossAttentionArgs), _vp], _i32),
        "lffw_self_attention": ([ctypes.POINTER(SelfAttentionArgs), _vp], _i32),
        "lffw_mel_frames": ([_vp, _i32, _i32, _i32, _vp, _vp], _i32),
        "lffw_conv1d_weight_layout": ([_vp, _i32, _i32, _vp, _vp], _i32),
        "lffw_conv1d_gelu": ([ctypes.POINTER(Conv1dArgs), _vp], _i32),
        "lffw_fp8_linear_heads": ([ctypes.POINTER(HeadsLinearArgs), _vp], _i32),
        "lffw_decoder_embed": ([_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp], _i32),
        "lffw_decoder_self_attention": ([ctypes.POINTER(DecoderSelfAttentionArgs), _vp], _i32),
        "lffw_greedy_select": ([_vp, _i64, _vp, _i64, _i32, _i32, _vp, _vp, _vp], _i32),
        "lffw_decoder_error": ([ctypes.POINTER(_i32)], _i32),
        "lffw_chain_create": ([ctypes.POINTER(LinearArgs), _i32, ctypes.POINTER(_vp)], _i32),
        "lffw_chain_run": ([_vp, _vp], _i32),
        "lffw_chain_destroy": ([_vp], None),
        "lffw_fp8_quantize_rows": ([_vp, _i64, _i64, _vp, _vp, _vp], _i32),
        "lffw_fp8_weight_scales": ([_vp, _i64, _i64, _vp, _vp], _i32),
        "lffw_fp8_dynamic_scale": ([_vp, _i64, _vp, _vp, _vp], _i32),
        "lffw_fp16_fc1": ([_vp, _vp, _vp, _vp, _i64, _i64, _vp], _i32),
        "lffw_fp16_qkv": ([_vp, _vp, _vp, _vp, _vp, _i64, _vp], _i32),
        "lffw_fp16_bias": ([_vp, ctypes.c_uint16, _vp, _i64, _vp], _i32),
        "lffw_fp16_gelu": ([_vp, _vp, _i64, _vp], _i32),
        "lffw_fp16_linear": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp], _i32),
        "lffw_skinny_packed_bytes": ([_i64, _i64, _i32], _i64),
        "lffw_pack_skinny_weights": ([_vp, _i64, _i64, _i32, _vp, _vp], _i32),
        "lffw_device_supported": ([_i32], _i32),
        "lffw_device_error": ([ctypes.POINTER(_i32)], _i32),
        "lffw_launch_count": ([], ctypes.c_uint64),
        "lffw_status_string": ([_i32], ctypes.c_char_p),
        "lffw_version": ([ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)], None),
        "lffw_plugin_creator_count": ([], _i32),
        "lffw_plugin_creator": (
            [_i32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p),
             ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.POINTER(PluginField)),
             ctypes.POINTER(_i32)], _i32),
        "lffw_plugin_create": (
            [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(PluginField), _i32, _i32], _vp),
        "lffw_plugin_clone": ([_vp], _vp),
        "lffw_plugin_destroy": ([_vp], None),
        "lffw_plugin_validate": ([_vp, ctypes.POINTER(TensorDesc), _i32, ctypes.POINTER(TensorDesc)], _i32),
        "lffw_plugin_workspace_size": ([_vp, ctypes.POINTER(TensorDesc), _i32], _i64),
        "lffw_plugin_enqueue": (
            [_vp, ctypes.POINTER(TensorDesc), ctypes.POINTER(TensorDesc), ctypes.POINTER(_vp),
             ctypes.POINTER(_vp), _vp, _vp], _i32),
    }
    for name, (argtypes, restype) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = L
    return L


def status_string(status: int) -> str:
    try:
        return library().lffw_status_string(status).decode()
    except FileNotFoundError:
        return f"status {status}"


def check(status: int, what: str) -> None:
    if status != SUCCESS:
        raise NativeError(status, what)


def bundle_sha256() -> str:
    """The library's tensoracle_bundle_sha256, read the way _plugins.py:33 reads it."""
    return (ctypes.c_char * 65).in_dll(library(), "tensoracle_bundle_sha256").value.decode()


def launch_count() -> int:
    return int(library().lffw_launch_count())


def device_error() -> int:
    """Reads and clears the device's sticky error word; returns the site code (0 = none)."""
    where = _i32(0)
    status = library().lffw_device_error(ctypes.byref(where))
    if status not in (SUCCESS, DEVICE_TIMEOUT):
        raise NativeError(status, "lffw_device_error")
    return int(where.value)


def declared_symbols() -> list[str]:
    """Every function/object the public header declares with LFFW_FP8_API."""
    text = "\n".join(line for line in HEADER.read_text().splitlines() if not line.lstrip().startswith("#"))
    names = re.findall(r"LFFW_FP8_API\s+(?:extern\s+)?[\w\s\*]*?\b(\w+)\s*(?:\(|\[)", text)
    return sorted(set(names))
