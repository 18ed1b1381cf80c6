"""Host side of the FP8 E4M3 quantized linear, mirroring the reference's FP8 graph.

`Fp8Graph` restates python/src/listenflow/fastest_whisper/_fp8.py:13-55
(``_Fp8Graph``) over device tensors instead of a TensorRT network: the same
constructor arguments (checkpoint + activation-scale mapping), the same
``linear(x, key, bias=True)`` / ``decoder_fc1(x, key)`` methods, the same
``ValueError("missing or invalid activation scale for <key>")`` on a missing,
non-finite or non-positive scale (_fp8.py:34-36, network_graph.cpp:137-139),
and the same weight-scale rule (max|W[n,:]|/448, zero rows -> 1).  Weights are
quantized once per key and kept on the device, as TensorRT folds the weight
Q into a constant at build time.

Tensors here are torch CUDA tensors used only as device memory; every byte of
arithmetic runs in liblffw_b200.so (sm_100a kernels) through the C ABI.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Mapping
from dataclasses import dataclass

import torch

from . import _native as native

E4M3_MAX = 448.0


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _require(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")


def _valid_scale(value) -> bool:
    try:
        v = float(value)
    except (TypeError, ValueError):
        return False
    return math.isfinite(v) and v > 0


def weight_scales(weight: torch.Tensor, stream=None) -> torch.Tensor:
    """Per-output-channel scales max|W[n,:]|/448 (0 -> 1) of an fp16 [N, K] weight."""
    _require(weight, torch.float16, "weight")
    rows, cols = weight.shape
    out = torch.empty(rows, dtype=torch.float32, device=weight.device)
    native.check(native.library().lffw_fp8_weight_scales(weight.data_ptr(), rows, cols, out.data_ptr(),
                                                         _stream(stream)), "lffw_fp8_weight_scales")
    return out


def quantize(x: torch.Tensor, scale, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """E4M3 codes of an fp16 tensor with one scale (float, or a 1-element fp32 CUDA tensor)."""
    _require(x, torch.float16, "x")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale_ptr = None
    value = 0.0
    if isinstance(scale, torch.Tensor):
        _require(scale, torch.float32, "scale")
        scale_ptr = scale.data_ptr()
    else:
        value = float(scale)
    native.check(native.library().lffw_fp8_quantize(x.data_ptr(), x.numel(), value, scale_ptr, out.data_ptr(),
                                                    _stream(stream)), "lffw_fp8_quantize")
    return out


def layer_norm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5, *,
               residual: torch.Tensor | None = None, code_scale=None, want_y: bool = True,
               want_sum: bool = False, stream=None):
    """LayerNorm producer (network_graph.cpp:160-166 after the residual add of :285-287).

    Returns (sum, y, codes): sum = x + residual in fp16 (if want_sum), y = the fp16
    LayerNorm of it over the last axis with fp32 gamma/beta (if want_y), and the
    E4M3 codes of y for the next linear when `code_scale` (float or 1-element fp32
    CUDA tensor) is given."""
    _require(x, torch.float16, "x")
    _require(gamma, torch.float32, "gamma")
    _require(beta, torch.float32, "beta")
    if x.dim() != 2:
        raise ValueError("x must be [rows, cols]")
    rows, cols = x.shape
    if gamma.numel() != cols or beta.numel() != cols:
        raise ValueError("gamma and beta must have cols elements")
    if residual is not None:
        _require(residual, torch.float16, "residual")
        if residual.shape != x.shape:
            raise ValueError("residual must match x")
    a = native.LayerNormArgs()
    a.struct_size = ctypes.sizeof(native.LayerNormArgs)
    a.rows, a.cols = rows, cols
    a.x = x.data_ptr()
    a.residual = residual.data_ptr() if residual is not None else None
    a.gamma, a.beta = gamma.data_ptr(), beta.data_ptr()
    a.epsilon = float(eps)
    total = torch.empty_like(x) if want_sum else None
    y = torch.empty_like(x) if want_y else None
    codes = None
    if code_scale is not None:
        codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
        if isinstance(code_scale, torch.Tensor):
            _require(code_scale, torch.float32, "code_scale")
            a.code_scale_ptr = code_scale.data_ptr()
        else:
            a.code_scale = float(code_scale)
        a.codes = codes.data_ptr()
    a.sum_out = total.data_ptr() if total is not None else None
    a.y = y.data_ptr() if y is not None else None
    native.check(native.library().lffw_layer_norm(ctypes.byref(a), _stream(stream)), "lffw_layer_norm")
    return total, y, codes


def cross_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, queries: int, *, code_scale=None,
                    want_out: bool = True, stream=None):
    """Decoder cross-attention over cached encoder K/V (network_graph.cpp:235-244, 401-404).

    q: fp16 [streams * queries, heads * 64] (q_proj output, beams of a stream adjacent);
    k, v: fp16 [streams, heads, keys, 64].  Returns (out, codes): out fp16 like q
    (out_proj's input), and its E4M3 codes when `code_scale` is given."""
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        _require(t, torch.float16, name)
    if k.dim() != 4 or v.shape != k.shape:
        raise ValueError("k and v must be [streams, heads, keys, head_dim] of one shape")
    streams, heads, keys, dim = k.shape
    if q.shape != (streams * queries, heads * dim):
        raise ValueError("q must be [streams * queries, heads * head_dim]")
    a = native.CrossAttentionArgs()
    a.struct_size = ctypes.sizeof(native.CrossAttentionArgs)
    a.streams, a.queries, a.heads, a.head_dim, a.keys = streams, queries, heads, dim, keys
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    out = torch.empty_like(q) if want_out else None
    codes = None
    if code_scale is not None:
        codes = torch.empty(q.shape, dtype=torch.uint8, device=q.device)
        if isinstance(code_scale, torch.Tensor):
            _require(code_scale, torch.float32, "code_scale")
            a.code_scale_ptr = code_scale.data_ptr()
        else:
            a.code_scale = float(code_scale)
        a.out_codes = codes.data_ptr()
    a.out = out.data_ptr() if out is not None else None
    native.check(native.library().lffw_cross_attention(ctypes.byref(a), _stream(stream)), "lffw_cross_attention")
    return out, codes


def self_attention(qkv: torch.Tensor, streams: int, heads: int, *, code_scale=None, want_out: bool = True,
                   stream=None):
    """Encoder self-attention (network_graph.cpp:235-247) read in place from the fused
    QKV linear output qkv [streams * tokens, 3 * heads * 64] (q | k | v columns).

    Returns (out, codes): out fp16 [streams * tokens, heads * 64] (out_proj's input),
    and its E4M3 codes when `code_scale` is given."""
    _require(qkv, torch.float16, "qkv")
    rows, cols = qkv.shape
    width = heads * 64
    if cols != 3 * width or rows % streams != 0:
        raise ValueError("qkv must be [streams * tokens, 3 * heads * 64]")
    a = native.SelfAttentionArgs()
    a.struct_size = ctypes.sizeof(native.SelfAttentionArgs)
    a.streams, a.tokens, a.heads, a.head_dim = streams, rows // streams, heads, 64
    base = qkv.data_ptr()
    a.q, a.k, a.v = base, base + 2 * width, base + 4 * width
    a.q_ld = a.k_ld = a.v_ld = cols
    out = torch.empty((rows, width), dtype=torch.float16, device=qkv.device) if want_out else None
    codes = None
    if code_scale is not None:
        codes = torch.empty((rows, width), dtype=torch.uint8, device=qkv.device)
        if isinstance(code_scale, torch.Tensor):
            _require(code_scale, torch.float32, "code_scale")
            a.code_scale_ptr = code_scale.data_ptr()
        else:
            a.code_scale = float(code_scale)
        a.out_codes = codes.data_ptr()
    a.out = out.data_ptr() if out is not None else None
    native.check(native.library().lffw_self_attention(ctypes.byref(a), _stream(stream)), "lffw_self_attention")
    return out, codes


def mel_frames(mel: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """fp32 log-mel [streams, mels, frames] -> fp16 [streams, frames + 2, mels], the
    time-major zero-padded input of conv1d_gelu (half(mel), network_graph.cpp:257)."""
    _require(mel, torch.float32, "mel")
    if mel.dim() != 3:
        raise ValueError("mel must be [streams, mels, frames]")
    streams, mels, frames = mel.shape
    if out is None:
        out = torch.empty((streams, frames + 2, mels), dtype=torch.float16, device=mel.device)
    native.check(native.library().lffw_mel_frames(mel.data_ptr(), streams, mels, frames, out.data_ptr(),
                                                  _stream(stream)), "lffw_mel_frames")
    return out


def conv1d_weight_layout(weight: torch.Tensor, stream=None) -> torch.Tensor:
    """Checkpoint conv1d weight fp16 [c_out, c_in, 3] -> tap-major [c_out, 3, c_in]."""
    _require(weight, torch.float16, "weight")
    c_out, c_in, taps = weight.shape
    if taps != 3:
        raise ValueError("kernel size 3 expected")
    out = torch.empty((c_out, 3, c_in), dtype=torch.float16, device=weight.device)
    native.check(native.library().lffw_conv1d_weight_layout(weight.data_ptr(), c_out, c_in, out.data_ptr(),
                                                            _stream(stream)), "lffw_conv1d_weight_layout")
    return out


def conv1d_gelu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, stride: int, *,
                positions: torch.Tensor | None = None, out: torch.Tensor | None = None, out_row0: int = 0,
                stream=None) -> torch.Tensor:
    """Encoder convolution + GELU (+ positional add) on padded time-major input
    x fp16 [streams, frames_in + 2, c_in] with the tap-major weight [c_out, 3, c_in]
    (network_graph.cpp:259-282).  Writes rows out_row0 .. out_row0 + frames_out - 1 of
    each stream block of `out` ([streams, rows, c_out]; allocated dense when None)."""
    for t, name in ((x, "x"), (weight, "weight"), (bias, "bias")):
        _require(t, torch.float16, name)
    streams, rows_in, c_in = x.shape
    c_out = weight.shape[0]
    frames_in = rows_in - 2
    frames_out = frames_in // stride
    if out is None:
        out = torch.empty((streams, frames_out, c_out), dtype=torch.float16, device=x.device)
    a = native.Conv1dArgs()
    a.struct_size = ctypes.sizeof(native.Conv1dArgs)
    a.streams, a.frames_in, a.c_in, a.c_out, a.stride = streams, frames_in, c_in, c_out, stride
    a.x, a.weight, a.bias = x.data_ptr(), weight.data_ptr(), bias.data_ptr()
    if positions is not None:
        _require(positions, torch.float16, "positions")
        a.positions = positions.data_ptr()
    a.y = out.data_ptr()
    a.y_rows, a.y_row0 = out.shape[1], out_row0
    native.check(native.library().lffw_conv1d_gelu(ctypes.byref(a), _stream(stream)), "lffw_conv1d_gelu")
    return out


def linear_heads(x_codes: torch.Tensor, w_codes: torch.Tensor, w_scales: torch.Tensor, act_scale, *,
                 streams: int, heads: int, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 stream=None) -> torch.Tensor:
    """FP8 linear over codes [streams * tokens, k] whose fp16 output is split by heads:
    [n / (64 heads), streams, heads, tokens, 64] (the cross_keys / cross_values layout,
    network_graph.cpp:231-234, 296-300)."""
    _require(x_codes, torch.uint8, "x_codes")
    _require(w_codes, torch.uint8, "w_codes")
    _require(w_scales, torch.float32, "w_scales")
    rows, k = x_codes.shape
    n = w_codes.shape[0]
    tokens = rows // streams
    if tokens * streams != rows or n % (64 * heads) != 0:
        raise ValueError("x_codes must be [streams * tokens, k] and n a multiple of 64 * heads")
    if out is None:
        out = torch.empty((n // (64 * heads), streams, heads, tokens, 64), dtype=torch.float16, device=x_codes.device)
    a = native.HeadsLinearArgs()
    a.struct_size = ctypes.sizeof(native.HeadsLinearArgs)
    a.streams, a.tokens, a.heads, a.n, a.k = streams, tokens, heads, n, k
    a.x_codes = x_codes.data_ptr()
    if isinstance(act_scale, torch.Tensor):
        _require(act_scale, torch.float32, "act_scale")
        a.act_scale_ptr = act_scale.data_ptr()
    else:
        a.act_scale = float(act_scale)
    a.w_codes, a.w_scales, a.bias, a.y = w_codes.data_ptr(), w_scales.data_ptr(), _ptr(bias), out.data_ptr()
    native.check(native.library().lffw_fp8_linear_heads(ctypes.byref(a), _stream(stream)), "lffw_fp8_linear_heads")
    return out


def decoder_embed(tokens: torch.Tensor, lengths: torch.Tensor, token_table: torch.Tensor,
                  position_table: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """x[s] = half(token_table[tokens[s]] + position_table[lengths[s]]) (network_graph.cpp:380-388)."""
    _require(tokens, torch.int32, "tokens")
    _require(lengths, torch.int32, "lengths")
    _require(token_table, torch.float16, "token_table")
    _require(position_table, torch.float16, "position_table")
    streams = tokens.numel()
    vocab, width = token_table.shape
    if out is None:
        out = torch.empty((streams, width), dtype=torch.float16, device=tokens.device)
    native.check(native.library().lffw_decoder_embed(tokens.data_ptr(), lengths.data_ptr(), token_table.data_ptr(),
                                                     position_table.data_ptr(), streams, width, vocab,
                                                     position_table.shape[0], out.data_ptr(), _stream(stream)),
                 "lffw_decoder_embed")
    return out


def decoder_self_attention(qkv: torch.Tensor, cache_k: torch.Tensor, cache_v: torch.Tensor, lengths: torch.Tensor,
                           *, code_scale=None, want_out: bool = True, out: torch.Tensor | None = None,
                           codes: torch.Tensor | None = None, stream=None):
    """One decoder layer's self-attention over its KV cache [streams, heads, capacity, 64],
    appending the step's k and v (rows of qkv [streams, >= 3 * heads * 64]) at row
    lengths[s] first (network_graph.cpp:390-399).  Returns (out fp16 or None, codes or None)."""
    _require(qkv, torch.float16, "qkv")
    _require(cache_k, torch.float16, "cache_k")
    _require(cache_v, torch.float16, "cache_v")
    _require(lengths, torch.int32, "lengths")
    streams, heads, capacity, dim = cache_k.shape
    width = heads * dim
    a = native.DecoderSelfAttentionArgs()
    a.struct_size = ctypes.sizeof(a)
    a.streams, a.heads, a.head_dim, a.capacity = streams, heads, dim, capacity
    a.qkv, a.qkv_ld = qkv.data_ptr(), qkv.shape[1]
    a.cache_k, a.cache_v, a.lengths = cache_k.data_ptr(), cache_v.data_ptr(), lengths.data_ptr()
    if want_out and out is None:
        out = torch.empty((streams, width), dtype=torch.float16, device=qkv.device)
    if code_scale is not None and codes is None:
        codes = torch.empty((streams, width), dtype=torch.uint8, device=qkv.device)
    a.out = out.data_ptr() if want_out else None
    a.code_scale = float(code_scale) if code_scale is not None else 0.0
    a.out_codes = _ptr(codes) if code_scale is not None else None
    native.check(native.library().lffw_decoder_self_attention(ctypes.byref(a), _stream(stream)),
                 "lffw_decoder_self_attention")
    return (out if want_out else None), (codes if code_scale is not None else None)


def greedy_select(logits: torch.Tensor, suppression: torch.Tensor, tokens: torch.Tensor | None = None,
                  lengths: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """tokens[s] = the first argmax of fp32(logits[s]) + suppression[s] (network_graph.cpp:332-339);
    lengths[s] += 1 when lengths is given."""
    _require(logits, torch.float16, "logits")
    _require(suppression, torch.float32, "suppression")
    streams, vocab = logits.shape
    if tokens is None:
        tokens = torch.empty(streams, dtype=torch.int32, device=logits.device)
    native.check(native.library().lffw_greedy_select(logits.data_ptr(), vocab, suppression.data_ptr(),
                                                     suppression.shape[1], streams, vocab, tokens.data_ptr(),
                                                     _ptr(lengths), _stream(stream)), "lffw_greedy_select")
    return tokens


def decoder_error() -> int:
    """Reads and clears the decoder kernels' error word (0 = none)."""
    code = ctypes.c_int32(0)
    native.check(native.library().lffw_decoder_error(ctypes.byref(code)), "lffw_decoder_error")
    return int(code.value)


def quantize_rows(w: torch.Tensor, scales: torch.Tensor, stream=None) -> torch.Tensor:
    """E4M3 codes of an fp16 [N, K] weight with one scale per row."""
    _require(w, torch.float16, "w")
    _require(scales, torch.float32, "scales")
    rows, cols = w.shape
    out = torch.empty(w.shape, dtype=torch.uint8, device=w.device)
    native.check(native.library().lffw_fp8_quantize_rows(w.data_ptr(), rows, cols, scales.data_ptr(),
                                                         out.data_ptr(), _stream(stream)),
                 "lffw_fp8_quantize_rows")
    return out


def dynamic_scale(x: torch.Tensor, stream=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(scale, amax) as 1-element fp32 device tensors: scale = amax/448, 0 -> 1."""
    _require(x, torch.float16, "x")
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    amax = torch.empty(1, dtype=torch.float32, device=x.device)
    native.check(native.library().lffw_fp8_dynamic_scale(x.data_ptr(), x.numel(), scale.data_ptr(),
                                                         amax.data_ptr(), _stream(stream)),
                 "lffw_fp8_dynamic_scale")
    return scale, amax


def pack_skinny(weight: torch.Tensor, stream=None) -> torch.Tensor:
    """Re-lays a row-major [N, K] weight (E4M3 codes as uint8, or fp16) into the
    contiguous 16 KB tiles the small-m (m <= 32) kernels stream sequentially."""
    if weight.dtype not in (torch.uint8, torch.float16) or not weight.is_cuda or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous CUDA uint8 (E4M3 codes) or float16 tensor")
    n, k = weight.shape
    elem = weight.element_size()
    size = native.library().lffw_skinny_packed_bytes(n, k, elem)
    out = torch.empty(size, dtype=torch.uint8, device=weight.device)
    native.check(native.library().lffw_pack_skinny_weights(weight.data_ptr(), n, k, elem, out.data_ptr(),
                                                           _stream(stream)), "lffw_pack_skinny_weights")
    return out


def linear(x_codes: torch.Tensor, w_codes: torch.Tensor, w_scales: torch.Tensor, act_scale, *,
           bias: torch.Tensor | None = None, gelu: bool = False, out: torch.Tensor | None = None,
           want_y: bool = True, next_scale: float | None = None, next_codes: torch.Tensor | None = None,
           w_packed: torch.Tensor | None = None, residual: torch.Tensor | None = None,
           stream=None) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """One FP8 Q/DQ linear on E4M3 codes: x_codes [..., K], w_codes [N, K].
    `w_packed` (from pack_skinny(w_codes)) replaces w_codes on the m <= 32 path.
    `residual` (fp16 [..., N]) is added to y after the bias, the graph's residual
    add (network_graph.cpp:285-287); `out` may be the residual itself.

    Returns (y fp16 [..., N] or None, next-linear E4M3 codes or None)."""
    _require(x_codes, torch.uint8, "x_codes")
    _require(w_packed if w_packed is not None else w_codes, torch.uint8, "w_codes")
    _require(w_scales, torch.float32, "w_scales")
    k = x_codes.shape[-1]
    m = x_codes.numel() // k
    n = w_scales.shape[0]  # one scale per output channel
    lead = tuple(x_codes.shape[:-1])
    if want_y and out is None:
        out = torch.empty(lead + (n,), dtype=torch.float16, device=x_codes.device)
    if next_scale is not None and next_codes is None:
        next_codes = torch.empty(lead + (n,), dtype=torch.uint8, device=x_codes.device)
    a = native.LinearArgs()
    a.struct_size = ctypes.sizeof(native.LinearArgs)
    a.m, a.n, a.k = m, n, k
    a.x_codes = x_codes.data_ptr()
    if isinstance(act_scale, torch.Tensor):
        _require(act_scale, torch.float32, "act_scale")
        a.act_scale_ptr = act_scale.data_ptr()
    else:
        a.act_scale = float(act_scale)
    a.w_codes = (w_codes if w_packed is None else w_packed).data_ptr()
    a.w_layout = native.WEIGHTS_ROW_MAJOR if w_packed is None else native.WEIGHTS_SKINNY_TILES
    a.w_scales = w_scales.data_ptr()
    a.bias = _ptr(bias)
    a.epilogue = native.EPILOGUE_GELU if gelu else native.EPILOGUE_NONE
    a.y = _ptr(out) if want_y else None
    a.next_scale = float(next_scale) if next_scale is not None else 0.0
    a.next_codes = _ptr(next_codes)
    if residual is not None:
        _require(residual, torch.float16, "residual")
        if residual.numel() != m * n:
            raise ValueError("residual must hold m x n fp16 values")
    a.residual = _ptr(residual)
    native.check(native.library().lffw_fp8_linear(ctypes.byref(a), _stream(stream)), "lffw_fp8_linear")
    return (out if want_y else None), next_codes


class LinearChain:
    """Dependent small-m linears (m <= 32, packed weights) run back to back in one
    persistent launch: link i reads what earlier links wrote.  Each link is a dict
    of fp8.linear's arguments: x_codes, w_packed, w_scales, act_scale and
    optionally bias, gelu, out (fp16 y), next_scale + next_codes.  The tensors are
    bound at construction (they must stay alive); run() launches the chain."""

    def __init__(self, links: list[dict]):
        self._handle = None
        self._keep = []  # tensors the device descriptors point to
        args = (native.LinearArgs * len(links))()
        for a, link in zip(args, links):
            x_codes, w_packed, w_scales = link["x_codes"], link["w_packed"], link["w_scales"]
            _require(x_codes, torch.uint8, "x_codes")
            _require(w_packed, torch.uint8, "w_packed")
            _require(w_scales, torch.float32, "w_scales")
            k = x_codes.shape[-1]
            a.struct_size = ctypes.sizeof(native.LinearArgs)
            a.m, a.n, a.k = x_codes.numel() // k, w_scales.shape[0], k
            a.x_codes = x_codes.data_ptr()
            scale = link["act_scale"]
            if isinstance(scale, torch.Tensor):
                _require(scale, torch.float32, "act_scale")
                a.act_scale_ptr = scale.data_ptr()
            else:
                a.act_scale = float(scale)
            a.w_codes = w_packed.data_ptr()
            a.w_layout = native.WEIGHTS_SKINNY_TILES
            a.w_scales = w_scales.data_ptr()
            a.bias = _ptr(link.get("bias"))
            a.epilogue = native.EPILOGUE_GELU if link.get("gelu") else native.EPILOGUE_NONE
            a.y = _ptr(link.get("out"))
            a.next_scale = float(link["next_scale"]) if link.get("next_codes") is not None else 0.0
            a.next_codes = _ptr(link.get("next_codes"))
            self._keep.append(link)
        handle = ctypes.c_void_p()
        native.check(native.library().lffw_chain_create(args, len(links), ctypes.byref(handle)), "lffw_chain_create")
        self._handle = handle

    def run(self, stream=None) -> None:
        native.check(native.library().lffw_chain_run(self._handle, _stream(stream)), "lffw_chain_run")

    def close(self) -> None:
        if self._handle is not None:
            native.library().lffw_chain_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class QuantizedWeight:
    """A linear's device-resident E4M3 weight, per-channel scales and fp16 bias."""

    codes: torch.Tensor
    scales: torch.Tensor
    bias: torch.Tensor | None

    @classmethod
    def from_half(cls, weight: torch.Tensor, bias: torch.Tensor | None = None, stream=None) -> "QuantizedWeight":
        scales = weight_scales(weight, stream)
        return cls(quantize_rows(weight, scales, stream), scales, bias)


class Fp8Graph:
    """Device-tensor counterpart of ``_Fp8Graph`` (_fp8.py:13-55).

    ``checkpoint`` maps ``"<key>.weight"`` -> fp16 [out, in] and
    ``"<key>.bias"`` -> fp16 [out] CUDA tensors; ``scales`` maps each linear key
    to its static activation scale (the calibrated amax/448 of
    assets/fp8-scales.json)."""

    def __init__(self, checkpoint: Mapping[str, torch.Tensor], scales: Mapping[str, float]):
        self.checkpoint = checkpoint
        self.scales = scales
        self._weights: dict[tuple[str, bool], QuantizedWeight] = {}

    def scale(self, key: str) -> float:
        scale = self.scales.get(key)
        if scale is None or not _valid_scale(scale):
            raise ValueError(f"missing or invalid activation scale for {key}")
        return float(scale)

    def weight(self, key: str, bias: bool = True) -> QuantizedWeight:
        cached = self._weights.get((key, bias))
        if cached is None:
            w = self.checkpoint[f"{key}.weight"].contiguous()
            b = self.checkpoint[f"{key}.bias"].contiguous() if bias else None
            cached = QuantizedWeight.from_half(w, b)
            self._weights[(key, bias)] = cached
        return cached

    def linear(self, x: torch.Tensor, key: str, *, bias: bool = True, gelu: bool = False) -> torch.Tensor:
        """fp16 x [..., in] -> fp16 [..., out]: Q(x) . DQ, Q(W) . DQ, MatMul, + bias."""
        scale = self.scale(key)  # validated before anything is quantized
        weight = self.weight(key, bias)
        codes = quantize(x.contiguous(), scale)
        y, _ = linear(codes, weight.codes, weight.scales, scale, bias=weight.bias, gelu=gelu)
        return y

    def decoder_fc1(self, x: torch.Tensor, key: str) -> torch.Tensor:
        """gelu(linear(x, key)) with the GELU fused into the GEMM epilogue (_fp8.py:53-55)."""
        return self.linear(x, key, gelu=True)

    def mlp(self, x: torch.Tensor, fc1: str, fc2: str) -> torch.Tensor:
        """fc2(gelu(fc1(x))): fc1's epilogue emits fc2's E4M3 input codes directly."""
        s1, s2 = self.scale(fc1), self.scale(fc2)
        w1, w2 = self.weight(fc1), self.weight(fc2)
        codes = quantize(x.contiguous(), s1)
        _, hidden = linear(codes, w1.codes, w1.scales, s1, bias=w1.bias, gelu=True, want_y=False,
                           next_scale=s2)
        y, _ = linear(hidden, w2.codes, w2.scales, s2, bias=w2.bias)
        return y


# ---- fp16 single-token projections (the reference plugins' kernels) ---------

def fp16_fc1(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, out: torch.Tensor | None = None,
             stream=None) -> torch.Tensor:
    rows, width = weight.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.float16, device=weight.device)
    native.check(native.library().lffw_fp16_fc1(x.data_ptr(), weight.data_ptr(), bias.data_ptr(),
                                                out.data_ptr(), rows, width, _stream(stream)), "lffw_fp16_fc1")
    return out


def fp16_qkv(x: torch.Tensor, weight: torch.Tensor, q_bias: torch.Tensor, v_bias: torch.Tensor,
             out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    width = weight.shape[1]
    if out is None:
        out = torch.empty(3 * width, dtype=torch.float16, device=weight.device)
    native.check(native.library().lffw_fp16_qkv(x.data_ptr(), weight.data_ptr(), q_bias.data_ptr(),
                                                v_bias.data_ptr(), out.data_ptr(), width, _stream(stream)),
                 "lffw_fp16_qkv")
    return out


def fp16_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                out: torch.Tensor | None = None, w_packed: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """fp16 [m <= 32, k] x fp16 [n, k]^T (+ bias) -> fp16 [m, n], fp32 accumulate (decoder logits).
    `w_packed` (from pack_skinny(weight)) streams the weight as contiguous tiles."""
    _require(x, torch.float16, "x")
    _require(weight, torch.float16, "weight")
    m, k = x.shape
    n = weight.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=x.device)
    w = weight if w_packed is None else w_packed
    layout = native.WEIGHTS_ROW_MAJOR if w_packed is None else native.WEIGHTS_SKINNY_TILES
    native.check(native.library().lffw_fp16_linear(x.data_ptr(), w.data_ptr(), _ptr(bias), out.data_ptr(),
                                                   m, n, k, layout, _stream(stream)), "lffw_fp16_linear")
    return out


def fp16_gelu(x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """GELU with fp16 graph edges (graph::gelu), elementwise."""
    _require(x, torch.float16, "x")
    if out is None:
        out = torch.empty_like(x)
    native.check(native.library().lffw_fp16_gelu(x.data_ptr(), out.data_ptr(), x.numel(), _stream(stream)),
                 "lffw_fp16_gelu")
    return out


def fp16_bias(x: torch.Tensor, bias_bits: int, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    native.check(native.library().lffw_fp16_bias(x.data_ptr(), int(bias_bits), out.data_ptr(), x.numel(),
                                                 _stream(stream)), "lffw_fp16_bias")
    return out
