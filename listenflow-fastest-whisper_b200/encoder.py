"""The Whisper encoder forward on this library's kernels.

Restates the FP8 encoder graph of cpp/src/network_graph.cpp:255-301:

    mel -> half -> conv1 (k3, s1) + GELU -> conv2 (k3, s2) + GELU -> + positions
        -> layers x [ LayerNorm -> fused q|k|v Q/DQ linear -> self-attention -> out_proj
                      -> residual add + LayerNorm -> fc1 + GELU -> fc2 -> residual add ]
        -> final LayerNorm -> "encoder" states
        -> k_proj / v_proj of every decoder layer's cross-attention -> cross_keys / cross_values

Every step is one launch of liblffw_b200.so; the launch arguments are built once
(an ``Encoder`` is a plan over preallocated device buffers, like an engine's
bindings), so a forward allocates nothing and can be captured in a CUDA graph.
The residual adds (the fp16 sums of network_graph.cpp:285-287) ride on the
epilogues of out_proj and fc2, so each LayerNorm reads one tensor, and every
LayerNorm or epilogue that feeds an FP8 linear writes that linear's E4M3 codes
directly.

Weights come from a checkpoint mapping with the reference's key names (fp16
device tensors) and the per-linear activation scales of assets/fp8-scales.json
(or ``calibrate``'s amax/448 for other weights).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Mapping

import torch

from . import _native as native
from . import fp8

NEG_ZERO_HALF = -32768  # int16 bits of fp16 -0.0: adding it leaves every fp16 value (and -0) unchanged


@dataclass(frozen=True)
class EncoderConfig:
    """Whisper large-v3 encoder shapes (128 mel bins, 3000 frames -> 1500 positions)."""

    layers: int = 32
    d_model: int = 1280
    heads: int = 20
    ffn: int = 5120
    mels: int = 128
    frames: int = 3000
    decoder_layers: int = 32  # cross-attention K/V projections computed from the states

    @property
    def positions(self) -> int:
        return self.frames // 2


def scale_keys(config: EncoderConfig) -> dict[str, list[str]]:
    """The activation-scale keys the encoder reads, by role (network_graph.cpp:124-139)."""
    layer = lambda i, op: f"model.encoder.layers.{i}.{op}"
    return {
        "qkv": [layer(i, "self_attn.q_proj") for i in range(config.layers)],
        "out": [layer(i, "self_attn.out_proj") for i in range(config.layers)],
        "fc1": [layer(i, "fc1") for i in range(config.layers)],
        "fc2": [layer(i, "fc2") for i in range(config.layers)],
        "cross": [f"model.decoder.layers.{j}.encoder_attn.{p}_proj" for j in range(config.decoder_layers)
                  for p in "kv"],
    }


def sinusoids(length: int, channels: int) -> torch.Tensor:
    """Whisper's fixed encoder position table: sin then cos of t / 10000^(i / (C/2 - 1))."""
    half = channels // 2
    step = math.log(10000.0) / (half - 1)
    inv = torch.exp(-step * torch.arange(half, dtype=torch.float64))
    t = torch.arange(length, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.sin(t), torch.cos(t)], dim=1)


def synthetic_checkpoint(config: EncoderConfig, seed: int, device) -> dict[str, torch.Tensor]:
    """Random-init fp16 weights under the reference's checkpoint names and shapes
    (no checkpoint is available here): linears and convolutions ~N(0, 0.02),
    biases ~N(0, 0.02), LayerNorm gamma 1 + N(0, 0.1) and beta N(0, 0.1), the
    sinusoidal position table."""
    g = torch.Generator(device=device).manual_seed(seed)
    d, f = config.d_model, config.ffn
    ck: dict[str, torch.Tensor] = {}

    def normal(shape, std):
        return (torch.randn(shape, generator=g, device=device) * std).half()

    ck["model.encoder.conv1.weight"] = normal((d, config.mels, 3), 0.02)
    ck["model.encoder.conv1.bias"] = normal((d,), 0.02)
    ck["model.encoder.conv2.weight"] = normal((d, d, 3), 0.02)
    ck["model.encoder.conv2.bias"] = normal((d,), 0.02)
    ck["model.encoder.embed_positions.weight"] = sinusoids(config.positions, d).half().to(device)
    for i in range(config.layers):
        root = f"model.encoder.layers.{i}"
        for p in ("q", "k", "v", "out"):
            ck[f"{root}.self_attn.{p}_proj.weight"] = normal((d, d), 0.02)
            if p != "k":
                ck[f"{root}.self_attn.{p}_proj.bias"] = normal((d,), 0.02)
        for name, (n, k) in (("fc1", (f, d)), ("fc2", (d, f))):
            ck[f"{root}.{name}.weight"] = normal((n, k), 0.02)
            ck[f"{root}.{name}.bias"] = normal((n,), 0.02)
        for norm in ("self_attn_layer_norm", "final_layer_norm"):
            ck[f"{root}.{norm}.weight"] = (1 + 0.1 * torch.randn(d, generator=g, device=device)).half()
            ck[f"{root}.{norm}.bias"] = normal((d,), 0.1)
    ck["model.encoder.layer_norm.weight"] = (1 + 0.1 * torch.randn(d, generator=g, device=device)).half()
    ck["model.encoder.layer_norm.bias"] = normal((d,), 0.1)
    for j in range(config.decoder_layers):
        root = f"model.decoder.layers.{j}.encoder_attn"
        ck[f"{root}.k_proj.weight"] = normal((d, d), 0.02)
        ck[f"{root}.v_proj.weight"] = normal((d, d), 0.02)
        ck[f"{root}.v_proj.bias"] = normal((d,), 0.02)
    return ck


@dataclass
class EncoderLayerWeights:
    ln1: tuple[torch.Tensor, torch.Tensor]
    qkv: fp8.QuantizedWeight
    out: fp8.QuantizedWeight
    ln2: tuple[torch.Tensor, torch.Tensor]
    fc1: fp8.QuantizedWeight
    fc2: fp8.QuantizedWeight


@dataclass
class EncoderWeights:
    """Device-resident encoder weights in the layouts the kernels read: tap-major
    fp16 convolutions, fp32 LayerNorm parameters (network_graph.cpp:160-163 keeps
    them fp32), fused q|k|v E4M3 rows with bias [b_q | -0 | b_v] (k_proj has no
    bias, :231-234), and every decoder layer's cross k|v E4M3 rows stacked."""

    config: EncoderConfig
    conv1: tuple[torch.Tensor, torch.Tensor]
    conv2: tuple[torch.Tensor, torch.Tensor]
    positions: torch.Tensor
    layers: list[EncoderLayerWeights]
    ln_post: tuple[torch.Tensor, torch.Tensor]
    cross_kv: fp8.QuantizedWeight
    keep: list = field(default_factory=list)

    @classmethod
    def from_checkpoint(cls, checkpoint: Mapping[str, torch.Tensor],
                        config: EncoderConfig = EncoderConfig()) -> "EncoderWeights":
        def get(name):
            t = checkpoint[name]
            if t.dtype != torch.float16 or not t.is_cuda:
                raise ValueError(f"{name}: fp16 CUDA tensor expected")
            return t.contiguous()

        def norm(name):
            return get(f"{name}.weight").float(), get(f"{name}.bias").float()

        def neg_zero(n, device):
            return torch.full((n,), NEG_ZERO_HALF, dtype=torch.int16, device=device).view(torch.float16)

        d = config.d_model
        conv1 = (fp8.conv1d_weight_layout(get("model.encoder.conv1.weight")), get("model.encoder.conv1.bias"))
        conv2 = (fp8.conv1d_weight_layout(get("model.encoder.conv2.weight")), get("model.encoder.conv2.bias"))
        positions = get("model.encoder.embed_positions.weight")[: config.positions].contiguous()
        device = positions.device
        layers = []
        for i in range(config.layers):
            root = f"model.encoder.layers.{i}"
            sa = f"{root}.self_attn"
            w_qkv = torch.cat([get(f"{sa}.{p}_proj.weight") for p in "qkv"])
            b_qkv = torch.cat([get(f"{sa}.q_proj.bias"), neg_zero(d, device), get(f"{sa}.v_proj.bias")])
            layers.append(EncoderLayerWeights(
                ln1=norm(f"{root}.self_attn_layer_norm"),
                qkv=fp8.QuantizedWeight.from_half(w_qkv, b_qkv),
                out=fp8.QuantizedWeight.from_half(get(f"{sa}.out_proj.weight"), get(f"{sa}.out_proj.bias")),
                ln2=norm(f"{root}.final_layer_norm"),
                fc1=fp8.QuantizedWeight.from_half(get(f"{root}.fc1.weight"), get(f"{root}.fc1.bias")),
                fc2=fp8.QuantizedWeight.from_half(get(f"{root}.fc2.weight"), get(f"{root}.fc2.bias")),
            ))
            del w_qkv
        rows, bias = [], []
        for j in range(config.decoder_layers):
            root = f"model.decoder.layers.{j}.encoder_attn"
            rows += [get(f"{root}.k_proj.weight"), get(f"{root}.v_proj.weight")]
            bias += [neg_zero(d, device), get(f"{root}.v_proj.bias")]
        cross = fp8.QuantizedWeight.from_half(torch.cat(rows), torch.cat(bias))
        return cls(config, conv1, conv2, positions, layers, norm("model.encoder.layer_norm"), cross)


def _scales_for(config: EncoderConfig, scales: Mapping[str, float]) -> dict[str, list[float]]:
    """Per-role scale lists; a missing, non-finite or non-positive scale is an error
    naming the key (network_graph.cpp:137-139), and the fused projections require
    the equal scales the reference's asset has (q = k = v; all cross k and v)."""
    out = {}
    keys = scale_keys(config)
    for role, names in keys.items():
        values = []
        for key in names:
            v = scales.get(key)
            if v is None or not isinstance(v, (int, float)) or not math.isfinite(v) or v <= 0:
                raise ValueError(f"missing or invalid activation scale for {key}")
            values.append(float(v))
        out[role] = values
    for i in range(config.layers):
        root = f"model.encoder.layers.{i}.self_attn"
        for p in "kv":
            v = scales.get(f"{root}.{p}_proj")
            if v is not None and float(v) != out["qkv"][i]:
                raise ValueError(f"{root}: q/k/v activation scales differ; the fused QKV linear needs one scale")
    if len(set(out["cross"])) != 1:
        raise ValueError("cross-attention k/v activation scales differ; the stacked projection needs one scale")
    return out


class Encoder:
    """A planned encoder forward for `streams` 30-second inputs on the current device.

    ``forward(mel)`` reads fp32 log-mel [streams, mels, frames] from device memory
    and returns (states fp16 [streams, positions, d_model], cross_kv fp16
    [2 * decoder_layers, streams, heads, positions, 64]); cross_kv[2j] and
    cross_kv[2j + 1] are decoder layer j's cross keys and values in the layout
    lffw_cross_attention reads.  The returned tensors are the plan's own buffers,
    overwritten by the next forward.

    Streams run through the layers in slices of `chunk` streams (default 32) that
    share one set of activation buffers.  Smaller slices keep more of a slice's
    activations in the 126 MB L2 between the kernels that write and read them;
    larger ones give each launch more tiles, so its last partial wave is a smaller
    part of it.  Measured on the 64-stream forward (one B200, states bit-identical
    across slice sizes), since the FP8 GEMM walks large-A linears in row-panel
    groups: chunk 8 132.6-133.1 ms, 16 127.5-127.9 ms, 32 125.4-126.0 ms on one box;
    32 127.9-128.3 ms and 64 127.9-128.4 ms on another."""

    def __init__(self, weights: EncoderWeights, scales: Mapping[str, float], streams: int, device=None,
                 chunk: int | None = None):
        c = weights.config
        self.config, self.weights, self.streams = c, weights, streams
        self.chunk = max(1, min(streams, chunk if chunk is not None else 32))
        self.scales = _scales_for(c, scales)
        device = torch.device(device) if device is not None else weights.positions.device
        d, f, t = c.d_model, c.ffn, c.positions
        n = self.chunk
        m = n * t
        self.rows = m
        empty = lambda shape, dtype=torch.float16: torch.empty(shape, dtype=dtype, device=device)
        self.mel = empty((streams, c.mels, c.frames), torch.float32)
        self.frames = empty((n, c.frames + 2, c.mels))
        self.h1 = torch.zeros((n, c.frames + 2, d), dtype=torch.float16, device=device)  # rows 0, -1: padding
        self.x0 = empty((n, t, d))
        self.stream_buf = [empty((m, d)), empty((m, d))]
        self.ln_codes = empty((m, d), torch.uint8)
        self.qkv = empty((m, 3 * d))
        self.attn_codes = empty((m, d), torch.uint8)
        self.fc2_codes = empty((m, f), torch.uint8)
        self.states = empty((streams, t, d))
        self.kv_codes = empty((m, d), torch.uint8)
        self.cross_kv = empty((2 * c.decoder_layers, streams, c.heads, t, 64))
        self._calls = []
        # (first stream, stream count, its launches in _calls, and the end of the
        # launch that writes its states: the final LayerNorm, before the cross K/V)
        self._slices = []
        for first in range(0, streams, n):
            count = min(n, streams - first)
            begin = len(self._calls)
            plan = self._plan(first, count)
            states_end = begin + max(i for i, (name, _) in enumerate(plan) if name == "lffw_layer_norm") + 1
            self._calls += plan
            self._slices.append((first, count, begin, states_end, len(self._calls)))
        self._copy_stream = None

    # -- launch plan ---------------------------------------------------------
    def _plan(self, first: int, count: int):
        """The launches of streams [first, first + count) (count <= chunk)."""
        c, w, sc = self.config, self.weights, self.scales
        lib = native.library()
        calls = []
        d, f, t = c.d_model, c.ffn, c.positions
        m = count * t
        p = lambda tensor: tensor.data_ptr() if tensor is not None else None
        mel = self.mel[first:first + count]
        states = self.states[first:first + count].view(m, d)

        calls.append(("lffw_mel_frames", lambda s, a=(p(mel), count, c.mels, c.frames, p(self.frames)):
                      lib.lffw_mel_frames(*a, s)))

        def conv(x, weight, bias, stride, y, y_rows, y_row0, frames_in, c_in, positions=None):
            a = native.Conv1dArgs()
            a.struct_size = ctypes.sizeof(a)
            a.streams, a.frames_in, a.c_in, a.c_out, a.stride = count, frames_in, c_in, d, stride
            a.x, a.weight, a.bias, a.positions, a.y = p(x), p(weight), p(bias), p(positions), p(y)
            a.y_rows, a.y_row0 = y_rows, y_row0
            return ("lffw_conv1d_gelu", lambda s, a=a: lib.lffw_conv1d_gelu(ctypes.byref(a), s))

        calls.append(conv(self.frames, *w.conv1, 1, self.h1, c.frames + 2, 1, c.frames, c.mels))
        calls.append(conv(self.h1, *w.conv2, 2, self.x0, t, 0, c.frames, d, positions=w.positions))

        def norm(x, residual, params, sum_out, y, code_scale, codes):
            a = native.LayerNormArgs()
            a.struct_size = ctypes.sizeof(a)
            a.rows, a.cols = m, d
            a.x, a.residual, a.sum_out = p(x), p(residual), p(sum_out)
            a.gamma, a.beta, a.epsilon = p(params[0]), p(params[1]), 1e-5
            a.y, a.code_scale, a.codes = p(y), code_scale, p(codes)
            return ("lffw_layer_norm", lambda s, a=a: lib.lffw_layer_norm(ctypes.byref(a), s))

        def linear(x_codes, weight, act_scale, y=None, gelu=False, next_scale=None, next_codes=None,
                   residual=None):
            a = native.LinearArgs()
            a.struct_size = ctypes.sizeof(a)
            a.m, a.n, a.k = m, weight.scales.shape[0], x_codes.shape[-1]
            a.x_codes, a.act_scale = p(x_codes), act_scale
            a.w_codes, a.w_scales, a.bias = p(weight.codes), p(weight.scales), p(weight.bias)
            a.epilogue = native.EPILOGUE_GELU if gelu else native.EPILOGUE_NONE
            a.y = p(y)
            a.next_scale = next_scale if next_scale is not None else 0.0
            a.next_codes = p(next_codes)
            a.w_layout = native.WEIGHTS_ROW_MAJOR
            a.residual = p(residual)
            return ("lffw_fp8_linear", lambda s, a=a: lib.lffw_fp8_linear(ctypes.byref(a), s))

        def attention(code_scale):
            a = native.SelfAttentionArgs()
            a.struct_size = ctypes.sizeof(a)
            a.streams, a.tokens, a.heads, a.head_dim = count, t, c.heads, 64
            base, step = self.qkv.data_ptr(), 2 * d  # bytes per d-wide column window
            a.q, a.k, a.v = base, base + step, base + 2 * step
            a.q_ld = a.k_ld = a.v_ld = 3 * d
            a.out, a.code_scale, a.out_codes = None, code_scale, p(self.attn_codes)
            return ("lffw_self_attention", lambda s, a=a: lib.lffw_self_attention(ctypes.byref(a), s))

        # The residual adds ride on the epilogues of out_proj and fc2 (y = linear +
        # residual, the same fp16 add), so each LayerNorm reads one tensor and
        # writes codes only.  Layer l's input x is stream_buf[0] (x0 for layer 0),
        # its mid-layer sum stream_buf[1], and fc2 writes layer l + 1's input over
        # stream_buf[0], which out_proj has finished reading.
        x = self.x0.view(-1, d)
        for i, L in enumerate(w.layers):
            s_qkv, s_out, s_fc1, s_fc2 = sc["qkv"][i], sc["out"][i], sc["fc1"][i], sc["fc2"][i]
            calls.append(norm(x, None, L.ln1, None, None, s_qkv, self.ln_codes))
            calls.append(linear(self.ln_codes, L.qkv, s_qkv, y=self.qkv))
            calls.append(attention(s_out))
            mid = self.stream_buf[1]
            calls.append(linear(self.attn_codes, L.out, s_out, y=mid, residual=x))
            calls.append(norm(mid, None, L.ln2, None, None, s_fc1, self.ln_codes))
            calls.append(linear(self.ln_codes, L.fc1, s_fc1, gelu=True, next_scale=s_fc2, next_codes=self.fc2_codes))
            nxt = self.stream_buf[0]
            calls.append(linear(self.fc2_codes, L.fc2, s_fc2, y=nxt, residual=mid))
            x = nxt
        s_cross = sc["cross"][0]
        calls.append(norm(x, None, w.ln_post, None, states, s_cross, self.kv_codes))

        a = native.HeadsLinearArgs()
        a.struct_size = ctypes.sizeof(a)
        a.streams, a.tokens, a.heads, a.n, a.k = count, t, c.heads, w.cross_kv.scales.shape[0], d
        a.x_codes, a.act_scale = p(self.kv_codes), s_cross
        a.w_codes, a.w_scales, a.bias = p(w.cross_kv.codes), p(w.cross_kv.scales), p(w.cross_kv.bias)
        a.y = p(self.cross_kv[:, first])  # this slice's first stream of every group
        a.y_streams = self.streams
        calls.append(("lffw_fp8_linear_heads", lambda s, a=a: lib.lffw_fp8_linear_heads(ctypes.byref(a), s)))
        return calls

    @property
    def launches(self) -> int:
        return len(self._calls)

    def run(self, stream=None) -> None:
        """One forward over the plan's mel buffer (``self.mel``) on `stream`."""
        s = fp8._stream(stream)
        for name, call in self._calls:
            native.check(call(s), name)

    def forward(self, mel: torch.Tensor, stream=None, states_out: torch.Tensor | None = None):
        """Copies mel (fp32 [streams, mels, frames], device or pinned host) into the
        plan and runs it; returns (states, cross_kv) on the device.

        With `states_out` (fp16 [streams, positions, d_model], pinned host memory)
        the states are also copied there.  Host copies run on a side stream slice
        by slice: every slice's log-mel is copied in up front and each slice starts
        once its own rows have arrived, and a slice's states go out as soon as its
        final LayerNorm has written them, while its cross K/V and the next slice
        run.  The copies wait for work already on `stream` before they
        touch the plan's buffers, and `stream` waits for the last copy, so stream
        order covers both (synchronise `stream` before reading `states_out`)."""
        if tuple(mel.shape) != tuple(self.mel.shape) or mel.dtype != torch.float32:
            raise ValueError(f"mel must be fp32 {tuple(self.mel.shape)}")
        if states_out is not None and (tuple(states_out.shape) != tuple(self.states.shape)
                                       or states_out.dtype != torch.float16):
            raise ValueError(f"states_out must be fp16 {tuple(self.states.shape)}")
        torch_stream = stream if stream is not None else torch.cuda.current_stream(self.mel.device)
        if mel.is_cuda and states_out is None:
            with torch.cuda.stream(torch_stream):
                self.mel.copy_(mel, non_blocking=True)
            self.run(torch_stream)
            return self.states, self.cross_kv
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.mel.device)
        side = self._copy_stream
        start = torch.cuda.Event()
        start.record(torch_stream)
        side.wait_event(start)
        arrived = []
        for first, count, _, _, _ in self._slices:
            with torch.cuda.stream(side):
                self.mel[first:first + count].copy_(mel[first:first + count], non_blocking=True)
            event = torch.cuda.Event()
            event.record(side)
            arrived.append(event)
        s = fp8._stream(torch_stream)
        for (first, count, begin, states_end, end), event in zip(self._slices, arrived):
            torch_stream.wait_event(event)
            for name, call in self._calls[begin:states_end]:
                native.check(call(s), name)
            if states_out is not None:
                done = torch.cuda.Event()
                done.record(torch_stream)
                side.wait_event(done)
                with torch.cuda.stream(side):
                    states_out[first:first + count].copy_(self.states[first:first + count], non_blocking=True)
            for name, call in self._calls[states_end:end]:
                native.check(call(s), name)
        finished = torch.cuda.Event()
        finished.record(side)
        torch_stream.wait_event(finished)
        return self.states, self.cross_kv

    def flops_per_forward(self) -> int:
        """Multiply-add work of one forward x 2: convolutions, linears, QK^T and P.V."""
        c = self.config
        t, d, f, s = c.positions, c.d_model, c.ffn, self.streams
        conv = 2 * s * (c.frames * c.mels * 3 * d + t * d * 3 * d)
        linears = 2 * s * t * c.layers * (3 * d * d + d * d + 2 * d * f)
        attention = 4 * s * c.layers * c.heads * t * t * 64
        cross = 2 * s * t * d * 2 * d * c.decoder_layers
        return conv + linears + attention + cross


def calibrate(weights: EncoderWeights, mel: torch.Tensor, stream=None) -> dict[str, float]:
    """Static activation scales amax/448 (python/scripts/calibrate_fp8.py:384-385)
    of every FP8 linear input of the encoder, observed on `mel` (fp32 [streams,
    mels, frames], device).  Runs the same kernels with fp16 outputs and dynamic
    scales; returns a mapping keyed like assets/fp8-scales.json."""
    c = weights.config
    streams = mel.shape[0]
    d, t = c.d_model, c.positions
    m = streams * t
    keys = scale_keys(c)
    out: dict[str, float] = {}

    def amax_scale(x):
        scale, _ = fp8.dynamic_scale(x.contiguous(), stream=stream)
        return scale

    frames = fp8.mel_frames(mel.contiguous(), stream=stream)
    h1 = torch.zeros((streams, c.frames + 2, d), dtype=torch.float16, device=mel.device)
    fp8.conv1d_gelu(frames, *weights.conv1, 1, out=h1, out_row0=1, stream=stream)
    x = fp8.conv1d_gelu(h1, *weights.conv2, 2, positions=weights.positions, stream=stream).view(m, d)
    residual = None
    for i, L in enumerate(weights.layers):
        total, y, _ = fp8.layer_norm(x, *L.ln1, residual=residual, want_sum=residual is not None, stream=stream)
        x = total if residual is not None else x
        s = amax_scale(y)
        qkv, _ = fp8.linear(fp8.quantize(y, s, stream=stream), L.qkv.codes, L.qkv.scales, s, bias=L.qkv.bias,
                            stream=stream)
        attn, _ = fp8.self_attention(qkv, streams, c.heads, stream=stream)
        s_out = amax_scale(attn)
        o, _ = fp8.linear(fp8.quantize(attn, s_out, stream=stream), L.out.codes, L.out.scales, s_out,
                          bias=L.out.bias, stream=stream)
        x, y2, _ = fp8.layer_norm(x, *L.ln2, residual=o, want_sum=True, stream=stream)
        s_fc1 = amax_scale(y2)
        h, _ = fp8.linear(fp8.quantize(y2, s_fc1, stream=stream), L.fc1.codes, L.fc1.scales, s_fc1,
                          bias=L.fc1.bias, gelu=True, stream=stream)
        s_fc2 = amax_scale(h)
        residual, _ = fp8.linear(fp8.quantize(h, s_fc2, stream=stream), L.fc2.codes, L.fc2.scales, s_fc2,
                                 bias=L.fc2.bias, stream=stream)
        root = f"model.encoder.layers.{i}"
        for p in "qkv":
            out[f"{root}.self_attn.{p}_proj"] = float(s.item())
        out[f"{root}.self_attn.out_proj"] = float(s_out.item())
        out[f"{root}.fc1"] = float(s_fc1.item())
        out[f"{root}.fc2"] = float(s_fc2.item())
    _, states, _ = fp8.layer_norm(x, *weights.ln_post, residual=residual, stream=stream)
    s_cross = float(amax_scale(states).item())
    for key in keys["cross"]:
        out[key] = s_cross
    return out
