"""Greedy Whisper decoding on this library's kernels, one token per stream per step.

Restates the FP8 decoder graph of cpp/src/network_graph.cpp:378-416 for a step of
`streams` independent streams (one beam each):

    x = half(token_table[token] + position_table[position])
    layers x [ LayerNorm -> fused q|k|v Q/DQ linear -> self-attention over the
               KV cache with the step's k, v appended -> out_proj -> residual add
               -> LayerNorm -> q_proj -> cross-attention over the encoder's
               cross K/V -> out_proj -> residual add -> LayerNorm -> fc1 + GELU
               -> fc2 -> residual add ]
    -> final LayerNorm -> fp16 logits against the token table -> greedy token
       (select_token, :332-339) -> the stream's cache length grows by one

and the greedy loop of python/src/listenflow/fastest_whisper/_inference.py:673-754
around it (every stream runs the fixed number of steps; tokens after a stream's
end-of-text are ignored by the caller).  The cache is a fixed-capacity fp16 buffer
[layers, streams, heads, capacity, 64] per K and V; the lengths (cached keys per
stream, also each new token's position) stay on the device, so one CUDA graph of
a step replays for every step.  A plan serves at most 32 streams (the small-M
tensor-core linears); more streams use several plans.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Mapping

import torch

from . import _native as native
from . import fp8
from .encoder import NEG_ZERO_HALF

MAX_STREAMS = 32
SOT = 50258  # <|startoftranscript|> of the multilingual large-v3 vocabulary
EOT = 50257


@dataclass(frozen=True)
class DecoderConfig:
    """Whisper large-v3 decoder shapes."""

    layers: int = 32
    d_model: int = 1280
    heads: int = 20
    ffn: int = 5120
    vocab: int = 51866
    positions: int = 448
    audio_positions: int = 1500


def scale_keys(config: DecoderConfig) -> dict[str, list[str]]:
    """The activation-scale keys of the decoder's FP8 linears, by role."""
    layer = lambda i, op: f"model.decoder.layers.{i}.{op}"
    r = range(config.layers)
    return {"qkv": [layer(i, "self_attn.q_proj") for i in r],
            "self_out": [layer(i, "self_attn.out_proj") for i in r],
            "cross_q": [layer(i, "encoder_attn.q_proj") for i in r],
            "cross_out": [layer(i, "encoder_attn.out_proj") for i in r],
            "fc1": [layer(i, "fc1") for i in r],
            "fc2": [layer(i, "fc2") for i in r]}


def add_synthetic_decoder(checkpoint: dict, config: DecoderConfig, seed: int, device) -> dict:
    """Adds random-init decoder weights under the reference's names (the cross-attention
    k/v projections come with the encoder's synthetic checkpoint): linears ~N(0, 0.02),
    biases ~N(0, 0.02), token and position tables ~N(0, 0.02), LayerNorm gamma
    1 + N(0, 0.1) and beta N(0, 0.1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    d, f = config.d_model, config.ffn

    def normal(shape, std):
        return (torch.randn(shape, generator=g, device=device) * std).half()

    ck = checkpoint
    ck["model.decoder.embed_tokens.weight"] = normal((config.vocab, d), 0.02)
    ck["model.decoder.embed_positions.weight"] = normal((config.positions, d), 0.02)
    for i in range(config.layers):
        root = f"model.decoder.layers.{i}"
        for p in ("q", "k", "v", "out"):
            ck[f"{root}.self_attn.{p}_proj.weight"] = normal((d, d), 0.02)
            if p != "k":
                ck[f"{root}.self_attn.{p}_proj.bias"] = normal((d,), 0.02)
        for p in ("q", "out"):
            ck[f"{root}.encoder_attn.{p}_proj.weight"] = normal((d, d), 0.02)
            ck[f"{root}.encoder_attn.{p}_proj.bias"] = normal((d,), 0.02)
        for name, (n, k) in (("fc1", (f, d)), ("fc2", (d, f))):
            ck[f"{root}.{name}.weight"] = normal((n, k), 0.02)
            ck[f"{root}.{name}.bias"] = normal((n,), 0.02)
        for norm in ("self_attn_layer_norm", "encoder_attn_layer_norm", "final_layer_norm"):
            ck[f"{root}.{norm}.weight"] = (1 + 0.1 * torch.randn(d, generator=g, device=device)).half()
            ck[f"{root}.{norm}.bias"] = normal((d,), 0.1)
    ck["model.decoder.layer_norm.weight"] = (1 + 0.1 * torch.randn(d, generator=g, device=device)).half()
    ck["model.decoder.layer_norm.bias"] = normal((d,), 0.1)
    return ck


@dataclass
class PackedLinear:
    """E4M3 weight, scales, bias, and the weight re-laid for the small-M kernels."""

    q: fp8.QuantizedWeight
    packed: torch.Tensor


def _packed(weight: torch.Tensor, bias: torch.Tensor | None) -> PackedLinear:
    q = fp8.QuantizedWeight.from_half(weight, bias)
    return PackedLinear(q, fp8.pack_skinny(q.codes))


@dataclass
class DecoderLayerWeights:
    ln1: tuple[torch.Tensor, torch.Tensor]
    qkv: PackedLinear
    self_out: PackedLinear
    ln2: tuple[torch.Tensor, torch.Tensor]
    cross_q: PackedLinear
    cross_out: PackedLinear
    ln3: tuple[torch.Tensor, torch.Tensor]
    fc1: PackedLinear
    fc2: PackedLinear


@dataclass
class DecoderWeights:
    config: DecoderConfig
    token_table: torch.Tensor   # fp16 [vocab, d]: embedding and (tied) logits weight
    logits_packed: torch.Tensor  # the same, re-laid for the small-M fp16 kernel
    position_table: torch.Tensor
    layers: list[DecoderLayerWeights]
    ln_post: tuple[torch.Tensor, torch.Tensor]

    @classmethod
    def from_checkpoint(cls, checkpoint: Mapping[str, torch.Tensor],
                        config: DecoderConfig = DecoderConfig()) -> "DecoderWeights":
        def get(name):
            t = checkpoint[name]
            if t.dtype != torch.float16 or not t.is_cuda:
                raise ValueError(f"{name}: fp16 CUDA tensor expected")
            return t.contiguous()

        def norm(name):
            return get(f"{name}.weight").float(), get(f"{name}.bias").float()

        d = config.d_model
        tokens = get("model.decoder.embed_tokens.weight")
        device = tokens.device
        neg_zero = torch.full((d,), NEG_ZERO_HALF, dtype=torch.int16, device=device).view(torch.float16)
        layers = []
        for i in range(config.layers):
            root = f"model.decoder.layers.{i}"
            sa, ca = f"{root}.self_attn", f"{root}.encoder_attn"
            w_qkv = torch.cat([get(f"{sa}.{p}_proj.weight") for p in "qkv"])
            b_qkv = torch.cat([get(f"{sa}.q_proj.bias"), neg_zero, get(f"{sa}.v_proj.bias")])
            layers.append(DecoderLayerWeights(
                ln1=norm(f"{root}.self_attn_layer_norm"),
                qkv=_packed(w_qkv, b_qkv),
                self_out=_packed(get(f"{sa}.out_proj.weight"), get(f"{sa}.out_proj.bias")),
                ln2=norm(f"{root}.encoder_attn_layer_norm"),
                cross_q=_packed(get(f"{ca}.q_proj.weight"), get(f"{ca}.q_proj.bias")),
                cross_out=_packed(get(f"{ca}.out_proj.weight"), get(f"{ca}.out_proj.bias")),
                ln3=norm(f"{root}.final_layer_norm"),
                fc1=_packed(get(f"{root}.fc1.weight"), get(f"{root}.fc1.bias")),
                fc2=_packed(get(f"{root}.fc2.weight"), get(f"{root}.fc2.bias")),
            ))
        return cls(config, tokens, fp8.pack_skinny(tokens), get("model.decoder.embed_positions.weight"), layers,
                   norm("model.decoder.layer_norm"))

    def weight_bytes(self) -> int:
        """Bytes a step streams: E4M3 weights, scales and biases of every linear, and the
        fp16 logits table."""
        total = self.token_table.numel() * 2
        for L in self.layers:
            for lin in (L.qkv, L.self_out, L.cross_q, L.cross_out, L.fc1, L.fc2):
                n, k = lin.q.codes.shape
                total += n * k + n * 4 + n * 2
        return total


def _scales_for(config: DecoderConfig, scales: Mapping[str, float]) -> dict[str, list[float]]:
    out = {}
    for role, names in scale_keys(config).items():
        values = []
        for key in names:
            v = scales.get(key)
            if v is None or not isinstance(v, (int, float)) or not math.isfinite(v) or v <= 0:
                raise ValueError(f"missing or invalid activation scale for {key}")
            values.append(float(v))
        out[role] = values
    return out


class Decoder:
    """A planned greedy decode step for `streams` (<= 32) streams that read the cross
    K/V of streams [first, first + streams) of an encoder's cross_kv buffer
    ([2 * layers, total streams, heads, positions, 64])."""

    def __init__(self, weights: DecoderWeights, scales: Mapping[str, float], cross_kv: torch.Tensor,
                 streams: int, first: int = 0, capacity: int | None = None):
        c = weights.config
        if not 1 <= streams <= MAX_STREAMS:
            raise ValueError(f"a decoder plan serves 1 to {MAX_STREAMS} streams")
        if cross_kv.shape[0] != 2 * c.layers or first + streams > cross_kv.shape[1]:
            raise ValueError("cross_kv must be [2 * layers, streams, heads, positions, 64] covering the streams")
        self.config, self.weights, self.streams, self.first = c, weights, streams, first
        self.capacity = capacity if capacity is not None else c.positions
        self.scales = _scales_for(c, scales)
        self.cross_kv = cross_kv
        device = cross_kv.device
        d, f, s = c.d_model, c.ffn, streams
        empty = lambda shape, dtype=torch.float16: torch.empty(shape, dtype=dtype, device=device)
        self.tokens = torch.zeros(s, dtype=torch.int32, device=device)
        self.lengths = torch.zeros(s, dtype=torch.int32, device=device)
        self.suppression = torch.zeros((s, c.vocab), dtype=torch.float32, device=device)
        self.cache_k = torch.zeros((c.layers, s, c.heads, self.capacity, 64), dtype=torch.float16, device=device)
        self.cache_v = torch.zeros_like(self.cache_k)
        self.x0 = empty((s, d))
        self.stream_buf = [empty((s, d)), empty((s, d))]
        self.ln_codes = empty((s, d), torch.uint8)
        self.qkv = empty((s, 3 * d))
        self.attn_codes = empty((s, d), torch.uint8)
        self.o = empty((s, d))
        self.q = empty((s, d))
        self.fc2_codes = empty((s, f), torch.uint8)
        self.r = empty((s, d))
        self.states = empty((s, d))
        self.logits = empty((s, c.vocab))
        self._calls = self._plan()

    def _plan(self):
        c, w, sc = self.config, self.weights, self.scales
        lib = native.library()
        calls = []
        d, s = c.d_model, self.streams
        p = lambda t: t.data_ptr() if t is not None else None

        calls.append(("lffw_decoder_embed", lambda st, a=(p(self.tokens), p(self.lengths), p(w.token_table),
                                                           p(w.position_table), s, d, c.vocab, c.positions,
                                                           p(self.x0)): lib.lffw_decoder_embed(*a, st)))

        def norm(x, residual, params, sum_out, y, code_scale, codes):
            a = native.LayerNormArgs()
            a.struct_size = ctypes.sizeof(a)
            a.rows, a.cols = s, d
            a.x, a.residual, a.sum_out = p(x), p(residual), p(sum_out)
            a.gamma, a.beta, a.epsilon = p(params[0]), p(params[1]), 1e-5
            a.y, a.code_scale, a.codes = p(y), code_scale if code_scale is not None else 0.0, p(codes)
            return ("lffw_layer_norm", lambda st, a=a: lib.lffw_layer_norm(ctypes.byref(a), st))

        def linear(x_codes, lin, act_scale, y=None, gelu=False, next_scale=None, next_codes=None):
            a = native.LinearArgs()
            a.struct_size = ctypes.sizeof(a)
            a.m, a.n, a.k = s, lin.q.scales.shape[0], x_codes.shape[-1]
            a.x_codes, a.act_scale = p(x_codes), act_scale
            a.w_codes, a.w_scales, a.bias = p(lin.packed), p(lin.q.scales), p(lin.q.bias)
            a.w_layout = native.WEIGHTS_SKINNY_TILES
            a.epilogue = native.EPILOGUE_GELU if gelu else native.EPILOGUE_NONE
            a.y = p(y)
            a.next_scale = next_scale if next_scale is not None else 0.0
            a.next_codes = p(next_codes)
            return ("lffw_fp8_linear", lambda st, a=a: lib.lffw_fp8_linear(ctypes.byref(a), st))

        def self_attention(layer, code_scale):
            a = native.DecoderSelfAttentionArgs()
            a.struct_size = ctypes.sizeof(a)
            a.streams, a.heads, a.head_dim, a.capacity = s, c.heads, 64, self.capacity
            a.qkv, a.qkv_ld = p(self.qkv), 3 * d
            a.cache_k, a.cache_v, a.lengths = p(self.cache_k[layer]), p(self.cache_v[layer]), p(self.lengths)
            a.out, a.code_scale, a.out_codes = None, code_scale, p(self.attn_codes)
            return ("lffw_decoder_self_attention",
                    lambda st, a=a: lib.lffw_decoder_self_attention(ctypes.byref(a), st))

        def cross_attention(layer, code_scale):
            a = native.CrossAttentionArgs()
            a.struct_size = ctypes.sizeof(a)
            a.streams, a.queries, a.heads, a.head_dim, a.keys = s, 1, c.heads, 64, c.audio_positions
            a.q = p(self.q)
            a.k = p(self.cross_kv[2 * layer, self.first])
            a.v = p(self.cross_kv[2 * layer + 1, self.first])
            a.out, a.code_scale, a.out_codes = None, code_scale, p(self.attn_codes)
            return ("lffw_cross_attention", lambda st, a=a: lib.lffw_cross_attention(ctypes.byref(a), st))

        x, residual, turn = self.x0, None, 0

        def next_buf():
            nonlocal turn
            b = self.stream_buf[turn]
            turn ^= 1
            return b

        for i, L in enumerate(w.layers):
            s_qkv, s_so, s_cq, s_co = sc["qkv"][i], sc["self_out"][i], sc["cross_q"][i], sc["cross_out"][i]
            s_fc1, s_fc2 = sc["fc1"][i], sc["fc2"][i]
            if residual is None:
                calls.append(norm(x, None, L.ln1, None, None, s_qkv, self.ln_codes))
            else:
                nxt = next_buf()
                calls.append(norm(x, residual, L.ln1, nxt, None, s_qkv, self.ln_codes))
                x = nxt
            calls.append(linear(self.ln_codes, L.qkv, s_qkv, y=self.qkv))
            calls.append(self_attention(i, s_so))
            calls.append(linear(self.attn_codes, L.self_out, s_so, y=self.o))
            nxt = next_buf()
            calls.append(norm(x, self.o, L.ln2, nxt, None, s_cq, self.ln_codes))
            x = nxt
            calls.append(linear(self.ln_codes, L.cross_q, s_cq, y=self.q))
            calls.append(cross_attention(i, s_co))
            calls.append(linear(self.attn_codes, L.cross_out, s_co, y=self.o))
            nxt = next_buf()
            calls.append(norm(x, self.o, L.ln3, nxt, None, s_fc1, self.ln_codes))
            x = nxt
            calls.append(linear(self.ln_codes, L.fc1, s_fc1, gelu=True, next_scale=s_fc2, next_codes=self.fc2_codes))
            calls.append(linear(self.fc2_codes, L.fc2, s_fc2, y=self.r))
            residual = self.r
        calls.append(norm(x, residual, w.ln_post, None, self.states, None, None))
        calls.append(("lffw_fp16_linear", lambda st, a=(p(self.states), p(w.logits_packed), None, p(self.logits), s,
                                                         c.vocab, d, native.WEIGHTS_SKINNY_TILES):
                      lib.lffw_fp16_linear(*a, st)))
        calls.append(("lffw_greedy_select", lambda st, a=(p(self.logits), c.vocab, p(self.suppression),
                                                           c.vocab, s, c.vocab, p(self.tokens), p(self.lengths)):
                      lib.lffw_greedy_select(*a, st)))
        return calls

    @property
    def launches(self) -> int:
        return len(self._calls)

    def reset(self, start_token: int = SOT) -> None:
        """Empties the caches and puts `start_token` at position 0 of every stream."""
        self.lengths.zero_()
        self.tokens.fill_(start_token)

    def step(self, stream=None) -> None:
        """One greedy step of every stream: reads tokens/lengths, writes the next tokens,
        appends to the caches and advances the lengths."""
        st = fp8._stream(stream)
        for name, call in self._calls:
            native.check(call(st), name)


def calibrate(weights: DecoderWeights, cross_kv: torch.Tensor, streams: int, steps: int,
              start_token: int = SOT) -> dict[str, float]:
    """Static activation scales amax/448 of every FP8 linear input of the decoder,
    observed over `steps` greedy steps of the first `streams` streams of cross_kv (the
    rule of python/scripts/calibrate_fp8.py:384-385, the maximum over the steps).  The
    same kernels run with fp16 outputs and dynamic scales."""
    c = weights.config
    d = c.d_model
    device = cross_kv.device
    amax: dict[str, float] = {}
    keys = scale_keys(c)
    tokens = torch.full((streams,), start_token, dtype=torch.int32, device=device)
    lengths = torch.zeros(streams, dtype=torch.int32, device=device)
    cache_k = torch.zeros((c.layers, streams, c.heads, steps, 64), dtype=torch.float16, device=device)
    cache_v = torch.zeros_like(cache_k)
    suppression = torch.zeros((streams, c.vocab), dtype=torch.float32, device=device)

    def observe(role, i, t):
        scale, _ = fp8.dynamic_scale(t.contiguous())
        key = keys[role][i]
        amax[key] = max(amax.get(key, 0.0), float(scale.item()))
        return scale

    for _ in range(steps):
        x = fp8.decoder_embed(tokens, lengths, weights.token_table, weights.position_table)
        residual = None
        for i, L in enumerate(weights.layers):
            total, y, _ = fp8.layer_norm(x, *L.ln1, residual=residual, want_sum=residual is not None)
            x = total if residual is not None else x
            s = observe("qkv", i, y)
            qkv, _ = fp8.linear(fp8.quantize(y, s), L.qkv.q.codes, L.qkv.q.scales, s, bias=L.qkv.q.bias)
            a, _ = fp8.decoder_self_attention(qkv, cache_k[i], cache_v[i], lengths)
            s = observe("self_out", i, a)
            o, _ = fp8.linear(fp8.quantize(a, s), L.self_out.q.codes, L.self_out.q.scales, s, bias=L.self_out.q.bias)
            x, y, _ = fp8.layer_norm(x, *L.ln2, residual=o, want_sum=True)
            s = observe("cross_q", i, y)
            q, _ = fp8.linear(fp8.quantize(y, s), L.cross_q.q.codes, L.cross_q.q.scales, s, bias=L.cross_q.q.bias)
            a, _ = fp8.cross_attention(q, cross_kv[2 * i, :streams].contiguous(),
                                       cross_kv[2 * i + 1, :streams].contiguous(), 1)
            s = observe("cross_out", i, a)
            o, _ = fp8.linear(fp8.quantize(a, s), L.cross_out.q.codes, L.cross_out.q.scales, s,
                              bias=L.cross_out.q.bias)
            x, y, _ = fp8.layer_norm(x, *L.ln3, residual=o, want_sum=True)
            s = observe("fc1", i, y)
            h, _ = fp8.linear(fp8.quantize(y, s), L.fc1.q.codes, L.fc1.q.scales, s, bias=L.fc1.q.bias, gelu=True)
            s = observe("fc2", i, h)
            residual, _ = fp8.linear(fp8.quantize(h, s), L.fc2.q.codes, L.fc2.q.scales, s, bias=L.fc2.q.bias)
        _, y, _ = fp8.layer_norm(x, *weights.ln_post, residual=residual)
        logits = fp8.fp16_linear(y, weights.token_table, w_packed=weights.logits_packed)
        fp8.greedy_select(logits, suppression, tokens, lengths)
    out = dict(amax)
    for i in range(c.layers):  # k_proj and v_proj read the same input as q_proj
        for part in "kv":
            out[f"model.decoder.layers.{i}.self_attn.{part}_proj"] = out[keys["qkv"][i]]
    return out
