"""The reference graph's FP8 Q/DQ arithmetic in PyTorch on the host CPU.  TEST AND
BENCHMARK INFRASTRUCTURE ONLY: the CPU baseline that bench.py times beside the
GPU path (and its --impl reference arm); the product never imports it.

The reference runs this path inside TensorRT (no CPU implementation exists), so
this restates its graph (cpp/src/network_graph.cpp) with torch's fp32 CPU
kernels, rounding to fp16 at every edge the graph declares fp16:

* Q (:115-123): codes = saturate(rne(x / scale)) as clamp(x / s, +-448) cast to
  float8_e4m3fn (torch's cast rounds to nearest even but does not saturate);
* the Q/DQ linear (:124-159): per-row weight scales amax/448 (zero rows -> 1),
  the E4M3 codes dequantized exactly to fp32, matmul in fp32, times
  s_x * s_w, rounded to fp16, then + bias in fp16;
* GELU (:168-180) with its fp16 edges and constant fp16(2^-1/2) = 0.70703125;
* LayerNorm (:160-166) in fp32 with fp32 gamma/beta, rounded to fp16;
* attention (:235-247): q' = half(q c), k' = half(k c) with c = 64^-1/4 in
  fp16, scores half(q' k'^T), p = half(softmax_fp32(scores)), out = half(p v);
* the convolutions (:259-275) in fp32 with their bias, rounded to fp16, then GELU.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

E4M3_MAX = 448.0


def quantize(x: torch.Tensor, scale: float) -> torch.Tensor:
    """fp16/fp32 tensor -> E4M3 codes (torch.float8_e4m3fn) with one scale."""
    return (x.float() / scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)


def weight_scales(w: torch.Tensor) -> torch.Tensor:
    s = w.float().abs().amax(dim=1) / E4M3_MAX
    return torch.where(s > 0, s, torch.ones_like(s))


def prepare_weight(w: torch.Tensor):
    """(E4M3 codes as exact fp32 values, per-row scales) of an fp16 [n, k] weight."""
    s = weight_scales(w)
    return quantize(w.float() / s[:, None], 1.0).float(), s


def gelu_fp16(x: torch.Tensor) -> torch.Tensor:
    """(x * 0.5) * (1 + erf(x * 0.70703125)) with every edge rounded to fp16."""
    x = x.half().float()
    scaled = (x * 0.70703125).half().float()
    erf = torch.erf(scaled).half().float()
    left = (x * 0.5).half().float()
    right = (1.0 + erf).half().float()
    return (left * right).half()


def linear(x_codes: torch.Tensor, w_prepared, act_scale: float, bias: torch.Tensor | None = None,
           gelu: bool = False) -> torch.Tensor:
    """The Q/DQ linear on E4M3 codes [m, k] (float8_e4m3fn) -> fp16 [m, n]."""
    wq, ws = w_prepared
    acc = x_codes.float() @ wq.t()
    y = (acc * (act_scale * ws)[None, :]).half()
    if bias is not None:
        y = (y.float() + bias.float()).half()
    return gelu_fp16(y) if gelu else y


def layer_norm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    return F.layer_norm(x.float(), (x.shape[-1],), gamma.float(), beta.float(), eps).half()


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """q [heads, tq, 64], k/v [heads, tk, 64] fp16 -> fp16 [heads, tq, 64]."""
    c = torch.tensor(64.0 ** -0.25).half().float()
    qs = (q.float() * c).half().float()
    ks = (k.float() * c).half().float()
    scores = (qs @ ks.transpose(1, 2)).half().float()
    p = torch.softmax(scores, dim=-1).half().float()
    return (p @ v.float()).half()


def conv_gelu(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, stride: int) -> torch.Tensor:
    """x fp16 [c_in, frames] -> GELU(half(conv1d(x, w, b))) fp16 [c_out, frames / stride]."""
    y = F.conv1d(x.float()[None], w.float(), b.float(), stride=stride, padding=1)[0]
    return gelu_fp16(y.half())


class EncoderCPU:
    """The FP8 encoder graph (network_graph.cpp:255-301) for one stream on the CPU.
    `weights` maps the reference checkpoint names to fp16 CPU tensors; `scales`
    the activation-scale keys to floats (as encoder.scale_keys lists them)."""

    def __init__(self, weights, scales, layers: int, decoder_layers: int):
        self.w, self.s = weights, scales
        self.layers, self.decoder_layers = layers, decoder_layers
        self.prepared = {}
        for i in range(layers):
            root = f"model.encoder.layers.{i}"
            sa = f"{root}.self_attn"
            qkv = torch.cat([weights[f"{sa}.{p}_proj.weight"] for p in "qkv"])
            self.prepared[f"{root}.qkv"] = prepare_weight(qkv)
            self.prepared[f"{sa}.out_proj"] = prepare_weight(weights[f"{sa}.out_proj.weight"])
            self.prepared[f"{root}.fc1"] = prepare_weight(weights[f"{root}.fc1.weight"])
            self.prepared[f"{root}.fc2"] = prepare_weight(weights[f"{root}.fc2.weight"])
        rows = []
        for j in range(decoder_layers):
            root = f"model.decoder.layers.{j}.encoder_attn"
            rows += [weights[f"{root}.k_proj.weight"], weights[f"{root}.v_proj.weight"]]
        self.prepared["cross"] = prepare_weight(torch.cat(rows))

    def front(self, mel: torch.Tensor) -> torch.Tensor:
        w = self.w
        x = conv_gelu(mel.half(), w["model.encoder.conv1.weight"], w["model.encoder.conv1.bias"], 1)
        x = conv_gelu(x, w["model.encoder.conv2.weight"], w["model.encoder.conv2.bias"], 2)
        pos = w["model.encoder.embed_positions.weight"][: x.shape[1]]
        return (x.t().float() + pos.float()).half()

    def layer(self, i: int, x: torch.Tensor) -> torch.Tensor:
        w, s, p = self.w, self.s, self.prepared
        root = f"model.encoder.layers.{i}"
        sa = f"{root}.self_attn"
        d = x.shape[1]
        h = layer_norm(x, w[f"{root}.self_attn_layer_norm.weight"], w[f"{root}.self_attn_layer_norm.bias"])
        s_q = s[f"{sa}.q_proj"]
        bias = torch.cat([w[f"{sa}.q_proj.bias"], torch.zeros(d, dtype=torch.float16), w[f"{sa}.v_proj.bias"]])
        qkv = linear(quantize(h, s_q), p[f"{root}.qkv"], s_q, bias)
        heads = d // 64
        split = lambda t: t.reshape(-1, heads, 64).transpose(0, 1)
        a = attention(split(qkv[:, :d]), split(qkv[:, d:2 * d]), split(qkv[:, 2 * d:]))
        a = a.transpose(0, 1).reshape(-1, d)
        s_o = s[f"{sa}.out_proj"]
        x = (x.float() + linear(quantize(a, s_o), p[f"{sa}.out_proj"], s_o, w[f"{sa}.out_proj.bias"]).float()).half()
        h = layer_norm(x, w[f"{root}.final_layer_norm.weight"], w[f"{root}.final_layer_norm.bias"])
        s1, s2 = s[f"{root}.fc1"], s[f"{root}.fc2"]
        f = linear(quantize(h, s1), p[f"{root}.fc1"], s1, w[f"{root}.fc1.bias"], gelu=True)
        return (x.float() + linear(quantize(f, s2), p[f"{root}.fc2"], s2, w[f"{root}.fc2.bias"]).float()).half()

    def tail(self, x: torch.Tensor):
        w, s = self.w, self.s
        states = layer_norm(x, w["model.encoder.layer_norm.weight"], w["model.encoder.layer_norm.bias"])
        s_c = s["model.decoder.layers.0.encoder_attn.k_proj"]
        d = x.shape[1]
        bias = []
        for j in range(self.decoder_layers):
            bias += [torch.zeros(d, dtype=torch.float16), w[f"model.decoder.layers.{j}.encoder_attn.v_proj.bias"]]
        return states, linear(quantize(states, s_c), self.prepared["cross"], s_c, torch.cat(bias))

    def forward(self, mel: torch.Tensor, layers: int | None = None):
        x = self.front(mel)
        for i in range(self.layers if layers is None else layers):
            x = self.layer(i, x)
        return self.tail(x)
