"""Benchmark of the FP8 E4M3 quantized-linear hot path on B200.

Workload: one Whisper large-v3 encoder layer's linear set on
M = 12000 rows (8 streams x 1500 positions): activation quantize -> QKV
[1280->3840] + bias, quantize -> out-proj [1280->1280] + bias, quantize ->
fc1 [1280->5120] + bias + GELU whose epilogue emits fc2's E4M3 input codes, and
fc2 [5120->1280] + bias.  A step is one pass over that set: 4 tcgen05 GEMMs and
3 quantize kernels = 471.86 GFLOP.  Inputs are seeded synthetic tensors
(activations ~N(0,1) as after LayerNorm, weights ~N(0,0.02)); static activation
scales are the calibration rule amax/448 applied once at set-up.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (under torchrun) every rank runs the same per-GPU workload on its own
GPU (independent stream batches, no collective on the data path); `value` is
the whole-job TFLOP/s over the max-over-ranks time.  `--impl reference` times
the CPU restatement of the reference's Q/DQ linear (oracle/, the reference has
no CPU implementation of this path) on host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PACKAGE = "listenflow-fastest-whisper_b200"

M = 12000  # 8 x 1500 encoder positions
D = 1280
FFN = 5120
LINEARS = (  # name, K, N, gelu
    ("qkv", D, 3 * D, False),
    ("out_proj", D, D, False),
    ("fc1", D, FFN, True),
    ("fc2", FFN, D, False),
)
FLOPS_PER_STEP = sum(2 * M * k * n for _, k, n, _ in LINEARS)  # 471.86e9
METRIC = "FP8 GEMM TFLOP/s (encoder layer linear set, M=12000)"
CONFIG = {
    "workload": "C2: Whisper large-v3 encoder layer FP8 linear set (QKV 1280->3840, out 1280->1280, "
                "fc1 1280->5120 +GELU -> fc2 codes, fc2 5120->1280), M=12000 (8 x 1500 positions)",
    "m": M,
    "flops_per_step": FLOPS_PER_STEP,
    "l2": "flushed between timed steps, outside the step events: a 256 MiB buffer is written, then a "
          "separate 256 MiB buffer is read so that the written lines go back to HBM before the step; the "
          "step's working set (~330 MB) also exceeds L2",
    "timing": "one CUDA event pair per step, no events between the step's kernels; per_gemm_ms and the "
              "roofline come from a second pass of the same steps with an event around every GEMM, each "
              "GEMM's time the median over that pass's launches (an interval can include the GPU idling "
              "until the host enqueues the next launch)",
}


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--decoder-steps", type=int, default=20,
                   help="timed replays of the C3 decoder-step graph (0 skips it)")
    p.add_argument("--decoder-layers", type=int, default=32,
                   help="decoder layers in the C3 step (32 is the measured configuration)")
    p.add_argument("--only", choices=("all", "c2", "ln", "attention", "self_attention", "decoder", "encoder"),
                   default="all",
                   help="run one section alone and print its line (profiling): 'c2' the timed C2 steps, "
                        "'ln' the LayerNorm producer, 'attention' the cross-attention, 'decoder' the C3 step, "
                        "'encoder' the 32-layer encoder forward")
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="target CPU-baseline sample time (0 skips the CPU baseline, for profiling runs)")
    return p.parse_args(argv)


def dist_env():
    return importlib.import_module(PACKAGE + ".replicas").env_rank()


def synthetic(seed: int):
    """Seeded inputs: three fp16 activation tensors and four fp16 weights/biases."""
    rng = np.random.default_rng(seed)
    acts = {
        "qkv": (rng.standard_normal((M, D), dtype=np.float32)).astype(np.float16),
        "out_proj": (rng.standard_normal((M, D), dtype=np.float32)).astype(np.float16),
        "fc1": (rng.standard_normal((M, D), dtype=np.float32)).astype(np.float16),
    }
    weights = {}
    for name, k, n, _ in LINEARS:
        w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16)
        b = (rng.standard_normal(n, dtype=np.float32) * 0.02).astype(np.float16)
        weights[name] = (w, b)
    return acts, weights


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.

class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every ~2 ms while
    the timed region runs (a thread; reading settings only)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, bus_id: str):
        self.bus_id = bus_id
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._nvml = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(self.bus_id)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:  # no NVML: report no samples
            self._nvml = None
        return self

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                clk = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                why = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._handle)
                self.samples.append((clk, why))
            except Exception:
                break
            time.sleep(0.002)

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self._thread.join(timeout=2)
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        clocks = [c for c, _ in self.samples]
        reasons = set()
        for _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(clocks) if clocks else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(clocks)}


def pci_bus_id(torch, device) -> str:
    """NVML bus id of a torch device (independent of CUDA_VISIBLE_DEVICES)."""
    props = torch.cuda.get_device_properties(device)
    return f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"


# ---------------------------------------------------------------------------
# Our arm.

def run_ours(args, rank, local_rank, world):
    import torch

    fp8 = importlib.import_module(PACKAGE + ".fp8")
    native = importlib.import_module(PACKAGE + "._native")
    replicas = importlib.import_module(PACKAGE + ".replicas")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = replicas.init("nccl", device=device) if world > 1 else None

    acts_np, weights_np = synthetic(seed=1234 + rank)
    # Static activation scales: the calibration rule (amax/448) applied once.
    scales = {name: float(np.float32(np.abs(a.astype(np.float32)).max()) / np.float32(448))
              for name, a in acts_np.items()}
    stream = torch.cuda.current_stream()
    acts = {name: torch.from_numpy(a).to(device) for name, a in acts_np.items()}
    weights = {}
    for name, k, n, _ in LINEARS:
        w, b = weights_np[name]
        weights[name] = fp8.QuantizedWeight.from_half(torch.from_numpy(w).to(device), torch.from_numpy(b).to(device))
    # fc2's input scale: calibrated on one fc1 pass (fp16 GELU output amax / 448).
    codes_fc1 = fp8.quantize(acts["fc1"], scales["fc1"])
    hidden, _ = fp8.linear(codes_fc1, weights["fc1"].codes, weights["fc1"].scales, scales["fc1"],
                           bias=weights["fc1"].bias, gelu=True)
    scales["fc2"] = float(hidden.abs().max().float().item()) / 448.0
    del hidden

    # Output / scratch buffers, allocated once.
    codes = {name: torch.empty((M, D), dtype=torch.uint8, device=device) for name in acts}
    fc2_codes = torch.empty((M, FFN), dtype=torch.uint8, device=device)
    outs = {"qkv": torch.empty((M, 3 * D), dtype=torch.float16, device=device),
            "out_proj": torch.empty((M, D), dtype=torch.float16, device=device),
            "fc2": torch.empty((M, D), dtype=torch.float16, device=device)}
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    scrub = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=device)  # 256 MiB, read to clean L2
    gemm_flops = {name: 2 * M * k * n for name, k, n, _ in LINEARS}

    def step(events=None, a=acts, o=outs):
        def mark(i):
            if events is not None:
                events[i].record(stream)
        fp8.quantize(a["qkv"], scales["qkv"], out=codes["qkv"])
        mark(0)
        fp8.linear(codes["qkv"], weights["qkv"].codes, weights["qkv"].scales, scales["qkv"],
                   bias=weights["qkv"].bias, out=o["qkv"])
        mark(1)
        fp8.quantize(a["out_proj"], scales["out_proj"], out=codes["out_proj"])
        mark(2)
        fp8.linear(codes["out_proj"], weights["out_proj"].codes, weights["out_proj"].scales, scales["out_proj"],
                   bias=weights["out_proj"].bias, out=o["out_proj"])
        mark(3)
        fp8.quantize(a["fc1"], scales["fc1"], out=codes["fc1"])
        mark(4)
        fp8.linear(codes["fc1"], weights["fc1"].codes, weights["fc1"].scales, scales["fc1"],
                   bias=weights["fc1"].bias, gelu=True, want_y=False, next_scale=scales["fc2"],
                   next_codes=fc2_codes)
        mark(5)
        fp8.linear(fc2_codes, weights["fc2"].codes, weights["fc2"].scales, scales["fc2"],
                   bias=weights["fc2"].bias, out=o["fc2"])
        mark(6)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if native.device_error() != 0:
        raise RuntimeError("device-side wait timed out during warm-up")

    def flush_l2():
        flush.zero_()  # evicts the step's tensors from L2
        scrub.sum()    # read-only pass: the memset's dirty lines are written back here, not in the step

    # Timed steps: one event pair per step and nothing between the kernels, so
    # each launch can overlap the previous one's tail (programmatic dependent
    # launch); the L2 flush sits outside the events.
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    launches_before = native.launch_count()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(pci_bus_id(torch, device)) as clocks:
        for s in range(args.steps):
            flush_l2()
            ev[s][0].record(stream)
            step()
            ev[s][1].record(stream)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    launches = native.launch_count() - launches_before
    step_ms = [ev[s][0].elapsed_time(ev[s][1]) for s in range(args.steps)]

    # Per-GEMM breakdown (roofline of the GEMM kernel): the same steps again with
    # an event around every GEMM launch.  Events between launches end the
    # launch overlap, so these steps are slower than the timed ones above.
    bd_steps = min(args.steps, 50)
    bev = [[torch.cuda.Event(enable_timing=True) for _ in range(8)] for _ in range(bd_steps)]
    for s in range(bd_steps):
        flush_l2()
        bev[s][7].record(stream)
        step(bev[s])
    torch.cuda.synchronize()
    # Median per GEMM over the pass: an event interval also holds any time the GPU
    # waits for the host to enqueue the next launch, which a median ignores.
    per_gemm = {
        "qkv": statistics.median(bev[s][0].elapsed_time(bev[s][1]) for s in range(bd_steps)),
        "out_proj": statistics.median(bev[s][2].elapsed_time(bev[s][3]) for s in range(bd_steps)),
        "fc1": statistics.median(bev[s][4].elapsed_time(bev[s][5]) for s in range(bd_steps)),
        "fc2": statistics.median(bev[s][5].elapsed_time(bev[s][6]) for s in range(bd_steps)),
    }
    total_ms = sum(step_ms)
    total_gemm_ms = bd_steps * sum(per_gemm.values())
    if native.device_error() != 0:
        raise RuntimeError("device-side wait timed out during the timed steps")

    # End to end through the public API with host buffers, every step: its
    # three fp16 activation tensors are copied in from pinned host memory and
    # its three fp16 outputs are copied back.  Copies in, the step's kernels
    # and copies out run on three streams with two device buffer sets, so
    # step i's outputs go out while step i+1 computes and step i+2's inputs
    # come in (PCIe is full duplex).
    import torch as _t

    host_in = {name: _t.from_numpy(a).pin_memory() for name, a in acts_np.items()}
    host_out = {name: _t.empty(tuple(t.shape), dtype=t.dtype).pin_memory() for name, t in outs.items()}
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out.values())
    sets = [(acts, outs), ({k: _t.empty_like(v) for k, v in acts.items()},
                           {k: _t.empty_like(v) for k, v in outs.items()})]
    s_in, s_out = _t.cuda.Stream(device), _t.cuda.Stream(device)

    def e2e_run(n):
        """n pipelined end-to-end steps; returns (start event on s_in, end event on s_out)."""
        start, end = _t.cuda.Event(enable_timing=True), _t.cuda.Event(enable_timing=True)
        loaded = [_t.cuda.Event() for _ in range(n)]
        computed = [_t.cuda.Event() for _ in range(n)]
        drained = [_t.cuda.Event() for _ in range(n)]
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        start.record(s_in)
        for i in range(n):
            a, o = sets[i % 2]
            with _t.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(computed[i - 2])  # set i%2's inputs are free once step i-2 ran
                for name, t in host_in.items():
                    a[name].copy_(t, non_blocking=True)
                loaded[i].record(s_in)
            stream.wait_event(loaded[i])
            if i >= 2:
                stream.wait_event(drained[i - 2])     # set i%2's outputs were copied out
            step(a=a, o=o)
            computed[i].record(stream)
            with _t.cuda.stream(s_out):
                s_out.wait_event(computed[i])
                for name, t in host_out.items():
                    t.copy_(o[name], non_blocking=True)
                drained[i].record(s_out)
        s_out.wait_stream(s_in)
        s_out.wait_stream(stream)
        end.record(s_out)
        return start, end

    e2e_steps = max(1, args.e2e_steps)
    e2e_run(2)
    _t.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e_start, e_end = e2e_run(e2e_steps)
    _t.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end)
    np.testing.assert_array_equal(host_out["fc2"].numpy(), sets[(e2e_steps - 1) % 2][1]["fc2"].cpu().numpy())

    full = args.only == "all" # 'c2': the timed C2 steps (and e2e) only
    ln = run_ln_producer(fp8, native, device, 20, seed=31 + rank) if full else None
    attention = run_cross_attention(fp8, native, device, 10, seed=41 + rank) if full else None
    self_attn = run_self_attention(fp8, native, device, 10, seed=51 + rank) if full else None
    encoder = run_encoder(fp8, native, device, 5, 2, seed=61 + rank) if full else None
    decoder = None
    if full and args.decoder_steps > 0:
        del flush, scrub
        decoder = run_decoder(fp8, native, device, args.decoder_steps, 3, seed=77 + rank,
                              layers_count=args.decoder_layers)
    # Max over ranks.
    total_ms, total_gemm_ms, e2e_ms = replicas.max_over_ranks([total_ms, total_gemm_ms, e2e_ms], dist, device)

    result = None
    if rank == 0:
        peaks = read_peaks()
        ms_per_step = total_ms / args.steps
        value = replicas.whole_job_rate(FLOPS_PER_STEP * args.steps, world, total_ms / 1e3) / 1e12
        gemm_launch_ms = total_gemm_ms / (4 * bd_steps)
        gemm_achieved = FLOPS_PER_STEP / 4 / (gemm_launch_ms / 1e3) / 1e12
        peak, peak_src = peaks
        traffic = read_traffic()
        result = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> fp32 accumulate, fp16 out",
            "data": "synthetic (seeded; activations ~N(0,1), weights ~N(0,0.02))",
            "config": dict(CONFIG, parallelism=f"replicas x{world} (no collective on the data path)"),
            "impl": "ours",
            "per_gemm_ms": {k: round(v, 4) for k, v in per_gemm.items()},
            "per_gemm_tflops": {k: round(gemm_flops[k] / (per_gemm[k] / 1e3) / 1e12, 1) for k in per_gemm},
            "roofline": {
                "bound": "tensor",
                "kernel": "fp8_gemm_kernel (tcgen05 kind::f8f6f4)",
                "achieved": round(gemm_achieved, 1),
                "peak": peak,
                "peak_source": peak_src,
                "unit": "TFLOP/s",
                "frac": round(gemm_achieved / peak, 4),
                "traffic": traffic,
            },
            "e2e": {
                "value": round(world * FLOPS_PER_STEP * e2e_steps / (e2e_ms / 1e3) / 1e12, 2),
                "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "fp8.quantize / fp8.linear (C ABI lffw_fp8_quantize / lffw_fp8_linear)",
                "pipelining": "copies in, kernels and copies out on three streams, two device buffer sets",
            },
            "encoder_linears_audio_s_per_s": round(
                replicas.whole_job_rate(8 * 30.0, world, 32 * ms_per_step / 1e3), 1),
            "encoder_linears_audio_note": "30 s streams/s through the FP8 linears of all 32 encoder layers "
                                          "(8 streams per step and GPU); attention, LayerNorm, conv and "
                                          "cross-K/V projections are not included",
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if full:
            result["ln_producer"] = ln
            result["cross_attention"] = attention
            result["self_attention"] = self_attn
            result["encoder_forward"] = encoder
        if decoder is not None:
            result["decoder_step"] = decoder
        if full and world == 1 and args.cpu_seconds > 0:
            result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ---------------------------------------------------------------------------
# Decoder step: M = 20 rows (4 streams x 5 beams), 32 layers
# of {self QKV 1280->3840, self out 1280->1280, cross q 1280->1280, cross out
# 1280->1280, fc1 1280->5120 + GELU (emits fc2's codes), fc2 5120->1280} with
# E4M3 weights, then the fp16 logits projection 1280->51866.  Memory-bound: the
# metric is weight bytes streamed per second.

DEC_M = 20
DEC_LAYERS = 32
VOCAB = 51866
DEC_LINEARS = (("qkv", 1280, 3840), ("self_out", 1280, 1280), ("cross_q", 1280, 1280),
               ("cross_out", 1280, 1280), ("fc1", 1280, 5120), ("fc2", 5120, 1280))


def run_decoder(fp8, native, device, steps: int, warmup: int, seed: int, layers_count: int = DEC_LAYERS):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    layers = []
    weight_bytes = 0
    for _ in range(layers_count):
        layer = {}
        for name, k, n in DEC_LINEARS:
            w = (torch.randn(n, k, generator=g, device=device) * 0.02).half()
            b = (torch.randn(n, generator=g, device=device) * 0.02).half()
            q = fp8.QuantizedWeight.from_half(w, b)
            layer[name] = (q, fp8.pack_skinny(q.codes))  # build-time re-layout for m <= 32
            weight_bytes += n * k + n * 4 + n * 2  # E4M3 codes + fp32 scales + fp16 bias
            del w, q.codes
        layers.append(layer)
    logits_w = (torch.randn(VOCAB, 1280, generator=g, device=device) * 0.02).half()
    logits_packed = fp8.pack_skinny(logits_w)
    weight_bytes += VOCAB * 1280 * 2
    x_codes = fp8.quantize(torch.randn(DEC_M, 1280, generator=g, device=device).half(), 0.01)
    x16 = torch.randn(DEC_M, 1280, generator=g, device=device).half()
    outs = {name: torch.empty(DEC_M, n, dtype=torch.float16, device=device) for name, _, n in DEC_LINEARS}
    fc2_in = torch.empty(DEC_M, 5120, dtype=torch.uint8, device=device)
    logits = torch.empty(DEC_M, VOCAB, dtype=torch.float16, device=device)

    def step():
        for layer in layers:
            for name in ("qkv", "self_out", "cross_q", "cross_out"):
                q, packed = layer[name]
                fp8.linear(x_codes, None, q.scales, 0.01, bias=q.bias, out=outs[name], w_packed=packed)
            q, packed = layer["fc1"]
            fp8.linear(x_codes, None, q.scales, 0.01, bias=q.bias, gelu=True, want_y=False, next_scale=0.02,
                       next_codes=fc2_in, w_packed=packed)
            q, packed = layer["fc2"]
            fp8.linear(fc2_in, None, q.scales, 0.02, bias=q.bias, out=outs["fc2"], w_packed=packed)
        fp8.fp16_linear(x16, logits_w, out=logits, w_packed=logits_packed)

    # The same linears as one persistent chain launch (link i starts reading
    # activations once link i-1 is complete), then the logits launch.
    links = []
    for layer in layers:
        for name in ("qkv", "self_out", "cross_q", "cross_out"):
            q, packed = layer[name]
            links.append(dict(x_codes=x_codes, w_packed=packed, w_scales=q.scales, act_scale=0.01, bias=q.bias,
                              out=outs[name]))
        q, packed = layer["fc1"]
        links.append(dict(x_codes=x_codes, w_packed=packed, w_scales=q.scales, act_scale=0.01, bias=q.bias,
                          gelu=True, next_scale=0.02, next_codes=fc2_in))
        q, packed = layer["fc2"]
        links.append(dict(x_codes=fc2_in, w_packed=packed, w_scales=q.scales, act_scale=0.02, bias=q.bias,
                          out=outs["fc2"]))
    chain = fp8.LinearChain(links)

    def chained_step():
        chain.run()
        fp8.fp16_linear(x16, logits_w, out=logits, w_packed=logits_packed)

    def measure(body):
        stream = torch.cuda.Stream(device)
        with torch.cuda.stream(stream):
            for _ in range(max(1, warmup)):
                body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body()
        for _ in range(max(1, warmup)):
            graph.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        if native.device_error() != 0:
            raise RuntimeError("device-side wait timed out in the decoder step")
        del graph
        return statistics.median(times)

    ms_calls = measure(step)
    calls_out = (outs["fc2"].clone(), logits.clone())
    ms_chain = measure(chained_step)
    # Same products, another fp32 summation order: a loose check against gross
    # errors (the tests bound both paths against the oracle).
    if not (torch.allclose(calls_out[0].float(), outs["fc2"].float(), rtol=2.0**-6, atol=2.0**-6)
            and torch.equal(calls_out[1], logits)):
        raise RuntimeError("the chained decoder step differs from the per-call step")
    chain.close()
    ms = min(ms_calls, ms_chain)
    hbm = read_hbm_peak()
    gbs = weight_bytes / (ms / 1e3) / 1e9
    mode = "one persistent chain launch + logits" if ms_chain <= ms_calls else \
        "one CUDA graph of per-linear launches with programmatic dependent launches"
    return {"workload": f"C3: decoder step, M=20 (4 streams x 5 beams), {layers_count} layers x 6 E4M3 linears + "
                        f"fp16 logits 1280->51866; {mode}",
            "ms_per_step": round(ms, 4), "weight_bytes_per_step": weight_bytes,
            "value": round(gbs, 1), "unit": "GB/s (weights streamed)",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm[0], "peak_source": hbm[1],
                         "unit": "GB/s", "frac": round(gbs / hbm[0], 4)},
            "per_call_ms": round(ms_calls, 4), "chain_ms": round(ms_chain, 4),
            "launches_per_step": 2 if ms_chain <= ms_calls else layers_count * 6 + 1}


def run_section_only(args, local_rank):
    """One secondary section alone on one GPU (profiling): the C3 decoder step,
    the LayerNorm producer or the cross-attention (--decoder-layers layers)."""
    import torch

    fp8 = importlib.import_module(PACKAGE + ".fp8")
    native = importlib.import_module(PACKAGE + "._native")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if args.only == "decoder":
        result = run_decoder(fp8, native, device, max(1, args.decoder_steps), max(1, args.warmup), seed=77,
                             layers_count=args.decoder_layers)
        result.update(metric="decoder-step weight streaming (C3)")
    elif args.only == "ln":
        result = run_ln_producer(fp8, native, device, max(1, args.steps), seed=31)
        result.update(metric="LayerNorm producer HBM throughput")
    elif args.only == "attention":
        result = run_cross_attention(fp8, native, device, max(1, args.steps), seed=41, layers=args.decoder_layers)
        result.update(metric="decoder cross-attention K/V throughput")
    elif args.only == "encoder":
        result = run_encoder(fp8, native, device, max(1, args.decoder_steps), max(1, args.warmup), seed=61)
        result.update(metric="encoder forward audio-s/s (32 layers, this library's kernels only)")
    else:
        result = run_self_attention(fp8, native, device, max(1, args.steps), seed=51)
        result.update(metric="encoder self-attention TFLOP/s")
    result.update(n_gpus=1, higher_is_better=True, impl="ours")
    return result


def run_encoder(fp8, native, device, steps: int, warmup: int, seed: int, layers_count: int = 32):
    """The Whisper large-v3 encoder's 32 transformer layers for 8 streams x 1500
    positions, every kernel this library's: LayerNorm -> E4M3 codes, QKV linear,
    self-attention -> codes, out_proj, residual add + LayerNorm -> codes, fc1 + GELU
    -> fc2 codes, fc2; the residual add after fc2 is done by the next layer's
    LayerNorm (network_graph.cpp:285-287).  One CUDA graph per forward.  Random
    weights (~N(0, 0.02), per-channel E4M3), fixed activation scales; the conv
    front-end and the log-mel are not included."""
    import torch

    streams, heads = 8, 20
    rows = streams * 1500
    g = torch.Generator(device=device).manual_seed(seed)

    def weight(n, k):
        w = (torch.randn(n, k, generator=g, device=device) * 0.02).half()
        b = (torch.randn(n, generator=g, device=device) * 0.02).half()
        q = fp8.QuantizedWeight.from_half(w, b)
        del w
        return q

    def norm_params():
        gamma = (1 + 0.1 * torch.randn(D, generator=g, device=device)).float()
        beta = (0.1 * torch.randn(D, generator=g, device=device)).float()
        return gamma, beta

    layers = [dict(qkv=weight(3840, D), out=weight(D, D), fc1=weight(5120, D), fc2=weight(D, 5120),
                   ln1=norm_params(), ln2=norm_params()) for _ in range(layers_count)]
    x0 = torch.randn(rows, D, generator=g, device=device).half()
    s_ln, s_attn, s_gelu = 0.012, 0.004, 0.006  # activation scales (amax / 448 of typical values)

    def forward():
        x, r = x0, None
        for L in layers:
            x, _, h = fp8.layer_norm(x, *L["ln1"], residual=r, code_scale=s_ln, want_y=False, want_sum=True)
            qkv, _ = fp8.linear(h, L["qkv"].codes, L["qkv"].scales, s_ln, bias=L["qkv"].bias)
            _, a = fp8.self_attention(qkv, streams, heads, code_scale=s_attn, want_out=False)
            o, _ = fp8.linear(a, L["out"].codes, L["out"].scales, s_attn, bias=L["out"].bias)
            x, _, h2 = fp8.layer_norm(x, *L["ln2"], residual=o, code_scale=s_ln, want_y=False, want_sum=True)
            _, f = fp8.linear(h2, L["fc1"].codes, L["fc1"].scales, s_ln, bias=L["fc1"].bias, gelu=True,
                              want_y=False, next_scale=s_gelu)
            r, _ = fp8.linear(f, L["fc2"].codes, L["fc2"].scales, s_gelu, bias=L["fc2"].bias)
        return x, r

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(max(1, warmup)):
            forward()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    launches_before = native.launch_count()
    with torch.cuda.graph(graph, stream=stream):
        out = forward()
    launches = native.launch_count() - launches_before
    for _ in range(max(1, warmup)):
        graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    if native.device_error() != 0:
        raise RuntimeError("device-side wait timed out in the encoder forward")
    if not bool(torch.isfinite(out[0]).all()):
        raise RuntimeError("non-finite encoder output")
    del graph, out
    ms = statistics.median(times)
    tokens = 1500
    flops = layers_count * (FLOPS_PER_STEP + 4 * tokens * tokens * 64 * heads * streams)
    return {"workload": f"Whisper large-v3 encoder, {layers_count} layers x (LayerNorm, QKV, self-attention, out_proj, "
                        "residual + LayerNorm, fc1 + GELU, fc2), 8 streams x 1500 positions, one CUDA graph; "
                        "conv front-end and log-mel not included",
            "ms_per_forward": round(ms, 3), "streams": streams,
            "value": round(streams * 30.0 / (ms / 1e3), 1), "unit": "audio-s/s (30 s streams)",
            "tflops": round(flops / (ms / 1e3) / 1e12, 1),
            "flops_note": "linears + QK^T + P.V (the second QK^T pass of the exact softmax not counted)",
            "launches_per_forward": int(launches)}


def run_ln_producer(fp8, native, device, reps: int, seed: int):
    """LayerNorm producer at C2 shapes (12000 x 1280, residual add): the fused
    kernel (residual sum + E4M3 codes for the next linear) against LayerNorm
    writing fp16 followed by a separate quantize."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, D, generator=g, device=device).half()
    r = torch.randn(M, D, generator=g, device=device).half()
    gamma = (1 + 0.1 * torch.randn(D, generator=g, device=device)).float()
    beta = (0.1 * torch.randn(D, generator=g, device=device)).float()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    scrub = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=device)

    def fused():
        fp8.layer_norm(x, gamma, beta, residual=r, code_scale=0.01, want_y=False, want_sum=True)

    def separate():
        _, y, _ = fp8.layer_norm(x, gamma, beta, residual=r, want_sum=True)
        fp8.quantize(y, 0.01)

    def timed(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(reps):
            flush.zero_()
            scrub.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    t_fused, t_sep = timed(fused), timed(separate)
    if native.device_error() != 0:
        raise RuntimeError("device-side wait timed out in the LayerNorm section")
    elems = M * D
    fused_bytes = elems * (2 + 2 + 2 + 1)  # x, residual in; sum, codes out
    gbs = fused_bytes / (t_fused / 1e3) / 1e9
    hbm = read_hbm_peak()
    return {"workload": "LayerNorm producer, 12000 x 1280 fp16 + residual -> fp16 sum + E4M3 codes",
            "fused_ms": round(t_fused, 4), "separate_ms": round(t_sep, 4),
            "separate": "LayerNorm writing fp16 y (and the sum), then lffw_fp8_quantize of y",
            "value": round(gbs, 1), "unit": "GB/s (algorithmic: 7 bytes per element)",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm[0], "peak_source": hbm[1],
                         "unit": "GB/s", "frac": round(gbs / hbm[0], 4)},
            "l2": "flushed before every launch (256 MiB written, then 256 MiB read)"}


def run_cross_attention(fp8, native, device, steps: int, seed: int, layers: int = DEC_LAYERS):
    """Decoder cross-attention over cached encoder K/V for all 32 layers of one
    decoder step, as one CUDA graph: C3 (4 streams x 5 beams) and C5 (16 greedy
    streams per GPU, 128 streams over 8 GPUs).  Each layer reads its own K/V
    (streams x 20 heads x 1500 keys x 64), so the step streams K/V from HBM;
    out_proj's E4M3 codes are the output."""
    import torch

    results = {}
    for name, streams, queries in (("c3_4x5", 4, 5), ("c5_16x1", 16, 1)):
        g = torch.Generator(device=device).manual_seed(seed)
        shape = (layers, streams, 20, 1500, 64)
        k = torch.randn(shape, generator=g, device=device).half()
        v = torch.randn(shape, generator=g, device=device).half()
        q = torch.randn((layers, streams * queries, 1280), generator=g, device=device).half()
        stream = torch.cuda.Stream(device)

        def step():
            for layer in range(layers):
                fp8.cross_attention(q[layer], k[layer], v[layer], queries, code_scale=0.004, want_out=False)

        with torch.cuda.stream(stream):
            for _ in range(3):
                step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        graph.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        if native.device_error() != 0:
            raise RuntimeError("device-side wait timed out in the cross-attention section")
        ms = statistics.median(times)
        kv_bytes = 2 * k.numel() * 2
        gbs = kv_bytes / (ms / 1e3) / 1e9
        hbm = read_hbm_peak()
        results[name] = {"streams": streams, "queries_per_stream": queries, "layers": layers,
                         "ms_per_step": round(ms, 4), "kv_bytes_per_step": kv_bytes,
                         "value": round(gbs, 1), "unit": "GB/s (K/V streamed)",
                         "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm[0],
                                      "peak_source": hbm[1], "unit": "GB/s", "frac": round(gbs / hbm[0], 4)}}
        del graph, k, v, q
        torch.cuda.empty_cache()
    results["workload"] = (f"decoder cross-attention, 20 heads x 1500 keys x 64, {layers} layers per step "
                           "(one graph), out_proj E4M3 codes out")
    return results


def run_self_attention(fp8, native, device, steps: int, seed: int):
    """Encoder self-attention for one layer at C2 shapes (8 streams x 1500 tokens x
    20 heads), read in place from a fused QKV output.  Work: 4 * tokens^2 * 64 flops
    per (stream, head) (QK^T and P.V); the kernel recomputes QK^T once more for the
    exact fp16 probabilities, which the rate does not count."""
    import torch

    streams, tokens, heads = 8, 1500, 20
    g = torch.Generator(device=device).manual_seed(seed)
    qkv = torch.randn((streams * tokens, 3 * heads * 64), generator=g, device=device).half()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    for _ in range(3):
        fp8.self_attention(qkv, streams, heads, code_scale=0.004, want_out=False)
    torch.cuda.synchronize()
    ts = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fp8.self_attention(qkv, streams, heads, code_scale=0.004, want_out=False)
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    if native.device_error() != 0:
        raise RuntimeError("device-side wait timed out in the self-attention section")
    ms = statistics.median(ts)
    flops = 4 * tokens * tokens * 64 * heads * streams
    tflops = flops / (ms / 1e3) / 1e12
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    return {"workload": "encoder self-attention, 8 streams x 1500 tokens x 20 heads x 64, one layer, "
                        "out_proj E4M3 codes out (tcgen05 kind::f16 MMAs, exact two-pass softmax; the second QK^T "
                        "pass is not counted in the flops)",
            "ms": round(ms, 4), "flops": flops, "value": round(tflops, 1), "unit": "TFLOP/s (QK^T + P.V)",
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak,
                         "peak_source": "measured dense bf16 of MEASURED_PEAKS.json (fp16 runs at the bf16 rate)",
                         "unit": "TFLOP/s", "frac": round(tflops / peak, 4)}}


def read_hbm_peak():
    try:
        return round(float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]), 1), \
            "MEASURED_PEAKS.json hbm_gbs (copy)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def read_peaks():
    """FP8 dense denominator: MEASURED_PEAKS.json has bf16 only; B200's dense FP8
    rate is twice its bf16 rate, so the measured burst bf16 figure x 2."""
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return round(2 * float(data["bf16_tflops"]), 1), "2 x measured bf16_tflops (burst) of MEASURED_PEAKS.json"
    except (OSError, KeyError, ValueError):
        return round(2 * 1590.0, 1), "2 x fallback bf16 1.59 PFLOP/s"


def read_traffic():
    """DRAM bytes per GEMM launch from the committed ncu summary, or None."""
    path = ROOT / "profiles" / "fp8_gemm_c2_traffic.json"
    try:
        return json.loads(path.read_text())["dram_bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        return None


# ---------------------------------------------------------------------------
# CPU baseline: the oracle restatement of the Q/DQ linear on host cores.

def cpu_sample(rows: int, seed: int = 4321):
    from oracle import oracle

    acts, weights = synthetic_small(rows, seed)
    prepared = []
    for name, k, n, gelu in LINEARS:
        w, b = weights[name]
        ws = oracle.weight_scales(w)
        wq = oracle.quantize_rows(w, ws)
        x = acts[name]
        s = np.float32(oracle.amax(x)) / np.float32(448)
        prepared.append((oracle.quantize(x, s), wq, s, ws, b, gelu))
    return prepared


def synthetic_small(rows, seed):
    rng = np.random.default_rng(seed)
    acts = {name: (rng.standard_normal((rows, k), dtype=np.float32)).astype(np.float16)
            for name, k, _, _ in LINEARS}
    weights = {name: ((rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16),
                      (rng.standard_normal(n, dtype=np.float32) * 0.02).astype(np.float16))
               for name, k, n, _ in LINEARS}
    return acts, weights


def cpu_step(prepared, threads: int):
    from oracle import oracle

    for xq, wq, s, ws, b, gelu in prepared:
        oracle.fp8_linear(xq, wq, s, ws, b, gelu=gelu, threads=threads)


def cpu_baseline(target_seconds: float):
    from oracle import oracle

    threads = oracle.threads()
    probe_rows = max(threads, 8)
    prepared = cpu_sample(probe_rows)
    t0 = time.perf_counter()
    cpu_step(prepared, threads)
    probe = time.perf_counter() - t0
    rows = int(min(M, max(probe_rows, probe_rows * target_seconds / max(probe, 1e-3) / 3)))
    prepared = cpu_sample(rows)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        cpu_step(prepared, threads)
        times.append(time.perf_counter() - t0)
    flops = FLOPS_PER_STEP * rows / M
    return {"value": round(flops / statistics.median(times) / 1e12, 6), "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": f"{rows} of {M} rows of each of the 4 linears (oracle/lffw_oracle.c, float64 exact "
                      f"accumulation, {threads} threads), median of 3"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    from oracle import oracle

    threads = oracle.threads()
    rows = 64
    prepared = cpu_sample(rows)
    t0 = time.perf_counter()
    cpu_step(prepared, threads)
    probe = time.perf_counter() - t0
    # Size each step so the whole --steps/--warmup run stays within ~2 minutes.
    per_step = min(4.0, 120.0 / max(1, args.steps + args.warmup))
    rows = int(min(M, max(rows, rows * per_step / max(probe, 1e-3))))
    prepared = cpu_sample(rows)
    for _ in range(args.warmup):
        cpu_step(prepared, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(prepared, threads)
    elapsed = time.perf_counter() - t0
    flops = FLOPS_PER_STEP * rows / M * args.steps
    value = round(flops / elapsed / 1e12, 6)
    sample = (f"{rows} of {M} rows of each of the 4 linears per step (CPU restatement oracle/lffw_oracle.c; "
              f"the reference runs this path inside TensorRT, which has no CPU implementation)")
    return {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> float64 exact accumulate, fp16 out",
        "data": "synthetic (seeded)", "config": dict(CONFIG, parallelism="host CPU, rank 0"),
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main(argv=None):
    args = parse_args(argv)
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        result = run_reference(args, rank, world)
    elif args.only in ("decoder", "ln", "attention", "self_attention", "encoder"):
        result = run_section_only(args, local_rank)
    else:
        result = run_ours(args, rank, local_rank, world)
    if result is not None and rank == 0:
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
