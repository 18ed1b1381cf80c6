"""Regenerate tests/golden/config1_fc1.npz, the seeded config-1 fc1 vectors.

    python tests/golden/make_config1.py

Config 1 is one encoder fc1 Q/DQ linear: X [1500, 1280] fp16 ~ N(0, 1),
W [5120, 1280] fp16 ~ N(0, 0.02), b [5120] fp16 ~ N(0, 0.02), drawn in that order
from torch.Generator().manual_seed(0); activation scale amax(X)/448, per-row
weight scales amax(W[n])/448 (0 -> 1), E4M3 codes of both operands, fp16 output
GELU(half(half(X.W^T * s_x * s_w) + b)) with the graph's fp16 edges
(cpp/src/network_graph.cpp:124-159, 168-183).

The inputs are regenerated from the seed, so the fixture stays small: it holds
the scales, SHA-256 digests of both code arrays and of the full output, and a
sample of output rows (with their activation codes) written by the oracle.
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

M, K, N = 1500, 1280, 5120
SAMPLE_ROWS = np.array([0, 1, 2, 127, 128, 255, 256, 511, 700, 1023, 1024, 1279, 1280, 1407, 1498, 1499])


def inputs():
    """X, W, b as float16 numpy arrays, drawn exactly as config 1 specifies."""
    import torch

    gen = torch.Generator().manual_seed(0)
    x = torch.randn(M, K, generator=gen).half()
    w = (torch.randn(N, K, generator=gen) * 0.02).half()
    b = (torch.randn(N, generator=gen) * 0.02).half()
    return x.numpy(), w.numpy(), b.numpy()


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    from oracle import oracle

    x, w, b = inputs()
    act_scale = np.float32(oracle.amax(x)) / np.float32(448)
    w_scales = oracle.weight_scales(w)
    xq = oracle.quantize(x, act_scale)
    wq = oracle.quantize_rows(w, w_scales)
    y, _ = oracle.fp8_linear(xq, wq, act_scale, w_scales, b, gelu=True)
    np.savez_compressed(
        HERE / "config1_fc1.npz",
        shape=np.array([M, K, N]),
        act_scale=np.array([act_scale], np.float32),
        w_scales=w_scales.astype(np.float32),
        x_codes_sha256=np.array(digest(xq)),
        w_codes_sha256=np.array(digest(wq)),
        y_sha256=np.array(digest(y)),
        rows=SAMPLE_ROWS,
        x_codes_rows=xq[SAMPLE_ROWS],
        y_rows=y[SAMPLE_ROWS],
    )
    print("wrote", HERE / "config1_fc1.npz")


if __name__ == "__main__":
    main()
