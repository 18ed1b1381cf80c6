"""The FP8 GEMM's tile order does not change its results.

A linear whose A operand exceeds 48 MB walks its tiles in groups of 8 M tiles
(every N tile of a group before the next group) so that A row panels are reused
from L2; smaller ones walk column by column.  Each output tile is still computed
by one CTA (or CTA pair) with the same K order, so both orders must give the same
bits.  LFFW_GEMM_GROUP forces an order for a whole process, so the column-order
run is a child process; the shapes cover a partial last group, a partial last N
tile and the single-CTA GELU code-table epilogue.
"""

from __future__ import annotations

import importlib
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = "listenflow-fastest-whisper_b200"

SHAPES = [
    (12000, 1280, 5120, False),  # 47 CTA-pair M tiles: 5 full groups and one of 7
    (10000, 1008, 5120, False),  # a partial last N tile (N a multiple of 16, as the ABI requires)
    (10000, 5120, 5120, True),   # GELU -> E4M3 codes only: single-CTA tiles, code table
]


def _run(fp8, m, n, k, gelu):
    """The linear's outputs on seeded inputs (fp16 y as bytes, or E4M3 codes with GELU)."""
    import torch

    gen = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k)
    x = (torch.randn(m, k, generator=gen, device="cuda") * 0.5).half()
    w = (torch.randn(n, k, generator=gen, device="cuda") * 0.02).half()
    b = (torch.randn(n, generator=gen, device="cuda") * 0.02).half()
    q = fp8.QuantizedWeight.from_half(w, b)
    codes = fp8.quantize(x, 0.01)
    if gelu:
        _, out = fp8.linear(codes, q.codes, q.scales, 0.01, bias=q.bias, gelu=True, want_y=False,
                            next_scale=0.02)
    else:
        out, _ = fp8.linear(codes, q.codes, q.scales, 0.01, bias=q.bias)
    torch.cuda.synchronize()
    return out.view(torch.uint8).cpu().numpy() if out.dtype != torch.uint8 else out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,gelu", SHAPES)
def test_grouped_raster_matches_column_order(cuda, fp8, tmp_path, m, n, k, gelu):
    assert m * k > (48 << 20), "the shape must take the grouped raster by default"
    grouped = _run(fp8, m, n, k, gelu)
    out_file = tmp_path / "column_order.npy"
    env = dict(os.environ, LFFW_GEMM_GROUP="0")
    subprocess.run([sys.executable, __file__, str(m), str(n), str(k), str(int(gelu)), str(out_file)],
                   env=env, check=True, cwd=ROOT, timeout=300)
    column = np.load(out_file)
    assert column.shape == grouped.shape
    assert np.array_equal(column, grouped)


if __name__ == "__main__":
    # Child process: the same linear in the order LFFW_GEMM_GROUP selects.
    sys.path.insert(0, str(ROOT))
    fp8_module = importlib.import_module(PACKAGE + ".fp8")
    m_, n_, k_, g_, path = sys.argv[1:6]
    np.save(path, _run(fp8_module, int(m_), int(n_), int(k_), bool(int(g_))))
