"""Regenerate the committed golden fixtures.

    python tests/golden/make_golden.py

e4m3_edges.json   E4M3 known answers: the format's own edge cases (OCP FP8
                  e4m3fn: max finite 448, min normal 2^-6, min subnormal 2^-9,
                  round to nearest even, saturation as TensorRT's Q clamps),
                  written by hand below, not computed by the oracle.
fp16_plugins.npz  The reference's own seeded fp16-plugin test data and expected
                  outputs (cpp/tests/kernel_reference.hpp: mt19937(3318), x ~ N(0,1),
                  W ~ N(0,1)/sqrt(1280), bias ~ U(-.5,.5)), produced by compiling
                  that header where it lies in the reference tree (oracle/_ref,
                  `make -C oracle`).  Only the first ROWS weight rows are kept.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
ROWS = 32


def f16(bits: int) -> float:
    return float(np.array([bits], np.uint16).view(np.float16)[0])


# (fp16 input bits, fp32 scale, expected E4M3 code, why).  E4M3 codes are
# S.EEEE.MMM with bias 7; exponent 0 holds subnormals m * 2^-9.
EDGES = [
    (0x0000, 1.0, 0x00, "+0"),
    (0x8000, 1.0, 0x80, "-0 keeps its sign"),
    (0x1400, 1.0, 0x00, "2^-10, half the smallest subnormal: tie to even -> 0"),
    (0x9400, 1.0, 0x80, "-2^-10: tie to even -> -0"),
    (0x1800, 1.0, 0x01, "2^-9: smallest subnormal"),
    (0x1A00, 1.0, 0x02, "3*2^-10: tie between 1*2^-9 (odd) and 2*2^-9 (even) -> 2^-8"),
    (0x1C00, 1.0, 0x02, "2^-8 = 2*2^-9"),
    (0x1E00, 1.0, 0x03, "3*2^-9"),
    (0x2300, 1.0, 0x07, "7*2^-9: largest subnormal"),
    (0x2380, 1.0, 0x08, "7.5*2^-9: tie between 7*2^-9 (odd) and 2^-6 (even) -> 2^-6"),
    (0x2400, 1.0, 0x08, "2^-6: smallest normal"),
    (0x3C00, 1.0, 0x38, "1.0"),
    (0x3C40, 1.0, 0x38, "1.0625: tie between 1.0 (even) and 1.125 (odd) -> 1.0"),
    (0x3C80, 1.0, 0x39, "1.125 = 1 + 1/8"),
    (0x3CC0, 1.0, 0x3A, "1.1875: tie between 1.125 (odd) and 1.25 (even) -> 1.25"),
    (0xBC00, 1.0, 0xB8, "-1.0"),
    (0x5F00, 1.0, 0x7E, "448: largest finite"),
    (0x5F40, 1.0, 0x7E, "464: tie between 448 (even) and 480 (not finite) -> 448"),
    (0x5F80, 1.0, 0x7E, "480: beyond the range, saturates to 448 (torch's cast gives NaN)"),
    (0xDF80, 1.0, 0xFE, "-480: saturates to -448"),
    (0x7BFF, 1.0, 0x7E, "65504 (fp16 max): saturates"),
    (0x7BFF, 2.0**-10, 0x7E, "65504 with a tiny scale: saturates"),
    (0x7C00, 1.0, 0x7E, "+inf: saturates to 448"),
    (0xFC00, 1.0, 0xFE, "-inf: saturates to -448"),
    (0x3C00, 1.0 / 448.0, 0x7E, "1 / fp32(1/448): the fp32 quotient is 448 to within an ulp"),
    (0x3800, 0.125, 0x48, "0.5 / 0.125 = 4 = 1.0 * 2^2"),
]


def fix_edges():
    out = []
    for bits, scale, code, why in EDGES:
        s, e, m = code >> 7, (code >> 3) & 15, code & 7
        value = (m / 8.0) * 2.0**-6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
        out.append({"x_bits": bits, "x": f16(bits), "scale": scale, "code": code, "why": why,
                    "code_value": -value if s else value})
    return out


def main() -> None:
    edges = fix_edges()
    (HERE / "e4m3_edges.json").write_text(json.dumps(edges, indent=1) + "\n")
    from oracle import oracle

    if not oracle.reference_available():
        raise SystemExit("oracle/_ref not built (reference tree not mounted): fp16_plugins.npz unchanged")
    arrays = {}
    for name, fc1 in (("fc1", True), ("qkv", False)):
        x, w, b, vb, expected = oracle.reference_projection(fc1)
        arrays[f"{name}_x"] = x
        arrays[f"{name}_w"] = w[:ROWS]
        arrays[f"{name}_bias"] = b if not fc1 else b[:ROWS]
        if vb is not None:
            arrays[f"{name}_v_bias"] = vb
        arrays[f"{name}_expected"] = expected
        arrays[f"{name}_expected_rows"] = np.array([ROWS])
    # The reference's fp16-edge GELU on a grid of (dot, bias) pairs.
    rng = np.random.default_rng(5)
    dots = rng.standard_normal(4096) * 3
    biases = rng.uniform(-0.5, 0.5, 4096)
    arrays["gelu_dot"] = dots
    arrays["gelu_bias"] = biases
    arrays["gelu_expected"] = np.array([oracle.reference_gelu(d, b) for d, b in zip(dots, biases)])
    np.savez_compressed(HERE / "fp16_plugins.npz", **arrays)
    print("wrote", HERE / "e4m3_edges.json", HERE / "fp16_plugins.npz")


if __name__ == "__main__":
    main()
