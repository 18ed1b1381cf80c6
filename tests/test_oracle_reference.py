"""The oracle against the reference's own CPU model of its fp16 plugins
(cpp/tests/kernel_reference.hpp), via the committed golden fixture and, where
the reference tree is mounted, the full compiled model (oracle/_ref)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = np.load(Path(__file__).parent / "golden" / "fp16_plugins.npz")


def expected_bits(values: np.ndarray) -> np.ndarray:
    # kernel_reference.hpp returns doubles that are already fp16 values.
    return values.astype(np.float16).view(np.uint16)


def test_fc1_rows_match_reference_golden(oracle):
    rows = int(GOLDEN["fc1_expected_rows"][0])
    got = oracle.fp16_fc1(GOLDEN["fc1_x"], GOLDEN["fc1_w"], GOLDEN["fc1_bias"])
    np.testing.assert_array_equal(got, expected_bits(GOLDEN["fc1_expected"][:rows]))


def test_qkv_rows_match_reference_golden(oracle):
    rows = int(GOLDEN["qkv_expected_rows"][0])
    width = GOLDEN["qkv_x"].size
    w = np.zeros((3 * width, width), np.uint16)
    w[:rows] = GOLDEN["qkv_w"]
    got = oracle.fp16_qkv(GOLDEN["qkv_x"], w, GOLDEN["qkv_bias"], GOLDEN["qkv_v_bias"])
    np.testing.assert_array_equal(got[:rows], expected_bits(GOLDEN["qkv_expected"][:rows]))


def test_gelu_edges_match_reference(oracle):
    dot, bias, want = GOLDEN["gelu_dot"], GOLDEN["gelu_bias"], GOLDEN["gelu_expected"]
    # kernel_reference.hpp:20-25: x = half(half(dot) + bias), then the GELU edges.
    x = oracle.half_from_double(
        oracle.halves(oracle.half_from_double(dot)).astype(np.float64) + bias)
    np.testing.assert_array_equal(oracle.gelu_fp16(x), expected_bits(want))


@pytest.mark.skipif(not __import__("oracle.oracle", fromlist=["x"]).reference_available(),
                    reason="reference tree not mounted (oracle/_ref not built)")
@pytest.mark.parametrize("fc1", [True, False])
def test_full_projection_matches_compiled_reference(oracle, fc1):
    x, w, b, vb, expected = oracle.reference_projection(fc1)
    got = oracle.fp16_fc1(x, w, b) if fc1 else oracle.fp16_qkv(x, w, b, vb)
    np.testing.assert_array_equal(got, expected_bits(expected))


def test_erf_table_matches_oracle(oracle):
    import importlib.util

    path = Path(__file__).parents[1] / "listenflow-fastest-whisper_b200" / "csrc" / "gen_erf_table.py"
    spec = importlib.util.spec_from_file_location("gen_erf_table", path)
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    table = gen.values()
    x = np.arange(gen.LO, gen.HI + 1, dtype=np.uint16)
    np.testing.assert_array_equal(table, oracle.erf_fp16(x))
    assert table[-1] == 0x3C00
    # Above the table erf rounds to 1.0; the committed .inc is the generator's output.
    above = np.arange(gen.HI, 0x7C01, dtype=np.uint16)
    assert np.all(oracle.erf_fp16(above) == 0x3C00)
    assert (path.with_name("erf_table.inc")).read_text() == gen.render()


@pytest.mark.parametrize("fc1", [True, False])
def test_kernel_order_projection_within_reference_tolerance(oracle, fc1):
    """The oracle's restatement of the reference kernel's fp32 summation order
    (cpp/kernels.cu:27-49) meets the reference's own GPU tolerance against its
    CPU model's expected rows (cpp/tests/kernel_gpu.cpp:95-202: atol 2^-11 for
    fc1, 2^-12 for qkv, plus 2^-10 relative)."""
    name = "fc1" if fc1 else "qkv"
    rows = int(GOLDEN[f"{name}_expected_rows"][0])
    x = GOLDEN[f"{name}_x"]
    if fc1:
        got = oracle.fp16_fc1_kernel_order(x, GOLDEN["fc1_w"], GOLDEN["fc1_bias"])[:rows]
    else:
        w = np.zeros((3 * x.size, x.size), np.uint16)
        w[:rows] = GOLDEN["qkv_w"]
        got = oracle.fp16_qkv_kernel_order(x, w, GOLDEN["qkv_bias"], GOLDEN["qkv_v_bias"])[:rows]
    want = GOLDEN[f"{name}_expected"][:rows].astype(np.float64)
    err = np.abs(got.view(np.float16).astype(np.float64) - want)
    atol = 2.0**-11 if fc1 else 2.0**-12
    assert np.all(err <= atol + 2.0**-10 * np.abs(want))


def test_kernel_order_sums_small_cases(oracle):
    """Hand-checked cases of the kernel order.  A single nonzero column is exact.
    Then, with DEPTH 256 (V = 8), lane 0 holds columns 0-3 and 128-131, lane 1
    columns 4-7 and lane 2 columns 8-11: products 2^-24 at columns 0 and 128 fold
    first into 2^-23, shfl_down adds lane 2's 2^-11 and then lane 1's 1.0, so the
    fp32 sum is exactly 1 + 2^-11 + 2^-23 and rounds up to 1 + 2^-10 in fp16.  A
    left-to-right fp32 sum would absorb each 2^-24 and land on the tie 1 + 2^-11,
    which rounds to 1.0."""
    width = 256
    zeros = np.zeros(width, np.float16)
    x = np.zeros(width, np.float16)
    w = np.zeros((3 * width, width), np.float16)
    x[5] = 3.0
    w[:, 5] = 0.5
    assert np.all(oracle.fp16_qkv_kernel_order(x, w, zeros, zeros).view(np.float16) == np.float16(1.5))
    x = np.zeros(width, np.float16)
    w = np.zeros((3 * width, width), np.float16)
    x[0] = x[128] = 2.0**-12
    w[:, 0] = w[:, 128] = 2.0**-12
    x[4], w[:, 4] = 1.0, 1.0
    x[8], w[:, 8] = 2.0**-11, 1.0
    got = oracle.fp16_qkv_kernel_order(x, w, zeros, zeros).view(np.float16)
    assert np.all(got == np.float16(1.0 + 2.0**-10))
