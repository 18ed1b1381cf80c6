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
