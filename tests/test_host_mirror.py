"""The Python host mirror of the reference's FP8 graph API and its scale file
(python/src/listenflow/fastest_whisper/_fp8.py, _assets.py), without a GPU."""

from __future__ import annotations

import importlib
import json
import math
from pathlib import Path

import pytest

from conftest import PACKAGE, reference_root

_ROOT = reference_root()
REFERENCE_SCALES = (_ROOT / "python/src/listenflow/fastest_whisper/assets/fp8-scales.json") if _ROOT else None


@pytest.fixture(scope="module")
def scales_mod(lffw):
    return importlib.import_module(PACKAGE + ".scales")


@pytest.mark.parametrize("invalid", [0, -0.1, float("nan"), float("inf"), None, "x"])
def test_fp8_graph_rejects_invalid_or_missing_scale_before_quantizing(fp8, invalid):
    # python/tests/test_fp8_graph.py:306-317: the error names the key, and no
    # weight is read or quantized first (the checkpoint here would raise).
    key = "model.decoder.layers.0.fc1"

    class Untouchable(dict):
        def __getitem__(self, item):
            raise AssertionError("weights must not be read before the scale is validated")

    for scales in ({}, {key: invalid}):
        graph = fp8.Fp8Graph(Untouchable(), scales)
        with pytest.raises(ValueError, match=key):
            graph.linear(None, key)
        with pytest.raises(ValueError, match=key):
            graph.decoder_fc1(None, key)


def test_read_fp8_scales(scales_mod, tmp_path):
    path = tmp_path / "scales.json"
    path.write_text(json.dumps({"a": 0.125}))
    assert scales_mod.read_fp8_scales(path) == {"a": 0.125}
    for bad in (None, [], 3):
        path.write_text(json.dumps(bad))
        with pytest.raises(ValueError, match="scales"):
            scales_mod.read_fp8_scales(path)


def test_calibration_rule_and_keys(scales_mod):
    assert scales_mod.scale_from_amax(0.0) == 1.0
    # python/tests/test_fp8_product.py:90-103: three pinned layer maxima / 448.
    for amax in (22.02214813232422, 12.829965591430664, 1.898099422454834):
        assert scales_mod.scale_from_amax(amax) == pytest.approx(amax / 448, rel=1e-12)
    keys = scales_mod.linear_keys()
    assert len(keys) == 512
    assert "model.decoder.layers.31.encoder_attn.v_proj" in keys
    with pytest.raises(ValueError, match="model.encoder.layers.0.fc1"):
        scales_mod.validate({}, {"model.encoder.layers.0.fc1"})


@pytest.mark.skipif(REFERENCE_SCALES is None or not REFERENCE_SCALES.exists(),
                    reason="reference checkout not found (set LFFW_REFERENCE_ROOT)")
def test_reference_scale_file_supports_fused_projections(scales_mod):
    scales = scales_mod.read_fp8_scales(REFERENCE_SCALES)
    assert set(scales) == scales_mod.linear_keys()
    assert all(math.isfinite(v) and v > 0 for v in scales.values())
    # q/k/v of one self-attention share their input, hence one activation
    # scale: a fused QKV GEMM (N = 3 * 1280) is exactly the three Q/DQ linears.
    for part in ("encoder", "decoder"):
        for layer in range(32):
            root = f"model.{part}.layers.{layer}.self_attn"
            assert scales[f"{root}.q_proj"] == scales[f"{root}.k_proj"] == scales[f"{root}.v_proj"]
    cross = {scales[f"model.decoder.layers.{i}.encoder_attn.{p}_proj"] for i in range(32) for p in "kv"}
    assert len(cross) == 1  # all 64 cross K/V projections read the encoder output
