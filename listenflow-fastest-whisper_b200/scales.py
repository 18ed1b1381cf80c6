"""FP8 activation-scale mapping, as shipped by the reference.

``read_fp8_scales`` restates python/src/listenflow/fastest_whisper/_assets.py:11-16:
the file is a JSON object mapping a linear's key (e.g.
``model.encoder.layers.0.fc1``) to its static activation scale, the calibrated
input amax/448 (python/scripts/calibrate_fp8.py:384-385; zero maximum -> 1).
"""

from __future__ import annotations

import json
import math
from pathlib import Path

E4M3_MAX = 448.0


def read_fp8_scales(path: Path | str) -> dict[str, float]:
    """Read the calibration mapping before handing model inputs to native code."""
    values = json.loads(Path(path).read_text())
    if not isinstance(values, dict):
        raise ValueError("FP8 scales must be a mapping of layer names to values")
    return values


def scale_from_amax(amax: float) -> float:
    """The calibration rule: observed absolute maximum / 448; a zero maximum uses 1."""
    return amax / E4M3_MAX if amax else 1.0


def linear_keys(layers: int = 32) -> set[str]:
    """All 512 large-v3 linear inputs that carry an activation scale."""
    keys = set()
    for part in ("encoder", "decoder"):
        for layer in range(layers):
            ops = ["fc1", "fc2"] + [f"self_attn.{p}_proj" for p in ("q", "k", "v", "out")]
            if part == "decoder":
                ops += [f"encoder_attn.{p}_proj" for p in ("q", "k", "v", "out")]
            keys.update(f"model.{part}.layers.{layer}.{op}" for op in ops)
    return keys


def validate(scales: dict[str, float], keys: set[str]) -> None:
    """Every required key present with a finite positive value (network_graph.cpp:137-139)."""
    for key in sorted(keys):
        value = scales.get(key)
        if value is None or not isinstance(value, (int, float)) or not math.isfinite(value) or value <= 0:
            raise ValueError(f"missing or invalid activation scale for {key}")
