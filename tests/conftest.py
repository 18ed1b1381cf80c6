"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and run on a B200 with
``pytest -m gpu``; everything else runs on a CPU-only host."""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PACKAGE = "listenflow-fastest-whisper_b200"


def reference_root() -> Path | None:
    """The reference checkout: $LFFW_REFERENCE_ROOT, else a directory named
    ``reference`` beside this repository; None when neither exists (tests that
    read the reference's own files then skip)."""
    import os

    env = os.environ.get("LFFW_REFERENCE_ROOT")
    candidate = Path(env) if env else ROOT.parent / "reference"
    return candidate if (candidate / "python").is_dir() else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def lffw():
    return importlib.import_module(PACKAGE)


@pytest.fixture(scope="session")
def fp8(lffw):
    return importlib.import_module(PACKAGE + ".fp8")


@pytest.fixture(scope="session")
def native(lffw):
    return importlib.import_module(PACKAGE + "._native")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda:0")
