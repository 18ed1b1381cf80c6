"""The host-side log-mel preparation (audio.py) against the reference's own
python/src/listenflow/fastest_whisper/_audio.py and assets/mel_filters.npz,
loaded from the reference checkout when it is present."""

from __future__ import annotations

import importlib
import importlib.util
import sys
import types

import numpy as np
import pytest

from conftest import PACKAGE, reference_root

_ROOT = reference_root()
_FW = (_ROOT / "python/src/listenflow/fastest_whisper") if _ROOT else None
needs_reference = pytest.mark.skipif(_FW is None or not (_FW / "_audio.py").exists(),
                                     reason="reference checkout not found (set LFFW_REFERENCE_ROOT)")


@pytest.fixture(scope="module")
def audio():
    return importlib.import_module(PACKAGE + ".audio")


@pytest.fixture(scope="module")
def ref_audio():
    # _audio.py and _assets.py only, as members of a stand-in package (the
    # reference package's __init__ needs TensorRT, which is absent).
    pkg = types.ModuleType("lffw_reference_fw")
    pkg.__path__ = [str(_FW)]
    sys.modules["lffw_reference_fw"] = pkg
    for name in ("_assets", "_audio"):
        spec = importlib.util.spec_from_file_location(f"lffw_reference_fw.{name}", _FW / f"{name}.py")
        module = importlib.util.module_from_spec(spec)
        sys.modules[f"lffw_reference_fw.{name}"] = module
        spec.loader.exec_module(module)
    return sys.modules["lffw_reference_fw._audio"]


@needs_reference
@pytest.mark.parametrize("n_mels", [80, 128])
def test_mel_filters_match_reference_asset(audio, n_mels):
    with np.load(_FW / "assets" / "mel_filters.npz") as f:
        expected = f[f"mel_{n_mels}"]
    got = audio.mel_filters(n_mels)
    assert got.shape == expected.shape == (n_mels, 201)
    # float32 rounding of the same formula: within 1e-7 of the largest weight
    np.testing.assert_allclose(got, expected, rtol=0, atol=1e-7 * float(expected.max()) * 10)
    assert ((got > 0) == (expected > 0)).all()


@needs_reference
@pytest.mark.parametrize("samples", [480_000, 100_000, 1])
def test_log_mel_matches_reference(audio, ref_audio, samples):
    pcm = audio.synthetic_pcm(11)[:samples]
    want = ref_audio.log_mel_spectrogram(pcm, n_mels=128)
    with np.load(_FW / "assets" / "mel_filters.npz") as f:
        filters = f["mel_128"]
    np.testing.assert_array_equal(audio.log_mel_spectrogram(pcm, n_mels=128, filters=filters), want)
    np.testing.assert_allclose(audio.log_mel_spectrogram(pcm, n_mels=128), want, rtol=0, atol=2.0**-20)


def test_log_mel_rejects_invalid_audio(audio):
    with pytest.raises(ValueError):
        audio.log_mel_spectrogram(np.zeros(480_001, np.float32), n_mels=128)
    with pytest.raises(ValueError):
        audio.log_mel_spectrogram(np.full(10, np.nan, np.float32), n_mels=128)


def test_synthetic_pcm_is_seeded_and_noisy(audio):
    a, b = audio.synthetic_pcm(5), audio.synthetic_pcm(5)
    np.testing.assert_array_equal(a, b)
    assert a.shape == (480_000,) and a.dtype == np.float32
    assert not np.array_equal(a, audio.synthetic_pcm(6))
    mel = audio.synthetic_mel_batch(2, seed=5)
    assert mel.shape == (2, 128, 3000) and np.isfinite(mel).all()
