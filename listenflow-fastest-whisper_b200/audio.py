"""Host-side audio preparation: the 30-second log-mel input of the encoder.

``log_mel_spectrogram`` restates python/src/listenflow/fastest_whisper/_audio.py:12-30
(reflect-padded 400-sample Hann frames every 160 samples, power spectrum, mel
filterbank, log10 clamped at 1e-10, an 8-decade floor below the maximum, then
(x + 4) / 4).  ``mel_filters`` computes the filterbank the reference ships as
assets/mel_filters.npz from its published definition: Slaney's mel scale
(linear below 1 kHz at 200/3 Hz per mel, logarithmic above with 27 steps per
factor 6.4) and triangular filters normalised to unit area per mel band
("slaney" normalisation), over the 201 bins of a 400-point FFT at 16 kHz.

``synthetic_pcm`` is the benchmark's seeded stand-in for speech: three
sinusoids at U(100, 4000) Hz plus white noise 20 dB below the tone power.
"""

from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16_000
N_SAMPLES = 480_000  # 30 s
FFT_SIZE = 400
HOP_SIZE = 160
N_FRAMES = N_SAMPLES // HOP_SIZE  # 3000


def _hz_to_mel(f):
    f = np.asarray(f, np.float64)
    f_sp = 200.0 / 3
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    mel = f / f_sp
    return np.where(f >= min_log_hz, min_log_mel + np.log(np.maximum(f, min_log_hz) / min_log_hz) / logstep, mel)


def _mel_to_hz(m):
    m = np.asarray(m, np.float64)
    f_sp = 200.0 / 3
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), f_sp * m)


def mel_filters(n_mels: int, sample_rate: int = SAMPLE_RATE, n_fft: int = FFT_SIZE) -> np.ndarray:
    """float32 [n_mels, n_fft // 2 + 1] Slaney-scale, Slaney-normalised triangular filters
    spanning 0 Hz to the Nyquist frequency."""
    bins = np.linspace(0.0, sample_rate / 2.0, n_fft // 2 + 1)
    edges = _mel_to_hz(np.linspace(_hz_to_mel(0.0), _hz_to_mel(sample_rate / 2.0), n_mels + 2))
    widths = np.diff(edges)
    offsets = edges[:, None] - bins[None, :]
    weights = np.zeros((n_mels, bins.size))
    for i in range(n_mels):
        rising = -offsets[i] / widths[i]
        falling = offsets[i + 2] / widths[i + 1]
        weights[i] = np.maximum(0.0, np.minimum(rising, falling))
    weights *= (2.0 / (edges[2:n_mels + 2] - edges[:n_mels]))[:, None]
    return weights.astype(np.float32)


_FILTER_CACHE: dict[int, np.ndarray] = {}


def log_mel_spectrogram(audio: np.ndarray, *, n_mels: int, filters: np.ndarray | None = None) -> np.ndarray:
    """fp32 [n_mels, 3000] log-mel of at most 30 s of 16 kHz mono audio (_audio.py:12-30)."""
    samples = np.asarray(audio, dtype=np.float32)
    if samples.ndim != 1 or samples.size > N_SAMPLES or not np.isfinite(samples).all():
        raise ValueError("audio must be a finite mono waveform of at most 30 seconds")
    if filters is None:
        filters = _FILTER_CACHE.setdefault(n_mels, mel_filters(n_mels))
    samples = np.pad(samples, (0, N_SAMPLES - samples.size))
    centered = np.pad(samples, (FFT_SIZE // 2, FFT_SIZE // 2), mode="reflect")
    frames = np.lib.stride_tricks.sliding_window_view(centered, FFT_SIZE)[::HOP_SIZE]
    window = np.hanning(FFT_SIZE + 1)[:-1].astype(np.float32)
    spectrum = np.fft.rfft(frames * window, axis=-1)[:-1].astype(np.complex64)
    power = (spectrum.real**2 + spectrum.imag**2).T
    mel = filters @ power
    log_mel = np.log10(np.maximum(mel, np.float32(1e-10)))
    log_mel = np.maximum(log_mel, log_mel.max() - np.float32(8.0))
    return ((log_mel + np.float32(4.0)) / np.float32(4.0)).astype(np.float32)


def synthetic_pcm(seed: int, samples: int = N_SAMPLES) -> np.ndarray:
    """fp32 mono 16 kHz: three sinusoids at U(100, 4000) Hz with random phases and
    amplitudes U(0.05, 0.3), plus white noise at -20 dB relative to their power."""
    rng = np.random.default_rng(seed)
    t = np.arange(samples, dtype=np.float64) / SAMPLE_RATE
    freqs = rng.uniform(100.0, 4000.0, 3)
    phases = rng.uniform(0.0, 2 * np.pi, 3)
    amps = rng.uniform(0.05, 0.3, 3)
    tone = (amps[:, None] * np.sin(2 * np.pi * freqs[:, None] * t[None, :] + phases[:, None])).sum(axis=0)
    noise_std = np.sqrt(np.mean(tone**2) * 10.0 ** (-20.0 / 10.0))
    return (tone + rng.standard_normal(samples) * noise_std).astype(np.float32)


def synthetic_mel_batch(streams: int, seed: int = 0, n_mels: int = 128) -> np.ndarray:
    """fp32 [streams, n_mels, 3000]: the log-mel of synthetic_pcm(seed + s) per stream."""
    return np.stack([log_mel_spectrogram(synthetic_pcm(seed + s), n_mels=n_mels) for s in range(streams)])
