"""Audio-side helpers: the Slaney mel filterbank the GPU front end needs, and seeded synthetic clips.

The filterbank is the one WhisperFeatureExtractor(feature_size=128) builds and custom/model.py:38
uploads (transformers audio_utils.mel_filter_bank, norm='slaney', mel_scale='slaney', 0-8000 Hz,
201 FFT bins): triangles on the Slaney mel scale (linear below 1 kHz, logarithmic above), each scaled
to unit area (2 / bandwidth in Hz).

No speech data is available offline, so benchmark and parity inputs are synthetic: 5 sinusoids with
frequencies U[100, 4000] Hz, random phases and amplitude 0.1 each, plus Gaussian noise with standard
deviation 0.01, from numpy.random.default_rng(seed).
"""

import numpy as np

SAMPLE_RATE = 16000
N_SAMPLES = 30 * SAMPLE_RATE
N_FFT, HOP, N_MELS = 400, 160, 128


def _hz_to_mel(f):
    f = np.asarray(f, np.float64)
    lin = 3.0 * f / 200.0
    return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-30) / 1000.0) * 27.0 / np.log(6.4), lin)


def _mel_to_hz(m):
    m = np.asarray(m, np.float64)
    return np.where(m >= 15.0, 1000.0 * np.exp((m - 15.0) * np.log(6.4) / 27.0), 200.0 * m / 3.0)


def mel_filters(n_mels=N_MELS, n_fft=N_FFT, sr=SAMPLE_RATE, f_max=8000.0):
    """[n_fft // 2 + 1, n_mels] float32 Slaney filterbank."""
    edges_hz = _mel_to_hz(np.linspace(_hz_to_mel(0.0), _hz_to_mel(f_max), n_mels + 2))
    bins_hz = np.linspace(0, sr // 2, n_fft // 2 + 1)
    lower = (bins_hz[:, None] - edges_hz[None, :-2]) / (edges_hz[1:-1] - edges_hz[:-2])[None, :]
    upper = (edges_hz[None, 2:] - bins_hz[:, None]) / (edges_hz[2:] - edges_hz[1:-1])[None, :]
    tri = np.clip(np.minimum(lower, upper), 0.0, None)
    return (tri * (2.0 / (edges_hz[2:] - edges_hz[:-2]))[None, :]).astype(np.float32)


def synthetic_audio(seed, seconds=30.0, sr=SAMPLE_RATE):
    """Seeded synthetic clip: 5 sinusoids (amp 0.1, f ~ U[100, 4000] Hz) + N(0, 0.01^2) noise, fp32."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * sr))
    t = np.arange(n) / sr
    freqs = rng.uniform(100.0, 4000.0, size=5)
    phases = rng.uniform(0.0, 2 * np.pi, size=5)
    x = np.zeros(n)
    for f, p in zip(freqs, phases):
        x += 0.1 * np.sin(2 * np.pi * f * t + p)
    x += rng.normal(0.0, 0.01, size=n)
    return x.astype(np.float32)


def pad_to_30s(audio):
    """Zero-pads a 1-D clip to 480000 samples (custom/model.py:182-183)."""
    out = np.zeros(N_SAMPLES, np.float32)
    out[:audio.size] = audio
    return out
