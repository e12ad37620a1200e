"""numpy restatement of the log-mel front end (test infrastructure).

custom/model.py:93-98 computes, on the GPU with torch:
    stft = torch.stft(wave, n_fft=400, hop=160, window=hann(400, periodic), center=True, reflect)
    mel  = clamp(filters.T @ |stft[..., :-1]|^2, min=1e-10).log10()
    mel  = maximum(mel, mel.max() - 8);  out = (mel + 4) / 4
which is WhisperFeatureExtractor._torch_extract_fbank_features (transformers
feature_extraction_whisper.py, per-clip max for a batch). The filterbank is
WhisperFeatureExtractor(feature_size=128).mel_filters: transformers audio_utils.mel_filter_bank with
Slaney mel scale and Slaney area normalisation (the librosa 'slaney' filterbank), restated below.
"""

import numpy as np

N_FFT, HOP, SAMPLE_RATE = 400, 160, 16000


def _hz_to_mel(f):
    f = np.asarray(f, np.float64)
    mel = 3.0 * f / 200.0
    log_region = f >= 1000.0
    return np.where(log_region, 15.0 + np.log(np.maximum(f, 1e-30) / 1000.0) * (27.0 / np.log(6.4)), mel)


def _mel_to_hz(m):
    m = np.asarray(m, np.float64)
    f = 200.0 * m / 3.0
    return np.where(m >= 15.0, 1000.0 * np.exp(np.log(6.4) / 27.0 * (m - 15.0)), f)


def mel_filter_bank(n_freqs=N_FFT // 2 + 1, n_mels=128, f_min=0.0, f_max=8000.0, sr=SAMPLE_RATE):
    """[n_freqs, n_mels] triangular filters on the Slaney mel scale, Slaney-normalised (float64)."""
    mel_pts = np.linspace(_hz_to_mel(f_min), _hz_to_mel(f_max), n_mels + 2)
    hz_pts = _mel_to_hz(mel_pts)
    fft_freqs = np.linspace(0, sr // 2, n_freqs)
    diff = np.diff(hz_pts)
    slopes = hz_pts[None, :] - fft_freqs[:, None]
    down = -slopes[:, :-2] / diff[:-1]
    up = slopes[:, 2:] / diff[1:]
    fb = np.maximum(0.0, np.minimum(down, up))
    return fb * (2.0 / (hz_pts[2:n_mels + 2] - hz_pts[:n_mels]))[None, :]


def log_mel(wave, filters=None, n_fft=N_FFT, hop=HOP):
    """Log-mel of one clip or a batch [b, n] (float64 math); returns float64 [.., n_mels, n // hop]."""
    wave = np.asarray(wave, np.float64)
    if wave.ndim == 2:
        return np.stack([log_mel(w, filters, n_fft, hop) for w in wave])
    if filters is None:
        filters = mel_filter_bank()
    pad = n_fft // 2
    x = np.pad(wave, (pad, pad), mode='reflect')
    n_frames = 1 + (x.size - n_fft) // hop
    idx = np.arange(n_fft)[None, :] + hop * np.arange(n_frames)[:, None]
    window = 0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(n_fft) / n_fft)
    spec = np.fft.rfft(x[idx] * window[None, :], axis=-1)[:-1]
    power = spec.real ** 2 + spec.imag ** 2
    mel = np.clip(power @ filters, 1e-10, None).T
    logm = np.log10(mel)
    logm = np.maximum(logm, logm.max() - 8.0)
    return (logm + 4.0) / 4.0


def synthetic_audio(seed, seconds=30.0, sr=SAMPLE_RATE):
    """Same generator as flash_whisper_b200.audio.synthetic_audio (restated so the oracle stands alone)."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * sr))
    t = np.arange(n) / sr
    freqs = rng.uniform(100.0, 4000.0, size=5)
    phases = rng.uniform(0.0, 2 * np.pi, size=5)
    x = sum(0.1 * np.sin(2 * np.pi * f * t + p) for f, p in zip(freqs, phases))
    x = x + rng.normal(0.0, 0.01, size=n)
    return x.astype(np.float32)
