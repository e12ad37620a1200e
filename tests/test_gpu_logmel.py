"""GPU parity of the log-mel front end against the numpy oracle (itself pinned to the reference's
_log_mel and the HF feature extractor): fp32 in, fp16 out, within 1e-2 relative / 1e-3 absolute."""

import numpy as np
import pytest
import torch

from flash_whisper_b200.audio import mel_filters, pad_to_30s, synthetic_audio
from oracle.mel import log_mel

pytestmark = pytest.mark.gpu


def _run(ext, waves, layout):
    b = waves.shape[0]
    wave = torch.from_numpy(waves).cuda()
    filt = torch.from_numpy(mel_filters()).cuda()
    scratch = torch.empty(b * 128 * 3000, device='cuda')
    cmax = torch.zeros(b, dtype=torch.int32, device='cuda')
    shape = (b, 128, 3000) if layout == 0 else (b, 3002, 128)
    out = torch.full(shape, 7.0, dtype=torch.float16, device='cuda')
    ext.log_mel(wave, filt, scratch, cmax, out, layout)
    return out.float().cpu().numpy()


@pytest.mark.parametrize('seconds', [30.0, 7.25, 0.5])
def test_log_mel_batch1_vs_oracle(ext, seconds):
    wave = pad_to_30s(synthetic_audio(0, seconds))
    ref = log_mel(wave)
    out = _run(ext, wave[None], 0)[0]
    np.testing.assert_allclose(out, ref, rtol=1e-2, atol=1e-3)
    tm = _run(ext, wave[None], 1)[0]
    assert np.all(tm[0] == 0) and np.all(tm[-1] == 0)
    np.testing.assert_allclose(tm[1:-1].T, ref, rtol=1e-2, atol=1e-3)


def test_log_mel_batch32_per_clip_max(ext):
    waves = np.stack([pad_to_30s(synthetic_audio(s, 30.0) * (0.5 + s / 16)) for s in range(32)])
    out = _run(ext, waves, 0)
    for i in (0, 7, 31):
        np.testing.assert_allclose(out[i], log_mel(waves[i]), rtol=1e-2, atol=1e-3)


def test_log_mel_silence_and_impulse(ext):
    wave = np.zeros((2, 480000), np.float32)
    wave[1, 12345] = 1.0
    out = _run(ext, wave, 0)
    np.testing.assert_allclose(out[0], log_mel(wave[0]), rtol=1e-2, atol=1e-3)
    np.testing.assert_allclose(out[1], log_mel(wave[1]), rtol=1e-2, atol=1e-3)
