"""Batched decode (fw_batch_decoder_step, flash_whisper_b200/batch.py) against decoding each clip
alone with the batch-1 step: every clip's tokens and its whole self-attention cache (the K/V rows every
layer wrote at every position) must be identical bit for bit, for a full batch of 8 clips and a
partial batch, on weights whose greedy output is not degenerate (varied_state_dict)."""

import numpy as np
import pytest
import torch

from flash_whisper_b200.audio import synthetic_audio
from flash_whisper_b200.weights import TURBO, varied_state_dict

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def model(cuda):
    from flash_whisper_b200.model import CustomModel
    return CustomModel(state_dict=varied_state_dict(0, TURBO), dims=TURBO, selftest=False)


@pytest.fixture(scope='module')
def batch(model):
    from flash_whisper_b200.batch import BatchDecoder
    return BatchDecoder(model, clips=8)


def _alone(model, audio, n_tokens):
    """Tokens and self cache of the clip decoded alone (batch-1 path)."""
    out = model.transcribe(audio, max_new_tokens=n_tokens, stop_at_eos=False)
    return out['token_ids'], model.self_kv.clone()


@pytest.mark.parametrize('n_clips,n_tokens', [(8, 40), (3, 75)])
@torch.inference_mode()
def test_batched_tokens_and_caches_equal_batch1(model, batch, n_clips, n_tokens):
    rng = np.random.default_rng(n_clips)
    audios = [synthetic_audio(100 + i, float(rng.uniform(5.0, 30.0))) for i in range(n_clips)]
    for c, a in enumerate(audios):
        model.load_audio(a)
        batch.encode_slot(c)
    batch.decode(n_clips, n_tokens)
    torch.cuda.synchronize()
    got = batch.tokens[:n_clips, :n_tokens].tolist()
    got_kv = batch.self_kv[:n_clips].clone()
    assert model.ext.device_error() == 0
    distinct = set()
    for c, a in enumerate(audios):
        want, kv = _alone(model, a, n_tokens)
        distinct.update(want)
        assert got[c] == want, f'clip {c}: first divergence at ' \
            f'{next(i for i, (x, y) in enumerate(zip(got[c], want)) if x != y)}'
        pos = len(TURBO.prompt) + n_tokens - 1  # positions written: the prompt and every fed-back token
        assert torch.equal(got_kv[c][..., :pos, :], kv[..., :pos, :]), f'clip {c}: self cache differs'
    assert len(distinct) > 10


@torch.inference_mode()
def test_batched_cross_cache_slots_match_encoder(model, batch):
    """encode_slot writes the same cross K/V as the batch-1 front end, into its own slot only."""
    a = synthetic_audio(7, 12.0)
    batch.cross_kv[5].zero_()
    before = batch.cross_kv[4].clone()
    model.load_audio(a)
    batch.encode_slot(5)
    model.run_front()
    torch.cuda.synchronize()
    assert torch.equal(batch.cross_kv[5], model.cross_kv)
    assert torch.equal(batch.cross_kv[4], before)


def test_batched_descriptor_checks(model, batch):
    from flash_whisper_b200 import _lib
    d = _lib.BatchDecoder()
    ctypes_copy = type(d).from_buffer_copy(batch._desc(2))
    ctypes_copy.clips = 9
    with pytest.raises(RuntimeError, match='clips must be 1..8'):
        model.ext.batch_decoder_step(ctypes_copy, 1)
    ctypes_copy.clips = 2
    ctypes_copy.lm_q = None
    with pytest.raises(RuntimeError, match='required pointer'):
        model.ext.batch_decoder_step(ctypes_copy, 1)


@torch.inference_mode()
def test_transcribe_batch_pipeline_equals_transcribe(model):
    """transcribe_batch (three batched decoders on three streams, encoders of the next groups overlapping
    the current decode, a partial last group) returns for every clip what transcribe() returns."""
    rng = np.random.default_rng(11)
    secs = sorted((float(rng.uniform(5.0, 30.0)) for _ in range(11)), reverse=True)
    audios = [synthetic_audio(200 + i, s) for i, s in enumerate(secs)]
    limits = [int(round(7.5 * s)) // 4 for s in secs]
    outs = model.transcribe_batch(audios, max_new_tokens=limits, stop_at_eos=False)
    assert len(outs) == len(audios)
    for i, (a, lim) in enumerate(zip(audios, limits)):
        want = model.transcribe(a, max_new_tokens=lim, stop_at_eos=False)['token_ids']
        assert outs[i]['token_ids'] == want, f'clip {i}'
        assert outs[i]['n_tokens'] == lim
