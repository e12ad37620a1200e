"""The on-device decode loop (fw_decode_loop_*: a CUDA graph whose WHILE node runs decode steps and
evaluates the stop condition on the GPU), which replaces the host loop of custom/model.py:208-215.

It must produce exactly the tokens of the chunked host loop, stop after exactly `limit` tokens, and
stop right after the first occurrence of the EOS id (here a token id taken from the clip's own output,
so the stop is exercised without changing the weights). The chunked variant (the stop checked every 8
steps, as transcribe(stop_at_eos=True) runs it) must give the same tokens up to the stop."""

import pytest
import torch

from flash_whisper_b200.audio import synthetic_audio
from flash_whisper_b200.weights import TURBO, varied_state_dict

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def model(cuda):
    from flash_whisper_b200.model import CustomModel
    m = CustomModel(state_dict=varied_state_dict(0, TURBO), dims=TURBO, selftest=False)
    assert m.loop is not None, m.selftest.get('decode_loop_error')
    return m


@torch.inference_mode()
def _loop(model, audio, limit, stop, eos=None, chunked=False):
    model.load_audio(audio)
    model.run_front()
    model.run_prompt()
    model.run_loop(limit, stop, eos, chunked=chunked)
    torch.cuda.synchronize()
    n = int(model.state[1])
    return n, model.tokens[:n].tolist(), int(model.loop_ctrl[3])


@torch.inference_mode()
def test_loop_matches_host_loop_and_limit(model):
    audio = synthetic_audio(6, 20.0)
    full = model.transcribe(audio, max_new_tokens=60, stop_at_eos=False)['token_ids']
    assert len(set(full)) > 10
    for limit in (1, 2, 37, 60):
        n, toks, iters = _loop(model, audio, limit, False)
        assert n == limit and toks == full[:limit], limit
        assert iters == max(0, limit - 1)  # one body iteration (one step) per token after the first


@torch.inference_mode()
def test_loop_stops_after_first_eos(model):
    audio = synthetic_audio(6, 20.0)
    full = model.transcribe(audio, max_new_tokens=60, stop_at_eos=False)['token_ids']
    k = next(i for i in range(3, len(full)) if full[i] not in full[:i])
    n, toks, _ = _loop(model, audio, 60, True, eos=full[k])
    assert n == k + 1 and toks == full[:k + 1]
    # a stop token that is already the first token (from the prompt) ends the loop before any step
    n, toks, _ = _loop(model, audio, 60, True, eos=full[0])
    assert n == 1 and toks == full[:1]


@torch.inference_mode()
def test_chunked_loop_keeps_tokens_and_stops_within_a_chunk(model):
    """The loop transcribe(stop_at_eos=True) uses checks the stop every `chunk` steps (EOS among all the
    tokens of the chunk): the tokens up to the limit or the first EOS are the exact loop's, and it
    decodes fewer than `chunk` tokens past them."""
    assert model.loop_chunk is not None
    audio = synthetic_audio(6, 20.0)
    full = model.transcribe(audio, max_new_tokens=60, stop_at_eos=False)['token_ids']
    c = model.chunk
    for limit in (1, 2, 37, 60):
        n, toks, _ = _loop(model, audio, limit, False, chunked=True)
        assert limit <= n < limit + c and toks[:limit] == full[:limit], limit
    k = next(i for i in range(3, len(full)) if full[i] not in full[:i])
    n, toks, _ = _loop(model, audio, 60, True, eos=full[k], chunked=True)
    assert k + 1 <= n < k + 1 + c and toks[:k + 1] == full[:k + 1]
    n, toks, _ = _loop(model, audio, 60, True, eos=full[0], chunked=True)
    assert n == 1 and toks == full[:1]


@torch.inference_mode()
def test_transcribe_stop_at_eos_uses_loop(model):
    audio = synthetic_audio(8, 15.0)
    full = model.transcribe(audio, max_new_tokens=50, stop_at_eos=False)['token_ids']
    out = model.transcribe(audio, max_new_tokens=50, stop_at_eos=True)
    if TURBO.eos_token_id in full:
        assert out['token_ids'] == full[:full.index(TURBO.eos_token_id) + 1]
    else:
        assert out['token_ids'] == full
    assert out['ttft_s'] <= out['ttlt_s']
