"""CPU tests: the oracle against the reference's golden vectors, and host-side logic."""

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from flash_whisper_b200.audio import mel_filters, pad_to_30s, synthetic_audio
from flash_whisper_b200.weights import TURBO, WhisperDims, random_state_dict, sinusoids
from oracle import kernels as K
from oracle import mel as M


def test_mel_filters_match_reference_filterbank():
    ref = np.load(GOLDEN / 'mel_filters.npy')
    assert np.abs(M.mel_filter_bank() - ref).max() < 1e-7
    assert np.abs(mel_filters() - ref).max() < 1e-7


@pytest.mark.parametrize('name,seconds', [('clip30', 30.0), ('clip7', 7.25)])
def test_logmel_oracle_matches_reference_log_mel(name, seconds):
    g = np.load(GOLDEN / 'logmel.npz')
    wave = pad_to_30s(synthetic_audio(0, seconds))
    mine = M.log_mel(wave)
    assert np.abs(mine[:, :160] - g[f'{name}_ref_head']).max() < 1e-4
    assert np.abs(mine[:, :160] - g[f'{name}_hf_head']).max() < 1e-4
    assert np.abs(mine[:, -4:] - g[f'{name}_ref_tail']).max() < 1e-4
    assert abs(mine.sum() - float(g[f'{name}_ref_sum'])) < 1e-6 * mine.size + 1e-3
    assert abs((mine ** 2).sum() - float(g[f'{name}_ref_sumsq'])) / float(g[f'{name}_ref_sumsq']) < 1e-6


def test_logmel_batch_uses_per_clip_max():
    a, b = pad_to_30s(synthetic_audio(1, 3.0)), pad_to_30s(0.01 * synthetic_audio(2, 3.0))
    batch = M.log_mel(np.stack([a, b]))
    assert np.allclose(batch[0], M.log_mel(a)) and np.allclose(batch[1], M.log_mel(b))


def test_synthetic_audio_is_seeded_and_shaped():
    x = synthetic_audio(0)
    assert x.dtype == np.float32 and x.shape == (480000,)
    assert np.array_equal(x, M.synthetic_audio(0))
    assert not np.array_equal(x, synthetic_audio(1))
    assert 0.1 < np.abs(x).max() < 0.6


def test_attention_oracle_matches_reference_attention_ref():
    from golden.make_golden import attention_inputs
    g = np.load(GOLDEN / 'attention.npz')
    q, k, v, kc, vc = attention_inputs()
    assert abs(float(q.double().sum()) - float(g['q_sum'])) < 1e-6
    out, _, _ = K.decode_attention(q.numpy(), k.numpy(), v.numpy(), 64, k[:, 64].numpy(), v[:, 64].numpy())
    assert np.abs(out - g['self_ref']).max() < 1e-5
    out, _, _ = K.decode_attention(q.numpy(), kc.numpy(), vc.numpy())
    assert np.abs(out - g['cross_ref']).max() < 1e-5


def test_attention_oracle_kv_write_is_exact():
    rng = np.random.default_rng(0)
    k = rng.standard_normal((20, 448, 64)).astype(np.float16)
    v = rng.standard_normal((20, 448, 64)).astype(np.float16)
    kn = rng.standard_normal((20, 64)).astype(np.float16)
    vn = rng.standard_normal((20, 64)).astype(np.float16)
    q = rng.standard_normal(1280).astype(np.float16)
    _, k2, v2 = K.decode_attention(q, k, v, 100, kn, vn)
    assert np.array_equal(k2[:, 100], kn) and np.array_equal(v2[:, 100], vn)
    mask = np.ones(448, bool)
    mask[100] = False
    assert np.array_equal(k2[:, mask], k[:, mask]) and np.array_equal(v2[:, mask], v[:, mask])


def test_pack_score_orders_scores_and_breaks_ties_low_index():
    vals = [-3.0, -0.0, 0.0, 1e-30, 2.5, 2.5, float('inf')]
    keys = [int(K.pack_score(v, i)) for i, v in enumerate(vals)]
    assert keys[4] > keys[5]  # tie -> lower index wins
    assert keys[6] == max(keys) and keys[0] == min(keys)
    assert keys[3] > keys[2] and keys[2] > keys[0]
    for i, key in enumerate(keys):
        assert K.unpack_index(key) == i


def test_argmax_first_and_suppress():
    logits = np.array([1, 5, 5, 2], np.float16)
    assert K.argmax_first(logits) == 1
    assert K.argmax_first(logits, [False, True, False, False]) == 2


def test_argmax_finalize_bookkeeping():
    tokens = np.zeros(8, np.int64)
    state = np.array([3, 0], np.int64)
    cur = np.zeros(1, np.int64)
    tok = K.argmax_finalize(int(K.pack_score(1.5, 1234)), tokens, state, cur, 448)
    assert tok == 1234 and tokens[0] == 1234 and state.tolist() == [4, 1] and cur[0] == 1234
    state = np.array([447, 447], np.int64)
    K.argmax_finalize(int(K.pack_score(1.0, 7)), np.zeros(448, np.int64), state, cur, 448)
    assert state.tolist() == [447, 448]
    state = np.array([447, 448], np.int64)
    K.argmax_finalize(int(K.pack_score(1.0, 7)), np.zeros(448, np.int64), state, cur, 448)
    assert state.tolist() == [447, 448]


def test_embed_pos_oracle_is_exact_fp16_sum():
    rng = np.random.default_rng(1)
    e = rng.standard_normal((50, 16)).astype(np.float16)
    p = rng.standard_normal((10, 16)).astype(np.float16)
    out = K.embed_pos(e, p, [3, 7], [0, 9])
    assert np.array_equal(out[0], (e[3].astype(np.float64) + p[0]).astype(np.float16))
    assert np.array_equal(out[1], (e[7].astype(np.float64) + p[9]).astype(np.float16))


def test_add_layernorm_oracle():
    rng = np.random.default_rng(2)
    h = rng.standard_normal(1280).astype(np.float16)
    x = rng.standard_normal(1280).astype(np.float16)
    g = rng.standard_normal(1280).astype(np.float16)
    b = rng.standard_normal(1280).astype(np.float16)
    h2, y = K.add_layernorm(h, x, g, b)
    ref = torch.nn.functional.layer_norm(torch.from_numpy((h + x).astype(np.float32)), (1280,),
                                         torch.from_numpy(g).float(), torch.from_numpy(b).float(), 1e-5)
    assert np.array_equal(h2, (h.astype(np.float32) + x).astype(np.float16))
    assert np.abs(y.astype(np.float32) - ref.numpy()).max() < 2e-2


def test_weights_are_seeded_and_hf_shaped():
    names = {'model.decoder.embed_tokens.weight', 'model.decoder.layers.0.fc1.bias',
             'model.encoder.embed_positions.weight', 'model.decoder.layer_norm.weight'}
    a = random_state_dict(0, TURBO, names=names)
    b = random_state_dict(0, TURBO, names=names)
    assert all(torch.equal(a[n], b[n]) for n in names)
    e = a['model.decoder.embed_tokens.weight']
    assert e.shape == (51866, 1280) and abs(float(e.std()) - 0.02) < 1e-3
    assert float(e[TURBO.pad_token_id].abs().max()) == 0.0
    assert torch.equal(a['model.encoder.embed_positions.weight'], sinusoids(1500, 1280))
    assert float(a['model.decoder.layers.0.fc1.bias'].abs().max()) == 0.0
    assert torch.equal(a['model.decoder.layer_norm.weight'], torch.ones(1280))


def test_numpy_model_matches_transformers_golden():
    from oracle.model_np import WhisperOracle
    g = np.load(GOLDEN / 'hf_small.npz')
    dims = WhisperDims(d_model=256, heads=4, encoder_layers=2, decoder_layers=2, ffn=512)
    sd = random_state_dict(int(g['seed']), dims, bias_std=0.02, ln_std=0.1)
    o = WhisperOracle(sd, dims, fp16=False)
    wave = pad_to_30s(synthetic_audio(int(g['audio_seed']), 5.0))
    enc = o.encoder(M.log_mel(wave).astype(np.float32))
    assert np.abs(enc[::100] - g['enc_rows']).max() < 2e-5
    o.set_cross(enc)
    o.reset()
    for i, t in enumerate(dims.prompt):
        logits = o.step(t, i)
    assert np.abs(logits - g['prompt_logits']).max() < 2e-5
    first = np.isin(np.arange(dims.vocab), dims.begin_suppress)
    tokens, _, _ = o.greedy(8, list(dims.prompt), None, first)
    assert tokens == g['tokens'].tolist()


def test_turbo_golden_tokens_recorded():
    g = json.loads((GOLDEN / 'turbo_tokens.json').read_text())
    assert g['n_tokens'] == 32 and len(g['tokens']) == 32
    assert all(0 <= t < TURBO.vocab for t in g['tokens'])
