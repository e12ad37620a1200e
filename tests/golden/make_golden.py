"""Generates the golden fixtures in tests/golden/ from the reference's own code (run in the build
container, where the read-only reference checkout and transformers are importable).

    python tests/golden/make_golden.py /path/to/reference

Fixtures (all small):
  mel_filters.npy     WhisperFeatureExtractor(feature_size=128).mel_filters (what custom/model.py:38
                      uploads), float32 [201, 128]
  logmel.npz          custom/model.py CustomModel._log_mel (called unbound on CPU torch tensors) and
                      the HF feature extractor on seeded synthetic audio: first 160 frames + checksums
  attention.npz       custom/selftest.py _attention_ref on seeded fp16 inputs (self L=65, cross 1500)
  hf_small.npz        transformers WhisperForConditionalGeneration (small dims, seeded weights from
                      flash_whisper_b200.weights) encoder output rows, prompt logits and 8 greedy tokens
                      of the reference's PyTorch loop (custom/pytorch_model.py:59-80 semantics, CPU fp32)
  turbo_tokens.json   the same loop at full large-v3-turbo size, seed-0 weights and seed-0 30 s audio,
                      forced to 32 tokens
  turbo_tokens_varied.json
                      the same loop on flash_whisper_b200.weights.varied_state_dict(0) (a decoder whose
                      greedy output changes from step to step), seed-1 30 s audio, 32 tokens, with the
                      fp32 top-2 logit gap of every step. The two token fixtures need only
                      transformers: `python tests/golden/make_golden.py --tokens-only`

The reference checkout is the first argument, or $FLASH_WHISPER_REFERENCE.
"""

import os

import json
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def attention_inputs(heads=20):
    """Seeded fp16 inputs of the attention fixture: q [heads*64], k/v [heads,448,64], kc/vc [heads,1500,64]."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(heads * 64, generator=g).half()
    k = torch.randn(heads, 448, 64, generator=g).half()
    v = torch.randn(heads, 448, 64, generator=g).half()
    kc = torch.randn(heads, 1500, 64, generator=g).half()
    vc = torch.randn(heads, 1500, 64, generator=g).half()
    return q, k, v, kc, vc


def main(reference):
    sys.path.insert(0, str(reference))
    from custom.model import CustomModel  # reference: only the pure-torch _log_mel method is used
    from custom.selftest import _attention_ref
    from transformers import WhisperFeatureExtractor

    from flash_whisper_b200.audio import synthetic_audio
    from flash_whisper_b200.weights import TURBO, WhisperDims, load_hf_model, random_state_dict
    from oracle.hf_cpu import transcribe_cpu

    fe = WhisperFeatureExtractor(feature_size=128)
    np.save(HERE / 'mel_filters.npy', fe.mel_filters.astype(np.float32))

    ns = SimpleNamespace(features=fe, window=torch.hann_window(400),
                         mel_filters=torch.from_numpy(fe.mel_filters).float())
    out = {}
    for name, seconds in (('clip30', 30.0), ('clip7', 7.25)):
        audio = synthetic_audio(0, seconds)
        wave = np.zeros(480000, np.float32)
        wave[:audio.size] = audio
        ref = CustomModel._log_mel(ns, torch.from_numpy(wave)).numpy()
        hf = fe(audio, sampling_rate=16000, return_tensors='np').input_features[0]
        out[f'{name}_ref_head'] = ref[:, :160].astype(np.float32)
        out[f'{name}_hf_head'] = hf[:, :160].astype(np.float32)
        out[f'{name}_ref_sum'] = np.float64(ref.astype(np.float64).sum())
        out[f'{name}_ref_sumsq'] = np.float64((ref.astype(np.float64) ** 2).sum())
        out[f'{name}_ref_tail'] = ref[:, -4:].astype(np.float32)
    np.savez_compressed(HERE / 'logmel.npz', **out)

    heads = 20
    q, k, v, kc, vc = attention_inputs()
    scale = 64 ** -0.5
    self_ref = _attention_ref(q.view(heads, 64), k, v, 65, scale).flatten()
    cross_ref = _attention_ref(q.view(heads, 64), kc, vc, 1500, scale).flatten()
    # inputs are regenerated from the seed by the tests (attention_inputs below); only outputs are stored
    np.savez_compressed(HERE / 'attention.npz', self_ref=self_ref.numpy(), cross_ref=cross_ref.numpy(),
                        q_sum=q.double().sum().numpy(), k_sum=k.double().sum().numpy(),
                        kc_sum=kc.double().sum().numpy())

    dims = WhisperDims(d_model=256, heads=4, encoder_layers=2, decoder_layers=2, ffn=512)
    sd = random_state_dict(3, dims, bias_std=0.02, ln_std=0.1)
    model = load_hf_model(sd, dims)
    from oracle.mel import log_mel
    audio = synthetic_audio(1, 5.0)
    wave = np.zeros(480000, np.float32)
    wave[:audio.size] = audio
    mel = torch.from_numpy(log_mel(wave).astype(np.float32))[None]
    with torch.inference_mode():
        enc = model.get_encoder()(mel).last_hidden_state[0]
        logits = model(encoder_outputs=(enc[None],), decoder_input_ids=torch.tensor([list(dims.prompt)])).logits[0, -1]
    tokens, _ = transcribe_cpu(model, audio, dims, n_tokens=8, begin_suppress=dims.begin_suppress)
    np.savez_compressed(HERE / 'hf_small.npz', enc_rows=enc[::100].numpy(), enc_sum=enc.double().sum().numpy(),
                        prompt_logits=logits.numpy(), tokens=np.array(tokens), seed=3, audio_seed=1)

    make_turbo_tokens()
    make_varied_tokens()


def make_turbo_tokens():
    """32 greedy tokens of the CPU fp32 reference loop at full size with the HF-init weights (seed 0)."""
    from flash_whisper_b200.audio import synthetic_audio
    from flash_whisper_b200.weights import TURBO, load_hf_model, random_state_dict
    from oracle.hf_cpu import transcribe_cpu

    model = load_hf_model(random_state_dict(0, TURBO), TURBO)
    audio = synthetic_audio(0, 30.0)
    gaps = []
    tokens, timing = transcribe_cpu(model, audio, TURBO, n_tokens=32, begin_suppress=TURBO.begin_suppress,
                                    logit_gaps=gaps)
    (HERE / 'turbo_tokens.json').write_text(json.dumps({
        'weights_seed': 0, 'audio_seed': 0, 'seconds': 30.0, 'n_tokens': 32, 'tokens': tokens,
        'top2_gap': [round(g, 6) for g in gaps],
        'generator': 'oracle.hf_cpu.transcribe_cpu (custom/pytorch_model.py loop, CPU fp32, HF feature extractor)',
        'timing_s': {k: round(v, 4) for k, v in timing.items() if k.endswith('_s')}}, indent=1) + '\n')
    print('tokens', tokens, 'min gap', min(gaps))


def make_varied_tokens():
    """32 greedy tokens of the CPU fp32 reference loop on weights whose output is not degenerate."""
    from flash_whisper_b200.audio import synthetic_audio
    from flash_whisper_b200.weights import TURBO, load_hf_model, varied_state_dict
    from oracle.hf_cpu import transcribe_cpu

    model = load_hf_model(varied_state_dict(0, TURBO), TURBO)
    audio = synthetic_audio(1, 30.0)
    gaps = []
    tokens, timing = transcribe_cpu(model, audio, TURBO, n_tokens=32, begin_suppress=TURBO.begin_suppress,
                                    logit_gaps=gaps)
    (HERE / 'turbo_tokens_varied.json').write_text(json.dumps({
        'weights': 'varied_state_dict(0)', 'audio_seed': 1, 'seconds': 30.0, 'n_tokens': 32, 'tokens': tokens,
        'top2_gap': [round(g, 6) for g in gaps],
        'generator': 'oracle.hf_cpu.transcribe_cpu (custom/pytorch_model.py loop, CPU fp32, HF feature extractor)',
        'timing_s': {k: round(v, 4) for k, v in timing.items() if k.endswith('_s')}}, indent=1) + '\n')
    print('varied tokens', tokens, 'min gap', min(gaps))


if __name__ == '__main__':
    if '--varied-only' in sys.argv:
        make_varied_tokens()
    elif '--tokens-only' in sys.argv:
        make_turbo_tokens()
        make_varied_tokens()
    else:
        ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('FLASH_WHISPER_REFERENCE')
        if not ref:
            sys.exit('usage: make_golden.py /path/to/reference  (or set FLASH_WHISPER_REFERENCE)')
        main(Path(ref))
