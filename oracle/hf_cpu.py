"""The reference's PyTorch backend restated for the CPU (test infrastructure + CPU baseline).

custom/pytorch_model.py:28-89 runs transformers' Whisper in fp16 on CUDA: CPU feature extraction
with transformers' WhisperFeatureExtractor (:37-41), encoder, then a greedy loop over the full HF
decoder with its KV cache, suppress masks applied to the fp32 logits, `argmax().item()` per token,
EOS break. That file hard-codes CUDA (:16-17,40,46,72,78), so this is the same loop on the CPU in
fp32, with the decode optionally forced to a fixed token count (EOS ignored).
The feature extractor is transformers' own (mel='hf', the default) or the numpy restatement
oracle/mel.py (mel='oracle').
"""

import time

import numpy as np
import torch

from .mel import log_mel


_EXTRACTORS = {}


def feature_extractor(n_mels=128):
    """transformers' WhisperFeatureExtractor, as custom/pytorch_model.py:37 builds it (cached)."""
    if n_mels not in _EXTRACTORS:
        from transformers import WhisperFeatureExtractor
        _EXTRACTORS[n_mels] = WhisperFeatureExtractor(feature_size=n_mels)
    return _EXTRACTORS[n_mels]


def transcribe_cpu(model, audio, dims, n_tokens=None, begin_suppress=(), suppress=(), stop_at_eos=False,
                   threads=None, mel='hf', logit_gaps=None):
    """Returns (token_ids, timings dict). `model` is a CPU WhisperForConditionalGeneration (fp32).
    With `logit_gaps` (a list), the top-2 gap of each step's masked logits is appended to it."""
    if threads:
        torch.set_num_threads(threads)
    fe = feature_extractor(dims.n_mels) if mel == 'hf' else None
    t0 = time.perf_counter()
    if fe is not None:  # custom/pytorch_model.py:37-41: 30 s padding inside the extractor
        feats = torch.from_numpy(fe(audio, sampling_rate=16000, return_tensors='np').input_features.astype(np.float32))
    else:
        wave = np.zeros(30 * 16000, np.float32)
        wave[:audio.size] = audio
        feats = torch.from_numpy(log_mel(wave).astype(np.float32))[None]
    t_mel = time.perf_counter()
    with torch.inference_mode():
        enc = model.get_encoder()(feats)
        t_enc = time.perf_counter()
        prompt = list(dims.prompt)
        decoder_input = torch.tensor([prompt], dtype=torch.long)
        past = None
        tokens = []
        limit = dims.max_pos - len(prompt) if n_tokens is None else n_tokens
        for step in range(limit):
            out = model(encoder_outputs=enc, decoder_input_ids=decoder_input, past_key_values=past, use_cache=True)
            logits = out.logits[0, -1].float()
            if suppress:
                logits[list(suppress)] = -float('inf')
            if step == 0 and begin_suppress:
                logits[list(begin_suppress)] = -float('inf')
            token = int(logits.argmax().item())
            if logit_gaps is not None:
                top2 = torch.topk(logits, 2).values
                logit_gaps.append(float(top2[0] - top2[1]))
            tokens.append(token)
            if stop_at_eos and token == dims.eos_token_id:
                break
            past = out.past_key_values
            decoder_input = torch.tensor([[token]], dtype=torch.long)
    t_end = time.perf_counter()
    return tokens, {'mel_s': t_mel - t0, 'encoder_s': t_enc - t_mel, 'decode_s': t_end - t_enc,
                    'e2e_s': t_end - t0, 'n_tokens': len(tokens)}
