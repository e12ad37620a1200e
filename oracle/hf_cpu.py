"""The reference's PyTorch backend restated for the CPU (test infrastructure + CPU baseline).

custom/pytorch_model.py:28-89 runs transformers' Whisper in fp16 on CUDA: CPU feature extraction,
encoder, then a greedy loop over the full HF decoder with its KV cache, suppress masks applied to
the fp32 logits, `argmax().item()` per token, EOS break. That file hard-codes CUDA
(:16-17,40,46,72,78), so this is the same loop on the CPU in fp32, with the
decode optionally forced to a fixed token count (EOS ignored).
"""

import time

import numpy as np
import torch

from .mel import log_mel


def transcribe_cpu(model, audio, dims, n_tokens=None, begin_suppress=(), suppress=(), stop_at_eos=False,
                   threads=None):
    """Returns (token_ids, timings dict). `model` is a CPU WhisperForConditionalGeneration (fp32)."""
    if threads:
        torch.set_num_threads(threads)
    t0 = time.perf_counter()
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
            tokens.append(token)
            if stop_at_eos and token == dims.eos_token_id:
                break
            past = out.past_key_values
            decoder_input = torch.tensor([[token]], dtype=torch.long)
    t_end = time.perf_counter()
    return tokens, {'mel_s': t_mel - t0, 'encoder_s': t_enc - t_mel, 'decode_s': t_end - t_enc,
                    'e2e_s': t_end - t0, 'n_tokens': len(tokens)}
