"""The reference's CUDA backend re-hosted for GPU parity and timing (test infrastructure).

custom/model.py cannot be imported on the GPU box (the reference checkout is not there) and needs a
checkpoint and tokenizer. This module runs the same pipeline on the same seeded random-init weights:

  * log-mel with torch.stft + the HF filterbank (custom/model.py:93-98),
  * the transformers WhisperEncoder in fp16 with SDPA + one cross-K/V F.linear, graph-captured
    (:143-171),
  * the decode step of :107-123 built from the reference's own kernels (oracle/_ref, compiled from
    custom/kernels/whisper_kernels.cu by oracle/build_ref.py) around cuBLAS F.linear / F.gelu /
    index_select, captured as 1-step and CHUNK-step CUDA graphs (:125-141),
  * the prompt handling and chunked greedy loop of transcribe (:196-215), here forced to a fixed
    token count with EOS ignored (BASELINE configs 3 and 4).
"""

import time
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn.functional as F

from .build_ref import load_ref
from .mel import mel_filter_bank

CHUNK = 8
SPLIT_KEYS = 64


class RefCudaBackend:
    @torch.inference_mode()
    def __init__(self, state_dict, dims):
        from flash_whisper_b200.weights import load_hf_model
        self.ext = load_ref()
        if self.ext is None:
            raise RuntimeError('oracle/_ref is not built (python -m oracle.build_ref)')
        hf = load_hf_model(state_dict, dims, dtype=torch.float16).cuda()
        hf.config._attn_implementation = 'sdpa'
        self.dims = dims
        self.encoder = hf.model.encoder
        self.window = torch.hann_window(400, device='cuda')
        self.mel_filters = torch.from_numpy(mel_filter_bank().astype(np.float32)).cuda()
        dec = hf.model.decoder
        self.heads, self.head_dim = dims.heads, dims.head_dim
        self.scale = self.head_dim ** -0.5
        self.max_pos, self.enc_len = dims.max_pos, dims.enc_len
        self.prompt = list(dims.prompt)
        self.embed, self.pos_embed = dec.embed_tokens.weight, dec.embed_positions.weight
        self.lm_head = hf.proj_out.weight.contiguous()
        self.final_ln = (dec.layer_norm.weight, dec.layer_norm.bias, dec.layer_norm.eps)
        self.layers = [self._pack(layer) for layer in dec.layers]
        cross = [layer.encoder_attn for layer in dec.layers]
        self.cross_w = torch.cat([torch.cat([a.k_proj.weight, a.v_proj.weight]) for a in cross]).contiguous()
        self.cross_b = torch.cat([torch.cat([torch.zeros_like(a.v_proj.bias), a.v_proj.bias]) for a in cross])
        vocab, n_layers, half = dims.vocab, dims.decoder_layers, torch.float16
        self.base_mask = torch.zeros(vocab, dtype=torch.bool, device='cuda')
        if dims.suppress:
            self.base_mask[list(dims.suppress)] = True
        self.first_mask = self.base_mask.clone()
        if dims.begin_suppress:
            self.first_mask[list(dims.begin_suppress)] = True
        self.suppress = self.base_mask.clone()
        self.self_kv = torch.zeros(n_layers, 2, self.heads, self.max_pos, self.head_dim, dtype=half, device='cuda')
        self.cross_kv = torch.zeros(n_layers, 2, self.heads, self.enc_len, self.head_dim, dtype=half, device='cuda')
        self.h = torch.zeros(1, dims.d_model, dtype=half, device='cuda')
        self.y = torch.zeros_like(self.h)
        self.attn = torch.zeros(dims.d_model, dtype=half, device='cuda')
        self.cur = torch.zeros(1, dtype=torch.long, device='cuda')
        self.state = torch.zeros(2, dtype=torch.long, device='cuda')
        self.tokens = torch.zeros(self.max_pos, dtype=torch.long, device='cuda')
        self.best = torch.zeros(1, dtype=torch.long, device='cuda')
        splits = -(-max(self.max_pos, self.enc_len) // SPLIT_KEYS)
        self.workspace = (torch.empty(self.heads * splits, device='cuda'), torch.empty(self.heads * splits, device='cuda'),
                          torch.empty(self.heads * splits * self.head_dim, device='cuda'))
        self.mel = torch.zeros(1, dims.n_mels, 2 * self.enc_len, dtype=half, device='cuda')
        self.graph_one, self.graph_chunk = self._capture()
        self.graph_enc = self._capture_encoder()

    @staticmethod
    def _pack(layer):
        sa, ca = layer.self_attn, layer.encoder_attn
        ln = lambda m: (m.weight, m.bias, m.eps)  # noqa: E731
        return SimpleNamespace(
            ln1=ln(layer.self_attn_layer_norm), ln2=ln(layer.encoder_attn_layer_norm), ln3=ln(layer.final_layer_norm),
            qkv_w=torch.cat([sa.q_proj.weight, sa.k_proj.weight, sa.v_proj.weight]).contiguous(),
            qkv_b=torch.cat([sa.q_proj.bias, torch.zeros_like(sa.q_proj.bias), sa.v_proj.bias]),
            out=(sa.out_proj.weight, sa.out_proj.bias), cross_q=(ca.q_proj.weight, ca.q_proj.bias),
            cross_out=(ca.out_proj.weight, ca.out_proj.bias),
            fc1=(layer.fc1.weight, layer.fc1.bias), fc2=(layer.fc2.weight, layer.fc2.bias))

    def log_mel(self, wave):
        stft = torch.stft(wave, 400, 160, window=self.window, return_complex=True)
        mel = torch.clamp(self.mel_filters.T @ (stft[..., :-1].abs() ** 2), min=1e-10).log10()
        mel = torch.maximum(mel, mel.max() - 8.0)
        return (mel + 4.0) / 4.0

    def _step(self):
        ext, state = self.ext, self.state
        torch.add(self.embed.index_select(0, self.cur), self.pos_embed.index_select(0, state[:1]), out=self.h)
        pending = None
        for i, L in enumerate(self.layers):
            ext.add_layernorm(self.h, pending, *L.ln1[:2], self.y, L.ln1[2])
            q, k, v = F.linear(self.y, L.qkv_w, L.qkv_b).view(3, self.heads, 1, self.head_dim)
            ext.decode_attention(q, self.self_kv[i, 0], self.self_kv[i, 1], self.attn, state, k, v, *self.workspace,
                                 self.scale)
            ext.add_layernorm(self.h, F.linear(self.attn.view(1, -1), *L.out), *L.ln2[:2], self.y, L.ln2[2])
            q = F.linear(self.y, *L.cross_q)
            ext.decode_attention(q, self.cross_kv[i, 0], self.cross_kv[i, 1], self.attn, None, None, None,
                                 *self.workspace, self.scale)
            ext.add_layernorm(self.h, F.linear(self.attn.view(1, -1), *L.cross_out), *L.ln3[:2], self.y, L.ln3[2])
            pending = F.linear(F.gelu(F.linear(self.y, *L.fc1)), *L.fc2)
        ext.add_layernorm(self.h, pending, *self.final_ln[:2], self.y, self.final_ln[2])
        ext.lm_head_argmax(self.y, self.lm_head, self.suppress, self.best)
        ext.argmax_finalize(self.best, self.tokens, self.state, self.cur, self.max_pos)

    def _capture(self):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                self._step()
        torch.cuda.current_stream().wait_stream(side)
        graphs = []
        for steps in (1, CHUNK):
            self.state.zero_()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(steps):
                    self._step()
            graphs.append(g)
        torch.cuda.synchronize()
        return graphs

    def _encode(self):
        enc = self.encoder(self.mel).last_hidden_state[0]
        kv = F.linear(enc, self.cross_w, self.cross_b)
        self.cross_kv.copy_(kv.view(self.enc_len, len(self.layers), 2, self.heads, self.head_dim)
                            .permute(1, 2, 3, 0, 4))
        return enc

    def _capture_encoder(self):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                self._encode()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.enc_out = self._encode()
        torch.cuda.synchronize()
        return g

    @torch.inference_mode()
    def transcribe(self, audio, n_tokens):
        """Forced decode of n_tokens (EOS ignored); returns (token_ids, timings)."""
        torch.cuda.synchronize()
        start = time.perf_counter()
        wave = torch.zeros(480000, device='cuda')
        wave[:audio.size] = torch.from_numpy(audio).cuda()
        mel = self.log_mel(wave)
        torch.cuda.synchronize()
        mel_s = time.perf_counter() - start
        self.mel.copy_(mel[None])
        self.graph_enc.replay()
        torch.cuda.synchronize()
        encoder_s = time.perf_counter() - start - mel_s
        decode_start = time.perf_counter()
        self.state.zero_()
        last = len(self.prompt) - 1
        for i, token in enumerate(self.prompt):
            self.cur.fill_(token)
            if i == last:
                self.suppress.copy_(self.first_mask)
            self.graph_one.replay()
            if i == last:
                self.suppress.copy_(self.base_mask)
            else:
                self.state[1].zero_()
        token_ids = [int(self.tokens[0])]
        ttft = time.perf_counter() - start
        while len(token_ids) < n_tokens:
            self.graph_chunk.replay()
            token_ids.extend(self.tokens[len(token_ids):len(token_ids) + CHUNK].tolist())
        token_ids = token_ids[:n_tokens]
        ttlt = time.perf_counter() - start
        return token_ids, {'mel_s': mel_s, 'encoder_s': encoder_s, 'decode_s': ttlt - (decode_start - start),
                           'ttft_s': ttft, 'e2e_s': ttlt}
