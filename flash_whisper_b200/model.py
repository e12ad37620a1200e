"""Batch-1 fp16 Whisper-large-v3-turbo on B200: the drop-in for the reference's custom/model.py.

`CustomModel(model_id, cache_dir)` and `.transcribe(audio)` keep the reference's call surface and
return dict (custom/model.py:26-225). Everything between the host waveform and the token ids runs
in this package's CUDA kernels, recorded into CUDA graphs:

  * front graph: GPU log-mel (fw_log_mel, time-major output with zero padding rows) and the whole
    encoder (fw_encoder_forward: implicit-GEMM convs, 32 layers of tcgen05 GEMMs + attention,
    final LN, cross-K/V GEMM scattered straight into the decoder's cross cache);
  * prompt graph: state reset + the 4 prompt steps (prompt ids are read on the device, so the
    host never writes `cur` between steps as custom/model.py:199-207 does);
  * chunk graph: CHUNK decode steps (fw_decoder_step, 17 PDL-chained launches per token).

The host reads tokens back once per chunk, one chunk behind the GPU, and stops at EOS like
custom/model.py:210-215; with `max_new_tokens` and `stop_at_eos=False` it replays all chunks and
reads once. No kernel allocates; all buffers are allocated here once.
"""

import ctypes
import time

import numpy as np
import torch

from . import _lib
from .audio import N_SAMPLES, mel_filters
from .ext import load_ext
from .selftest import SPLIT_KEYS, run_selftest
from .weights import TURBO, pack_decoder, pack_encoder, random_state_dict

CHUNK = 8  # decode steps per graph replay


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


class _StubTokenizer:
    """Stand-in when no tokenizer files are available offline: text is the id list."""

    def decode(self, ids, skip_special_tokens=True):
        return ' '.join(str(i) for i in ids)


def _load_pretrained(model_id, cache_dir):
    from transformers import AutoTokenizer, WhisperForConditionalGeneration
    hf = WhisperForConditionalGeneration.from_pretrained(model_id, cache_dir=cache_dir, dtype=torch.float16)
    sd = {k: v for k, v in hf.state_dict().items() if k != 'proj_out.weight'}
    tok = AutoTokenizer.from_pretrained(model_id, cache_dir=cache_dir)
    gen, cfg = hf.generation_config, hf.config
    eos = gen.eos_token_id if gen.eos_token_id is not None else cfg.eos_token_id
    prompt = tuple(tok.convert_tokens_to_ids(['<|startoftranscript|>', '<|en|>', '<|transcribe|>',
                                              '<|notimestamps|>']))
    from .weights import WhisperDims
    dims = WhisperDims(d_model=cfg.d_model, heads=cfg.decoder_attention_heads, encoder_layers=cfg.encoder_layers,
                       decoder_layers=cfg.decoder_layers, ffn=cfg.decoder_ffn_dim, vocab=cfg.vocab_size,
                       n_mels=cfg.num_mel_bins, enc_len=cfg.max_source_positions, max_pos=cfg.max_target_positions,
                       pad_token_id=cfg.pad_token_id, eos_token_id=eos if isinstance(eos, int) else eos[0],
                       prompt=prompt, begin_suppress=tuple(gen.begin_suppress_tokens or ()),
                       suppress=tuple(gen.suppress_tokens or ()))
    return sd, dims, tok


class CustomModel:
    @torch.inference_mode()
    def __init__(self, model_id=None, cache_dir=None, *, state_dict=None, dims=None, seed=0, tokenizer=None,
                 chunk=CHUNK, selftest=True, capture=True, lm_prune=True):
        if not torch.cuda.is_available():
            raise RuntimeError('CustomModel requires a CUDA device')
        self.ext = load_ext()
        if state_dict is None:
            if model_id is None or str(model_id).startswith('random'):
                dims = dims or TURBO
                state_dict = random_state_dict(seed, dims)
            else:
                state_dict, dims, tokenizer = _load_pretrained(model_id, cache_dir)
        self.dims = dims = dims or TURBO
        self.tokenizer = tokenizer or _StubTokenizer()
        self.chunk = chunk
        dev, half = 'cuda', torch.float16
        self.dec = pack_decoder(state_dict, dims, dev)
        self.enc = pack_encoder(state_dict, dims, dev)
        # int8 copy of the LM head with per-row bounds: each step streams it and rescores exactly only
        # the rows that can still win (fw_lm_head_argmax_q; the chosen token is unchanged)
        self.lm_q, self.lm_rp = self.ext.lm_quantize(self.dec.lm_head) if lm_prune else (None, None)
        self.heads, self.head_dim = dims.heads, dims.head_dim
        self.scale = self.head_dim ** -0.5
        self.max_pos, self.enc_len = dims.max_pos, dims.enc_len
        self.prompt = list(dims.prompt)
        self.max_new = self.max_pos - len(self.prompt)
        self.eos = {dims.eos_token_id}

        vocab, n_layers = dims.vocab, dims.decoder_layers
        self.base_mask = torch.zeros(vocab, dtype=torch.bool, device=dev)
        if dims.suppress:
            self.base_mask[list(dims.suppress)] = True
        self.first_mask = self.base_mask.clone()
        if dims.begin_suppress:
            self.first_mask[list(dims.begin_suppress)] = True

        # decode state (custom/model.py:64-74)
        self.self_kv = torch.zeros(n_layers, 2, self.heads, self.max_pos, self.head_dim, dtype=half, device=dev)
        self.cross_kv = torch.zeros(n_layers, 2, self.heads, self.enc_len, self.head_dim, dtype=half, device=dev)
        d = dims.d_model
        self.h = torch.zeros(d, dtype=half, device=dev)
        self.qkv = torch.zeros(3 * d, dtype=half, device=dev)
        self.attn = torch.zeros(d, dtype=half, device=dev)
        self.cq = torch.zeros(d, dtype=half, device=dev)
        self.ffn = torch.zeros(dims.ffn, dtype=half, device=dev)
        self.cur = torch.zeros(1, dtype=torch.long, device=dev)
        self.state = torch.zeros(2, dtype=torch.long, device=dev)  # [position, generated count]
        self.tokens = torch.zeros(self.max_pos, dtype=torch.long, device=dev)
        self.best = torch.zeros(1, dtype=torch.long, device=dev)
        self.prompt_t = torch.tensor(self.prompt, dtype=torch.long, device=dev)
        # split-attention workspace; the fused step also keeps two blocks' output-projection partials
        # (2 * heads * 1280 floats) in part_acc
        self.splits = max(-(-max(self.max_pos, self.enc_len) // SPLIT_KEYS), 2 * d // self.head_dim)
        self.part_m = torch.empty(self.heads * self.splits, device=dev)
        self.part_l = torch.empty(self.heads * self.splits, device=dev)
        self.part_acc = torch.empty(self.heads * self.splits * self.head_dim, device=dev)
        self.counters = torch.zeros(self.heads + 1, dtype=torch.int32, device=dev)

        # front end + encoder buffers
        T, F = self.enc_len, dims.n_frames
        self.wave = torch.zeros(N_SAMPLES, dtype=torch.float32, device=dev)
        self.wave_host = torch.zeros(N_SAMPLES, dtype=torch.float32).pin_memory()
        self.filters = torch.from_numpy(mel_filters(dims.n_mels)).to(dev)
        self.mel_scratch = torch.empty(dims.n_mels * F, dtype=torch.float32, device=dev)
        self.clip_max = torch.zeros(1, dtype=torch.int32, device=dev)
        self.mel = torch.zeros(F + 2, dims.n_mels, dtype=half, device=dev)  # time-major, zero pad rows
        self.conv1_out = torch.zeros(F + 2, d, dtype=half, device=dev)
        self.ex = torch.zeros(T, d, dtype=half, device=dev)
        self.ey = torch.zeros(T, d, dtype=half, device=dev)
        self.eqkv = torch.zeros(T, 3 * d, dtype=half, device=dev)
        self.eattn = torch.zeros(T, d, dtype=half, device=dev)
        self.effn = torch.zeros(T, dims.ffn, dtype=half, device=dev)
        self.enc_out = torch.zeros(T, d, dtype=half, device=dev)
        self.evt = torch.zeros(d, -(-T // 8) * 8, dtype=half, device=dev)  # V^T of the encoder attention
        self.tokens_host = torch.zeros(self.max_pos, dtype=torch.long).pin_memory()
        self._wave_copied = None  # event after the last asynchronous copy out of wave_host

        self.dec_desc = self._decoder_desc()
        self.enc_desc = self._encoder_desc()
        self.selftest = run_selftest(self.ext, self) if selftest else {'ok': None, 'checks': []}
        if selftest:
            self.selftest['mel_max_abs_diff'] = self._mel_diff()
        self.graph_mel = self.graph_enc = self.graph_prompt = self.graph_chunk = None
        self.loop = self.loop_chunk = None
        if capture:
            self._capture()

    # ---- descriptors -------------------------------------------------------------------------
    def _decoder_desc(self):
        dims, dec = self.dims, self.dec
        desc = _lib.Decoder()
        desc.n_layers, desc.heads, desc.max_pos = dims.decoder_layers, self.heads, self.max_pos
        desc.enc_len, desc.vocab, desc.prompt_len = self.enc_len, dims.vocab, len(self.prompt)
        desc.eps, desc.scale = dims.eps, self.scale
        desc.embed, desc.pos_embed, desc.lm_head = _p(dec.embed), _p(dec.pos_embed), _p(dec.lm_head)
        desc.final_g, desc.final_b = _p(dec.final_ln[0]), _p(dec.final_ln[1])
        desc.base_mask, desc.first_mask, desc.prompt = _p(self.base_mask), _p(self.first_mask), _p(self.prompt_t)
        for i, L in enumerate(dec.layers):
            dl = desc.layers[i]
            dl.ln1_g, dl.ln1_b = _p(L.ln1[0]), _p(L.ln1[1])
            dl.ln2_g, dl.ln2_b = _p(L.ln2[0]), _p(L.ln2[1])
            dl.ln3_g, dl.ln3_b = _p(L.ln3[0]), _p(L.ln3[1])
            dl.qkv_w, dl.qkv_b = _p(L.qkv_w), _p(L.qkv_b)
            dl.out_w, dl.out_b = _p(L.out[0]), _p(L.out[1])
            dl.cq_w, dl.cq_b = _p(L.cross_q[0]), _p(L.cross_q[1])
            dl.co_w, dl.co_b = _p(L.cross_out[0]), _p(L.cross_out[1])
            dl.fc1_w, dl.fc1_b = _p(L.fc1[0]), _p(L.fc1[1])
            dl.fc2_w, dl.fc2_b = _p(L.fc2[0]), _p(L.fc2[1])
            dl.self_k, dl.self_v = _p(self.self_kv[i, 0]), _p(self.self_kv[i, 1])
            dl.cross_k, dl.cross_v = _p(self.cross_kv[i, 0]), _p(self.cross_kv[i, 1])
        desc.h, desc.qkv, desc.attn, desc.cq, desc.ffn = (_p(self.h), _p(self.qkv), _p(self.attn), _p(self.cq),
                                                          _p(self.ffn))
        desc.part_m, desc.part_l, desc.part_acc = _p(self.part_m), _p(self.part_l), _p(self.part_acc)
        desc.ws_splits = self.splits
        desc.counters, desc.cur, desc.state = _p(self.counters), _p(self.cur), _p(self.state)
        desc.tokens, desc.best, desc.n_tokens = _p(self.tokens), _p(self.best), self.tokens.numel()
        if self.lm_q is not None:
            desc.lm_q, desc.lm_rp = _p(self.lm_q), _p(self.lm_rp)
        return desc

    def _encoder_desc(self):
        dims, enc = self.dims, self.enc
        desc = _lib.Encoder()
        desc.n_layers, desc.n_frames, desc.n_pos = dims.encoder_layers, dims.n_frames, self.enc_len
        desc.n_dec_layers, desc.heads, desc.eps = dims.decoder_layers, self.heads, dims.eps
        desc.mel = _p(self.mel)
        desc.conv1_w, desc.conv1_b = _p(enc.conv1[0]), _p(enc.conv1[1])
        desc.conv2_w, desc.conv2_b = _p(enc.conv2[0]), _p(enc.conv2[1])
        desc.pos = _p(enc.pos)
        for i, L in enumerate(enc.layers):
            el = desc.layers[i]
            el.ln1_g, el.ln1_b = _p(L.ln1[0]), _p(L.ln1[1])
            el.ln2_g, el.ln2_b = _p(L.ln2[0]), _p(L.ln2[1])
            el.qkv_w, el.qkv_b = _p(L.qkv_w), _p(L.qkv_b)
            el.out_w, el.out_b = _p(L.out[0]), _p(L.out[1])
            el.fc1_w, el.fc1_b = _p(L.fc1[0]), _p(L.fc1[1])
            el.fc2_w, el.fc2_b = _p(L.fc2[0]), _p(L.fc2[1])
        desc.final_g, desc.final_b = _p(enc.final_ln[0]), _p(enc.final_ln[1])
        desc.cross_w, desc.cross_b = _p(self.dec.cross_w), _p(self.dec.cross_b)
        desc.conv1_out, desc.x, desc.y = _p(self.conv1_out), _p(self.ex), _p(self.ey)
        desc.qkv, desc.attn, desc.ffn = _p(self.eqkv), _p(self.eattn), _p(self.effn)
        desc.enc_out, desc.cross_kv, desc.vt = _p(self.enc_out), _p(self.cross_kv), _p(self.evt)
        return desc

    # ---- stages (eager; also what the graphs record) -----------------------------------------
    def _mel(self):
        self.ext.log_mel(self.wave, self.filters, self.mel_scratch, self.clip_max, self.mel, layout=1)

    def _encode(self):
        self.ext.encoder_forward(self.enc_desc)

    def _front(self):
        self._mel()
        self._encode()

    def _prompt(self):
        self.state.zero_()
        self.ext.decoder_step(self.dec_desc, len(self.prompt))

    def _chunk(self):
        self.ext.decoder_step(self.dec_desc, self.chunk)

    def _mel_diff(self):
        """Largest |GPU log-mel - transformers' WhisperFeatureExtractor| on 10 s of seeded noise, the
        load-time front-end check of custom/model.py:77,100-105 (None if transformers is absent)."""
        try:
            from transformers import WhisperFeatureExtractor
        except ImportError:
            return None
        audio = np.random.default_rng(0).standard_normal(10 * 16000).astype(np.float32) * 0.1
        ref = WhisperFeatureExtractor(feature_size=self.dims.n_mels)(audio, sampling_rate=16000,
                                                                      return_tensors='np').input_features[0]
        self.load_audio(audio)
        self._mel()
        got = self.mel[1:-1].float().T.cpu().numpy()
        return float(np.abs(got - ref).max())

    def _capture(self):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                self._front()
                self._prompt()
                self._chunk()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graphs = []
        for name, fn in (('mel', self._mel), ('encoder', self._encode), ('prompt', self._prompt),
                         ('chunk', self._chunk)):
            try:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    fn()
            except Exception as exc:  # a stage whose capture fails runs eagerly (custom/model.py:165-168)
                torch.cuda.synchronize()
                g = None
                self.selftest[f'{name}_graph'] = False
                self.selftest[f'{name}_graph_error'] = f'{type(exc).__name__}: {exc}'
            graphs.append(g)
        torch.cuda.synchronize()
        self.graph_mel, self.graph_enc, self.graph_prompt, self.graph_chunk = graphs
        if self.graph_enc is not None:
            # graph replay vs eager on the same random input (custom/model.py:158-164)
            mel_saved = self.mel.clone()
            self.mel[1:-1].normal_()
            self._encode()
            eager = self.enc_out.clone()
            self.enc_out.zero_()
            self.graph_enc.replay()
            torch.cuda.synchronize()
            self.selftest['encoder_graph_max_abs_diff'] = float((self.enc_out.float() - eager.float()).abs().max())
            self.selftest['encoder_graph'] = True
            self.mel.copy_(mel_saved)
        self._make_loop()

    def _make_loop(self):
        """The on-device decode loops (fw_decode_loop_*): one graph launch decodes until EOS or the token
        limit, the stop condition evaluated on the GPU. `loop` evaluates it after every step (it stops
        exactly at the limit or the EOS token); `loop_chunk` after every `chunk` steps, like the
        reference's 8-step graphs (custom/model.py:208-215), which spends a conditional-node iteration
        per chunk instead of per token and may decode up to chunk - 1 tokens past the stop, which the
        caller drops. transcribe(stop_at_eos=True) uses `loop_chunk`."""
        self.loop_ctrl = torch.zeros(5, dtype=torch.long, device='cuda')
        self.loop_ctrl_host = torch.zeros(5, dtype=torch.long).pin_memory()
        self._ctrl_copied = None
        self._loop_destroy = _lib.lib().fw_decode_loop_destroy  # held: module globals may be gone at exit
        self.loop = self.loop_chunk = None
        try:
            for name, steps in (('loop', 1), ('loop_chunk', self.chunk)):
                handle = ctypes.c_void_p()
                _lib.call('fw_decode_loop_create', ctypes.byref(self.dec_desc), _p(self.loop_ctrl), int(steps),
                          ctypes.byref(handle))
                setattr(self, name, handle)
            self.selftest['decode_loop'] = True
        except RuntimeError as exc:  # the host loop of chunk graphs is used instead
            self.selftest['decode_loop'] = False
            self.selftest['decode_loop_error'] = str(exc)

    def __del__(self):
        destroy = getattr(self, '_loop_destroy', None)
        for name in ('loop', 'loop_chunk'):
            loop = getattr(self, name, None)
            if loop is not None and destroy is not None:
                destroy(loop)
                setattr(self, name, None)

    def run_loop(self, limit, stop_at_eos, eos=None, chunked=False):
        """Decode steps on the GPU until state[1] (tokens generated) reaches `limit` or, with
        stop_at_eos, the last generated token is `eos` (default: the model's EOS id); one graph
        launch, no host synchronisation. chunked=True runs `loop_chunk`, which checks the stop only
        every `chunk` steps (up to chunk - 1 extra tokens, to be dropped by the caller)."""
        loop = self.loop_chunk if chunked else self.loop
        if self._ctrl_copied is not None:
            self._ctrl_copied.synchronize()
        eos = self.dims.eos_token_id if eos is None else int(eos)
        self.loop_ctrl_host.copy_(torch.tensor([int(limit), eos, int(bool(stop_at_eos)), 0,
                                                self.max_pos + len(self.prompt)]))
        self.loop_ctrl.copy_(self.loop_ctrl_host, non_blocking=True)
        self._ctrl_copied = torch.cuda.Event()
        self._ctrl_copied.record()
        _lib.call('fw_decode_loop_launch', loop, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))

    def run_mel(self):
        self.graph_mel.replay() if self.graph_mel else self._mel()

    def run_encoder(self):
        self.graph_enc.replay() if self.graph_enc else self._encode()

    def run_front(self):
        self.run_mel()
        self.run_encoder()

    def run_prompt(self):
        self.graph_prompt.replay() if self.graph_prompt else self._prompt()

    def run_chunk(self):
        self.graph_chunk.replay() if self.graph_chunk else self._chunk()

    @torch.inference_mode()
    def load_audio(self, audio):
        """Copies a host clip (zero-padded to 30 s) into the device waveform buffer. The copy from the
        pinned staging buffer is asynchronous; the staging buffer is rewritten only after the previous
        copy from it has completed."""
        if self._wave_copied is not None:
            self._wave_copied.synchronize()
        host = self.wave_host.numpy()
        host[:audio.size] = audio
        host[audio.size:] = 0.0
        self.wave.copy_(self.wave_host, non_blocking=True)
        self._wave_copied = torch.cuda.Event()
        self._wave_copied.record()

    def run_steps(self, n):
        """n decode steps: whole CHUNK-step graphs, then the remainder launched directly."""
        for _ in range(n // self.chunk):
            self.run_chunk()
        if n % self.chunk:
            self.ext.decoder_step(self.dec_desc, n % self.chunk)

    @torch.inference_mode()
    def decode_device(self, n_tokens, loop=False):
        """Device-resident pipeline after the waveform is in self.wave: front, prompt (which yields
        the first token) and exactly n_tokens - 1 further decode steps, as chunk-graph replays or
        (loop=True) one launch of the on-device decode loop."""
        self.run_front()
        self.run_prompt()
        if loop and self.loop is not None:
            self.run_loop(n_tokens, False)
        else:
            self.run_steps(max(0, n_tokens - 1))

    # ---- public API --------------------------------------------------------------------------
    @staticmethod
    def _check_audio(audio):
        """custom/model.py:175-178."""
        if not isinstance(audio, np.ndarray) or audio.dtype != np.float32 or audio.ndim != 1:
            raise ValueError('audio must be a one-dimensional float32 NumPy array')
        if not 0 < audio.size <= N_SAMPLES or not np.isfinite(audio).all():
            raise ValueError('audio must contain finite samples and be between 0 and 30 seconds')

    def batch_decoders(self, count=3):
        """The batched decoders (flash_whisper_b200.batch.BatchDecoder, 8 clips each) that
        transcribe_batch rotates through, one decode stream each, created on first use. Three
        streams measured best for the 256-clip stream (1 / 2 / 3 / 4: 1722 / 2081 / 2152 / 2123
        audio-s/s on one B200)."""
        if getattr(self, '_batch', None) is None:
            from .batch import BatchDecoder
            self._batch = [BatchDecoder(self) for _ in range(count)]
        return self._batch

    def batch_decoder(self):
        """The first batched decoder (8 clips per weight read)."""
        return self.batch_decoders()[0]

    @torch.inference_mode()
    def transcribe_batch(self, audios, max_new_tokens=None, stop_at_eos=True):
        """Transcribes several clips with the batched decoders (flash_whisper_b200.batch): 8 clips per
        decoder weight read, three groups decoding on their own streams while the encoders of the next
        groups run.

        Returns one dict per clip with transcribe()'s keys; each clip's token ids are exactly those
        transcribe() returns for it alone. `max_new_tokens` is one limit or one per clip; clips are
        grouped in the given order (give them longest first to waste the fewest steps). A group is
        decoded to its longest limit and every clip is then cut at its limit and, with stop_at_eos, at
        its first EOS. Times: mel_s / encoder_s are the clip's own device times; ttft_s, ttlt_s and
        e2e_s are those of the whole call, whose decode_s is its wall time minus the clip's front end."""
        from .batch import run_clips
        for a in audios:
            self._check_audio(a)
        n_all = len(audios)
        if isinstance(max_new_tokens, (list, tuple)):
            limits = [min(int(x), self.max_new) for x in max_new_tokens]
        else:
            limits = [self.max_new if max_new_tokens is None else min(int(max_new_tokens), self.max_new)] * n_all
        decoders = self.batch_decoders()
        if getattr(self, '_staging', None) is None:
            from .batch import HostStaging
            self._staging = HostStaging(len(decoders) * decoders[0].clips, N_SAMPLES)
        torch.cuda.synchronize()
        start = time.perf_counter()
        tokens, times = run_clips(self, decoders, None, limits, host_audio=audios, staging=self._staging)
        ttlt = time.perf_counter() - start
        rows = tokens.tolist()
        results = []
        for i in range(n_all):
            ids = rows[i][:limits[i]]
            if stop_at_eos:
                cut = next((k + 1 for k, t in enumerate(ids) if t in self.eos), len(ids))
                ids = ids[:cut]
            d0 = time.perf_counter()
            text = self.tokenizer.decode(ids, skip_special_tokens=True)
            results.append({'text': text, 'token_ids': ids, 'ttft_s': ttlt, 'ttlt_s': ttlt,
                            'e2e_s': time.perf_counter() - start, 'mel_s': times[i][0], 'encoder_s': times[i][1],
                            'decode_s': ttlt - times[i][0] - times[i][1], 'detok_s': time.perf_counter() - d0,
                            'n_tokens': len(ids)})
        return results

    @torch.inference_mode()
    def transcribe(self, audio, max_new_tokens=None, stop_at_eos=True):
        self._check_audio(audio)
        limit = self.max_new if max_new_tokens is None else min(int(max_new_tokens), self.max_new)
        stream = torch.cuda.current_stream()
        torch.cuda.synchronize()
        start = time.perf_counter()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        host = self.wave_host.numpy()
        host[:audio.size] = audio
        host[audio.size:] = 0.0
        ev[0].record(stream)
        self.wave.copy_(self.wave_host, non_blocking=True)
        self.run_mel()
        ev[1].record(stream)
        self.run_encoder()
        ev[2].record(stream)
        self.run_prompt()
        ev[3].record(stream)
        n_chunks = -(-(limit - 1) // self.chunk) if limit > 1 else 0
        token_ids = []
        if not stop_at_eos:
            self.run_steps(max(0, limit - 1))
            self.tokens_host[:limit].copy_(self.tokens[:limit], non_blocking=True)
            ev[3].synchronize()
            ttft = time.perf_counter() - start
            stream.synchronize()
            token_ids = self.tokens_host[:limit].tolist()
        elif self.loop_chunk is not None:
            # prompt -> first token read back (TTFT) while the on-device loop decodes to EOS / limit
            # (chunks of `chunk` steps; the tokens past the limit or the first EOS are dropped below)
            self.tokens_host[:1].copy_(self.tokens[:1], non_blocking=True)
            first = torch.cuda.Event()
            first.record(stream)
            self.run_loop(limit, True, chunked=True)
            self.tokens_host[:limit].copy_(self.tokens[:limit], non_blocking=True)
            state_host = self.state.to('cpu', non_blocking=True)
            first.synchronize()
            ttft = time.perf_counter() - start
            stream.synchronize()
            n = min(int(state_host[1]), limit)
            token_ids = self.tokens_host[:n].tolist()
            cut = next((i + 1 for i, t in enumerate(token_ids) if t in self.eos), len(token_ids))
            token_ids = token_ids[:cut]
        else:
            done_events = []
            issued = 0

            def issue():
                nonlocal issued
                self.run_chunk()
                lo = 1 + issued * self.chunk
                hi = min(lo + self.chunk, limit)
                self.tokens_host[lo:hi].copy_(self.tokens[lo:hi], non_blocking=True)
                e = torch.cuda.Event()
                e.record(stream)
                done_events.append((e, lo, hi))
                issued += 1

            self.tokens_host[:1].copy_(self.tokens[:1], non_blocking=True)
            first = torch.cuda.Event()
            first.record(stream)
            if issued < n_chunks:
                issue()  # keep the GPU busy while the host waits for the first token
            first.synchronize()
            ttft = time.perf_counter() - start
            token_ids = [int(self.tokens_host[0])]
            k = 0
            while token_ids[-1] not in self.eos and len(token_ids) < limit and k < n_chunks:
                if issued < n_chunks:
                    issue()
                e, lo, hi = done_events[k]
                e.synchronize()
                for tok in self.tokens_host[lo:hi].tolist():
                    token_ids.append(tok)
                    if tok in self.eos or len(token_ids) >= limit:
                        break
                k += 1
            stream.synchronize()
        ttlt = time.perf_counter() - start
        mel_s = ev[0].elapsed_time(ev[1]) / 1e3
        encoder_s = ev[1].elapsed_time(ev[2]) / 1e3
        detok_start = time.perf_counter()
        text = self.tokenizer.decode(token_ids, skip_special_tokens=True)
        e2e = time.perf_counter() - start
        # Stage times come from CUDA events (the pipeline is not synchronised between stages);
        # mel_s includes the host->device copy of the waveform as in custom/model.py:182-186.
        return {
            'text': text, 'token_ids': token_ids, 'ttft_s': ttft, 'ttlt_s': ttlt, 'e2e_s': e2e,
            'mel_s': mel_s, 'encoder_s': encoder_s, 'decode_s': ttlt - mel_s - encoder_s,
            'detok_s': time.perf_counter() - detok_start, 'n_tokens': len(token_ids),
        }
