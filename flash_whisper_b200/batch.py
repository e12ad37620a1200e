"""Batched decode: up to 8 clips per decoder weight read (the throughput path for many clips on one GPU).

The reference decodes one clip per step and reads every decoder weight once per token
(custom/model.py:107-123). `BatchDecoder` keeps up to `FW_MAX_CLIPS` clips in flight: each clip gets
its own self and cross caches, residual stream, position and token row, its encoder output is
scattered into its own cross-cache slot, and `fw_batch_decoder_step` advances all of them by one
token with one pass over the weights (33 PDL-chained launches per step). Every clip's arithmetic is
the batch-1 step's, so its tokens are exactly those of `CustomModel.transcribe` on the same clip.

Clips of a batch advance in lockstep from the prompt: a batch decodes max(n_tokens) steps and each
clip keeps its first n_tokens tokens. Grouping clips of similar length (longest first) keeps the
wasted steps small.
"""

import ctypes

import torch

from . import _lib

MAX_CLIPS = _lib.MAX_CLIPS


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


class BatchDecoder:
    """Batched decoder sharing a CustomModel's weights, front end and encoder scratch."""

    @torch.inference_mode()
    def __init__(self, model, clips=MAX_CLIPS, chunk=8):
        if not 1 <= clips <= MAX_CLIPS:
            raise ValueError(f'clips must be 1..{MAX_CLIPS}')
        if model.lm_q is None:
            raise ValueError('the batched decoder needs the pruned LM head (CustomModel(lm_prune=True))')
        self.model, self.clips, self.chunk = model, clips, chunk
        dims, dev, half = model.dims, 'cuda', torch.float16
        L, H, HD, d = dims.decoder_layers, model.heads, model.head_dim, dims.d_model
        self.self_kv = torch.zeros(clips, L, 2, H, model.max_pos, HD, dtype=half, device=dev)
        self.cross_kv = torch.zeros(clips, L, 2, H, model.enc_len, HD, dtype=half, device=dev)
        self.h = torch.zeros(clips, d, dtype=half, device=dev)
        self.qkv = torch.zeros(clips, 3 * d, dtype=half, device=dev)
        self.attn = torch.zeros(clips, d, dtype=half, device=dev)
        self.ffn = torch.zeros(clips, dims.ffn, dtype=half, device=dev)
        self.ws_splits = -(-max(model.max_pos, model.enc_len) // 64)
        n = clips * H * self.ws_splits
        self.part_m = torch.empty(n, device=dev)
        self.part_l = torch.empty(n, device=dev)
        self.part_acc = torch.empty(n * HD, device=dev)
        self.counters = torch.zeros(clips * H + 1, dtype=torch.int32, device=dev)
        self.cur = torch.zeros(clips, dtype=torch.long, device=dev)
        self.state = torch.zeros(clips, 2, dtype=torch.long, device=dev)
        self.tokens = torch.zeros(clips, model.max_pos, dtype=torch.long, device=dev)
        self.best = torch.zeros(clips, dtype=torch.long, device=dev)
        self.descs = {}
        self.graphs = {}
        self.enc_descs = [self._encoder_desc(c) for c in range(clips)]
        self.enc_graphs = [None] * clips

    def _desc(self, n):
        """Descriptor of the first n clips."""
        if n in self.descs:
            return self.descs[n]
        m, dims = self.model, self.model.dims
        src = m.dec_desc
        d = _lib.BatchDecoder()
        d.n_layers, d.heads, d.max_pos, d.enc_len = src.n_layers, src.heads, src.max_pos, src.enc_len
        d.vocab, d.prompt_len, d.clips, d.eps, d.scale = src.vocab, src.prompt_len, n, src.eps, src.scale
        for name in ('embed', 'pos_embed', 'lm_head', 'final_g', 'final_b', 'base_mask', 'first_mask', 'prompt',
                     'lm_q', 'lm_rp'):
            setattr(d, name, getattr(src, name))
        for i in range(dims.decoder_layers):
            ctypes.memmove(ctypes.byref(d.layers[i]), ctypes.byref(src.layers[i]), ctypes.sizeof(_lib.DecoderLayer))
            dl = d.layers[i]
            dl.self_k, dl.self_v = _p(self.self_kv[0, i, 0]), _p(self.self_kv[0, i, 1])
            dl.cross_k, dl.cross_v = _p(self.cross_kv[0, i, 0]), _p(self.cross_kv[0, i, 1])
        d.self_clip_stride = self.self_kv[0].numel()
        d.cross_clip_stride = self.cross_kv[0].numel()
        d.h, d.qkv, d.attn, d.ffn = _p(self.h), _p(self.qkv), _p(self.attn), _p(self.ffn)
        d.part_m, d.part_l, d.part_acc, d.ws_splits = _p(self.part_m), _p(self.part_l), _p(self.part_acc), self.ws_splits
        d.counters, d.cur, d.state = _p(self.counters), _p(self.cur), _p(self.state)
        d.tokens, d.best, d.n_tokens = _p(self.tokens), _p(self.best), self.tokens.size(1)
        self.descs[n] = d
        return d

    def _encoder_desc(self, slot):
        e = _lib.Encoder()
        ctypes.memmove(ctypes.byref(e), ctypes.byref(self.model.enc_desc), ctypes.sizeof(_lib.Encoder))
        e.cross_kv = _p(self.cross_kv[slot])
        return e

    # ---- front end -------------------------------------------------------------------------
    def encode_slot(self, slot):
        """Log-mel of the model's waveform buffer, then the encoder into clip `slot`'s cross cache."""
        self.model.run_mel()
        self.encoder_slot(slot)

    def encoder_slot(self, slot):
        """The encoder on the model's mel buffer, its cross K/V scattered into clip `slot`'s cache."""
        m = self.model
        g = self.enc_graphs[slot]
        if g is None:
            m.ext.encoder_forward(self.enc_descs[slot])  # warm (first launches set kernel attributes)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                m.ext.encoder_forward(self.enc_descs[slot])
            self.enc_graphs[slot] = g
        g.replay()

    # ---- decode ----------------------------------------------------------------------------
    def _chunk_graph(self, n):
        """CUDA graph of `chunk` steps of the first n clips, captured on first use. The warm-up steps
        before the capture advance the clips' state, so call this only before `prompt` resets it."""
        g = self.graphs.get(n)
        if g is None:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self.model.ext.batch_decoder_step(self._desc(n), self.chunk)
            torch.cuda.current_stream().wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.model.ext.batch_decoder_step(self._desc(n), self.chunk)
            self.graphs[n] = g
        return g

    def prompt(self, n):
        """Resets the first n clips and runs the prompt steps (the last one yields each clip's first token)."""
        self.state[:n].zero_()
        self.model.ext.batch_decoder_step(self._desc(n), self.model.dec_desc.prompt_len)

    def steps(self, n, count):
        """`count` further decode steps of the first n clips (whole-chunk graphs, then the remainder)."""
        if count >= self.chunk:
            g = self.graphs[n]
            for _ in range(count // self.chunk):
                g.replay()
        if count % self.chunk:
            self.model.ext.batch_decoder_step(self._desc(n), count % self.chunk)

    def prepare(self, n):
        """Captures, before any use, the encoder graphs of slots 0..n-1 and the chunk graph of n clips
        (the warm-up launches they need change this decoder's state)."""
        m = self.model
        for slot in range(n):
            if self.enc_graphs[slot] is None:
                m.ext.encoder_forward(self.enc_descs[slot])
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    m.ext.encoder_forward(self.enc_descs[slot])
                self.enc_graphs[slot] = g
        self._chunk_graph(n)
        torch.cuda.synchronize()

    def decode(self, n, n_tokens):
        """Prompt + n_tokens - 1 steps of the first n clips, whose cross caches are already filled.
        Clip c's tokens are then self.tokens[c, :n_tokens]."""
        if n_tokens - 1 >= self.chunk:
            self._chunk_graph(n)
        self.prompt(n)
        self.steps(n, max(0, n_tokens - 1))


class HostStaging:
    """Pinned host buffers for clips copied in asynchronously: buffer k is rewritten only after the
    copy that last read it has completed."""

    def __init__(self, count, n_samples):
        self.bufs = [torch.zeros(n_samples, dtype=torch.float32).pin_memory() for _ in range(count)]
        self.events = [None] * count
        self.next = 0

    def copy_in(self, audio, dst, stream):
        k = self.next
        self.next = (k + 1) % len(self.bufs)
        if self.events[k] is not None:
            self.events[k].synchronize()
        buf = self.bufs[k].numpy()
        buf[:audio.size] = audio
        buf[audio.size:] = 0.0
        dst.copy_(self.bufs[k], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.events[k] = ev


@torch.inference_mode()
def run_clips(model, decoders, waves, n_tokens, host_audio=None, staging=None):
    """Decodes many clips through several batched decoders, each on its own CUDA stream.

    Clips are taken in order, `decoders[0].clips` at a time (group g uses decoders[g % len(decoders)],
    each decoder on its own stream). On the front-end stream the log-mel and encoders of the next
    groups run while the decode streams decode the current ones, so the tensor-core encoder and
    several latency-bound decodes share the GPU. waves: device
    float32 [n, 480000], or None with host_audio (float32 numpy clips, copied in on the front-end
    stream through `staging`, a HostStaging). Returns the token tensor [n, max_pos] on the host (clip
    i's tokens in its first n_tokens[i] entries) and per-clip (log-mel, encoder) device times in s.
    """
    clips = decoders[0].clips
    n_all = len(n_tokens)
    groups = [list(range(g, min(g + clips, n_all))) for g in range(0, n_all, clips)]
    for bd in decoders:
        bd.prepare(clips)
    for g, grp in enumerate(groups):
        if len(grp) != clips:
            decoders[g % len(decoders)].prepare(len(grp))
    cur = torch.cuda.current_stream()
    front = torch.cuda.Stream()
    backs = [torch.cuda.Stream() for _ in decoders]  # each decoder decodes on its own stream
    front.wait_stream(cur)
    for b in backs:
        b.wait_stream(cur)
    tokens = torch.zeros(n_all, model.max_pos, dtype=torch.long).pin_memory()
    enc_done = [torch.cuda.Event() for _ in groups]
    dec_done = [torch.cuda.Event() for _ in groups]
    stage_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_all)]
    nd = len(decoders)
    for g, grp in enumerate(groups):
        bd = decoders[g % nd]
        with torch.cuda.stream(front):
            if g >= nd:
                front.wait_event(dec_done[g - nd])  # the slot set of group g - nd is free again
            for c, i in enumerate(grp):
                stage_ev[i][0].record(front)
                if waves is not None:
                    model.wave.copy_(waves[i])
                else:
                    staging.copy_in(host_audio[i], model.wave, front)
                model.run_mel()
                stage_ev[i][1].record(front)
                bd.encoder_slot(c)
                stage_ev[i][2].record(front)
            enc_done[g].record(front)
        back = backs[g % len(backs)]
        with torch.cuda.stream(back):
            back.wait_event(enc_done[g])
            bd.decode(len(grp), max(n_tokens[i] for i in grp))
            tokens[grp[0]:grp[-1] + 1].copy_(bd.tokens[:len(grp)], non_blocking=True)
            dec_done[g].record(back)
    cur.wait_stream(front)
    for b in backs:
        cur.wait_stream(b)
    torch.cuda.synchronize()
    times = [(e[0].elapsed_time(e[1]) / 1e3, e[1].elapsed_time(e[2]) / 1e3) for e in stage_ev]
    return tokens, times
