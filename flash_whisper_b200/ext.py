"""Kernel boundary for PyTorch callers: the drop-in for the reference's custom/ext.py.

`load_ext()` returns an object exposing the reference's four kernels with the same names, argument
order and error behaviour as its pybind module (custom/kernels/whisper_kernels.cu:278-363, loaded by
custom/ext.py:13-18):

    add_layernorm(h, x, gamma, beta, y, eps)
    decode_attention(q, k, v, out, len_state, k_new, v_new, part_m, part_l, part_acc, scale)
    lm_head_argmax(h, w, suppress, best)
    argmax_finalize(best, tokens, state, cur, max_pos)

plus the fused decode, log-mel and encoder ops of this package. Each method validates dtype,
device, contiguity and shape like the reference's TORCH_CHECKs (RuntimeError with the same
messages), then calls the C ABI of libflashwhisper.so with raw pointers on the current CUDA
stream. There is no CPU path: without a CUDA tensor the checks fail.
"""

import ctypes

import torch

from . import _lib

HIDDEN, HEAD_DIM, SPLIT_KEYS = 1280, 64, 64


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _check_half(t, name):
    _check(t.is_cuda and t.is_contiguous() and t.dtype == torch.float16, f'{name} must be contiguous CUDA fp16')


def _check_cuda(t, dtype, name, what):
    _check(t.is_cuda and t.is_contiguous() and t.dtype == dtype, f'{name} must be contiguous CUDA {what}')


class Ext:
    """Reference-compatible kernel module backed by libflashwhisper.so."""

    SPLIT_KEYS = SPLIT_KEYS

    def __init__(self):
        self.lib = _lib.lib()

    # ---- reference surface -----------------------------------------------------------------
    def add_layernorm(self, h, x, gamma, beta, y, eps):
        """h += x (stored back in fp16) when x is given, then y = LayerNorm(h)."""
        for t, n in ((h, 'h'), (gamma, 'gamma'), (beta, 'beta'), (y, 'y')):
            _check_half(t, n)
        _check(h.numel() == HIDDEN, f'hidden size must be {HIDDEN}')
        if x is not None:
            _check_half(x, 'x')
        _lib.call('fw_add_layernorm', _ptr(h), _ptr(x), _ptr(gamma), _ptr(beta), _ptr(y), HIDDEN, float(eps),
                  _stream())

    def decode_attention(self, q, k, v, out, len_state, k_new, v_new, part_m, part_l, part_acc, scale):
        """Split-K single-query attention; self attention (len_state given) also writes k_new/v_new."""
        for t, n in ((q, 'q'), (k, 'k'), (v, 'v'), (out, 'out')):
            _check_half(t, n)
        _check(k.dim() == 3 and k.size(2) == HEAD_DIM and k.shape == v.shape, 'k, v must be [heads, max_len, 64]')
        heads, max_len = k.size(0), k.size(1)
        splits = -(-max_len // SPLIT_KEYS)
        _check(q.numel() == heads * HEAD_DIM and out.numel() == heads * HEAD_DIM, 'q, out must be [heads * 64]')
        _check((k_new is None) == (v_new is None) == (len_state is None),
               'len_state, k_new and v_new must be given together')
        if k_new is not None:
            _check_half(k_new, 'k_new')
            _check_half(v_new, 'v_new')
            _check(k_new.numel() == heads * HEAD_DIM and v_new.numel() == heads * HEAD_DIM,
                   'k_new, v_new must be [heads, 64]')
            _check(len_state.is_cuda and len_state.dtype == torch.long, 'len_state must be CUDA int64')
        for t in (part_m, part_l, part_acc):
            _check(t.is_cuda and t.is_contiguous() and t.dtype == torch.float32,
                   'workspace must be contiguous CUDA fp32')
        _check(part_m.numel() >= heads * splits and part_l.numel() >= heads * splits
               and part_acc.numel() >= heads * splits * HEAD_DIM, f'workspace too small for {splits} splits')
        _lib.call('fw_decode_attention', _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(len_state), _ptr(k_new),
                  _ptr(v_new), _ptr(part_m), part_m.numel(), _ptr(part_l), part_l.numel(), _ptr(part_acc),
                  part_acc.numel(), heads, max_len, float(scale), _stream())

    def decode_attention_noalloc(self, q, k, v, out, len_state, k_new, v_new, scale):
        """decode_attention without a workspace: the split partials live in the library's fixed device
        array (heads * ceil(max_len / 64) <= 2048; calls that overlap on the GPU race on it)."""
        for t, n in ((q, 'q'), (k, 'k'), (v, 'v'), (out, 'out')):
            _check_half(t, n)
        _check(k.dim() == 3 and k.size(2) == HEAD_DIM and k.shape == v.shape, 'k, v must be [heads, max_len, 64]')
        heads, max_len = k.size(0), k.size(1)
        _check(q.numel() == heads * HEAD_DIM and out.numel() == heads * HEAD_DIM, 'q, out must be [heads * 64]')
        _check((k_new is None) == (v_new is None) == (len_state is None),
               'len_state, k_new and v_new must be given together')
        if k_new is not None:
            _check_half(k_new, 'k_new')
            _check_half(v_new, 'v_new')
            _check(k_new.numel() == heads * HEAD_DIM and v_new.numel() == heads * HEAD_DIM,
                   'k_new, v_new must be [heads, 64]')
            _check(len_state.is_cuda and len_state.dtype == torch.long, 'len_state must be CUDA int64')
        _lib.call('fw_decode_attention_noalloc', _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(len_state), _ptr(k_new),
                  _ptr(v_new), heads, max_len, float(scale), _stream())

    def lm_head_argmax(self, h, w, suppress, best):
        """best <- max(best, packed key of the unsuppressed argmax of fp16(w @ h))."""
        _check_half(h, 'h')
        _check_half(w, 'w')
        _check(h.numel() == HIDDEN and w.dim() == 2 and w.size(1) == HIDDEN, f'hidden size must be {HIDDEN}')
        _check(suppress.dtype == torch.bool and suppress.numel() == w.size(0) and suppress.is_cuda
               and suppress.is_contiguous(), 'suppress must be bool [vocab]')
        _check(best.dtype == torch.long and best.numel() == 1 and best.is_cuda, 'best must be int64 [1]')
        _lib.call('fw_lm_head_argmax', _ptr(h), _ptr(w), _ptr(suppress), w.size(0), HIDDEN, _ptr(best), _stream())

    def lm_quantize(self, w):
        """(wq int8 [vocab, 1280], rp fp32 [vocab, 4]): the int8 LM head and per-row bounds that
        lm_head_argmax_q and the decode step's pruned argmax stream instead of w."""
        _check_half(w, 'w')
        _check(w.dim() == 2 and w.size(1) == HIDDEN, f'hidden size must be {HIDDEN}')
        wq = torch.empty(w.shape, dtype=torch.int8, device=w.device)
        rp = torch.empty(w.size(0), 4, dtype=torch.float32, device=w.device)
        _lib.call('fw_lm_quantize', _ptr(w), w.size(0), HIDDEN, _ptr(wq), _ptr(rp), _stream())
        return wq, rp

    def lm_head_argmax_q(self, h, w, wq, rp, suppress, best):
        """As lm_head_argmax (same key), streaming the lm_quantize output and recomputing exactly
        only the rows that can still win."""
        _check_half(h, 'h')
        _check_half(w, 'w')
        _check(h.numel() == HIDDEN and w.dim() == 2 and w.size(1) == HIDDEN, f'hidden size must be {HIDDEN}')
        _check(wq.dtype == torch.int8 and wq.shape == w.shape and wq.is_cuda and wq.is_contiguous(),
               'wq must be int8 like w')
        _check(rp.dtype == torch.float32 and rp.shape == (w.size(0), 4) and rp.is_cuda and rp.is_contiguous(),
               'rp must be fp32 [vocab, 4]')
        _check(suppress.dtype == torch.bool and suppress.numel() == w.size(0) and suppress.is_cuda
               and suppress.is_contiguous(), 'suppress must be bool [vocab]')
        _check(best.dtype == torch.long and best.numel() == 1 and best.is_cuda, 'best must be int64 [1]')
        _lib.call('fw_lm_head_argmax_q', _ptr(h), _ptr(w), _ptr(wq), _ptr(rp), _ptr(suppress), w.size(0), HIDDEN,
                  _ptr(best), _stream())

    def argmax_finalize(self, best, tokens, state, cur, max_pos):
        """Appends the decoded token, feeds it back, advances the position and resets best."""
        _check(tokens.dtype == torch.long and state.dtype == torch.long and cur.dtype == torch.long,
               'tokens, state and cur must be int64')
        _check(best.dtype == torch.long and best.numel() == 1, 'best must be int64 [1]')
        for t in (best, tokens, state, cur):
            _check(t.is_cuda and t.is_contiguous(), 'tokens, state and cur must be int64')
        _lib.call('fw_argmax_finalize', _ptr(best), _ptr(tokens), tokens.numel(), _ptr(state), _ptr(cur),
                  int(max_pos), _stream())

    # ---- fused / stand-alone decode ops ------------------------------------------------------
    def embed_pos(self, embed, pos_embed, ids, positions, out):
        """out[i] = fp16(embed[ids[i]] + pos_embed[positions[i]])."""
        for t, n in ((embed, 'embed'), (pos_embed, 'pos_embed'), (out, 'out')):
            _check_half(t, n)
        for t, n in ((ids, 'ids'), (positions, 'positions')):
            _check_cuda(t, torch.long, n, 'int64')
        n = ids.numel()
        _check(positions.numel() == n and out.numel() == n * embed.size(1) and pos_embed.size(1) == embed.size(1),
               'embed_pos: shape mismatch')
        _lib.call('fw_embed_pos', _ptr(embed), _ptr(pos_embed), _ptr(ids), _ptr(positions), _ptr(out), n,
                  embed.size(0), pos_embed.size(0), embed.size(1), _stream())

    def gelu(self, x, y):
        _check_half(x, 'x')
        _check_half(y, 'y')
        _check(x.numel() == y.numel(), 'gelu: x and y must have the same size')
        _lib.call('fw_gelu', _ptr(x), _ptr(y), x.numel(), _stream())

    def argmax_f16(self, logits, suppress, key, out_index):
        """out_index = first argmax of unsuppressed fp16 logits; key is an int64 scratch word (0)."""
        _check_half(logits, 'logits')
        if suppress is not None:
            _check(suppress.dtype == torch.bool and suppress.numel() == logits.numel() and suppress.is_cuda,
                   'suppress must be bool [n]')
        _check_cuda(key, torch.long, 'key', 'int64')
        _check_cuda(out_index, torch.long, 'out_index', 'int64')
        _lib.call('fw_argmax_f16', _ptr(logits), logits.numel(), _ptr(suppress), _ptr(key), _ptr(out_index),
                  _stream())

    def ln_gemv(self, h, gamma, beta, eps, w, b, out, act=0):
        """out = act(w @ LayerNorm(h) + b); act 0 none, 1 exact GELU."""
        for t, n in ((h, 'h'), (gamma, 'gamma'), (beta, 'beta'), (w, 'w'), (out, 'out')):
            _check_half(t, n)
        _check(h.numel() == HIDDEN and w.dim() == 2 and w.size(1) == HIDDEN, f'hidden size must be {HIDDEN}')
        _check(out.numel() == w.size(0), 'ln_gemv: out must have w.size(0) elements')
        if b is not None:
            _check_half(b, 'b')
        _lib.call('fw_ln_gemv', _ptr(h), _ptr(gamma), _ptr(beta), float(eps), _ptr(w), _ptr(b), _ptr(out),
                  w.size(0), HIDDEN, int(act), _stream())

    def gemv_residual(self, x, w, b, h):
        """h = fp16(h + fp16(w @ x + b))."""
        for t, n in ((x, 'x'), (w, 'w'), (h, 'h')):
            _check_half(t, n)
        _check(w.dim() == 2 and w.size(1) == x.numel() and h.numel() == w.size(0), 'gemv_residual: shape mismatch')
        if b is not None:
            _check_half(b, 'b')
        _lib.call('fw_gemv_residual', _ptr(x), x.numel(), _ptr(w), _ptr(b), _ptr(h), w.size(0), _stream())

    # ---- front end and encoder ---------------------------------------------------------------
    def log_mel(self, wave, filters, scratch, clip_max, out, layout=0):
        """fp16 log-mel of fp32 wave [batch, n_samples]; layout 0 [b,128,T], 1 [b,T+2,128] padded."""
        _check_cuda(wave, torch.float32, 'wave', 'fp32')
        _check_cuda(filters, torch.float32, 'filters', 'fp32')
        _check_cuda(scratch, torch.float32, 'scratch', 'fp32')
        _check(clip_max.is_cuda and clip_max.dtype == torch.int32, 'clip_max must be CUDA int32')
        _check_half(out, 'out')
        wave2 = wave.view(-1, wave.size(-1))
        batch, n = wave2.shape
        frames = n // 160
        _check(filters.shape == (201, 128), 'filters must be [201, 128]')
        _check(scratch.numel() >= batch * 128 * frames and clip_max.numel() >= batch, 'log_mel: scratch too small')
        want = batch * 128 * frames if layout == 0 else batch * (frames + 2) * 128
        _check(out.numel() == want, 'log_mel: output has the wrong size')
        _lib.call('fw_log_mel', _ptr(wave2), batch, n, _ptr(filters), _ptr(scratch), _ptr(clip_max), _ptr(out),
                  int(layout), _stream())

    def gemm(self, a, b, bias, c, epilogue=_lib.FW_EPI_BIAS, r=None, scale=1.0, scale_cols=0, m=None):
        """c = epilogue(a @ b.T + bias) on tcgen05 tensor cores."""
        _check_half(a, 'a')
        _check_half(b, 'b')
        _check_half(c, 'c')
        m = a.size(0) if m is None else m
        n, k = b.shape
        ldc = c.stride(0) if c.dim() == 2 else 0
        ldr = r.stride(0) if r is not None else 0
        _lib.call('fw_gemm_f16', _ptr(a), a.stride(0), _ptr(b), b.stride(0), _ptr(bias), _ptr(c), ldc, _ptr(r), ldr,
                  m, n, k, int(epilogue), float(scale), int(scale_cols), _stream())

    def conv1d_k3(self, x_padded, w_taps, bias, out, stride, epilogue=_lib.FW_EPI_BIAS_GELU, r=None, m=None):
        """Conv1d(k=3, pad=1) over a zero-padded time-major input as an implicit tcgen05 GEMM."""
        _check_half(x_padded, 'x')
        _check_half(w_taps, 'w')
        rows, ch = x_padded.shape
        n = w_taps.size(0)
        m = (rows - 2 + stride - 1) // stride if m is None else m
        ldr = r.stride(0) if r is not None else 0
        _lib.call('fw_conv1d_k3_f16', _ptr(x_padded), ch, rows, int(stride), _ptr(w_taps), _ptr(bias), _ptr(out),
                  out.stride(0), _ptr(r), ldr, m, n, int(epilogue), _stream())

    def layernorm_rows(self, x, g, b, y, eps):
        for t, n in ((x, 'x'), (g, 'g'), (b, 'b'), (y, 'y')):
            _check_half(t, n)
        _lib.call('fw_layernorm_rows', _ptr(x), _ptr(g), _ptr(b), _ptr(y), x.size(0), x.size(1), float(eps),
                  _stream())

    def encoder_attention(self, qkv, out, heads, kcol=HIDDEN, vcol=2 * HIDDEN, vt=None):
        """vt: optional fp16 scratch [heads * 64, round_up(seq, 8)] for V transposed (allocated if None)."""
        _check_half(qkv, 'qkv')
        _check_half(out, 'out')
        if vt is None:
            vt = torch.empty(int(heads) * 64, -(-qkv.size(0) // 8) * 8, dtype=torch.float16, device=qkv.device)
        _check_half(vt, 'vt')
        _lib.call('fw_encoder_attention', _ptr(qkv), qkv.stride(0), int(kcol), int(vcol), _ptr(out), qkv.size(0),
                  int(heads), _ptr(vt), _stream())

    def decoder_step(self, desc, steps=1):
        _lib.call('fw_decoder_step', ctypes.byref(desc), int(steps), _stream())

    def batch_decoder_step(self, desc, steps=1):
        """`steps` decode steps of every clip of a batched decoder descriptor (_lib.BatchDecoder)."""
        _lib.call('fw_batch_decoder_step', ctypes.byref(desc), int(steps), _stream())

    def batch_decoder_launch(self, desc, layer, block):
        """One launch of the batched step (0 qkv, 1 self attention, 2 out_proj, 3 cross q, 4 cross
        attention, 5 cross out_proj, 6 fc1, 7 fc2, 8 LM head)."""
        _lib.call('fw_batch_decoder_launch', ctypes.byref(desc), int(layer), int(block), _stream())

    def decoder_launch(self, desc, layer, block):
        """One launch of the decode step (block 0 self, 1 cross, 2 fc1, 3 fc2, 4 LM head)."""
        _lib.call('fw_decoder_launch', ctypes.byref(desc), int(layer), int(block), _stream())

    def decoder_step_trace(self, desc, trace):
        """One decode step that also records each block's output into `trace` (fp16, at least
        n_layers * TRACE_LAYER + 1280 elements; layout in include/flash_whisper.h)."""
        _check_half(trace, 'trace')
        need = desc.n_layers * _lib.TRACE_LAYER + HIDDEN
        if trace.numel() < need:
            raise RuntimeError(f'trace must hold at least {need} fp16 elements')
        _lib.call('fw_decoder_step_trace', ctypes.byref(desc), _ptr(trace), _stream())

    def encoder_forward(self, desc):
        _lib.call('fw_encoder_forward', ctypes.byref(desc), _stream())

    def device_error(self, clear=True):
        bits = ctypes.c_uint(0)
        _lib.call('fw_device_error', ctypes.byref(bits), int(clear))
        return bits.value


_EXT = None


def load_ext(verbose=False):
    """Returns the kernel module (the library is built ahead of time by flash_whisper_b200.build)."""
    global _EXT
    if _EXT is None:
        _EXT = Ext()
    return _EXT
