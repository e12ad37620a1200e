"""Load-time kernel self-check (the role of custom/selftest.py:32-88 in the reference).

`run_selftest(ext)` runs every kernel of the drop-in surface once on small seeded inputs and checks
it against a float32 PyTorch computation of the same op on the same GPU; `run_selftest(ext, model)`
also runs one traced decode step of the model's own fused decoder (fw_decoder_step_trace) and checks
its first layer block by block. It returns the reference's result shape, {'ok': bool, 'checks':
[{'name', 'max_err', 'ok'}, ...]}, which CustomModel stores as `model.selftest`.

Tolerances: fp16 activations within rtol 1e-2 / atol 1e-3 (reported as the largest excess over that
bound, 0 when inside it); cache writes, token bookkeeping and the pruned-vs-full LM-head argmax
key are exact. The interface names SPLIT_KEYS, workspace and run_selftest are those
custom/model.py:18 imports.

`python -m flash_whisper_b200.selftest --out DIR` writes the result as JSON.
"""

import argparse
import json
from pathlib import Path

import torch
import torch.nn.functional as F

SPLIT_KEYS = 64  # keys per attention split (whisper_kernels.cu split size)
_D, _HD = 1280, 64
_RTOL, _ATOL = 1e-2, 1e-3


def workspace(heads, splits, device='cuda'):
    """fp32 split partials of decode_attention: (max [heads*splits], sum [heads*splits],
    value accumulators [heads*splits*64])."""
    n = int(heads) * int(splits)
    return (torch.empty(n, device=device), torch.empty(n, device=device), torch.empty(n * _HD, device=device))


class _Checks:
    def __init__(self):
        self.items = []

    def close(self, name, got, want):
        """Largest amount by which |got - want| exceeds atol + rtol |want| (0 when within)."""
        got, want = got.float().flatten(), want.float().flatten()
        excess = ((got - want).abs() - (_ATOL + _RTOL * want.abs())).clamp_min(0)
        err = float(excess.max()) if excess.numel() else 0.0
        if not torch.isfinite(got).all():
            err = float('inf')
        self.items.append({'name': name, 'max_err': err, 'ok': err == 0.0})

    def exact(self, name, ok, detail=0.0):
        self.items.append({'name': name, 'max_err': float(detail), 'ok': bool(ok)})

    def result(self):
        return {'ok': all(c['ok'] for c in self.items), 'checks': self.items}


def _ln(x, g, b, eps=1e-5):
    return F.layer_norm(x.float(), (x.shape[-1],), g.float(), b.float(), eps)


def _attend(q, k, v, length, scale):
    """float32 single-query attention per head: q [heads, 64], k/v [heads, >=length, 64]."""
    s = torch.einsum('hd,hld->hl', q.float(), k[:, :length].float()) * scale
    return torch.einsum('hl,hld->hd', torch.softmax(s, -1), v[:, :length].float())


def _check_kernels(ext, c, gen, dev):
    half = torch.float16

    def randn(*shape, std=1.0):
        return (torch.randn(*shape, generator=gen, device=dev) * std).to(half)

    # residual add + LayerNorm: the residual write is exact, the normalised row within tolerance
    h, x = randn(1, _D), randn(1, _D)
    gamma, beta = randn(_D, std=0.3) + 1, randn(_D, std=0.3)
    want_h = (h.float() + x.float()).half()
    y = torch.empty_like(h)
    ext.add_layernorm(h, x, gamma, beta, y, 1e-5)
    c.exact('add_layernorm residual write', torch.equal(h, want_h))
    c.close('add_layernorm', y, _ln(want_h, gamma, beta))

    # split-K attention: lengths on both sides of each 64-key split boundary, the last cache row,
    # and the 1500-key cross cache; the workspace-free entry point must agree bit for bit
    heads, max_len, scale = 20, 448, _HD ** -0.5
    ws = workspace(heads, -(-1500 // SPLIT_KEYS), dev)
    for length in (1, 2, 64, 65, 128, 129, 333, 448):
        pos = length - 1
        q = randn(heads * _HD)
        k, v = randn(heads, max_len, _HD), randn(heads, max_len, _HD)
        k_new, v_new = randn(heads, 1, _HD), randn(heads, 1, _HD)
        k_want, v_want = k.clone(), v.clone()
        k_want[:, pos], v_want[:, pos] = k_new[:, 0], v_new[:, 0]
        k2, v2 = k.clone(), v.clone()
        out, out2 = torch.empty_like(q), torch.empty_like(q)
        state = torch.tensor([pos, 0], device=dev, dtype=torch.long)
        ext.decode_attention(q, k, v, out, state, k_new, v_new, *ws, scale)
        ext.decode_attention_noalloc(q, k2, v2, out2, state, k_new, v_new, scale)
        c.close(f'self attention L={length}', out, _attend(q.view(heads, _HD), k_want, v_want, length, scale))
        c.exact(f'cache write L={length}', torch.equal(k, k_want) and torch.equal(v, v_want))
        c.exact(f'noalloc attention L={length}', torch.equal(out, out2) and torch.equal(k2, k_want))
    q = randn(heads * _HD)
    kc, vc = randn(heads, 1500, _HD), randn(heads, 1500, _HD)
    out = torch.empty_like(q)
    ext.decode_attention(q, kc, vc, out, None, None, None, *ws, scale)
    c.close('cross attention 1500', out, _attend(q.view(heads, _HD), kc, vc, 1500, scale))

    # LM-head argmax: the chosen row is a maximum of the fp16 logits (up to an fp16 tie), the pruned
    # int8 head returns the same packed key, and the finalize bookkeeping is exact
    vocab = 51866
    row = _ln(randn(1, _D), torch.ones(_D, device=dev), torch.zeros(_D, device=dev)).half()
    w = randn(vocab, _D, std=0.05)
    suppress = torch.rand(vocab, generator=gen, device=dev) < 0.02
    logits = (row.float() @ w.float().T)[0].half().float().masked_fill(suppress, float('-inf'))
    best = torch.zeros(1, device=dev, dtype=torch.long)
    ext.lm_head_argmax(row, w, suppress, best)
    key_full = int(best)
    token = 0xFFFFFFFF - (key_full & 0xFFFFFFFF)
    top = float(logits.max())
    gap = top - float(logits[token]) if 0 <= token < vocab else float('inf')
    c.exact('lm_head_argmax is a maximum', gap <= 2 * 2.0 ** -10 * max(1.0, abs(top)), gap)
    wq, rp = ext.lm_quantize(w)
    best.zero_()
    ext.lm_head_argmax_q(row, w, wq, rp, suppress, best)
    c.exact('pruned lm_head_argmax key', int(best) == key_full)
    tokens = torch.zeros(16, device=dev, dtype=torch.long)
    state = torch.tensor([9, 5], device=dev, dtype=torch.long)
    cur = torch.zeros(1, device=dev, dtype=torch.long)
    ext.argmax_finalize(best, tokens, state, cur, 448)
    ok = (int(tokens[5]) == token and int(cur) == token and state.tolist() == [10, 6] and int(best) == 0
          and int(tokens.count_nonzero()) == (1 if token else 0))
    c.exact('argmax_finalize bookkeeping', ok)


def _check_decoder(ext, model, c, gen, dev):
    """One traced step of the model's fused decoder at position 70 (a 71-key self attention over two
    splits) on seeded caches; layer 0 is recomputed in float32 from the packed weights."""
    from . import _lib
    d = model.dims
    pos, tok = 70, 1234 % d.vocab
    saved = [t.clone() for t in (model.self_kv, model.cross_kv, model.state, model.cur, model.tokens)]
    try:
        model.self_kv.copy_((torch.randn(model.self_kv.shape, generator=gen, device=dev) * 0.5).half())
        model.cross_kv.copy_((torch.randn(model.cross_kv.shape, generator=gen, device=dev) * 0.5).half())
        model.state.copy_(torch.tensor([pos, 0]))
        model.cur.fill_(tok)
        k_before = model.self_kv[0, :, :, :pos].clone()
        trace = torch.zeros(d.decoder_layers * _lib.TRACE_LAYER + d.d_model, dtype=torch.float16, device=dev)
        ext.decoder_step_trace(model.dec_desc, trace)
        torch.cuda.synchronize()
        L, dec = model.dec.layers[0], model.dec
        heads, scale = d.heads, d.head_dim ** -0.5
        h0 = (dec.embed[tok].float() + dec.pos_embed[pos].float()).half()
        qkv = (_ln(h0, *L.ln1).half().float() @ L.qkv_w.float().T + L.qkv_b.float()).half()
        q, k, v = qkv.view(3, heads, d.head_dim)
        c.close('decoder cache write K', model.self_kv[0, 0, :, pos], k)
        c.close('decoder cache write V', model.self_kv[0, 1, :, pos], v)
        c.exact('decoder cache rows below the position untouched', torch.equal(model.self_kv[0, :, :, :pos], k_before))
        o = _attend(q, model.self_kv[0, 0], model.self_kv[0, 1], pos + 1, scale).half().flatten()
        t = trace[:_lib.TRACE_LAYER]
        o_gpu = t[_lib.TRACE_SELF_ATTN:_lib.TRACE_SELF_ATTN + d.d_model]
        c.close('decoder self attention', o_gpu, o)
        w_out = L.out[0].permute(1, 0, 2).reshape(d.d_model, d.d_model)  # head-major -> [out, in]
        h1 = (h0.float() + (o_gpu.float() @ w_out.float().T + L.out[1].float()).half().float()).half()
        h1_gpu = t[_lib.TRACE_H_SELF:_lib.TRACE_H_SELF + d.d_model]
        c.close('decoder self block residual', h1_gpu, h1)
        cq = (_ln(h1_gpu, *L.ln2).half().float() @ L.cross_q[0].float().T + L.cross_q[1].float()).half()
        co = _attend(cq.view(heads, d.head_dim), model.cross_kv[0, 0], model.cross_kv[0, 1], d.enc_len,
                     scale).half().flatten()
        co_gpu = t[_lib.TRACE_CROSS_ATTN:_lib.TRACE_CROSS_ATTN + d.d_model]
        c.close('decoder cross attention', co_gpu, co)
        h2_gpu = t[_lib.TRACE_H_CROSS:_lib.TRACE_H_CROSS + d.d_model]
        f = F.gelu((_ln(h2_gpu, *L.ln3).half().float() @ L.fc1[0].float().T + L.fc1[1].float()).half().float())
        c.close('decoder fc1 + gelu', t[_lib.TRACE_FFN:_lib.TRACE_FFN + d.ffn], f.half())
        ffn_gpu = t[_lib.TRACE_FFN:_lib.TRACE_FFN + d.ffn]
        h3 = (h2_gpu.float() + (ffn_gpu.float() @ L.fc2[0].float().T + L.fc2[1].float()).half().float()).half()
        c.close('decoder fc2 residual', t[_lib.TRACE_H_FFN:_lib.TRACE_H_FFN + d.d_model], h3)
        c.exact('decoder device error word', ext.device_error() == 0)
    finally:
        for dst, src in zip((model.self_kv, model.cross_kv, model.state, model.cur, model.tokens), saved):
            dst.copy_(src)
        torch.cuda.synchronize()


@torch.inference_mode()
def run_selftest(ext, model=None, seed=20240607):
    """Runs the kernel checks (and, with `model`, the traced decoder-step check)."""
    dev = 'cuda'
    gen = torch.Generator(device=dev).manual_seed(seed)
    c = _Checks()
    _check_kernels(ext, c, gen, dev)
    if model is not None:
        _check_decoder(ext, model, c, gen, dev)
    return c.result()


def main():
    from .ext import load_ext

    parser = argparse.ArgumentParser()
    parser.add_argument('--out', type=Path, required=True)
    args = parser.parse_args()
    args.out.mkdir(parents=True, exist_ok=True)
    result = run_selftest(load_ext())
    (args.out / 'selftest.json').write_text(json.dumps(result, indent=2) + '\n')
    print(json.dumps(result))


if __name__ == '__main__':
    main()
