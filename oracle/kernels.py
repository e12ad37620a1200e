"""numpy restatement of the reference's decode kernels and torch ops (test infrastructure).

fp16 tensors are numpy float16; math runs in float64 unless noted, and results are rounded to fp16
at the points where the reference stores fp16.
"""

import numpy as np

HIDDEN, HEAD_DIM, SPLIT_KEYS = 1280, 64, 64


def f16(x):
    return np.asarray(x, dtype=np.float64).astype(np.float16)


def add_layernorm(h, x, gamma, beta, eps=1e-5):
    """custom/kernels/whisper_kernels.cu:217-267: h <- fp16(h + x) (when x given), y = LN(h).

    Returns (h_new fp16, y fp16). Two-pass mean / biased variance as the kernel does."""
    h = np.asarray(h, np.float16).reshape(-1)
    r = h.astype(np.float64)
    if x is not None:
        r = f16(r + np.asarray(x, np.float16).reshape(-1).astype(np.float64)).astype(np.float64)
    mean = r.mean()
    var = ((r - mean) ** 2).mean()
    y = (r - mean) / np.sqrt(var + eps) * gamma.astype(np.float64) + beta.astype(np.float64)
    return f16(r), f16(y)


def decode_attention(q, k, v, length_pos=None, k_new=None, v_new=None, scale=HEAD_DIM ** -0.5):
    """custom/kernels/whisper_kernels.cu:108-213 / host :300-339.

    q [heads*64] fp16, k/v [heads, max_len, 64] fp16 (copied, not mutated). With length_pos = pos
    the row pos is replaced by k_new/v_new and keys 0..pos attend; else all max_len keys.
    Returns (out float64 [heads*64], k_after, v_after)."""
    k = np.array(k, dtype=np.float16, copy=True)
    v = np.array(v, dtype=np.float16, copy=True)
    heads, max_len, _ = k.shape
    if length_pos is not None:
        k[:, length_pos] = np.asarray(k_new, np.float16).reshape(heads, HEAD_DIM)
        v[:, length_pos] = np.asarray(v_new, np.float16).reshape(heads, HEAD_DIM)
        length = length_pos + 1
    else:
        length = max_len
    qh = np.asarray(q, np.float16).reshape(heads, HEAD_DIM).astype(np.float64)
    s = np.einsum('hd,hld->hl', qh, k[:, :length].astype(np.float64)) * scale
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    out = np.einsum('hl,hld->hd', p, v[:, :length].astype(np.float64)).reshape(-1)
    return out, k, v


def pack_score(value, index):
    """custom/kernels/whisper_kernels.cu:22-26: order-preserving (fp32 score, ~index) u64 key."""
    u = np.float32(value).view(np.uint32)
    u = np.uint32(~u) if u & np.uint32(0x80000000) else np.uint32(u | np.uint32(0x80000000))
    return (np.uint64(u) << np.uint64(32)) | np.uint64(0xFFFFFFFF - int(index))


def unpack_index(key):
    return 0xFFFFFFFF - (int(key) & 0xFFFFFFFF)


def argmax_first(logits, suppress=None):
    """torch.argmax semantics on fp16 logits (first index of the maximum), masked by suppress."""
    vals = np.asarray(logits, np.float16).astype(np.float32).copy()
    if suppress is not None:
        vals[np.asarray(suppress, bool)] = -np.inf
    return int(np.argmax(vals))


def lm_head_logits(h, w):
    """Logits rounded to fp16 (whisper_kernels.cu:70-71), accumulated in float64 here."""
    return f16(np.asarray(w, np.float16).astype(np.float64) @ np.asarray(h, np.float16).reshape(-1).astype(np.float64))


def argmax_finalize(best_key, tokens, state, cur, max_pos):
    """custom/kernels/whisper_kernels.cu:90-100 on int64 numpy arrays (mutated in place)."""
    tok = 0xFFFFFFFF - (int(best_key) & 0xFFFFFFFF)
    n = int(state[1])
    if n < max_pos and n < len(tokens):
        tokens[n] = tok
    state[1] = n + 1 if n < max_pos else n
    state[0] = state[0] + 1 if state[0] + 1 < max_pos else max_pos - 1
    cur[0] = tok
    return tok


def embed_pos(embed, pos_embed, ids, positions):
    """custom/model.py:110: fp16(embed[id] + pos_embed[pos]) (exact: one fp16 rounding of an exact sum)."""
    e = np.asarray(embed, np.float16)[np.asarray(ids)].astype(np.float32)
    p = np.asarray(pos_embed, np.float16)[np.asarray(positions)].astype(np.float32)
    return (e + p).astype(np.float16)


def gelu(x):
    """Exact-erf GELU (F.gelu default, custom/model.py:120) in float64."""
    from scipy.special import erf
    x = np.asarray(x, np.float64)
    return x * 0.5 * (1.0 + erf(x / np.sqrt(2.0)))


def linear(x, w, b=None):
    """F.linear with fp32 accumulation and one fp16 rounding (cuBLAS GEMV in custom/model.py)."""
    y = np.asarray(w, np.float16).astype(np.float64) @ np.asarray(x, np.float16).reshape(-1).astype(np.float64)
    if b is not None:
        y = y + np.asarray(b, np.float16).astype(np.float64)
    return f16(y)


def lm_quantize(w):
    """Checker for fw_lm_quantize (no reference counterpart: the reference streams the fp16 LM head
    every step, custom/kernels/whisper_kernels.cu:30-86). Per row: s = fp32(max|w| / 127) (1 for an
    all-zero row), q = rint(fp32(w / s)) clipped to +-127, a = max|w - s q| + 1e-5 max|w|,
    c2 = 0.51 s sum|q|, both in float64 (the device rounds them up to fp32)."""
    w32 = np.asarray(w, np.float16).astype(np.float32)
    wmax = np.abs(w32).max(1)
    s = np.where(wmax > 0, wmax / np.float32(127), np.float32(1)).astype(np.float32)
    q = np.clip(np.rint(w32 / s[:, None]), -127, 127).astype(np.int8)
    err = np.abs(w32.astype(np.float64) - q.astype(np.float64) * s[:, None].astype(np.float64)).max(1)
    a = err + 1e-5 * wmax.astype(np.float64)
    c2 = 0.51 * s.astype(np.float64) * np.abs(q.astype(np.int64)).sum(1)
    return q, s, a, c2


def lm_bounds(x, q, s, a, c2, xq_max=8191):
    """The pass-1 quantities of the pruned LM head for fp16 x: (approx, bound) per row, float64,
    such that |w_r . x - approx_r| <= bound_r (fp32 rounding slack of the device omitted)."""
    x = np.asarray(x, np.float16).astype(np.float64).reshape(-1)
    xmax = np.abs(x).max()
    sx = xmax / xq_max if xmax > 0 else 0.0
    xq = np.clip(np.rint(x / sx), -xq_max, xq_max) if xmax > 0 else np.zeros_like(x)
    S = q.astype(np.int64) @ xq.astype(np.int64)
    approx = s.astype(np.float64) * sx * S
    bound = np.abs(x).sum() * a + sx * c2 + 4e-7 * np.abs(approx)
    return approx, bound


def lm_prune_rows(approx, bound, suppress, rows_per_block):
    """Rows kept for exact rescoring: per block of rows_per_block rows, U_r >= T - m with
    T = max L_r over unsuppressed rows and m = 2^-9 (|T| + 2 max bound) + 2^-23 (every unsuppressed
    row of the block when |T| >= 32768 or T is not finite)."""
    keep = np.zeros(approx.size, bool)
    sup = np.asarray(suppress, bool)
    for b0 in range(0, approx.size, rows_per_block):
        sl = slice(b0, min(approx.size, b0 + rows_per_block))
        ok = ~sup[sl]
        if not ok.any():
            continue
        lo, hi = approx[sl] - bound[sl], approx[sl] + bound[sl]
        t = lo[ok].max()
        bm = bound[sl][ok].max()
        if not np.isfinite(t) or abs(t) >= 32768 or not bm < 32768:
            keep[sl] = ok
            continue
        keep[sl] = ok & (hi >= t - (2.0 ** -9 * (abs(t) + 2 * bm) + 2.0 ** -23))
    return keep
