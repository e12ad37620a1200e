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
