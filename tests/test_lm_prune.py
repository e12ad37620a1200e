"""CPU tests of the pruned LM-head argmax (fw_lm_head_argmax_q): the per-row bound holds, and the
rows kept for exact rescoring always contain the argmax the exact kernel returns, including
planted fp16 ties and suppressed rows."""

import numpy as np
import pytest

from oracle import kernels as K

V, D = 4096, 1280


def _w(rng, scale=0.02):
    return (rng.standard_normal((V, D)) * scale).astype(np.float16)


def _ln_like(rng):
    h = rng.standard_normal(D)
    return ((h - h.mean()) / h.std()).astype(np.float16)


def test_quantize_reconstructs_within_a():
    rng = np.random.default_rng(0)
    w = _w(rng)
    w[3] = 0  # all-zero row
    q, s, a, c2 = K.lm_quantize(w)
    assert q.dtype == np.int8 and np.abs(q.astype(int)).max() <= 127
    err = np.abs(w.astype(np.float64) - q * s[:, None].astype(np.float64)).max(1)
    assert np.all(err <= a) and np.all(err <= s * (0.5 + 1e-5))  # fp32 division can cross a midpoint
    assert s[3] == 1 and not q[3].any() and a[3] == 0 and c2[3] == 0


@pytest.mark.parametrize('kind', ['ln', 'adversarial', 'sparse'])
def test_bound_holds(kind):
    rng = np.random.default_rng(1)
    w = _w(rng)
    q, s, a, c2 = K.lm_quantize(w)
    for trial in range(4):
        if kind == 'ln':
            x = _ln_like(rng)
        elif kind == 'adversarial':  # x aligned with row r's quantisation error: the L1 bound is tight there
            r = rng.integers(V)
            e = w[r].astype(np.float64) - q[r] * np.float64(s[r])
            x = (np.sign(e) * 3.0).astype(np.float16)
        else:
            x = np.zeros(D, np.float16)
            x[rng.integers(D, size=5)] = rng.standard_normal(5) * 8
        exact = w.astype(np.float64) @ x.astype(np.float64)
        approx, bound = K.lm_bounds(x, q, s, a, c2)
        assert np.all(np.abs(exact - approx) <= bound)


def _exact_argmax(w, x, sup):
    logits = K.lm_head_logits(x, w).astype(np.float32)
    logits[sup] = -np.inf
    return int(np.argmax(logits))


@pytest.mark.parametrize('seed', range(6))
def test_kept_rows_contain_the_argmax(seed):
    rng = np.random.default_rng(seed)
    w = _w(rng)
    x = _ln_like(rng)
    sup = rng.random(V) < 0.01
    if seed % 2:  # plant exact fp16 ties across blocks: the lower index must stay reachable
        top = int(np.argmax(K.lm_head_logits(x, w).astype(np.float32)))
        for r in (5, 1000, 3000):
            w[r] = w[top]
        sup[[5, 1000, 3000, top]] = False
    q, s, a, c2 = K.lm_quantize(w)
    approx, bound = K.lm_bounds(x, q, s, a, c2)
    keep = K.lm_prune_rows(approx, bound, sup, rows_per_block=28)
    want = _exact_argmax(w, x, sup)
    assert keep[want]
    logits = K.lm_head_logits(x, w).astype(np.float32)
    logits[~keep] = -np.inf
    assert int(np.argmax(logits)) == want
    assert keep.sum() < V // 4  # the bound actually prunes on LayerNorm-like inputs


def test_zero_input_keeps_every_unsuppressed_row():
    rng = np.random.default_rng(9)
    w = _w(rng)
    q, s, a, c2 = K.lm_quantize(w)
    sup = np.zeros(V, bool)
    sup[:10] = True
    approx, bound = K.lm_bounds(np.zeros(D, np.float16), q, s, a, c2)
    keep = K.lm_prune_rows(approx, bound, sup, rows_per_block=28)
    assert np.array_equal(keep, ~sup)


def test_overflowing_logits_keep_every_row():
    rng = np.random.default_rng(10)
    w = _w(rng, scale=6.0)
    x = (_ln_like(rng).astype(np.float32) * 60).astype(np.float16)
    q, s, a, c2 = K.lm_quantize(w)
    approx, bound = K.lm_bounds(x, q, s, a, c2)
    keep = K.lm_prune_rows(approx, bound, np.zeros(V, bool), rows_per_block=28)
    blocks_over = [b for b in range(0, V, 28) if (approx[b:b + 28] - bound[b:b + 28]).max() >= 32768]
    assert blocks_over and all(keep[b:b + 28].all() for b in blocks_over)
