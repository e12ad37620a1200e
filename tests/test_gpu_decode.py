"""GPU parity of the decode kernels: against the numpy oracle, PyTorch fp32, and the reference's own
kernels built from its source (oracle/_ref) on identical inputs."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import kernels as K

pytestmark = pytest.mark.gpu
HIDDEN, HEADS, HD, VOCAB = 1280, 20, 64, 51866


def _ws(splits=24):
    return (torch.empty(HEADS * splits, device='cuda'), torch.empty(HEADS * splits, device='cuda'),
            torch.empty(HEADS * splits * HD, device='cuda'))


def test_selftest_passes(ext):
    from flash_whisper_b200.selftest import run_selftest
    res = run_selftest(ext)
    assert res['ok'], res


def test_add_layernorm_vs_oracle_and_reference(ext, ref_ext):
    g = torch.Generator(device='cuda').manual_seed(1)
    for with_x in (True, False):
        h = torch.randn(1, HIDDEN, device='cuda', generator=g).half()
        x = torch.randn(1, HIDDEN, device='cuda', generator=g).half() if with_x else None
        gamma = torch.randn(HIDDEN, device='cuda', generator=g).half()
        beta = torch.randn(HIDDEN, device='cuda', generator=g).half()
        h_ref, y_ref = h.clone(), torch.empty_like(h)
        y = torch.empty_like(h)
        h2_np, y_np = K.add_layernorm(h.cpu().numpy(), None if x is None else x.cpu().numpy(), gamma.cpu().numpy(),
                                      beta.cpu().numpy())
        ext.add_layernorm(h, x, gamma, beta, y, 1e-5)
        ref_ext.add_layernorm(h_ref, x, gamma, beta, y_ref, 1e-5)
        assert np.array_equal(h.cpu().numpy().ravel(), h2_np)
        np.testing.assert_allclose(y.float().cpu().numpy().ravel(), y_np.astype(np.float32), rtol=1e-2, atol=1e-3)
        assert torch.equal(h, h_ref)
        assert torch.equal(y, y_ref), 'LayerNorm output differs bitwise from the reference kernel'


@pytest.mark.parametrize('length', [1, 63, 64, 65, 200, 448])
def test_self_attention_vs_oracle_and_reference(ext, ref_ext, length):
    g = torch.Generator(device='cuda').manual_seed(length)
    pos = length - 1
    q = torch.randn(HEADS * HD, device='cuda', generator=g).half()
    k = torch.randn(HEADS, 448, HD, device='cuda', generator=g).half()
    v = torch.randn_like(k)
    kn = torch.randn(HEADS, 1, HD, device='cuda', generator=g).half()
    vn = torch.randn_like(kn)
    state = torch.tensor([pos, 0], device='cuda', dtype=torch.long)
    k0, v0 = k.clone(), v.clone()
    out_np, k_np, v_np = K.decode_attention(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), pos,
                                            kn.cpu().numpy(), vn.cpu().numpy())
    out = torch.empty_like(q)
    ext.decode_attention(q, k, v, out, state, kn, vn, *_ws(), HD ** -0.5)
    np.testing.assert_allclose(out.float().cpu().numpy(), out_np, rtol=1e-2, atol=1e-3)
    assert np.array_equal(k.cpu().numpy(), k_np) and np.array_equal(v.cpu().numpy(), v_np)
    kr, vr, outr = k0.clone(), v0.clone(), torch.empty_like(q)
    ref_ext.decode_attention(q, kr, vr, outr, state, kn, vn, *_ws(), HD ** -0.5)
    assert torch.equal(kr, k) and torch.equal(vr, v)
    assert torch.equal(out, outr), f'max diff vs reference {(out.float() - outr.float()).abs().max()}'


def test_cross_attention_vs_golden_and_reference(ext, ref_ext):
    from conftest import GOLDEN
    from golden.make_golden import attention_inputs
    gold = np.load(GOLDEN / 'attention.npz')
    q, _, _, kc, vc = (t.cuda() for t in attention_inputs())
    out = torch.empty_like(q)
    ext.decode_attention(q, kc, vc, out, None, None, None, *_ws(), HD ** -0.5)
    np.testing.assert_allclose(out.float().cpu().numpy(), gold['cross_ref'], rtol=1e-2, atol=1e-3)
    outr = torch.empty_like(q)
    ref_ext.decode_attention(q, kc, vc, outr, None, None, None, *_ws(), HD ** -0.5)
    assert torch.equal(out, outr)


def test_lm_head_argmax_bitexact_vs_reference(ext, ref_ext):
    g = torch.Generator(device='cuda').manual_seed(7)
    w = (torch.randn(VOCAB, HIDDEN, device='cuda', generator=g) * 0.02).half()
    for trial in range(4):
        h = torch.randn(1, HIDDEN, device='cuda', generator=g).half()
        sup = torch.rand(VOCAB, device='cuda', generator=g) < 0.01
        best, best_r = torch.zeros(1, device='cuda', dtype=torch.long), torch.zeros(1, device='cuda', dtype=torch.long)
        ext.lm_head_argmax(h, w, sup, best)
        ref_ext.lm_head_argmax(h, w, sup, best_r)
        assert int(best) == int(best_r)
        tok = K.unpack_index(int(best) & 0xFFFFFFFFFFFFFFFF)
        logits = F.linear(h, w).float()[0].masked_fill(sup, float('-inf'))
        assert float(logits.max() - logits[tok]) <= 1e-3


def test_lm_head_argmax_ties_go_to_lower_index(ext):
    w = torch.zeros(VOCAB, HIDDEN, device='cuda', dtype=torch.float16)
    w[100, 0] = 1.0
    w[50000, 0] = 1.0
    w[7, 0] = 0.5
    h = torch.zeros(1, HIDDEN, device='cuda', dtype=torch.float16)
    h[0, 0] = 2.0
    best = torch.zeros(1, device='cuda', dtype=torch.long)
    ext.lm_head_argmax(h, w, torch.zeros(VOCAB, dtype=torch.bool, device='cuda'), best)
    assert K.unpack_index(int(best) & 0xFFFFFFFFFFFFFFFF) == 100
    sup = torch.zeros(VOCAB, dtype=torch.bool, device='cuda')
    sup[100] = True
    best.zero_()
    ext.lm_head_argmax(h, w, sup, best)
    assert K.unpack_index(int(best) & 0xFFFFFFFFFFFFFFFF) == 50000


def test_lm_quantize_matches_oracle(ext):
    g = torch.Generator(device='cuda').manual_seed(11)
    w = (torch.randn(4096, HIDDEN, device='cuda', generator=g) * 0.02).half()
    w[17] = 0
    wq, rp = ext.lm_quantize(w)
    q, s, a, c2 = K.lm_quantize(w.cpu().numpy())
    assert np.array_equal(wq.cpu().numpy(), q)
    rp = rp.cpu().numpy()
    assert np.array_equal(rp[:, 0], s)
    for col, want in ((1, a), (2, c2)):  # rounded up from the float64 value: >= it and < one fp32 step above
        got = rp[:, col].astype(np.float64)
        assert np.all(got >= want)
        assert np.all(got <= np.nextafter(want.astype(np.float32), np.float32(np.inf)).astype(np.float64))


def _best_pair(ext, h, w, wq, rp, sup):
    b, bq = torch.zeros(1, device='cuda', dtype=torch.long), torch.zeros(1, device='cuda', dtype=torch.long)
    ext.lm_head_argmax(h, w, sup, b)
    ext.lm_head_argmax_q(h, w, wq, rp, sup, bq)
    return int(b), int(bq)


def test_lm_head_argmax_q_equals_exact_kernel(ext, ref_ext):
    """Same packed key as the full fp16 LM head (itself bit-exact with the reference kernel) on
    LayerNorm-like inputs, suppressed rows, planted fp16 ties, a zero input and overflowing logits."""
    g = torch.Generator(device='cuda').manual_seed(12)
    w = (torch.randn(VOCAB, HIDDEN, device='cuda', generator=g) * 0.02).half()
    wq, rp = ext.lm_quantize(w)
    for trial in range(6):
        h = torch.randn(HIDDEN, device='cuda', generator=g)
        h = ((h - h.mean()) / h.std()).half().view(1, HIDDEN)
        sup = torch.rand(VOCAB, device='cuda', generator=g) < 0.01
        b, bq = _best_pair(ext, h, w, wq, rp, sup)
        assert b == bq
        if trial == 0:
            br = torch.zeros(1, device='cuda', dtype=torch.long)
            ref_ext.lm_head_argmax(h, w, sup, br)
            assert bq == int(br)
    # ties: copies of the winning row in other blocks of rows; the lowest index must win
    h = torch.randn(1, HIDDEN, device='cuda', generator=g).half()
    none = torch.zeros(VOCAB, dtype=torch.bool, device='cuda')
    top = K.unpack_index(_best_pair(ext, h, w, wq, rp, none)[0] & 0xFFFFFFFFFFFFFFFF)
    w2 = w.clone()
    for r in (3, 20000, 51000):
        w2[r] = w2[top]
    wq2, rp2 = ext.lm_quantize(w2)
    b, bq = _best_pair(ext, h, w2, wq2, rp2, none)
    assert b == bq and K.unpack_index(bq & 0xFFFFFFFFFFFFFFFF) == min(3, top)
    if top != 3:
        sup = none.clone()
        sup[3] = True
        b, bq = _best_pair(ext, h, w2, wq2, rp2, sup)
        assert b == bq and K.unpack_index(bq & 0xFFFFFFFFFFFFFFFF) == min(20000, top)
    # zero input: every logit is 0, the first unsuppressed row wins
    sup = none.clone()
    sup[:5] = True
    b, bq = _best_pair(ext, torch.zeros(1, HIDDEN, device='cuda', dtype=torch.float16), w, wq, rp, sup)
    assert b == bq and K.unpack_index(bq & 0xFFFFFFFFFFFFFFFF) == 5
    # logits beyond the fp16 range tie at +inf
    w3 = (torch.randn(VOCAB, HIDDEN, device='cuda', generator=g) * 6).half()
    wq3, rp3 = ext.lm_quantize(w3)
    h = (torch.randn(1, HIDDEN, device='cuda', generator=g) * 60).half()
    b, bq = _best_pair(ext, h, w3, wq3, rp3, none)
    assert b == bq


def test_argmax_finalize_bookkeeping(ext):
    key = int(K.pack_score(0.75, 4321))
    best = torch.tensor([key - (1 << 64) if key >= 1 << 63 else key], dtype=torch.long, device='cuda')
    tokens = torch.zeros(8, dtype=torch.long, device='cuda')
    state = torch.tensor([3, 0], dtype=torch.long, device='cuda')
    cur = torch.zeros(1, dtype=torch.long, device='cuda')
    ext.argmax_finalize(best, tokens, state, cur, 448)
    assert int(tokens[0]) == 4321 and state.tolist() == [4, 1] and int(cur) == 4321 and int(best) == 0
    state = torch.tensor([447, 448], dtype=torch.long, device='cuda')
    ext.argmax_finalize(best, torch.zeros(448, dtype=torch.long, device='cuda'), state, cur, 448)
    assert state.tolist() == [447, 448]


def test_embed_pos_bitexact(ext):
    g = torch.Generator(device='cuda').manual_seed(3)
    embed = torch.randn(VOCAB, HIDDEN, device='cuda', generator=g).half()
    pos = torch.randn(448, HIDDEN, device='cuda', generator=g).half()
    ids = torch.randint(0, VOCAB, (448,), device='cuda', generator=g)
    positions = torch.arange(448, device='cuda')
    out = torch.empty(448, HIDDEN, device='cuda', dtype=torch.float16)
    ext.embed_pos(embed, pos, ids, positions, out)
    ref = K.embed_pos(embed.cpu().numpy(), pos.cpu().numpy(), ids.cpu().numpy(), positions.cpu().numpy())
    assert np.array_equal(out.cpu().numpy(), ref)
    assert torch.equal(out, embed[ids] + pos[positions])


def test_gelu_vs_oracle_and_torch(ext):
    x = torch.randn(5120, device='cuda').half() * 3
    y = torch.empty_like(x)
    ext.gelu(x, y)
    np.testing.assert_allclose(y.float().cpu().numpy(), K.gelu(x.cpu().numpy()), rtol=1e-2, atol=1e-3)
    assert (y.float() - F.gelu(x.float()).half().float()).abs().max() <= 2e-3


@pytest.mark.parametrize('n', [51866, 1000, 7])
def test_argmax_f16_bitexact(ext, n):
    g = torch.Generator(device='cuda').manual_seed(n)
    logits = (torch.randn(n, device='cuda', generator=g) * 2).half()  # N(0, 4)
    logits[n // 2] = logits.max()  # force a tie
    key = torch.zeros(1, dtype=torch.long, device='cuda')
    out = torch.zeros(1, dtype=torch.long, device='cuda')
    ext.argmax_f16(logits, None, key, out)
    assert int(out) == K.argmax_first(logits.cpu().numpy()) == int(torch.argmax(logits.float()))
    assert int(key) == 0
    sup = torch.rand(n, device='cuda', generator=g) < 0.3
    ext.argmax_f16(logits, sup, key, out)
    assert int(out) == K.argmax_first(logits.cpu().numpy(), sup.cpu().numpy())


@pytest.mark.parametrize('n_out,act', [(3840, 0), (1280, 0), (5120, 1)])
def test_ln_gemv_vs_oracle(ext, ref_ext, n_out, act):
    g = torch.Generator(device='cuda').manual_seed(n_out)
    h = torch.randn(HIDDEN, device='cuda', generator=g).half()
    gamma = (1 + 0.1 * torch.randn(HIDDEN, device='cuda', generator=g)).half()
    beta = (0.1 * torch.randn(HIDDEN, device='cuda', generator=g)).half()
    w = (0.02 * torch.randn(n_out, HIDDEN, device='cuda', generator=g)).half()
    b = (0.02 * torch.randn(n_out, device='cuda', generator=g)).half()
    out = torch.empty(n_out, device='cuda', dtype=torch.float16)
    ext.ln_gemv(h, gamma, beta, 1e-5, w, b, out, act)
    # reference composition: its LayerNorm kernel then cuBLAS F.linear (+ F.gelu)
    y = torch.empty(1, HIDDEN, device='cuda', dtype=torch.float16)
    ref_ext.add_layernorm(h.clone().view(1, -1), None, gamma, beta, y, 1e-5)
    ref = F.linear(y, w, b)
    if act:
        ref = F.gelu(ref)
    _, y_np = K.add_layernorm(h.cpu().numpy(), None, gamma.cpu().numpy(), beta.cpu().numpy())
    o_np = K.linear(y.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy()).astype(np.float64)
    if act:
        o_np = K.gelu(o_np)
    np.testing.assert_allclose(out.float().cpu().numpy(), o_np, rtol=1e-2, atol=1e-3)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy().ravel(), rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize('k', [1280, 5120])
def test_gemv_residual_vs_oracle(ext, k):
    g = torch.Generator(device='cuda').manual_seed(k)
    x = torch.randn(k, device='cuda', generator=g).half()
    w = (0.02 * torch.randn(HIDDEN, k, device='cuda', generator=g)).half()
    b = (0.02 * torch.randn(HIDDEN, device='cuda', generator=g)).half()
    h = torch.randn(HIDDEN, device='cuda', generator=g).half()
    h0 = h.cpu().numpy()
    ext.gemv_residual(x, w, b, h)
    proj = K.linear(x.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy())
    ref = (h0.astype(np.float32) + proj.astype(np.float32)).astype(np.float16)
    np.testing.assert_allclose(h.float().cpu().numpy(), ref.astype(np.float32), rtol=1e-2, atol=1e-3)


def test_device_error_word_is_clear(ext):
    torch.cuda.synchronize()
    assert ext.device_error(clear=True) == 0
