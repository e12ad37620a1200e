"""CPU tests of the kernel weight layouts built by flash_whisper_b200.weights (no GPU needed).

The decode kernels read the attention output projections head-major ([heads, d_model, 64]), the
self-attention q/k/v rows fused with a zeroed k bias (custom/model.py:87-88), and the cross-attention
K/V projections of all layers stacked for one encoder-side GEMM; the encoder's k=3 convolutions run
as implicit GEMMs over (tap, channel)-ordered weights and a time-major input with one zero row at
each end. Each layout is checked element-wise and by the product the kernels form with it, on a
narrow model (2 heads of 64) so the test runs in milliseconds.
"""

import sys
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from flash_whisper_b200.weights import WhisperDims, pack_decoder, pack_encoder, random_state_dict  # noqa: E402

DIMS = WhisperDims(d_model=128, heads=2, encoder_layers=1, decoder_layers=2, ffn=256, vocab=300, n_mels=16,
                   enc_len=20, max_pos=32, pad_token_id=299, eos_token_id=298)


@pytest.fixture(scope='module')
def sd():
    return random_state_dict(3, DIMS, bias_std=0.02)


def test_decoder_fused_qkv_and_zero_k_bias(sd):
    dec = pack_decoder(sd, DIMS, device='cpu', dtype=torch.float32)
    d = DIMS.d_model
    for i, L in enumerate(dec.layers):
        p = f'model.decoder.layers.{i}.self_attn'
        assert L.qkv_w.shape == (3 * d, d)
        assert torch.equal(L.qkv_w[:d], sd[f'{p}.q_proj.weight'])
        assert torch.equal(L.qkv_w[d:2 * d], sd[f'{p}.k_proj.weight'])
        assert torch.equal(L.qkv_w[2 * d:], sd[f'{p}.v_proj.weight'])
        assert torch.equal(L.qkv_b[:d], sd[f'{p}.q_proj.bias'])
        assert torch.count_nonzero(L.qkv_b[d:2 * d]) == 0  # HF's k_proj has no bias
        assert torch.equal(L.qkv_b[2 * d:], sd[f'{p}.v_proj.bias'])


@pytest.mark.parametrize('which', ['self_attn', 'encoder_attn'])
def test_decoder_output_projection_is_head_major(sd, which):
    dec = pack_decoder(sd, DIMS, device='cpu', dtype=torch.float32)
    H, hd, d = DIMS.heads, DIMS.head_dim, DIMS.d_model
    g = torch.Generator().manual_seed(5)
    for i, L in enumerate(dec.layers):
        w = sd[f'model.decoder.layers.{i}.{which}.out_proj.weight']
        hm, b = L.out if which == 'self_attn' else L.cross_out
        assert hm.shape == (H, d, hd) and hm.is_contiguous()
        for h in range(H):  # head h's slice W[:, 64h:64h+64] is one contiguous [d, 64] block
            assert torch.equal(hm[h], w[:, h * hd:(h + 1) * hd])
        # the product the attention block forms: sum over heads of (slice of head h) x (head h's output)
        a = torch.randn(H * hd, generator=g)
        by_head = sum(hm[h] @ a[h * hd:(h + 1) * hd] for h in range(H))
        torch.testing.assert_close(by_head + b, F.linear(a, w, sd[f'model.decoder.layers.{i}.{which}.out_proj.bias']))


def test_decoder_cross_kv_stack_and_tied_lm_head(sd):
    dec = pack_decoder(sd, DIMS, device='cpu', dtype=torch.float32)
    d = DIMS.d_model
    assert dec.cross_w.shape == (DIMS.decoder_layers * 2 * d, d)
    for i in range(DIMS.decoder_layers):
        p = f'model.decoder.layers.{i}.encoder_attn'
        base = 2 * d * i
        assert torch.equal(dec.cross_w[base:base + d], sd[f'{p}.k_proj.weight'])
        assert torch.equal(dec.cross_w[base + d:base + 2 * d], sd[f'{p}.v_proj.weight'])
        assert torch.count_nonzero(dec.cross_b[base:base + d]) == 0
        assert torch.equal(dec.cross_b[base + d:base + 2 * d], sd[f'{p}.v_proj.bias'])
    assert dec.lm_head is dec.embed  # tied, as the reference's proj_out
    assert torch.count_nonzero(dec.embed[DIMS.pad_token_id]) == 0


@pytest.mark.parametrize('conv,stride', [('conv1', 1), ('conv2', 2)])
def test_encoder_conv_as_implicit_gemm(sd, conv, stride):
    """y[t] = sum over taps j of W2[:, j*C:(j+1)*C] x_pad[stride*t + j], x_pad = time-major input with one
    zero row at each end: the product the conv GEMM's tensor map forms, equal to Conv1d(k=3, pad=1)."""
    enc = pack_encoder(sd, DIMS, device='cpu', dtype=torch.float32)
    w2, b = enc.conv1 if conv == 'conv1' else enc.conv2
    w = sd[f'model.encoder.{conv}.weight']  # [out, in, 3]
    out_c, in_c, k = w.shape
    assert w2.shape == (out_c, k * in_c)
    for j in range(k):
        assert torch.equal(w2[:, j * in_c:(j + 1) * in_c], w[:, :, j])
    T = 2 * DIMS.enc_len
    x = torch.randn(in_c, T, generator=torch.Generator().manual_seed(7))  # channel-major, as HF takes it
    ref = F.conv1d(x[None], w, b, stride=stride, padding=1)[0].T  # [T_out, out]
    xpad = torch.cat([torch.zeros(1, in_c), x.T, torch.zeros(1, in_c)])  # time-major + zero rows
    t_out = ref.shape[0]
    rows = torch.stack([xpad[stride * t:stride * t + k].reshape(-1) for t in range(t_out)])  # (tap, channel)
    torch.testing.assert_close(rows @ w2.T + b, ref)
