"""GPU parity of the encoder kernels: the tcgen05 GEMM with every epilogue, the implicit-GEMM
convolutions, row LayerNorm and encoder attention against PyTorch fp32, and the whole encoder
against the numpy oracle."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from flash_whisper_b200 import _lib

pytestmark = pytest.mark.gpu


def _close(out, ref, rtol=1e-2, atol=1e-3, inner=None):
    """|out - ref| <= atol + rtol |ref| (+ one fp16 ulp of `inner`, the fp16-rounded accumulator an
    epilogue rounds before adding a residual or applying GELU: a different fp32 summation order may
    round it one ulp apart, and that ulp survives cancellation in the sum)."""
    out, ref = out.float(), ref.float()
    tol = atol + rtol * ref.abs()
    if inner is not None:
        tol = tol + inner.float().abs() * 2.0 ** -10
    bad = (out - ref).abs() > tol
    assert not bool(bad.any()), (f'{int(bad.sum())} / {bad.numel()} mismatches, max abs diff '
                                 f'{float((out - ref).abs().max())}')


def _rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device='cuda').manual_seed(seed)
    return (torch.randn(*shape, device='cuda', generator=g) * scale).half()


@pytest.mark.parametrize('m,n,k', [(1500, 3840, 1280), (1500, 1280, 1280), (1500, 5120, 1280), (1500, 1280, 5120),
                                   (128, 256, 64), (300, 640, 192), (3000, 1280, 384)])
def test_gemm_bias_vs_torch(ext, m, n, k):
    a = _rand(m, k, seed=1)
    b = _rand(n, k, scale=k ** -0.5, seed=2)
    bias = _rand(n, scale=0.1, seed=3)
    c = torch.full((m, n), 9.0, device='cuda', dtype=torch.float16)
    ext.gemm(a, b, bias, c)
    ref = (a.float() @ b.float().T + bias.float()).half()
    _close(c, ref)


def test_gemm_epilogues(ext):
    m, n, k = 1500, 1280, 1280
    a, b, bias = _rand(m, k, seed=4), _rand(n, k, scale=k ** -0.5, seed=5), _rand(n, scale=0.1, seed=6)
    acc = (a.float() @ b.float().T + bias.float()).half().float()
    c = torch.empty(m, n, device='cuda', dtype=torch.float16)
    ext.gemm(a, b, bias, c, _lib.FW_EPI_BIAS_GELU)
    _close(c, F.gelu(acc).half(), inner=acc)
    r = _rand(m, n, seed=7)
    c = r.clone()
    ext.gemm(a, b, bias, c, _lib.FW_EPI_BIAS_RESID, r=c)  # in place, as the encoder residual does
    _close(c, (r.float() + acc).half(), inner=acc)
    pos = _rand(m, n, seed=8)
    ext.gemm(a, b, bias, c, _lib.FW_EPI_GELU_POS, r=pos)
    _close(c, (F.gelu(acc).half().float() + pos.float()).half(), inner=acc)
    ext.gemm(a, b, bias, c, _lib.FW_EPI_BIAS_SCALE, scale=0.125, scale_cols=640)
    ref = acc.clone()
    ref[:, :640] *= 0.125
    _close(c, ref.half())


def test_gemm_qkv_transposed_v_epilogue(ext):
    m, n, k = 1500, 3840, 1280
    a, b, bias = _rand(m, k, seed=21), _rand(n, k, scale=k ** -0.5, seed=22), _rand(n, scale=0.1, seed=23)
    acc = (a.float() @ b.float().T + bias.float()).half().float()
    c = torch.full((m, n), 7.0, device='cuda', dtype=torch.float16)
    ldv = 1504
    vt = torch.zeros(1280, ldv, device='cuda', dtype=torch.float16)
    ext.gemm(a, b, bias, c, _lib.FW_EPI_QKV_VT, r=vt, scale=0.125, scale_cols=1280)
    ref = acc.clone()
    ref[:, :1280] *= 0.125
    _close(c[:, :2560], ref[:, :2560].half())
    assert bool((c[:, 2560:] == 7.0).all()), 'v columns must not be written to C'
    _close(vt[:, :m], acc[:, 2560:].T.contiguous().half())
    assert float(vt[:, m:].abs().max()) == 0.0


def test_gemm_cross_kv_scatter(ext):
    m, layers, heads = 1500, 4, 20
    n, k = layers * 2 * 1280, 1280
    a, b, bias = _rand(m, k, seed=9), _rand(n, k, scale=k ** -0.5, seed=10), _rand(n, scale=0.1, seed=11)
    out = torch.empty(layers, 2, heads, m, 64, device='cuda', dtype=torch.float16)
    ext.gemm(a, b, bias, out, _lib.FW_EPI_CROSS_KV)
    kv = (a.float() @ b.float().T + bias.float()).half()
    ref = kv.view(m, layers, 2, heads, 64).permute(1, 2, 3, 0, 4)
    _close(out, ref)


@pytest.mark.parametrize('cin,stride,rows', [(128, 1, 3000), (1280, 2, 3000)])
def test_conv1d_implicit_gemm_vs_torch(ext, cin, stride, rows):
    x = _rand(rows, cin, seed=12)
    w = _rand(1280, cin, 3, scale=(3 * cin) ** -0.5, seed=13)
    bias = _rand(1280, scale=0.1, seed=14)
    xp = torch.zeros(rows + 2, cin, device='cuda', dtype=torch.float16)
    xp[1:-1] = x
    w_taps = w.permute(0, 2, 1).reshape(1280, -1).contiguous()
    m = (rows - 1) // stride + 1
    out = torch.empty(m, 1280, device='cuda', dtype=torch.float16)
    ext.conv1d_k3(xp, w_taps, bias, out, stride, _lib.FW_EPI_BIAS_GELU)
    ref = F.gelu(F.conv1d(x.float().T[None], w.float(), bias.float(), stride=stride, padding=1)[0].T.half().float())
    _close(out, ref.half())


def test_layernorm_rows_vs_torch(ext):
    x = _rand(1500, 1280, seed=15)
    g, b = (1 + 0.1 * _rand(1280, seed=16).float()).half(), _rand(1280, scale=0.1, seed=17)
    y = torch.empty_like(x)
    ext.layernorm_rows(x, g, b, y, 1e-5)
    _close(y, F.layer_norm(x.float(), (1280,), g.float(), b.float(), 1e-5).half())


@pytest.mark.parametrize('seq', [1500, 200, 77, 33, 20, 1])
def test_encoder_attention_vs_torch(ext, seq):
    heads = 20
    qkv = _rand(seq, 3 * 1280, seed=seq)
    qkv[:, :1280] = (qkv[:, :1280].float() * 0.125).half()  # q arrives pre-scaled (HF WhisperAttention)
    out = torch.empty(seq, 1280, device='cuda', dtype=torch.float16)
    ext.encoder_attention(qkv, out, heads)
    q, k, v = (qkv[:, i * 1280:(i + 1) * 1280].float().view(seq, heads, 64).transpose(0, 1) for i in range(3))
    ref = F.scaled_dot_product_attention(q, k, v, scale=1.0).transpose(0, 1).reshape(seq, 1280)
    _close(out, ref.half(), rtol=2e-2, atol=2e-3)


def test_encoder_forward_vs_numpy_oracle(ext):
    from flash_whisper_b200.audio import pad_to_30s, synthetic_audio
    from flash_whisper_b200.model import CustomModel
    from flash_whisper_b200.weights import WhisperDims, random_state_dict
    from oracle.mel import log_mel
    from oracle.model_np import WhisperOracle
    dims = WhisperDims(encoder_layers=4, decoder_layers=2)
    sd = random_state_dict(5, dims, bias_std=0.02, ln_std=0.05)
    model = CustomModel(state_dict=sd, dims=dims, selftest=False, capture=False)
    wave = pad_to_30s(synthetic_audio(3, 30.0))
    model.load_audio(wave)
    with torch.inference_mode():
        model._mel()
        model._encode()
    torch.cuda.synchronize()
    o = WhisperOracle(sd, dims)
    mel16 = model.mel[1:-1].float().cpu().numpy().T
    np.testing.assert_allclose(mel16, log_mel(wave), rtol=1e-2, atol=1e-3)
    enc = o.encoder(mel16)
    got = model.enc_out.float().cpu().numpy()
    rel = np.linalg.norm(got - enc) / np.linalg.norm(enc)
    assert rel < 1e-2, rel
    o.set_cross(enc)
    ck = model.cross_kv[:, 0].float().cpu().numpy()
    rel_k = np.linalg.norm(ck - o.cross_k) / np.linalg.norm(o.cross_k)
    assert rel_k < 1e-2, rel_k
