"""The no-allocation attention entry point (fw_decode_attention_noalloc), called through the C ABI.

Some callers cannot allocate device memory: a host in the middle of recording a CUDA graph, a
plug-in whose device memory is owned by the host application's allocator or a fixed budget, or a
real-time audio thread that must not stall on cudaMalloc / cudaFree. For them the library keeps
the attention split partials in a fixed device array of its own (at most 2048 head-splits, i.e.
heads * ceil(max_len / 64)). This test checks that variant against fw_decode_attention with a
caller-allocated workspace (bit for bit: both run the same kernels) on calls in a row (the shared array
keeps the previous call's contents, which must not leak into the next result): self attention with
the fused KV-cache write, 1500-key cross attention, a call that fills the array exactly, and a
smaller call after a larger one; and that oversize requests are rejected. It lives in a file
of its own that pytest collects last.
"""

import ctypes

import pytest
import torch

from flash_whisper_b200 import _lib

pytestmark = pytest.mark.gpu
HEADS, HD = 20, 64
vp = ctypes.c_void_p


def _p(t):
    return vp(t.data_ptr()) if t is not None else vp(0)


def _stream():
    return vp(torch.cuda.current_stream().cuda_stream)


def _with_workspace(q, k, v, out, state, kn, vn, max_len, heads=HEADS):
    splits = -(-max_len // 64)
    pm = torch.empty(heads * splits, device='cuda')
    pl = torch.empty(heads * splits, device='cuda')
    pa = torch.empty(heads * splits * HD, device='cuda')
    rc = _lib.lib().fw_decode_attention(_p(q), _p(k), _p(v), _p(out), _p(state), _p(kn), _p(vn), _p(pm), pm.numel(),
                                        _p(pl), pl.numel(), _p(pa), pa.numel(), heads, max_len, HD ** -0.5,
                                        _stream())
    assert rc == 0, _lib.lib().fw_last_error_string()


def _no_alloc(q, k, v, out, state, kn, vn, max_len, heads=HEADS):
    rc = _lib.lib().fw_decode_attention_noalloc(_p(q), _p(k), _p(v), _p(out), _p(state), _p(kn), _p(vn), heads,
                                                max_len, HD ** -0.5, _stream())
    assert rc == 0, _lib.lib().fw_last_error_string()


def _inputs(seed, max_len, self_attn, heads=HEADS):
    g = torch.Generator(device='cuda').manual_seed(seed)
    q = torch.randn(heads * HD, device='cuda', generator=g).half()
    k = torch.randn(heads, max_len, HD, device='cuda', generator=g).half()
    v = torch.randn(heads, max_len, HD, device='cuda', generator=g).half()
    if not self_attn:
        return q, k, v, None, None, None
    kn = torch.randn(heads, HD, device='cuda', generator=g).half()
    vn = torch.randn(heads, HD, device='cuda', generator=g).half()
    state = torch.tensor([(seed * 37) % max_len, 0], device='cuda', dtype=torch.long)
    return q, k, v, state, kn, vn


def _compare(seed, max_len, self_attn, heads=HEADS, tag=''):
    """One call of each entry point on the same inputs; both run the same kernels, so the outputs and
    the cache writes must be identical bit for bit."""
    q, k, v, state, kn, vn = _inputs(seed, max_len, self_attn, heads)
    k2, v2 = k.clone(), v.clone()
    want, got = torch.empty_like(q), torch.full_like(q, float('nan'))
    _with_workspace(q, k, v, want, state, kn, vn, max_len, heads)
    _no_alloc(q, k2, v2, got, state, kn, vn, max_len, heads)
    torch.cuda.synchronize()
    assert torch.equal(got, want), f'{tag}: max diff {(got.float() - want.float()).abs().max()}'
    assert torch.equal(k2, k) and torch.equal(v2, v), f'{tag}: KV-cache write differs'


@pytest.mark.parametrize('max_len,self_attn', [(448, True), (1500, False)])
def test_no_alloc_matches_workspace_entry_point_twice(cuda, max_len, self_attn):
    for call, seed in enumerate((1, 2)):  # two calls in a row, different inputs
        _compare(seed + 10 * max_len, max_len, self_attn, tag=f'call {call}')


def test_no_alloc_full_scratch_and_shrinking_calls(cuda):
    """Exactly 2048 head-splits (16 heads x 8192 keys fill the fixed array), then a 1500-key cross call
    followed by a 448-key self-attention call: a smaller call after a larger one must not pick up the
    earlier call's partials left in the array."""
    _compare(5, 8192, True, heads=16, tag='2048 head-splits, self')
    _compare(6, 8192, False, heads=16, tag='2048 head-splits, cross')
    _compare(7, 1500, False, tag='cross 1500')
    _compare(8, 448, True, tag='self 448 after cross 1500')


def test_no_alloc_rejects_oversize(cuda):
    q = torch.zeros(HEADS * HD, device='cuda', dtype=torch.float16)
    kv = torch.zeros(HEADS, 64 * 103, HD, device='cuda', dtype=torch.float16)  # 20 * 103 > 2048 splits
    rc = _lib.lib().fw_decode_attention_noalloc(_p(q), _p(kv), _p(kv), _p(q), vp(0), vp(0), vp(0), HEADS,
                                                kv.size(1), HD ** -0.5, _stream())
    assert rc == 2
    assert b'exceeds the fixed scratch' in _lib.lib().fw_last_error_string()
    rc = _lib.lib().fw_decode_attention_noalloc(_p(q), _p(kv), _p(kv), _p(q), vp(0), vp(0), vp(0), 1, 64 * 129,
                                                HD ** -0.5, _stream())
    assert rc == 2
    assert b'decode_attention_noalloc: max_len' in _lib.lib().fw_last_error_string()
