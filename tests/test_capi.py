"""CPU tests of the C-ABI boundary: the library loads, exports everything the header declares, and
rejects bad arguments with the reference's error messages before touching a GPU."""

import ctypes

import pytest
import torch

from flash_whisper_b200 import _lib
from flash_whisper_b200.ext import Ext


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _lib.header_symbols()
    assert len(declared) >= 19
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert set(declared) == set(_lib._SIGNATURES)
    assert lib.fw_version() == 1


def _c_class(decl):
    """Argument class of one C parameter declaration: pointer, i32, i64 or f32."""
    decl = decl.strip()
    if '*' in decl or decl.startswith('fw_stream_t'):
        return 'ptr'
    base = decl.rsplit(None, 1)[0] if ' ' in decl else decl
    return {'int': 'i32', 'int64_t': 'i64', 'float': 'f32'}[base.replace('const ', '').strip()]


def _ctypes_class(t):
    if t in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(t, ctypes._Pointer):
        return 'ptr'
    return {ctypes.c_int: 'i32', ctypes.c_int64: 'i64', ctypes.c_float: 'f32'}[t]


def test_ctypes_signatures_match_header_prototypes():
    """Every prototype in include/flash_whisper.h against the ctypes binding: same return type and the
    same number and kind of arguments (a wrong count or an int passed as int64 would otherwise show up
    only as wrong results on a GPU)."""
    import re
    text = re.sub(r'/\*.*?\*/', '', _lib.HEADER.read_text(), flags=re.S)
    protos = re.findall(r'^(const char\*|int)\s+(fw_\w+)\((.*?)\);', text, flags=re.M | re.S)
    assert len(protos) == len(_lib._SIGNATURES)
    for ret, name, args in protos:
        res, argtypes = _lib._SIGNATURES[name]
        assert (res is ctypes.c_char_p) == (ret == 'const char*'), name
        params = [] if args.strip() in ('', 'void') else [a for a in args.replace('\n', ' ').split(',')]
        assert [_c_class(a) for a in params] == [_ctypes_class(t) for t in argtypes], name


def test_null_pointers_return_status_and_message():
    lib = _lib.lib()
    rc = lib.fw_add_layernorm(None, None, None, None, None, 1280, 1e-5, None)
    assert rc == 1  # FW_ERR_NULL
    assert b'required' in lib.fw_last_error_string()
    p = ctypes.c_void_p(16)
    rc = lib.fw_add_layernorm(p, None, p, p, p, 1024, 1e-5, None)
    assert rc == 2 and b'hidden size must be 1280' in lib.fw_last_error_string()
    rc = lib.fw_decode_attention(p, p, p, p, None, p, None, p, 100, p, 100, p, 6400, 20, 448, 0.125, None)
    assert rc == 4 and b'given together' in lib.fw_last_error_string()
    rc = lib.fw_decode_attention(p, p, p, p, None, None, None, p, 10, p, 10, p, 640, 20, 448, 0.125, None)
    assert rc == 2 and b'workspace too small for 7 splits' in lib.fw_last_error_string()
    rc = lib.fw_gemm_f16(p, 64, p, 64, None, p, 64, None, 0, 100, 60, 64, 0, 1.0, 0, None)
    assert rc == 2
    rc = lib.fw_log_mel(p, 1, 1000, p, p, p, p, 0, None)
    assert rc == 2


def test_decoder_struct_matches_header_layout():
    # offsets the C struct would have: ints, floats, pointers in declaration order (x86-64 LP64)
    assert ctypes.sizeof(_lib.DecoderLayer) == 22 * 8
    assert _lib.Decoder.layers.offset == 8 * 4 + 8 * 8
    assert ctypes.sizeof(_lib.EncoderLayer) == 12 * 8
    assert _lib.Decoder.lm_q.offset == _lib.Decoder.n_tokens.offset + 8
    assert _lib.Decoder.lm_rp.offset == _lib.Decoder.lm_q.offset + 8
    assert ctypes.sizeof(_lib.Decoder) == _lib.Decoder.lm_rp.offset + 8


def test_pruned_lm_head_argument_checks():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)
    assert lib.fw_lm_quantize(None, 51866, 1280, p, p, None) == 1
    assert b'required' in lib.fw_last_error_string()
    assert lib.fw_lm_quantize(p, 51866, 1024, p, p, None) == 2
    assert b'hidden size must be 1280' in lib.fw_last_error_string()
    assert lib.fw_lm_quantize(ctypes.c_void_p(18), 51866, 1280, p, p, None) == 3  # FW_ERR_ALIGN
    assert lib.fw_lm_head_argmax_q(p, p, None, p, p, 51866, 1280, p, None) == 1
    assert b'wq' in lib.fw_last_error_string()
    assert lib.fw_lm_head_argmax_q(p, p, p, p, p, 0, 1280, p, None) == 2


def test_decoder_step_needs_both_pruned_lm_buffers():
    lib = _lib.lib()
    d = _lib.Decoder()
    d.n_layers, d.heads, d.max_pos, d.enc_len, d.vocab = 4, 20, 448, 1500, 51866
    d.ws_splits = 24
    for name in ('embed', 'pos_embed', 'lm_head', 'final_g', 'final_b', 'h', 'cq', 'ffn', 'part_acc', 'counters',
                 'cur', 'state', 'tokens', 'best'):
        setattr(d, name, 16)
    d.lm_q = 16  # lm_rp left NULL
    assert lib.fw_decoder_step(ctypes.byref(d), 1, None) == 1
    assert b'set both lm_q and lm_rp' in lib.fw_last_error_string()


def test_decoder_step_needs_residual_scratch_and_two_partial_sets():
    """The fused step keeps the self and cross blocks' output-projection partials in part_acc (the next
    launch forms the residual from them) and the residual after each self block in cq."""
    lib = _lib.lib()
    d = _lib.Decoder()
    d.n_layers, d.heads, d.max_pos, d.enc_len, d.vocab = 4, 20, 448, 1500, 51866
    for name in ('embed', 'pos_embed', 'lm_head', 'final_g', 'final_b', 'h', 'ffn', 'part_acc', 'counters',
                 'cur', 'state', 'tokens', 'best'):
        setattr(d, name, 16)
    d.ws_splits = 40
    assert lib.fw_decoder_step(ctypes.byref(d), 1, None) == 1  # cq left NULL
    assert b'required pointer' in lib.fw_last_error_string()
    d.cq = 16
    d.ws_splits = 24  # enough for the attention splits, not for two sets of partials
    assert lib.fw_decoder_step(ctypes.byref(d), 1, None) == 2
    assert b'2 * heads * 1280' in lib.fw_last_error_string()
    d.ws_splits = 40
    d.cq = 18  # misaligned
    assert lib.fw_decoder_step(ctypes.byref(d), 1, None) == 3
    assert b'16-byte aligned' in lib.fw_last_error_string()


def test_wrapper_checks_mirror_reference_messages():
    ext = Ext()
    h = torch.zeros(1280, dtype=torch.float16)
    with pytest.raises(RuntimeError, match='h must be contiguous CUDA fp16'):
        ext.add_layernorm(h, None, h, h, h, 1e-5)
    with pytest.raises(RuntimeError, match='q must be contiguous CUDA fp16'):
        ext.decode_attention(h, h, h, h, None, None, None, h, h, h, 0.125)
    with pytest.raises(RuntimeError, match='tokens, state and cur must be int64'):
        ext.argmax_finalize(torch.zeros(1, dtype=torch.long), torch.zeros(4, dtype=torch.int32),
                            torch.zeros(2, dtype=torch.long), torch.zeros(1, dtype=torch.long), 448)


def test_model_requires_cuda_without_fallback():
    if torch.cuda.is_available():
        pytest.skip('CUDA present')
    from flash_whisper_b200.model import CustomModel
    with pytest.raises(RuntimeError, match='requires a CUDA device'):
        CustomModel()


def test_audio_checks_match_the_reference():
    """transcribe's input checks (custom/model.py:175-178), which run before anything touches the GPU:
    a 1-D float32 array of 1..480000 finite samples, ValueError otherwise."""
    import numpy as np
    from flash_whisper_b200.model import CustomModel
    check = CustomModel._check_audio
    check(np.zeros(1, np.float32))
    check(np.zeros(480000, np.float32))
    bad = [np.zeros(16000, np.float64), np.zeros((2, 8000), np.float32), [0.0] * 16000, np.zeros(0, np.float32),
           np.zeros(480001, np.float32), np.array([0.0, np.nan], np.float32), np.array([np.inf], np.float32)]
    for audio in bad:
        with pytest.raises(ValueError):
            check(audio)
