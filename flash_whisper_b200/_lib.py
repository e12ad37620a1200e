"""ctypes binding of libflashwhisper.so (declared in include/flash_whisper.h).

This is the only place the package touches the shared library. Every call returns an int status;
`call()` turns a non-zero status into RuntimeError carrying fw_last_error_string(), the same
exception type the reference's TORCH_CHECKs raise (custom/kernels/whisper_kernels.cu:272-347).
"""

import ctypes
import os
from ctypes import POINTER, c_bool, c_char_p, c_float, c_int, c_int64, c_uint, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / 'libflashwhisper.so'
HEADER = PKG.parent / 'include' / 'flash_whisper.h'

FW_OK = 0
FW_EPI_BIAS, FW_EPI_BIAS_GELU, FW_EPI_BIAS_RESID, FW_EPI_GELU_POS, FW_EPI_CROSS_KV, FW_EPI_BIAS_SCALE, FW_EPI_QKV_VT = range(7)
MAX_LAYERS = 8
# fw_decoder_step_trace buffer layout (fp16 element offsets within one layer's record)
TRACE_SELF_ATTN, TRACE_H_SELF, TRACE_CROSS_ATTN, TRACE_H_CROSS, TRACE_FFN, TRACE_H_FFN = 0, 1280, 2560, 3840, 5120, 10240
TRACE_LAYER = 11520
MAX_ENC_LAYERS = 32

vp = c_void_p
i64p = POINTER(c_int64)


class DecoderLayer(ctypes.Structure):
    _fields_ = [(name, vp) for name in (
        'ln1_g', 'ln1_b', 'ln2_g', 'ln2_b', 'ln3_g', 'ln3_b', 'qkv_w', 'qkv_b', 'out_w', 'out_b', 'cq_w', 'cq_b',
        'co_w', 'co_b', 'fc1_w', 'fc1_b', 'fc2_w', 'fc2_b', 'self_k', 'self_v', 'cross_k', 'cross_v')]


class Decoder(ctypes.Structure):
    _fields_ = [
        ('n_layers', c_int), ('heads', c_int), ('max_pos', c_int), ('enc_len', c_int), ('vocab', c_int),
        ('prompt_len', c_int), ('eps', c_float), ('scale', c_float),
        ('embed', vp), ('pos_embed', vp), ('lm_head', vp), ('final_g', vp), ('final_b', vp),
        ('base_mask', vp), ('first_mask', vp), ('prompt', vp),
        ('layers', DecoderLayer * MAX_LAYERS),
        ('h', vp), ('qkv', vp), ('attn', vp), ('cq', vp), ('ffn', vp),
        ('part_m', vp), ('part_l', vp), ('part_acc', vp), ('ws_splits', c_int64),
        ('counters', vp), ('cur', vp), ('state', vp), ('tokens', vp), ('best', vp), ('n_tokens', c_int64),
        ('lm_q', vp), ('lm_rp', vp),
    ]


MAX_CLIPS = 8


class BatchDecoder(ctypes.Structure):
    _fields_ = [
        ('n_layers', c_int), ('heads', c_int), ('max_pos', c_int), ('enc_len', c_int), ('vocab', c_int),
        ('prompt_len', c_int), ('clips', c_int), ('eps', c_float), ('scale', c_float),
        ('embed', vp), ('pos_embed', vp), ('lm_head', vp), ('final_g', vp), ('final_b', vp),
        ('base_mask', vp), ('first_mask', vp), ('prompt', vp),
        ('layers', DecoderLayer * MAX_LAYERS),
        ('self_clip_stride', c_int64), ('cross_clip_stride', c_int64),
        ('h', vp), ('qkv', vp), ('attn', vp), ('ffn', vp),
        ('part_m', vp), ('part_l', vp), ('part_acc', vp), ('ws_splits', c_int64),
        ('counters', vp), ('cur', vp), ('state', vp), ('tokens', vp), ('best', vp), ('n_tokens', c_int64),
        ('lm_q', vp), ('lm_rp', vp),
    ]


class EncoderLayer(ctypes.Structure):
    _fields_ = [(name, vp) for name in (
        'ln1_g', 'ln1_b', 'ln2_g', 'ln2_b', 'qkv_w', 'qkv_b', 'out_w', 'out_b', 'fc1_w', 'fc1_b', 'fc2_w', 'fc2_b')]


class Encoder(ctypes.Structure):
    _fields_ = [
        ('n_layers', c_int), ('n_frames', c_int), ('n_pos', c_int), ('n_dec_layers', c_int), ('heads', c_int),
        ('eps', c_float),
        ('mel', vp), ('conv1_w', vp), ('conv1_b', vp), ('conv2_w', vp), ('conv2_b', vp), ('pos', vp),
        ('layers', EncoderLayer * MAX_ENC_LAYERS),
        ('final_g', vp), ('final_b', vp), ('cross_w', vp), ('cross_b', vp),
        ('conv1_out', vp), ('x', vp), ('y', vp), ('qkv', vp), ('attn', vp), ('ffn', vp), ('enc_out', vp),
        ('cross_kv', vp),
        ('vt', vp),
    ]


_SIGNATURES = {
    'fw_last_error_string': (c_char_p, []),
    'fw_version': (c_int, []),
    'fw_device_error': (c_int, [POINTER(c_uint), c_int]),
    'fw_add_layernorm': (c_int, [vp, vp, vp, vp, vp, c_int, c_float, vp]),
    'fw_decode_attention': (c_int, [vp, vp, vp, vp, vp, vp, vp, vp, c_int64, vp, c_int64, vp, c_int64, c_int, c_int,
                                    c_float, vp]),
    'fw_decode_attention_noalloc': (c_int, [vp, vp, vp, vp, vp, vp, vp, c_int, c_int, c_float, vp]),
    'fw_lm_head_argmax': (c_int, [vp, vp, vp, c_int, c_int, vp, vp]),
    'fw_lm_quantize': (c_int, [vp, c_int, c_int, vp, vp, vp]),
    'fw_lm_head_argmax_q': (c_int, [vp, vp, vp, vp, vp, c_int, c_int, vp, vp]),
    'fw_argmax_finalize': (c_int, [vp, vp, c_int64, vp, vp, c_int, vp]),
    'fw_embed_pos': (c_int, [vp, vp, vp, vp, vp, c_int, c_int, c_int, c_int, vp]),
    'fw_gelu': (c_int, [vp, vp, c_int64, vp]),
    'fw_argmax_f16': (c_int, [vp, c_int64, vp, vp, vp, vp]),
    'fw_ln_gemv': (c_int, [vp, vp, vp, c_float, vp, vp, vp, c_int, c_int, c_int, vp]),
    'fw_gemv_residual': (c_int, [vp, c_int, vp, vp, vp, c_int, vp]),
    'fw_decoder_step': (c_int, [POINTER(Decoder), c_int, vp]),
    'fw_decoder_step_trace': (c_int, [POINTER(Decoder), vp, vp]),
    'fw_decoder_launch': (c_int, [POINTER(Decoder), c_int, c_int, vp]),
    'fw_batch_decoder_step': (c_int, [POINTER(BatchDecoder), c_int, vp]),
    'fw_batch_decoder_launch': (c_int, [POINTER(BatchDecoder), c_int, c_int, vp]),
    'fw_decode_loop_create': (c_int, [POINTER(Decoder), vp, c_int, POINTER(vp)]),
    'fw_decode_loop_launch': (c_int, [vp, vp]),
    'fw_decode_loop_destroy': (c_int, [vp]),
    'fw_log_mel': (c_int, [vp, c_int, c_int, vp, vp, vp, vp, c_int, vp]),
    'fw_gemm_f16': (c_int, [vp, c_int64, vp, c_int64, vp, vp, c_int64, vp, c_int64, c_int, c_int, c_int, c_int,
                            c_float, c_int, vp]),
    'fw_conv1d_k3_f16': (c_int, [vp, c_int, c_int, c_int, vp, vp, vp, c_int64, vp, c_int64, c_int, c_int, c_int,
                                 vp]),
    'fw_layernorm_rows': (c_int, [vp, vp, vp, vp, c_int, c_int, c_float, vp]),
    'fw_encoder_attention': (c_int, [vp, c_int64, c_int, c_int, vp, c_int, c_int, vp, vp]),
    'fw_encoder_forward': (c_int, [POINTER(Encoder), vp]),
}

_lib = None


def header_symbols():
    """Names of every `fw_*` function declared in include/flash_whisper.h."""
    import re
    text = HEADER.read_text()
    return sorted(set(re.findall(r'^\s*(?:const\s+)?\w+\s*\*?\s*(fw_\w+)\s*\(', text, flags=re.M)))


def lib():
    """Loads the library once. Raises RuntimeError if it has not been built (no CPU fallback)."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get('FLASH_WHISPER_LIB', LIB_PATH))
        if not path.exists():
            raise RuntimeError(f'{path} is missing: build it with `python -m flash_whisper_b200.build`')
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def call(name, *args):
    """Calls fw_<name> and raises RuntimeError with the library's message on a non-zero status."""
    fn = getattr(lib(), name)
    rc = fn(*args)
    if rc != FW_OK:
        msg = lib().fw_last_error_string().decode(errors='replace')
        raise RuntimeError(msg or f'{name} failed with status {rc}')
    return rc
