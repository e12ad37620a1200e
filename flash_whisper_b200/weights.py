"""Whisper-large-v3-turbo dimensions, seeded random-init weights and device packing.

No checkpoint or tokenizer is available offline, so every test, bench and parity run uses the
architecture of openai/whisper-large-v3-turbo with weights drawn here: N(0, std) for every linear,
conv and embedding weight (std 0.02, transformers' WhisperConfig.init_std), LayerNorm gamma 1 and
beta 0, biases 0 (or N(0, bias_std) to exercise the bias paths), the encoder's sinusoid position
table, and a zero padding row in the token embedding, i.e. what
WhisperForConditionalGeneration(WhisperConfig(...)) initialises. Each tensor is drawn from its own
CPU torch.Generator seeded from (seed, name), so the weights are identical on every machine and
independent of transformers' init order. Names follow the HF state dict so the same dict loads
into the transformers model used by the oracle.

`pack_decoder` / `pack_encoder` build the fp16 device tensors in the layouts the kernels read:
the fused QKV matrix with a zeroed K bias (custom/model.py:87-88), the stacked cross K/V matrix of
all decoder layers (custom/model.py:54-55), and conv weights reordered (tap, channel).
"""

import hashlib
import math
from dataclasses import dataclass, field
from types import SimpleNamespace

import torch


@dataclass(frozen=True)
class WhisperDims:
    d_model: int = 1280
    heads: int = 20
    encoder_layers: int = 32
    decoder_layers: int = 4
    ffn: int = 5120
    vocab: int = 51866
    n_mels: int = 128
    enc_len: int = 1500
    max_pos: int = 448
    pad_token_id: int = 50256
    eos_token_id: int = 50257
    # '<|startoftranscript|>', '<|en|>', '<|transcribe|>', '<|notimestamps|>' of the large-v3 vocab
    prompt: tuple = (50258, 50259, 50360, 50364)
    begin_suppress: tuple = (220, 50257)
    suppress: tuple = field(default_factory=tuple)
    eps: float = 1e-5

    @property
    def head_dim(self):
        return self.d_model // self.heads

    @property
    def n_frames(self):
        return 2 * self.enc_len


TURBO = WhisperDims()


def hf_config(dims=TURBO):
    """transformers WhisperConfig of these dimensions."""
    from transformers import WhisperConfig
    return WhisperConfig(
        vocab_size=dims.vocab, num_mel_bins=dims.n_mels, d_model=dims.d_model,
        encoder_layers=dims.encoder_layers, decoder_layers=dims.decoder_layers,
        encoder_attention_heads=dims.heads, decoder_attention_heads=dims.heads,
        encoder_ffn_dim=dims.ffn, decoder_ffn_dim=dims.ffn, max_source_positions=dims.enc_len,
        max_target_positions=dims.max_pos, pad_token_id=dims.pad_token_id, eos_token_id=dims.eos_token_id,
        bos_token_id=dims.eos_token_id, decoder_start_token_id=dims.prompt[0],
        begin_suppress_tokens=list(dims.begin_suppress), activation_function='gelu', init_std=0.02,
        scale_embedding=False)


def sinusoids(length, channels, max_timescale=10000):
    """Whisper's encoder position table: [sin | cos] over geometric timescales."""
    log_inc = math.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-log_inc * torch.arange(channels // 2, dtype=torch.float32))
    scaled = torch.arange(length, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cat([scaled.sin(), scaled.cos()], dim=1)


def param_shapes(dims=TURBO):
    """HF state-dict names and shapes of WhisperForConditionalGeneration (without tied proj_out)."""
    d, f = dims.d_model, dims.ffn
    shapes = {
        'model.encoder.conv1.weight': (d, dims.n_mels, 3), 'model.encoder.conv1.bias': (d,),
        'model.encoder.conv2.weight': (d, d, 3), 'model.encoder.conv2.bias': (d,),
        'model.encoder.embed_positions.weight': (dims.enc_len, d),
    }

    def attn(prefix):
        shapes.update({f'{prefix}.q_proj.weight': (d, d), f'{prefix}.q_proj.bias': (d,),
                       f'{prefix}.k_proj.weight': (d, d),
                       f'{prefix}.v_proj.weight': (d, d), f'{prefix}.v_proj.bias': (d,),
                       f'{prefix}.out_proj.weight': (d, d), f'{prefix}.out_proj.bias': (d,)})

    def ln(prefix):
        shapes.update({f'{prefix}.weight': (d,), f'{prefix}.bias': (d,)})

    def mlp(prefix):
        shapes.update({f'{prefix}.fc1.weight': (f, d), f'{prefix}.fc1.bias': (f,),
                       f'{prefix}.fc2.weight': (d, f), f'{prefix}.fc2.bias': (d,)})

    for i in range(dims.encoder_layers):
        p = f'model.encoder.layers.{i}'
        attn(f'{p}.self_attn')
        ln(f'{p}.self_attn_layer_norm')
        mlp(p)
        ln(f'{p}.final_layer_norm')
    ln('model.encoder.layer_norm')
    shapes['model.decoder.embed_tokens.weight'] = (dims.vocab, d)
    shapes['model.decoder.embed_positions.weight'] = (dims.max_pos, d)
    for i in range(dims.decoder_layers):
        p = f'model.decoder.layers.{i}'
        attn(f'{p}.self_attn')
        ln(f'{p}.self_attn_layer_norm')
        attn(f'{p}.encoder_attn')
        ln(f'{p}.encoder_attn_layer_norm')
        mlp(p)
        ln(f'{p}.final_layer_norm')
    ln('model.decoder.layer_norm')
    return shapes


def _generator(seed, name):
    digest = hashlib.sha256(f'{seed}:{name}'.encode()).digest()
    return torch.Generator().manual_seed(int.from_bytes(digest[:8], 'little') & ((1 << 63) - 1))


def random_state_dict(seed=0, dims=TURBO, std=0.02, bias_std=0.0, ln_std=0.0, names=None):
    """Seeded random-init weights (fp32, CPU) keyed by HF names. `names` limits which are built."""
    out = {}
    for name, shape in param_shapes(dims).items():
        if names is not None and name not in names:
            continue
        if name == 'model.encoder.embed_positions.weight':
            t = sinusoids(*shape)
        elif name.endswith('layer_norm.weight'):
            t = torch.ones(shape)
            if ln_std:
                t += ln_std * torch.randn(shape, generator=_generator(seed, name))
        elif name.endswith('layer_norm.bias') or name.endswith('.bias'):
            t = torch.zeros(shape)
            if bias_std and not name.endswith('layer_norm.bias'):
                t = bias_std * torch.randn(shape, generator=_generator(seed, name))
            elif ln_std and name.endswith('layer_norm.bias'):
                t = ln_std * torch.randn(shape, generator=_generator(seed, name))
        else:
            t = std * torch.randn(shape, generator=_generator(seed, name))
            if name == 'model.decoder.embed_tokens.weight' and dims.pad_token_id < dims.vocab:
                t[dims.pad_token_id] = 0
        out[name] = t
    return out


def varied_state_dict(seed=0, dims=TURBO, decoder_std=0.05):
    """Seeded weights whose greedy decode is not degenerate, for token-level parity tests.

    With the HF init (std 0.02 everywhere, tied LM head) a random decoder's residual stream stays
    dominated by the current token's embedding, so greedy decoding repeats one token and a token
    match says little about the layers. Here the decoder weights are drawn with `decoder_std`, the
    biases with std 0.02 and the LayerNorm parameters perturbed by 0.1, which makes the layers move the
    argmax from step to step; the encoder keeps the HF init."""
    names = param_shapes(dims)
    enc = [n for n in names if not n.startswith('model.decoder')]
    dec = [n for n in names if n.startswith('model.decoder')]
    out = random_state_dict(seed, dims, names=enc)
    out.update(random_state_dict(seed, dims, std=decoder_std, bias_std=0.02, ln_std=0.1, names=dec))
    return out


def load_hf_model(state_dict, dims=TURBO, dtype=torch.float32):
    """transformers WhisperForConditionalGeneration holding `state_dict` (oracle / CPU baseline)."""
    from transformers import WhisperForConditionalGeneration
    with torch.device('meta'):
        model = WhisperForConditionalGeneration(hf_config(dims))
    model.load_state_dict(state_dict, strict=False, assign=True)
    model.tie_weights()
    model.proj_out.weight = model.model.decoder.embed_tokens.weight
    return model.to(dtype).eval()


def pack_decoder(sd, dims=TURBO, device='cuda', dtype=torch.float16):
    """Decoder weights in kernel layout (fp16 on `device`). The attention output projections are
    head-major [heads, d_model, head_dim]: the slice of head h, W[:, h*64:(h+1)*64], is contiguous,
    so the per-head attention block streams it with one bulk copy."""
    def t(name):
        return sd[name].to(device=device, dtype=dtype).contiguous()

    def head_major(w):
        return w.view(w.size(0), dims.heads, dims.head_dim).permute(1, 0, 2).contiguous()

    layers = []
    for i in range(dims.decoder_layers):
        p = f'model.decoder.layers.{i}'
        zeros = torch.zeros(dims.d_model, device=device, dtype=dtype)
        layers.append(SimpleNamespace(
            ln1=(t(f'{p}.self_attn_layer_norm.weight'), t(f'{p}.self_attn_layer_norm.bias')),
            ln2=(t(f'{p}.encoder_attn_layer_norm.weight'), t(f'{p}.encoder_attn_layer_norm.bias')),
            ln3=(t(f'{p}.final_layer_norm.weight'), t(f'{p}.final_layer_norm.bias')),
            qkv_w=torch.cat([t(f'{p}.self_attn.q_proj.weight'), t(f'{p}.self_attn.k_proj.weight'),
                             t(f'{p}.self_attn.v_proj.weight')]).contiguous(),
            qkv_b=torch.cat([t(f'{p}.self_attn.q_proj.bias'), zeros, t(f'{p}.self_attn.v_proj.bias')]).contiguous(),
            out=(head_major(t(f'{p}.self_attn.out_proj.weight')), t(f'{p}.self_attn.out_proj.bias')),
            cross_q=(t(f'{p}.encoder_attn.q_proj.weight'), t(f'{p}.encoder_attn.q_proj.bias')),
            cross_out=(head_major(t(f'{p}.encoder_attn.out_proj.weight')), t(f'{p}.encoder_attn.out_proj.bias')),
            fc1=(t(f'{p}.fc1.weight'), t(f'{p}.fc1.bias')),
            fc2=(t(f'{p}.fc2.weight'), t(f'{p}.fc2.bias'))))
    cross_w = torch.cat([torch.cat([t(f'model.decoder.layers.{i}.encoder_attn.k_proj.weight'),
                                    t(f'model.decoder.layers.{i}.encoder_attn.v_proj.weight')])
                         for i in range(dims.decoder_layers)]).contiguous()
    cross_b = torch.cat([torch.cat([torch.zeros(dims.d_model, device=device, dtype=dtype),
                                    t(f'model.decoder.layers.{i}.encoder_attn.v_proj.bias')])
                         for i in range(dims.decoder_layers)]).contiguous()
    embed = t('model.decoder.embed_tokens.weight')
    return SimpleNamespace(layers=layers, embed=embed, lm_head=embed, pos_embed=t('model.decoder.embed_positions.weight'),
                           final_ln=(t('model.decoder.layer_norm.weight'), t('model.decoder.layer_norm.bias')),
                           cross_w=cross_w, cross_b=cross_b)


def pack_encoder(sd, dims=TURBO, device='cuda', dtype=torch.float16):
    """Encoder weights in kernel layout: conv weights [out, 3*in] ordered (tap, channel)."""
    def t(name):
        return sd[name].to(device=device, dtype=dtype).contiguous()

    def conv(name):
        w = sd[name]
        return w.permute(0, 2, 1).reshape(w.size(0), -1).to(device=device, dtype=dtype).contiguous()

    layers = []
    for i in range(dims.encoder_layers):
        p = f'model.encoder.layers.{i}'
        zeros = torch.zeros(dims.d_model, device=device, dtype=dtype)
        layers.append(SimpleNamespace(
            ln1=(t(f'{p}.self_attn_layer_norm.weight'), t(f'{p}.self_attn_layer_norm.bias')),
            ln2=(t(f'{p}.final_layer_norm.weight'), t(f'{p}.final_layer_norm.bias')),
            qkv_w=torch.cat([t(f'{p}.self_attn.q_proj.weight'), t(f'{p}.self_attn.k_proj.weight'),
                             t(f'{p}.self_attn.v_proj.weight')]).contiguous(),
            qkv_b=torch.cat([t(f'{p}.self_attn.q_proj.bias'), zeros, t(f'{p}.self_attn.v_proj.bias')]).contiguous(),
            out=(t(f'{p}.self_attn.out_proj.weight'), t(f'{p}.self_attn.out_proj.bias')),
            fc1=(t(f'{p}.fc1.weight'), t(f'{p}.fc1.bias')),
            fc2=(t(f'{p}.fc2.weight'), t(f'{p}.fc2.bias'))))
    return SimpleNamespace(layers=layers, conv1=(conv('model.encoder.conv1.weight'), t('model.encoder.conv1.bias')),
                           conv2=(conv('model.encoder.conv2.weight'), t('model.encoder.conv2.bias')),
                           pos=t('model.encoder.embed_positions.weight'),
                           final_ln=(t('model.encoder.layer_norm.weight'), t('model.encoder.layer_norm.bias')))
