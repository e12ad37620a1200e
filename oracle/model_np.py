"""numpy restatement of the reference CUDA backend's model math (test infrastructure).

Follows custom/model.py: the fp16 HF encoder + cross-K/V projection (_encode, :143-147, with the
transformers WhisperEncoder / WhisperEncoderLayer / WhisperAttention math: conv1+GELU, conv2+GELU,
+ sinusoid positions, pre-LN layers with q_proj(x) * head_dim**-0.5, final LN), the per-token
decode step (_step, :107-123) and the prompt / greedy handling of transcribe (:196-215). Matmuls run
in float32 (the fp32 accumulators of the tensor-core / cuBLAS path); every value the reference
stores as fp16 is rounded to fp16 here at the same point, so activations track the GPU pipeline to
fp16 rounding noise.
"""

import numpy as np
from scipy.special import erf


def r16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def gelu(x):
    x = np.asarray(x, np.float32)
    return x * 0.5 * (1.0 + erf(x * np.float32(0.7071067811865476)))


def layer_norm(x, g, b, eps=1e-5):
    x = np.asarray(x, np.float32)
    mean = x.mean(axis=-1, keepdims=True, dtype=np.float64)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True, dtype=np.float64)
    return ((x - mean) / np.sqrt(var + eps) * g + b).astype(np.float32)


def linear(x, w, b=None):
    y = np.asarray(x, np.float32) @ w.T
    if b is not None:
        y = y + b
    return y


def softmax(s, axis=-1):
    s = s - s.max(axis=axis, keepdims=True)
    e = np.exp(s)
    return e / e.sum(axis=axis, keepdims=True)


class WhisperOracle:
    """numpy Whisper for parity checks. `sd` is a torch state dict (HF names).

    fp16=True rounds weights and every stored activation to fp16 like the GPU pipelines;
    fp16=False is plain fp32 (used to pin this restatement against transformers on the CPU)."""

    def __init__(self, sd, dims, decoder_only=False, fp16=True):
        self.dims = dims
        self.r = r16 if fp16 else (lambda x: np.asarray(x, np.float32))
        self.w = {}
        for k, v in sd.items():
            if decoder_only and k.startswith('model.encoder'):
                continue
            self.w[k] = self.r(v.float().numpy())
        self.reset()

    def reset(self):
        d = self.dims
        self.self_k = np.zeros((d.decoder_layers, d.heads, d.max_pos, d.head_dim), np.float32)
        self.self_v = np.zeros_like(self.self_k)

    # ---- encoder -------------------------------------------------------------------------
    def _conv(self, x, name, stride):
        """Conv1d(k=3, pad=1) on time-major x [T, C] -> [T', N], fp32 accumulate, fp16 out."""
        w = self.w[f'{name}.weight']  # [N, C, 3]
        xp = np.concatenate([np.zeros((1, x.shape[1]), np.float32), x, np.zeros((1, x.shape[1]), np.float32)])
        t_out = (x.shape[0] - 1) // stride + 1
        cols = np.concatenate([xp[j:j + stride * (t_out - 1) + 1:stride] for j in range(3)], axis=1)  # [T', 3C]
        wk = w.transpose(0, 2, 1).reshape(w.shape[0], -1)
        return self.r(linear(cols, wk, self.w[f'{name}.bias']))

    def encoder(self, mel16):
        """mel [n_mels, 2*enc_len] (fp16 values) -> final-LN encoder states [enc_len, d_model]."""
        d = self.dims
        p = 'model.encoder'
        x = np.asarray(mel16, np.float32).T
        x = self.r(gelu(self._conv(x, f'{p}.conv1', 1)))
        x = self.r(gelu(self._conv(x, f'{p}.conv2', 2)))
        x = self.r(x + self.w[f'{p}.embed_positions.weight'][:x.shape[0]])
        hd, nh = d.head_dim, d.heads
        for i in range(d.encoder_layers):
            q_ = f'{p}.layers.{i}'
            y = self.r(layer_norm(x, self.w[f'{q_}.self_attn_layer_norm.weight'], self.w[f'{q_}.self_attn_layer_norm.bias']))
            q = self.r(self.r(linear(y, self.w[f'{q_}.self_attn.q_proj.weight'], self.w[f'{q_}.self_attn.q_proj.bias']))
                    * np.float32(hd ** -0.5))
            k = self.r(linear(y, self.w[f'{q_}.self_attn.k_proj.weight']))
            v = self.r(linear(y, self.w[f'{q_}.self_attn.v_proj.weight'], self.w[f'{q_}.self_attn.v_proj.bias']))
            T = x.shape[0]
            qh = q.reshape(T, nh, hd).transpose(1, 0, 2)
            kh = k.reshape(T, nh, hd).transpose(1, 0, 2)
            vh = v.reshape(T, nh, hd).transpose(1, 0, 2)
            attn = softmax(qh @ kh.transpose(0, 2, 1)) @ vh
            attn = self.r(attn.transpose(1, 0, 2).reshape(T, -1))
            x = self.r(x + self.r(linear(attn, self.w[f'{q_}.self_attn.out_proj.weight'],
                                   self.w[f'{q_}.self_attn.out_proj.bias'])))
            y = self.r(layer_norm(x, self.w[f'{q_}.final_layer_norm.weight'], self.w[f'{q_}.final_layer_norm.bias']))
            f = self.r(gelu(self.r(linear(y, self.w[f'{q_}.fc1.weight'], self.w[f'{q_}.fc1.bias']))))
            x = self.r(x + self.r(linear(f, self.w[f'{q_}.fc2.weight'], self.w[f'{q_}.fc2.bias'])))
        return self.r(layer_norm(x, self.w[f'{p}.layer_norm.weight'], self.w[f'{p}.layer_norm.bias']))

    def set_cross(self, enc):
        """Cross K/V per decoder layer: [layers, heads, enc_len, head_dim] (custom/model.py:145-146)."""
        d = self.dims
        ks, vs = [], []
        for i in range(d.decoder_layers):
            a = f'model.decoder.layers.{i}.encoder_attn'
            k = self.r(linear(enc, self.w[f'{a}.k_proj.weight']))
            v = self.r(linear(enc, self.w[f'{a}.v_proj.weight'], self.w[f'{a}.v_proj.bias']))
            ks.append(k.reshape(-1, d.heads, d.head_dim).transpose(1, 0, 2))
            vs.append(v.reshape(-1, d.heads, d.head_dim).transpose(1, 0, 2))
        self.cross_k, self.cross_v = np.stack(ks), np.stack(vs)

    # ---- decoder -------------------------------------------------------------------------
    def embed(self, token, pos):
        """Layer-0 input: fp16(embed_tokens[token] + embed_positions[pos]) (custom/model.py:110)."""
        return self.r(self.w['model.decoder.embed_tokens.weight'][token] + self.w['model.decoder.embed_positions.weight'][pos])

    def self_block(self, i, h, pos):
        """LN1 -> q/k/v -> cache write at `pos` -> attention over pos + 1 keys -> out_proj -> residual
        (custom/model.py:113-116). Returns (attention output, new h, k row, v row)."""
        d = self.dims
        hd, nh = d.head_dim, d.heads
        p = f'model.decoder.layers.{i}'
        y = self.r(layer_norm(h, self.w[f'{p}.self_attn_layer_norm.weight'], self.w[f'{p}.self_attn_layer_norm.bias']))
        q = self.r(linear(y, self.w[f'{p}.self_attn.q_proj.weight'], self.w[f'{p}.self_attn.q_proj.bias']))
        k = self.r(linear(y, self.w[f'{p}.self_attn.k_proj.weight']))
        v = self.r(linear(y, self.w[f'{p}.self_attn.v_proj.weight'], self.w[f'{p}.self_attn.v_proj.bias']))
        self.self_k[i, :, pos] = k.reshape(nh, hd)
        self.self_v[i, :, pos] = v.reshape(nh, hd)
        K, V = self.self_k[i, :, :pos + 1], self.self_v[i, :, :pos + 1]
        s = np.einsum('hd,hld->hl', q.reshape(nh, hd), K) * np.float32(hd ** -0.5)
        attn = self.r(np.einsum('hl,hld->hd', softmax(s), V).reshape(-1))
        h = self.r(h + self.r(linear(attn, self.w[f'{p}.self_attn.out_proj.weight'], self.w[f'{p}.self_attn.out_proj.bias'])))
        return attn, h, k, v

    def cross_block(self, i, h):
        """LN2 -> cross q -> attention over the encoder cache -> out_proj -> residual
        (custom/model.py:116-119). Returns (attention output, new h)."""
        d = self.dims
        hd, nh = d.head_dim, d.heads
        p = f'model.decoder.layers.{i}'
        y = self.r(layer_norm(h, self.w[f'{p}.encoder_attn_layer_norm.weight'], self.w[f'{p}.encoder_attn_layer_norm.bias']))
        q = self.r(linear(y, self.w[f'{p}.encoder_attn.q_proj.weight'], self.w[f'{p}.encoder_attn.q_proj.bias']))
        s = np.einsum('hd,hld->hl', q.reshape(nh, hd), self.cross_k[i]) * np.float32(hd ** -0.5)
        attn = self.r(np.einsum('hl,hld->hd', softmax(s), self.cross_v[i]).reshape(-1))
        h = self.r(h + self.r(linear(attn, self.w[f'{p}.encoder_attn.out_proj.weight'],
                                     self.w[f'{p}.encoder_attn.out_proj.bias'])))
        return attn, h

    def fc1(self, i, h):
        """LN3 -> fc1 -> GELU (custom/model.py:119-120)."""
        p = f'model.decoder.layers.{i}'
        y = self.r(layer_norm(h, self.w[f'{p}.final_layer_norm.weight'], self.w[f'{p}.final_layer_norm.bias']))
        return self.r(gelu(self.r(linear(y, self.w[f'{p}.fc1.weight'], self.w[f'{p}.fc1.bias']))))

    def fc2(self, i, h, f):
        """fc2 -> residual (custom/model.py:120-121)."""
        p = f'model.decoder.layers.{i}'
        return self.r(h + self.r(linear(f, self.w[f'{p}.fc2.weight'], self.w[f'{p}.fc2.bias'])))

    def final(self, h):
        """Final LayerNorm and fp16 logits over the tied vocab matrix (custom/model.py:122)."""
        y = self.r(layer_norm(h, self.w['model.decoder.layer_norm.weight'], self.w['model.decoder.layer_norm.bias']))
        return y, self.r(self.w['model.decoder.embed_tokens.weight'] @ y)

    def step(self, token, pos):
        """One decode step (custom/model.py:107-122): returns fp16-valued logits [vocab] (float32)."""
        h = self.embed(token, pos)
        for i in range(self.dims.decoder_layers):
            _, h, _, _ = self.self_block(i, h, pos)
            _, h = self.cross_block(i, h)
            h = self.fc2(i, h, self.fc1(i, h))
        return self.final(h)[1]

    def greedy(self, n_tokens, prompt, base_mask=None, first_mask=None, forced=None):
        """Greedy decode after the prompt (custom/model.py:196-215, EOS ignored).

        Returns (tokens, gaps) where gaps[i] is the fp16-logit margin between the chosen token and
        the best other unsuppressed token at step i. With `forced`, the given tokens are fed back
        instead of the oracle's own choices (teacher forcing) and gaps are measured for them."""
        self.reset()
        tokens, gaps, chosen_logit_gap = [], [], []
        pos = 0
        for t in prompt[:-1]:
            self.step(t, pos)
            pos += 1
        cur = prompt[-1]
        for i in range(n_tokens):
            logits = self.step(cur, pos)
            mask = first_mask if i == 0 else base_mask
            vals = logits.copy()
            if mask is not None:
                vals[np.asarray(mask, bool)] = -np.inf
            best = int(np.argmax(vals))
            top = vals[best]
            vals2 = vals.copy()
            vals2[best] = -np.inf
            gaps.append(float(top - vals2.max()))
            tok = best if forced is None else int(forced[i])
            chosen_logit_gap.append(float(top - vals[tok]))
            tokens.append(best)
            cur = tok
            pos = min(pos + 1, self.dims.max_pos - 1)
        return tokens, gaps, chosen_logit_gap
