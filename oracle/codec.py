"""12.5 Hz codec decoder restated on the CPU: module stack and incremental state.

TEST INFRASTRUCTURE ONLY (see the package docstring).

Two parts:

1. Stand-in modules for the qwen-tts tokenizer-v2 decoder (absent here),
   with the class names and attributes the reference dispatches on
   (incremental_codec.py:51-96, codec_slots.py:63-99, cached_quantizer.py:12-30):
   ``Qwen3TTSTokenizerV2CausalConvNet`` (conv, stride, padding),
   ``Qwen3TTSTokenizerV2CausalTransConvNet`` (conv, right_pad),
   ``Qwen3TTSTokenizerV2ConvNeXtBlock``, ``Qwen3TTSTokenizerV2DecoderDecoderResidualUnit``,
   ``Qwen3TTSTokenizerV2DecoderDecoderBlock``, ``SnakeBeta`` and a split RVQ
   quantizer. Their full-sequence ``forward`` defines the codec (unpinned at
   the qwen-tts boundary: restated from these call sites and BASELINE shapes).

2. ``IncrementalOracle``: the reference's per-slot streaming state restated -
   causal-conv histories (incremental_codec.py:53-65), transposed-conv
   overlap tails with the bias removed (incremental_codec.py:66-79), the
   sliding-window transformer with a (window - 1)-entry KV tail and absolute
   frame positions (codec_slots.py:27-39, 63-99), frame counters and the
   final clamp. It is pinned against the reference's own IncrementalCodec /
   CodecSlotGraph run on these modules (tests/golden/make_golden.py), and
   chunked decoding must equal the full-sequence forward.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from types import SimpleNamespace

import torch
from torch import nn
from torch.nn import functional as F


# ====================================================================== modules
class SnakeBeta(nn.Module):
    """x + 1 / (exp(beta) + 1e-9) * sin(x * exp(alpha))^2, log-scale parameters."""

    def __init__(self, channels):
        super().__init__()
        self.alpha = nn.Parameter(torch.zeros(channels))
        self.beta = nn.Parameter(torch.zeros(channels))
        self.no_div_by_zero = 1e-9

    def forward(self, x):
        alpha = torch.exp(self.alpha)[None, :, None]
        beta = torch.exp(self.beta)[None, :, None]
        return x + 1.0 / (beta + self.no_div_by_zero) * torch.pow(torch.sin(x * alpha), 2)


class Qwen3TTSTokenizerV2CausalConvNet(nn.Module):
    """Left-padded (causal) Conv1d; `padding` history frames feed the next chunk."""

    def __init__(self, in_channels, out_channels, kernel_size, dilation=1, stride=1, groups=1):
        super().__init__()
        self.conv = nn.Conv1d(in_channels, out_channels, kernel_size, stride=stride, dilation=dilation, groups=groups)
        self.stride = stride
        self.padding = (kernel_size - 1) * dilation - (stride - 1)

    def forward(self, x):
        return self.conv(F.pad(x, (self.padding, 0)))


class Qwen3TTSTokenizerV2CausalTransConvNet(nn.Module):
    """ConvTranspose1d trimmed on the right by kernel - stride (the overlap tail)."""

    def __init__(self, in_channels, out_channels, kernel_size, stride):
        super().__init__()
        self.conv = nn.ConvTranspose1d(in_channels, out_channels, kernel_size, stride=stride)
        self.right_pad = kernel_size - stride

    def forward(self, x):
        y = self.conv(x)
        return y[..., :y.shape[-1] - self.right_pad] if self.right_pad else y


class Qwen3TTSTokenizerV2ConvNeXtBlock(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.dwconv = Qwen3TTSTokenizerV2CausalConvNet(dim, dim, 7, groups=dim)
        self.norm = nn.LayerNorm(dim, eps=1e-6)
        self.pwconv1 = nn.Linear(dim, 4 * dim)
        self.act = nn.GELU()
        self.pwconv2 = nn.Linear(4 * dim, dim)
        self.gamma = nn.Parameter(torch.full((dim,), 1e-6))

    def forward(self, x):
        h = self.dwconv(x).permute(0, 2, 1)
        h = self.pwconv2(self.act(self.pwconv1(self.norm(h))))
        return x + (self.gamma * h).permute(0, 2, 1)


class Qwen3TTSTokenizerV2DecoderDecoderResidualUnit(nn.Module):
    def __init__(self, dim, dilation):
        super().__init__()
        self.act1 = SnakeBeta(dim)
        self.conv1 = Qwen3TTSTokenizerV2CausalConvNet(dim, dim, 7, dilation=dilation)
        self.act2 = SnakeBeta(dim)
        self.conv2 = Qwen3TTSTokenizerV2CausalConvNet(dim, dim, 1)

    def forward(self, x):
        return x + self.conv2(self.act2(self.conv1(self.act1(x))))


class Qwen3TTSTokenizerV2DecoderDecoderBlock(nn.Module):
    def __init__(self, in_dim, out_dim, rate):
        super().__init__()
        self.block = nn.ModuleList([SnakeBeta(in_dim), Qwen3TTSTokenizerV2CausalTransConvNet(in_dim, out_dim, 2 * rate, rate)]
                                   + [Qwen3TTSTokenizerV2DecoderDecoderResidualUnit(out_dim, d) for d in (1, 3, 9)])

    def forward(self, x):
        for m in self.block:
            x = m(x)
        return x


class _Codebook(nn.Module):
    def __init__(self, bins, dim):
        super().__init__()
        self.register_buffer("embedding_sum", torch.zeros(bins, dim))
        self.register_buffer("cluster_usage", torch.ones(bins))
        self.epsilon = 1e-5


class _VQLayer(nn.Module):
    def __init__(self, bins, dim):
        super().__init__()
        self._codebook = _Codebook(bins, dim)
        self.project_out = nn.Identity()


class _RVQGroup(nn.Module):
    def __init__(self, layers, bins, dim, out_dim):
        super().__init__()
        self.vq = SimpleNamespace(layers=nn.ModuleList([_VQLayer(bins, dim) for _ in range(layers)]))
        self._layers = self.vq.layers
        self.output_proj = nn.Conv1d(dim, out_dim, 1, bias=False)

    def decode(self, codes):
        """codes [B, n, T] -> [B, out, T]: normalised codebook rows summed in layer order."""
        quantized = torch.zeros([1])[0]
        for i, layer_codes in enumerate(codes.transpose(0, 1)):
            book = self.vq.layers[i]._codebook
            table = book.embedding_sum / book.cluster_usage.clamp(min=book.epsilon)[:, None]
            quantized = quantized + self.vq.layers[i].project_out(F.embedding(layer_codes, table)).transpose(1, 2)
        return self.output_proj(quantized)


class SplitRVQ(nn.Module):
    """rvq_first (semantic) + rvq_rest groups (cached_quantizer.py:25-30 call shape)."""

    def __init__(self, n_q, n_semantic, bins, dim, out_dim):
        super().__init__()
        self.n_q_semantic = n_semantic
        self.rvq_first = _RVQGroup(n_semantic, bins, dim, out_dim)
        self.rvq_rest = _RVQGroup(n_q - n_semantic, bins, dim, out_dim)
        self.training = False

    def decode(self, codes):
        out = self.rvq_first.decode(codes[:, :self.n_q_semantic])
        if codes.shape[1] > self.n_q_semantic:
            out = out + self.rvq_rest.decode(codes[:, self.n_q_semantic:])
        return out


class RMSNorm(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return self.weight * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype)


def _rotate(x, cos, sin):
    half = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., half:], x[..., :half]], -1) * sin


class Rotary(nn.Module):
    def __init__(self, dim, theta):
        super().__init__()
        self.register_buffer("inv_freq", 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim)), persistent=False)

    def forward(self, x, positions):
        freqs = positions.float()[..., None] * self.inv_freq
        emb = torch.cat([freqs, freqs], -1)
        return emb.cos().to(x.dtype), emb.sin().to(x.dtype)


class TransformerLayer(nn.Module):
    """Pre-norm attention + SwiGLU MLP, each branch scaled by a per-channel layer scale."""

    def __init__(self, hidden, heads, head_dim, ffn, eps, layer_idx, scale):
        super().__init__()
        self.heads, self.head_dim, self.layer_idx = heads, head_dim, layer_idx
        self.input_layernorm = RMSNorm(hidden, eps)
        self.q_proj = nn.Linear(hidden, heads * head_dim, bias=False)
        self.k_proj = nn.Linear(hidden, heads * head_dim, bias=False)
        self.v_proj = nn.Linear(hidden, heads * head_dim, bias=False)
        self.o_proj = nn.Linear(heads * head_dim, hidden, bias=False)
        self.attn_scale = nn.Parameter(torch.full((hidden,), scale))
        self.post_attention_layernorm = RMSNorm(hidden, eps)
        self.gate_proj = nn.Linear(hidden, ffn, bias=False)
        self.up_proj = nn.Linear(hidden, ffn, bias=False)
        self.down_proj = nn.Linear(ffn, hidden, bias=False)
        self.mlp_scale = nn.Parameter(torch.full((hidden,), scale))

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None, use_cache=False,
                cache_position=None, position_embeddings=None, **kwargs):
        B, T, _ = hidden_states.shape
        x = self.input_layernorm(hidden_states)
        q = self.q_proj(x).view(B, T, self.heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.heads, self.head_dim).transpose(1, 2)
        cos, sin = position_embeddings
        q = _rotate(q, cos[:, None], sin[:, None])
        k = _rotate(k, cos[:, None], sin[:, None])
        if past_key_values is not None:
            k, v = past_key_values.update(k, v, self.layer_idx, {"cos": cos, "sin": sin})
        scores = q @ k.transpose(-1, -2) * self.head_dim ** -0.5
        if attention_mask is not None:
            scores = scores + attention_mask
        attn = (torch.softmax(scores.float(), -1).to(q.dtype) @ v).transpose(1, 2).reshape(B, T, -1)
        h = hidden_states + self.attn_scale * self.o_proj(attn)
        y = self.post_attention_layernorm(h)
        return h + self.mlp_scale * self.down_proj(F.silu(self.gate_proj(y)) * self.up_proj(y))


class Transformer(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.input_proj = nn.Linear(cfg.latent, cfg.hidden)
        self.layers = nn.ModuleList([TransformerLayer(cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.eps, i,
                                                      cfg.layer_scale) for i in range(cfg.layers)])
        self.norm = RMSNorm(cfg.hidden, cfg.eps)
        self.output_proj = nn.Linear(cfg.hidden, cfg.latent)
        self.rotary_emb = Rotary(cfg.head_dim, cfg.theta)
        self.window = cfg.window

    def forward(self, inputs_embeds):
        """Full sequence: causal sliding-window attention over positions 0..T-1."""
        B, T, _ = inputs_embeds.shape
        h = self.input_proj(inputs_embeds)
        pos = torch.arange(T)
        allowed = (pos[None, :] <= pos[:, None]) & (pos[None, :] > pos[:, None] - self.window)
        mask = torch.where(allowed, 0.0, torch.finfo(h.dtype).min).to(h.dtype)[None, None]
        rot = self.rotary_emb(h, pos[None].expand(B, T))
        for layer in self.layers:
            h = layer(h, attention_mask=mask, position_embeddings=rot)
        return SimpleNamespace(last_hidden_state=self.output_proj(self.norm(h)))


class CodecDecoder(nn.Module):
    """Tokenizer-v2 decoder: RVQ -> causal conv -> transformer -> upsampling -> decoder blocks -> PCM."""

    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        self.config = SimpleNamespace(num_quantizers=cfg.codebooks, sliding_window=cfg.window,
                                      num_key_value_heads=cfg.heads, head_dim=cfg.head_dim)
        self.quantizer = SplitRVQ(cfg.codebooks, cfg.semantic_codebooks, cfg.codebook_size, cfg.codebook_dim,
                                  cfg.codebook_dim)
        self.pre_conv = Qwen3TTSTokenizerV2CausalConvNet(cfg.codebook_dim, cfg.latent, 3)
        self.pre_transformer = Transformer(cfg)
        self.upsample = nn.ModuleList([nn.ModuleList([Qwen3TTSTokenizerV2CausalTransConvNet(cfg.latent, cfg.latent, r, r),
                                                      Qwen3TTSTokenizerV2ConvNeXtBlock(cfg.latent)])
                                       for r in cfg.upsampling_ratios])
        blocks = [Qwen3TTSTokenizerV2CausalConvNet(cfg.latent, cfg.decoder_dim, 7)]
        dim = cfg.decoder_dim
        for rate in cfg.upsample_rates:
            blocks.append(Qwen3TTSTokenizerV2DecoderDecoderBlock(dim, dim // 2, rate))
            dim //= 2
        blocks += [SnakeBeta(dim), Qwen3TTSTokenizerV2CausalConvNet(dim, 1, 7)]
        self.decoder = nn.ModuleList(blocks)

    def forward(self, codes):
        h = self.quantizer.decode(codes)
        h = self.pre_conv(h).transpose(1, 2)
        h = self.pre_transformer(inputs_embeds=h).last_hidden_state.permute(0, 2, 1)
        for blocks in self.upsample:
            for block in blocks:
                h = block(h)
        for block in self.decoder:
            h = block(h)
        return h.clamp(min=-1, max=1)


def randomize(decoder: CodecDecoder, seed: int, alpha_range=(0.5, 1.5)) -> CodecDecoder:
    """Seeded random init: N(0, 0.02) weights (conv weights scaled by fan-in so audio stays O(1)),
    SnakeBeta alpha ~ U[alpha_range] (stored as log), beta ~ N(0, 0.1), codebooks N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in decoder.named_parameters():
            if name.endswith("alpha"):
                lo, hi = alpha_range
                p.copy_(torch.log(lo + (hi - lo) * torch.rand(p.shape, generator=g)))
            elif name.endswith("beta"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
            elif p.ndim == 1 and ("norm" in name or "scale" in name or name.endswith("gamma")):
                p.copy_(1.0 + 0.02 * torch.randn(p.shape, generator=g) if "norm" in name
                        else 0.1 + 0.02 * torch.randn(p.shape, generator=g))
            elif p.ndim == 1:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
            else:
                fan_in = p[0].numel() if p.ndim > 1 else 1
                p.copy_(torch.randn(p.shape, generator=g) * (0.5 / math.sqrt(fan_in)))
        for group in (decoder.quantizer.rvq_first, decoder.quantizer.rvq_rest):
            for layer in group.vq.layers:
                book = layer._codebook
                book.embedding_sum.copy_(torch.randn(book.embedding_sum.shape, generator=g))
                book.cluster_usage.copy_(0.5 + torch.rand(book.cluster_usage.shape, generator=g))
    return decoder.eval()


# ====================================================================== incremental state (oracle)
@dataclass
class SlotState:
    history: dict = field(default_factory=dict)   # module -> [C, width]
    keys: list = None                             # per layer [heads, window-1, head_dim]
    values: list = None
    frames: int = 0


class IncrementalOracle:
    """Per-slot streaming decode of a CodecDecoder (the reference's state logic restated)."""

    def __init__(self, decoder: CodecDecoder):
        self.d = decoder
        self.window = decoder.cfg.window
        self.history = self.window - 1

    def new_state(self) -> SlotState:
        c = self.d.cfg
        zeros = [torch.zeros(c.heads, self.history, c.head_dim) for _ in range(c.layers)]
        return SlotState(keys=zeros, values=[z.clone() for z in zeros])

    def _module(self, m, x, st: SlotState):
        kind = type(m).__name__
        if kind == "Qwen3TTSTokenizerV2CausalConvNet":
            if m.padding:
                prev = st.history.get(m, torch.zeros(x.shape[0], x.shape[1], m.padding))
                joined = torch.cat([prev, x], -1)
                st.history[m] = joined[..., -m.padding:].clone()
            else:
                joined = x
            return m.conv(joined)
        if kind == "Qwen3TTSTokenizerV2CausalTransConvNet":
            y = m.conv(x)
            if m.right_pad:
                prev = st.history.get(m)
                if prev is not None:
                    y[..., :m.right_pad] += prev
                tail = y[..., -m.right_pad:]
                if m.conv.bias is not None:
                    tail = tail - m.conv.bias.view(1, -1, 1)
                st.history[m] = tail.clone()
                y = y[..., :-m.right_pad]
            return y
        if kind == "Qwen3TTSTokenizerV2ConvNeXtBlock":
            h = self._module(m.dwconv, x, st).permute(0, 2, 1)
            h = m.pwconv2(m.act(m.pwconv1(m.norm(h))))
            return x + (m.gamma * h).permute(0, 2, 1)
        if kind == "Qwen3TTSTokenizerV2DecoderDecoderResidualUnit":
            h = self._module(m.conv1, m.act1(x), st)
            return x + self._module(m.conv2, m.act2(h), st)
        if kind == "Qwen3TTSTokenizerV2DecoderDecoderBlock":
            for child in m.block:
                x = self._module(child, x, st)
            return x
        if kind == "SnakeBeta":
            return m(x)
        raise TypeError(kind)

    @torch.inference_mode()
    def decode(self, codes, st: SlotState):
        """codes [1, n_q, T] of one slot -> PCM [1, 1, T * samples_per_frame]."""
        d, c = self.d, self.d.cfg
        T = codes.shape[-1]
        h = d.quantizer.decode(codes)
        h = self._module(d.pre_conv, h, st).transpose(1, 2)
        tr = d.pre_transformer
        h = tr.input_proj(h)
        pos = st.frames + torch.arange(T)
        key_pos = st.frames + torch.arange(-self.history, T)
        allowed = (key_pos[None, :] >= 0) & (key_pos[None, :] <= pos[:, None]) & \
                  (key_pos[None, :] > pos[:, None] - self.window)
        mask = torch.where(allowed, 0.0, torch.finfo(h.dtype).min).to(h.dtype)[None, None]
        rot = tr.rotary_emb(h, pos[None])
        state = self

        class _Cache:
            def update(self_, k, v, layer_idx, kw):
                kk = torch.cat([st.keys[layer_idx][None], k], 2)
                vv = torch.cat([st.values[layer_idx][None], v], 2)
                st.keys[layer_idx] = kk[0, :, -state.history:].clone()
                st.values[layer_idx] = vv[0, :, -state.history:].clone()
                return kk, vv

        cache = _Cache()
        for layer in tr.layers:
            h = layer(h, attention_mask=mask, position_embeddings=rot, past_key_values=cache)
        h = tr.output_proj(tr.norm(h)).permute(0, 2, 1)
        for blocks in d.upsample:
            for block in blocks:
                h = self._module(block, h, st)
        for block in d.decoder:
            h = self._module(block, h, st)
        st.frames += T
        return h.clamp(min=-1, max=1)
