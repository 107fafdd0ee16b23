"""Stand-ins for the qwen-tts module classes the plugin installers look for (by class name).

qwen-tts is not installed here, so these small torch modules carry the same class
names, attributes and call signatures as the qwen-tts decoder modules the
reference's install functions match (packed_attention.py:88-95, packed_mlp.py:30-37,
operators.py:26-38, fused_decoder.py:40-47). Their forward passes compute in fp32
whatever the parameter dtype (q/k RMSNorm, rotate-half RoPE, causal GQA attention,
SwiGLU MLP) and serve as the reference numerics of the plugin tests.
"""
from types import SimpleNamespace

import torch
import torch.nn.functional as F


class Qwen3TTSRMSNorm(torch.nn.Module):
    def __init__(self, width, eps=1e-6):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(width))
        self.variance_epsilon = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
                * self.weight.float()).to(x.dtype)


def rotate_half(x):
    a, b = x.chunk(2, dim=-1)
    return torch.cat((-b, a), dim=-1)


class Qwen3TTSAttention(torch.nn.Module):
    def __init__(self, hidden, q_heads, kv_heads, head_dim, layer_idx=0, bias=False):
        super().__init__()
        self.q_proj = torch.nn.Linear(hidden, q_heads * head_dim, bias=bias)
        self.k_proj = torch.nn.Linear(hidden, kv_heads * head_dim, bias=bias)
        self.v_proj = torch.nn.Linear(hidden, kv_heads * head_dim, bias=bias)
        self.o_proj = torch.nn.Linear(q_heads * head_dim, hidden, bias=False)
        self.q_norm, self.k_norm = Qwen3TTSRMSNorm(head_dim), Qwen3TTSRMSNorm(head_dim)
        self.head_dim, self.layer_idx, self.scaling = head_dim, layer_idx, head_dim ** -0.5
        self.sliding_window, self.attention_dropout = None, 0.0
        self.config = SimpleNamespace(_attn_implementation="sdpa")

    def forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None, cache_position=None,
                **kwargs):
        b, s, _ = hidden_states.shape
        d = self.head_dim
        x = hidden_states.float()

        def proj(layer):
            return F.linear(x, layer.weight.float(), None if layer.bias is None else layer.bias.float())

        q = self.q_norm(proj(self.q_proj).view(b, s, -1, d)).float()
        k = self.k_norm(proj(self.k_proj).view(b, s, -1, d)).float()
        v = proj(self.v_proj).view(b, s, -1, d)
        cos, sin = position_embeddings
        if cos.ndim == 4:   # multimodal: identical axes, take the first
            cos, sin = cos[0], sin[0]
        cos, sin = cos.float()[:, :, None], sin.float()[:, :, None]
        q, k = q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if past_key_values is not None:
            k, v = past_key_values.update(k, v, self.layer_idx, {})
        lengths = getattr(past_key_values, "actual_seq_lengths_kv", None)
        total = k.shape[2]
        if lengths is not None:
            visible = torch.arange(total, device=x.device)[None, :] < torch.as_tensor(lengths, device=x.device)[:, None]
            mask = visible[:, None, None, :]
        else:
            mask = (torch.arange(total, device=x.device)[None, :]
                    <= torch.arange(s, device=x.device)[:, None] + (total - s))[None, None]
        out = F.scaled_dot_product_attention(q, k.float(), v.float(), attn_mask=mask, scale=self.scaling,
                                             enable_gqa=True)
        out = out.transpose(1, 2).reshape(b, s, -1)
        return F.linear(out, self.o_proj.weight.float()).to(hidden_states.dtype), None


class Qwen3TTSTalkerAttention(Qwen3TTSAttention):
    """The talker's attention: multimodal position embeddings [3, B, S, D]."""


class Qwen3TTSTalkerTextMLP(torch.nn.Module):
    def __init__(self, hidden, ffn, act="silu", bias=False):
        super().__init__()
        self.config = SimpleNamespace(hidden_act=act)
        self.gate_proj = torch.nn.Linear(hidden, ffn, bias=bias)
        self.up_proj = torch.nn.Linear(hidden, ffn, bias=bias)
        self.down_proj = torch.nn.Linear(ffn, hidden, bias=False)
        self.act_fn = torch.nn.SiLU()

    def forward(self, x):
        xf = x.float()
        h = F.silu(F.linear(xf, self.gate_proj.weight.float())) * F.linear(xf, self.up_proj.weight.float())
        return F.linear(h, self.down_proj.weight.float()).to(x.dtype)


class Qwen3TTSDecoderLayer(torch.nn.Module):
    def __init__(self, hidden, q_heads, kv_heads, head_dim, ffn, layer_idx=0, talker=False):
        super().__init__()
        attention = Qwen3TTSTalkerAttention if talker else Qwen3TTSAttention
        self.input_layernorm = Qwen3TTSRMSNorm(hidden)
        self.self_attn = attention(hidden, q_heads, kv_heads, head_dim, layer_idx)
        self.post_attention_layernorm = Qwen3TTSRMSNorm(hidden)
        self.mlp = Qwen3TTSTalkerTextMLP(hidden, ffn)

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                output_attentions=False, use_cache=False, cache_position=None, position_embeddings=None, **kwargs):
        attended, weights = self.self_attn(hidden_states=self.input_layernorm(hidden_states),
                                           position_embeddings=position_embeddings, attention_mask=attention_mask,
                                           past_key_values=past_key_values, cache_position=cache_position)
        h = hidden_states + attended
        out = h + self.mlp(self.post_attention_layernorm(h))
        return (out, weights) if output_attentions else (out,)


class Qwen3TTSTalkerDecoderLayer(Qwen3TTSDecoderLayer):
    def __init__(self, *args, **kwargs):
        super().__init__(*args, talker=True, **kwargs)


class TinyDecoder(torch.nn.Module):
    """Layers plus their rotary table: forward(hidden, positions, cache) -> hidden."""

    def __init__(self, layers=2, hidden=256, q_heads=16, kv_heads=8, head_dim=128, ffn=512, talker=False,
                 theta=1e6):
        super().__init__()
        layer = Qwen3TTSTalkerDecoderLayer if talker else Qwen3TTSDecoderLayer
        self.layers = torch.nn.ModuleList([layer(hidden, q_heads, kv_heads, head_dim, ffn, layer_idx=i)
                                           for i in range(layers)])
        self.norm = Qwen3TTSRMSNorm(hidden)
        self.head_dim, self.theta, self.talker = head_dim, theta, talker

    def rotary(self, positions, dtype):
        inv = 1.0 / self.theta ** (torch.arange(0, self.head_dim, 2, device=positions.device).float() / self.head_dim)
        angles = positions.float()[..., None] * inv
        emb = torch.cat((angles, angles), dim=-1)
        cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
        if self.talker:
            cos, sin = cos.expand(3, *cos.shape), sin.expand(3, *sin.shape)
        return cos, sin

    def forward(self, hidden, positions, cache=None):
        embeddings = self.rotary(positions, hidden.dtype)
        for layer in self.layers:
            hidden = layer(hidden, position_embeddings=embeddings, past_key_values=cache)[0]
        return self.norm(hidden)


def randomize(module, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            if p.ndim == 1 and "norm" in name:
                p.copy_(1.0 + 0.05 * torch.randn(p.shape, generator=g))
            elif p.ndim == 1:
                p.copy_(0.02 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) / p.shape[1] ** 0.5)
    return module


class ConcatCache:
    """HF dynamic-cache contract: update() appends along the sequence and returns the whole."""

    def __init__(self):
        self.keys, self.values = {}, {}

    def update(self, key, value, layer_idx, kwargs):
        if layer_idx in self.keys:
            self.keys[layer_idx] = torch.cat([self.keys[layer_idx], key], dim=2)
            self.values[layer_idx] = torch.cat([self.values[layer_idx], value], dim=2)
        else:
            self.keys[layer_idx], self.values[layer_idx] = key, value
        return self.keys[layer_idx], self.values[layer_idx]


class SlotCache:
    """Slot-arena contract (continuous.py:135-169): rows advance independently; update() writes each
    row's new key at its own position and returns the whole arena with the per-row lengths."""

    def __init__(self, keys, values, positions):
        self.arena_keys, self.arena_values = keys, values          # per layer [B, Hkv, cap, D]
        self.positions = positions
        self.actual_seq_lengths_kv = (positions + 1).tolist()

    def update(self, key, value, layer_idx, kwargs):
        rows = torch.arange(key.shape[0], device=key.device)
        self.arena_keys[layer_idx][rows, :, self.positions] = key[:, :, 0].to(self.arena_keys[layer_idx].dtype)
        self.arena_values[layer_idx][rows, :, self.positions] = value[:, :, 0].to(self.arena_values[layer_idx].dtype)
        return self.arena_keys[layer_idx], self.arena_values[layer_idx]


# ---------------------------------------------------------------------------------------------
# The qwen-tts functions the reference's PackedAttention imports at module level
# (packed_attention.py:5-8), restated from the Qwen3 decoder they come from (transformers'
# rotate-half RoPE with cos/sin broadcast over heads, repeat-KV GQA attention returning
# [batch, seq, heads, dim]). Registered under `qwen_tts.core.models.modeling_qwen3_tts` so that
# the reference module imports and its own forward runs on the CPU.

def _apply_rotary_pos_emb(q, k, cos, sin, position_ids=None, unsqueeze_dim=1):
    cos, sin = cos.unsqueeze(unsqueeze_dim), sin.unsqueeze(unsqueeze_dim)
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def _apply_multimodal_rotary_pos_emb(*args, **kwargs):
    raise NotImplementedError("the fixtures run the talker with text_only_rope=True")


def _repeat_kv(x, groups):
    if groups == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None].expand(b, h, groups, s, d).reshape(b, h * groups, s, d)


def _eager_attention_forward(module, query, key, value, attention_mask, scaling, dropout=0.0, **kwargs):
    groups = query.shape[1] // key.shape[1]
    key, value = _repeat_kv(key, groups), _repeat_kv(value, groups)
    scores = torch.matmul(query, key.transpose(2, 3)) * scaling
    if attention_mask is not None:
        scores = scores + attention_mask[:, :, :, :key.shape[-2]]
    weights = torch.softmax(scores.float(), dim=-1).to(query.dtype)
    out = torch.matmul(weights, value).transpose(1, 2).contiguous()
    return out, weights


def _sdpa_attention_forward(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    groups = query.shape[1] // key.shape[1]
    key, value = _repeat_kv(key, groups), _repeat_kv(value, groups)
    mask = None if attention_mask is None else attention_mask[:, :, :, :key.shape[-2]]
    out = F.scaled_dot_product_attention(query, key, value, attn_mask=mask, dropout_p=dropout, scale=scaling)
    return out.transpose(1, 2).contiguous(), None


def install_modeling_stub():
    """Register the stand-in `qwen_tts.core.models.modeling_qwen3_tts` module (idempotent)."""
    import sys
    import types
    name = "qwen_tts.core.models.modeling_qwen3_tts"
    if name in sys.modules:
        return sys.modules[name]
    parts = name.split(".")
    for i in range(1, len(parts)):
        sys.modules.setdefault(".".join(parts[:i]), types.ModuleType(".".join(parts[:i])))
    module = types.ModuleType(name)
    module.apply_rotary_pos_emb = _apply_rotary_pos_emb
    module.apply_multimodal_rotary_pos_emb = _apply_multimodal_rotary_pos_emb
    module.eager_attention_forward = _eager_attention_forward
    module.ALL_ATTENTION_FUNCTIONS = {"sdpa": _sdpa_attention_forward, "eager": _eager_attention_forward}
    sys.modules[name] = module
    return module


class TalkerModel(torch.nn.Module):
    """The talker's inner model as the reference's graphs drive it: `layers`, `norm` and
    `rotary_emb(hidden, position_ids [3, B, S]) -> (cos, sin) [3, B, S, D]` (identical axes).
    With talker=False the layers are the code predictor's (single-axis RoPE: position_ids
    [B, S] -> (cos, sin) [B, S, D])."""

    def __init__(self, layers, hidden, q_heads, kv_heads, head_dim, ffn, theta, talker=True):
        super().__init__()
        layer = Qwen3TTSTalkerDecoderLayer if talker else Qwen3TTSDecoderLayer
        self.layers = torch.nn.ModuleList([layer(hidden, q_heads, kv_heads, head_dim, ffn, layer_idx=i)
                                           for i in range(layers)])
        self.norm = Qwen3TTSRMSNorm(hidden)
        self.head_dim, self.theta = head_dim, theta
        self.config = SimpleNamespace(hidden_size=hidden, num_key_value_heads=kv_heads, head_dim=head_dim)

    def rotary_emb(self, hidden, position_ids):
        inv = 1.0 / self.theta ** (torch.arange(0, self.head_dim, 2, dtype=torch.int64).float() / self.head_dim)
        angles = position_ids.float()[..., None] * inv
        emb = torch.cat((angles, angles), dim=-1)
        return emb.cos().to(hidden.dtype), emb.sin().to(hidden.dtype)


class Talker(torch.nn.Module):
    """`model` plus the codec head, with the attributes PrefillGraph reads (prefill_graph.py:18-50)."""

    def __init__(self, model, vocab):
        super().__init__()
        self.model = model
        self.codec_head = torch.nn.Linear(model.config.hidden_size, vocab, bias=False)
        self.config = model.config


def load_oracle_weights(talker, weights):
    """Copy oracle-format weights (oracle/decoder.py) into a Talker's modules."""
    with torch.no_grad():
        for layer, w in zip(talker.model.layers, weights["layers"]):
            attn = layer.self_attn
            layer.input_layernorm.weight.copy_(w["input_norm"])
            layer.post_attention_layernorm.weight.copy_(w["post_norm"])
            attn.q_proj.weight.copy_(w["q"])
            attn.k_proj.weight.copy_(w["k"])
            attn.v_proj.weight.copy_(w["v"])
            attn.o_proj.weight.copy_(w["o"])
            attn.q_norm.weight.copy_(w["q_norm"])
            attn.k_norm.weight.copy_(w["k_norm"])
            layer.mlp.gate_proj.weight.copy_(w["gate"])
            layer.mlp.up_proj.weight.copy_(w["up"])
            layer.mlp.down_proj.weight.copy_(w["down"])
        talker.model.norm.weight.copy_(weights["norm"])
        talker.codec_head.weight.copy_(weights["head"])
