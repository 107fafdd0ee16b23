"""Qwen3-style decoder (talker and code predictor) restated on the CPU.

TEST INFRASTRUCTURE ONLY (see the package docstring).

The layer is the one the reference drives through HF modules and replaces
piecewise: RMSNorm (operators.py:16-23), packed QKV projection, per-head
q_norm/k_norm, rotate-half RoPE, cache update and GQA attention
(packed_attention.py:42-85), residual add, post-attention RMSNorm, SwiGLU MLP
(packed_mlp.py:19-27), final norm and LM head (continuous.py:188-198, 613).
Layer internals belong to qwen-tts==0.1.1 (absent here), so they are restated
from those call sites. Pinned: the fp32 mode reproduces, to fp32 accuracy
(tests/test_oracle_decoder_pinned.py), the reference's own PackedAttention and
PackedMLP forwards run inside its SlotGraph decode step, its PrefillGraph and
the predictor's position/mask pattern (tests/golden/make_golden.py), with the
four qwen-tts functions PackedAttention imports (rotate-half RoPE, repeat-KV
attention) restated in tests/qwen_tts_fakes.py.

Three precisions:
  mode="fp32"  every op in fp32 from the bf16 weights (the parity truth);
  mode="bf16"  fp32 math with bf16 rounding at each point the reference's
               bf16 tensors round (linear outputs, norms, RoPE ops, residuals);
  mode="bf16f" as "bf16", with the input and post-attention RMSNorms folded
               into the following projections the way the GPU path computes
               them (norm weight premultiplied into the bf16 weight, row scale
               on the fp32 product).
"""
from __future__ import annotations

import torch

from .elementwise import bf, rope_tables
from .sampling import categorical


def _rounds(mode):
    return mode in ("bf16", "bf16f")


def _r(x, mode):
    return bf(x) if _rounds(mode) else x


def _rms(x, w, eps, mode):
    r = 1.0 / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    if _rounds(mode):
        return bf(w.float() * bf(x * r))
    return w.float() * (x * r)


def _normed_proj(h, norm_w, weight, eps, mode):
    """RMSNorm of h followed by a projection. In mode "bf16f" the norm weight is
    folded into the projection (bf16(W * w)) and the row scale rsqrt(mean(h^2)+eps)
    multiplies the fp32 product before the bf16 rounding: the GPU's fused
    q3t_linear_rownorm path. The other modes normalise first (operators.py:16-23)."""
    if mode == "bf16f":
        r = 1.0 / torch.sqrt(h.pow(2).mean(-1, keepdim=True) + eps)
        folded = bf(weight.float() * norm_w.float()[None, :])
        return bf((h @ folded.T) * r)
    x = _rms(h, norm_w, eps, mode)
    return _r(x @ weight.float().T, mode)


def _rope(x, cos, sin, mode):
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    if _rounds(mode):
        return bf(bf(x * cos) + bf(rot * sin))
    return x * cos + rot * sin


class Tables:
    """RoPE cos/sin tables (bf16-rounded as the model's bf16 rotary embedding returns them)."""

    def __init__(self, positions: int, dim: int, theta: float):
        cos, sin = rope_tables(positions, dim, theta)
        self.cos = bf(cos)
        self.sin = bf(sin)


def layer_forward(cfg, w, h, rot_pos, cache_k, cache_v, cache_pos, tables, mode):
    """One decoder layer. h [B, L, H] fp32; rot_pos/cache_pos [B, L] int64;
    cache_k/cache_v [B, Hkv, cap, D] fp32 (written in place). Query (b, t)
    attends to cache positions 0..cache_pos[b, t]."""
    B, L, H = h.shape
    D, Hq, Hkv = cfg.head_dim, cfg.q_heads, cfg.kv_heads
    q = _normed_proj(h, w["input_norm"], w["q"], cfg.eps, mode).view(B, L, Hq, D)
    k = _normed_proj(h, w["input_norm"], w["k"], cfg.eps, mode).view(B, L, Hkv, D)
    v = _normed_proj(h, w["input_norm"], w["v"], cfg.eps, mode).view(B, L, Hkv, D)
    q = _rms(q, w["q_norm"], cfg.eps, mode)
    k = _rms(k, w["k_norm"], cfg.eps, mode)
    cos = tables.cos[rot_pos][:, :, None, :]
    sin = tables.sin[rot_pos][:, :, None, :]
    q = _rope(q, cos, sin, mode)
    k = _rope(k, cos, sin, mode)
    for b in range(B):
        for t in range(L):
            p = int(cache_pos[b, t])
            cache_k[b, :, p] = k[b, t]
            cache_v[b, :, p] = v[b, t]
    group = Hq // Hkv
    attn = torch.empty(B, L, Hq, D)
    for b in range(B):
        for t in range(L):
            n = int(cache_pos[b, t]) + 1
            kk = cache_k[b, :, :n].repeat_interleave(group, 0)
            vv = cache_v[b, :, :n].repeat_interleave(group, 0)
            s = torch.einsum("hd,hnd->hn", q[b, t], kk) * (D ** -0.5)
            attn[b, t] = torch.einsum("hn,hnd->hd", torch.softmax(s, -1), vv)
    attn = _r(attn, mode).reshape(B, L, Hq * D)
    h = _r(h + _r(attn @ w["o"].float().T, mode), mode)
    gate = _normed_proj(h, w["post_norm"], w["gate"], cfg.eps, mode)
    up = _normed_proj(h, w["post_norm"], w["up"], cfg.eps, mode)
    act = _r(_r(torch.nn.functional.silu(gate), mode) * up, mode)
    h = _r(h + _r(act @ w["down"].float().T, mode), mode)
    return h


def decoder_layers(cfg, weights, h, rot_pos, cache, cache_pos, tables, mode="fp32"):
    """All layers, without the final norm. cache: list of (K, V) per layer."""
    h = h.float()
    for w, (ck, cv) in zip(weights["layers"], cache):
        h = layer_forward(cfg, w, h, rot_pos, ck, cv, cache_pos, tables, mode)
    return h


def decoder_forward(cfg, weights, h, rot_pos, cache, cache_pos, tables, mode="fp32"):
    """All layers then the final norm. cache: list of (K, V) per layer."""
    return _rms(decoder_layers(cfg, weights, h, rot_pos, cache, cache_pos, tables, mode), weights["norm"], cfg.eps,
                mode)


def new_cache(cfg, batch, capacity):
    return [(torch.zeros(batch, cfg.kv_heads, capacity, cfg.head_dim),
             torch.zeros(batch, cfg.kv_heads, capacity, cfg.head_dim)) for _ in range(cfg.layers)]


def talker_decode_step(cfg, weights, embeds, positions, rope_deltas, cache, tables, mode="fp32"):
    """SlotGraph.compute + codec_head (continuous.py:188-198, 612-613).

    embeds [B, H]; positions [B] (KV write position); rotary = position + rope_delta.
    Returns (hidden [B, H], logits [B, vocab])."""
    pos = positions.view(-1, 1).long()
    rot = (positions + rope_deltas).view(-1, 1).long()
    hidden = decoder_forward(cfg, weights, embeds.view(embeds.shape[0], 1, -1), rot, cache, pos, tables, mode)
    logits = _r(hidden @ weights["head"].float().T, mode)
    return hidden[:, 0], logits[:, 0]


def predictor_frame(cfg, weights, hidden, first, draws, tables, mode="fp32", *, temperature=0.9, top_k=50,
                    top_p=1.0, uniforms_fn=None, forced_codes=None):
    """The 15-codebook loop of UniformPredictor.run (continuous.py:49-68).

    hidden/first [B, talker_hidden]; draws [B, 16] (column step+1 feeds step).
    Step 0 runs (hidden, first) at positions [0, 1]; step i runs the embedding
    of the previous code (codebook i-1 table) at position i+1; head i samples
    code i+1. Returns (subcodes [B, 15], summed embeddings [B, talker_hidden]).
    """
    B = hidden.shape[0]
    cache = new_cache(cfg, B, cfg.groups + 1)
    inputs = torch.stack([hidden, first], dim=1).float()
    codes = []
    all_logits = []
    token = None
    for step in range(cfg.groups):
        if step == 0:
            x = inputs
            pos = torch.tensor([[0, 1]]).expand(B, 2)
        else:
            x = weights["embeddings"][step - 1][token[:, 0]].float()[:, None, :]
            pos = torch.full((B, 1), step + 1)
        x = _r(x @ weights["proj"].float().T + weights["proj_bias"].float(), mode)
        if mode == "bf16f":
            # the predictor's final norm feeds only the heads: folded into them on the GPU
            out = decoder_layers(cfg, weights, x, pos, cache, pos, tables, mode)
            logits = _normed_proj(out[:, -1], weights["norm"], weights["heads"][step], cfg.eps, mode)
        else:
            out = decoder_forward(cfg, weights, x, pos, cache, pos, tables, mode)
            logits = _r(out[:, -1] @ weights["heads"][step].float().T, mode)
        u = draws[:, step + 1] if uniforms_fn is None else uniforms_fn(step)
        token = categorical(logits, u, temperature=temperature, top_k=top_k, top_p=top_p)
        codes.append(token)
        all_logits.append(logits)
        if forced_codes is not None:
            token = forced_codes[:, step:step + 1]
    subcodes = torch.cat(codes, dim=-1)
    # The frame embedding sums the codes the frame actually carries: the forced ones
    # under teacher forcing, else this chain's own draws (continuous.py:590-597).
    carried = forced_codes if forced_codes is not None else subcodes
    acc = first.float()
    for i in range(cfg.groups):
        acc = acc + weights["embeddings"][i][carried[:, i]].float()
    return subcodes, acc, torch.stack(all_logits)
