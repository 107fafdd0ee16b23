"""Elementwise and normalisation ops restated on the CPU, including the
reference's explicit bf16-rounding variants.

TEST INFRASTRUCTURE ONLY (see the package docstring).
"""
from __future__ import annotations

import torch

BF16 = torch.bfloat16


def bf(x: torch.Tensor) -> torch.Tensor:
    """Round fp32 values to bf16 and back (one rounding step)."""
    return x.to(BF16).float()


def rms_norm(x, weight, eps, mode="reference"):
    """RMSNorm (operators.py:16-23 and the HF Qwen3 RMSNorm it wraps).

    reference: bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))   (operators.py:21-23)
    native:    bf16(w * x * rsqrt(...)) with one rounding   (operators.py:19-20)
    fp32:      no rounding at all (the oracle's own precision)
    """
    xf = x.float()
    r = 1.0 / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if mode == "fp32":
        return weight.float() * (xf * r)
    if mode == "native":
        return bf(weight.float() * (xf * r))
    return bf(weight.float() * bf(xf * r))


def add_rms_norm(a, h, weight, eps, mode="reference"):
    """(normalized, residual): residual = a + h (fused_decoder.py:34-35).

    native normalises the unrounded fp32 sum; reference rounds the sum first.
    """
    raw = a.float() + h.float()
    residual = bf(raw)
    source = raw if mode == "native" else residual
    return rms_norm(source, weight, eps, "native" if mode == "native" else "reference"), residual


def rotary_bf16(x, cos, sin):
    """BSND rotary with bf16 rounding after every product and sum (rotary_triton_ascend.py:19-24)."""
    half = x.shape[-1] // 2
    xf = x.float()
    c = cos.float()[:, :, None, :]
    s = sin.float()[:, :, None, :]
    x1, x2 = xf[..., :half], xf[..., half:]
    out1 = bf(bf(x1 * c[..., :half]) + bf(-x2 * s[..., :half]))
    out2 = bf(bf(x2 * c[..., half:]) + bf(x1 * s[..., half:]))
    return torch.cat([out1, out2], dim=-1).to(BF16)


def rope_tables(positions: int, dim: int, theta: float, dtype=torch.float32):
    """cos/sin [positions, dim] of default RoPE: freqs = p * theta^(-2i/dim), duplicated halves."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    freqs = torch.arange(positions, dtype=torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x, cos, sin):
    """x * cos + rotate_half(x) * sin (the qwen-tts apply_rotary_pos_emb form), fp32."""
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


def swiglu(packed):
    """act_fn(gate) * up over packed [.., 2w] with bf16 rounding per op (packed_mlp.py:25-26)."""
    gate, up = packed.float().chunk(2, dim=-1)
    return bf(bf(torch.nn.functional.silu(gate)) * up).to(BF16)


def snake(x, alpha, inverse_beta):
    """SnakeBeta with cached constants (incremental_codec.py:49; snake_triton_ascend.py:20-24).

    bf16 input: bf16 rounding after each of x*alpha, sin, square, scale, add.
    fp32 input: x + inverse_beta * sin(x * alpha)^2.
    """
    a = alpha.float().reshape(1, -1, 1)
    r = inverse_beta.float().reshape(1, -1, 1)
    xf = x.float()
    if x.dtype == BF16:
        phase = bf(xf * a)
        sine = bf(torch.sin(phase))
        square = bf(sine * sine)
        scaled = bf(r * square)
        return (xf + scaled).to(BF16)
    return xf + r * torch.pow(torch.sin(xf * a), 2)


def scatter_rows(target, indices, source) -> None:
    """target[indices[i]] = source[i] (codec_row_scatter.py:41-45)."""
    for i, row in enumerate(indices.tolist()):
        target[row] = source[i]


def frame_embed(codes, first_table, group_tables, text=None):
    """E_first[c0] + sum_g E_g[c_{g+1}] summed in fp32, rounded once, then + text in bf16
    (continuous.py:584-601: cat(...).sum(1) then `embeds + text`)."""
    acc = first_table[codes[:, 0]].float()
    for g in range(group_tables.shape[0]):
        acc = acc + group_tables[g][codes[:, g + 1]].float()
    if text is None:
        return acc.to(BF16)
    return (bf(acc) + text.float()).to(BF16)
