"""Seeded random-init weights and their device layouts.

``decoder_weights`` draws the logical tensors (N(0, 0.02) projections and
embeddings, 1 + N(0, 0.02) norm scales) from one torch generator, in a fixed
order, so the same seed gives the same model on any device.
``pack_decoder`` lays them out for the kernels:

* ``qkv``: q|k|v rows concatenated ([q_width + 2*kv_width, hidden]), as
  PackedAttention concatenates them (packed_attention.py:17).
* ``gate_up``: gate and up rows interleaved per 128-row tile
  ([64 gate; 64 up] per tile), so one GEMM tile owns both halves of 64 FFN
  features and the SwiGLU runs in the GEMM epilogue.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .config import DecoderConfig, PredictorConfig, TalkerConfig

STD = 0.02


def _gen(seed: int, device) -> torch.Generator:
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return g


def _normal(g, shape, device, dtype, std=STD):
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)


def _norm(g, n, device, dtype):
    return (1.0 + torch.randn(n, generator=g, device=device, dtype=torch.float32) * STD).to(dtype)


def decoder_weights(cfg: DecoderConfig, seed: int, device="cpu", dtype=torch.bfloat16) -> dict:
    """Logical (unpacked) decoder weights: one dict per layer plus shared tensors."""
    g = _gen(seed, device)
    layers = []
    for _ in range(cfg.layers):
        layers.append({
            "input_norm": _norm(g, cfg.hidden, device, dtype),
            "q": _normal(g, (cfg.q_width, cfg.hidden), device, dtype),
            "k": _normal(g, (cfg.kv_width, cfg.hidden), device, dtype),
            "v": _normal(g, (cfg.kv_width, cfg.hidden), device, dtype),
            "q_norm": _norm(g, cfg.head_dim, device, dtype),
            "k_norm": _norm(g, cfg.head_dim, device, dtype),
            "o": _normal(g, (cfg.hidden, cfg.q_width), device, dtype),
            "post_norm": _norm(g, cfg.hidden, device, dtype),
            "gate": _normal(g, (cfg.ffn, cfg.hidden), device, dtype),
            "up": _normal(g, (cfg.ffn, cfg.hidden), device, dtype),
            "down": _normal(g, (cfg.hidden, cfg.ffn), device, dtype),
        })
    out = {"layers": layers, "norm": _norm(g, cfg.hidden, device, dtype)}
    if isinstance(cfg, PredictorConfig):
        out["heads"] = _normal(g, (cfg.groups, cfg.vocab, cfg.hidden), device, dtype)
        out["embeddings"] = _normal(g, (cfg.groups, cfg.vocab, cfg.talker_hidden), device, dtype)
        out["proj"] = _normal(g, (cfg.hidden, cfg.talker_hidden), device, dtype)
        out["proj_bias"] = _normal(g, (cfg.hidden,), device, dtype)
    else:
        out["head"] = _normal(g, (cfg.vocab, cfg.hidden), device, dtype)
        out["embedding"] = _normal(g, (cfg.vocab, cfg.hidden), device, dtype)
    return out


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = 64) -> torch.Tensor:
    """[F, H] x 2 -> [2F, H] with rows [gate[64t:64t+64]; up[64t:64t+64]] per tile t."""
    ffn, hidden = gate.shape
    if ffn % group:
        raise ValueError("FFN width must be a multiple of 64 for the paired SwiGLU epilogue")
    g = gate.reshape(ffn // group, group, hidden)
    u = up.reshape(ffn // group, group, hidden)
    return torch.stack([g, u], dim=1).reshape(2 * ffn, hidden).contiguous()


@dataclass
class PackedLayer:
    input_norm: torch.Tensor
    qkv: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o: torch.Tensor
    post_norm: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    folded: bool = False   # input/post norm weights are premultiplied into qkv/gate_up


def fold_norm(weight: torch.Tensor, norm_weight: torch.Tensor) -> torch.Tensor:
    """W[n, k] * w[k] in fp32, rounded to bf16: the RMSNorm weight moved into the next projection."""
    return (weight.float() * norm_weight.float()[None, :].to(weight.device)).to(torch.bfloat16)


def pack_decoder(weights: dict, device, tiled: bool = True, fold_norms: bool = True) -> dict:
    """Kernel layouts on `device` (bf16, contiguous).

    With ``tiled`` the projection matrices are re-laid out as contiguous
    pre-swizzled 16 KB GEMM tiles (``ops.pack_tiles``), so every pipeline stage
    of the weight-streaming GEMM reads one contiguous block of HBM. With
    ``fold_norms`` the input and post-attention RMSNorm weights are folded
    into the QKV and gate/up projections; the step then runs those GEMMs on the
    raw residual stream with the row RMS applied in the GEMM
    (``q3t_linear_rownorm``) and launches no separate norm kernels."""
    from . import ops

    def dev(t):
        return t.to(device=device, dtype=torch.bfloat16).contiguous()

    def mat(t):
        t = dev(t)
        return ops.pack_tiles(t) if tiled else t

    def maybe_fold(w, norm):
        return fold_norm(dev(w), dev(norm)) if fold_norms else w

    layers = [PackedLayer(
        input_norm=dev(l["input_norm"]),
        qkv=mat(maybe_fold(torch.cat([l["q"], l["k"], l["v"]], dim=0), l["input_norm"])),
        q_norm=dev(l["q_norm"]),
        k_norm=dev(l["k_norm"]),
        o=mat(l["o"]),
        post_norm=dev(l["post_norm"]),
        gate_up=mat(maybe_fold(interleave_gate_up(l["gate"], l["up"]), l["post_norm"])),
        down=mat(l["down"]),
        folded=fold_norms,
    ) for l in weights["layers"]]
    packed = {"layers": layers, "norm": dev(weights["norm"])}
    for key in ("embedding", "embeddings", "proj_bias"):
        if key in weights:
            packed[key] = dev(weights[key])
    if "head" in weights:
        packed["head"] = mat(weights["head"])
    if "proj" in weights:
        packed["proj"] = mat(weights["proj"])
    if "heads" in weights:
        # the predictor's final norm feeds only the codebook heads: fold it into them too
        packed["heads"] = [mat(maybe_fold(h, weights["norm"])) for h in weights["heads"]]
        packed["heads_folded"] = fold_norms
    if "proj" in weights and "embeddings" in weights:
        # Step i >= 1 of the predictor projects one row of codebook table i-1: project
        # every row once here, so that the step gathers the projected row instead.
        packed["proj_tables"] = torch.stack([
            ops.linear(packed["embeddings"][g], packed["proj"], packed["proj_bias"])
            for g in range(packed["embeddings"].shape[0])]).contiguous()
    return packed
