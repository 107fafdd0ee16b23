"""Sampling restated on the CPU (torch fp32 ops, as the reference calls them).

TEST INFRASTRUCTURE ONLY (see the package docstring).
"""
from __future__ import annotations

import numpy as np
import torch


def random_table(seed: int, steps: int) -> torch.Tensor:
    """Per-request uniform table [steps + 1, 16] from a CPU mt19937 stream (sampling.py:17-19)."""
    generator = torch.Generator(device="cpu").manual_seed(seed)
    return torch.rand(steps + 1, 16, generator=generator)


def top_p_filter(probabilities: torch.Tensor, top_p: float) -> torch.Tensor:
    """Zero the smallest-probability tail whose cumulative mass is <= 1 - top_p.

    Not part of the reference (it rejects top_p != 1.0, continuous.py:388-393);
    this is the HF TopP rule (ascending sort, keep at least the largest token)
    used for the code-predictor benchmark configuration. Ties sort by index.
    """
    out = probabilities.clone()
    for r in range(out.shape[0]):
        row = out[r]
        idx = torch.nonzero(row > 0).flatten()
        vals = row[idx]
        order = sorted(range(len(idx)), key=lambda i: (float(vals[i]), int(idx[i])))
        cum = np.float32(0)
        cut = np.float32(1) - np.float32(top_p)
        for rank, i in enumerate(order):
            cum = np.float32(cum + np.float32(vals[i]))
            if cum <= cut and rank < len(order) - 1:
                row[idx[i]] = 0
    return out


def categorical(scores, uniform, *, temperature=0.9, top_k=50, top_p=1.0) -> torch.Tensor:
    """Inverse-CDF draw over the top-k tempered softmax (sampling.py:5-14).

    scores [rows, vocab] -> tokens [rows, 1]; `uniform` [rows] in [0, 1).
    The CDF is the running sum in vocabulary order, normalised by its last
    entry, and the token is the count of entries <= u (sampling.py:9-14).
    """
    scores = scores.float() / temperature
    threshold = torch.topk(scores, top_k, dim=-1).values[..., -1:]
    probabilities = torch.softmax(scores.masked_fill(scores < threshold, -float("inf")), dim=-1)
    if top_p < 1.0:
        kept = top_p_filter(probabilities, top_p)
        e = torch.exp(scores - scores.max(-1, keepdim=True).values)
        e = torch.where(kept > 0, e, torch.zeros_like(e))
        probabilities = e * (1.0 / e.sum(-1, keepdim=True))
    cdf = probabilities.cumsum(-1)
    cdf = cdf / cdf[..., -1:]
    return (cdf <= uniform.unsqueeze(-1)).sum(-1, keepdim=True)


def cdf_select(cdf: torch.Tensor, uniforms: torch.Tensor) -> torch.Tensor:
    """token = #{ j : cdf[j] / cdf[-1] <= u } with fp32 division (cdf_triton_ascend.py:13-17)."""
    normalized = cdf / cdf[:, -1:]
    return (normalized <= uniforms[:, None]).sum(-1, keepdim=True)


def allowed_mask(vocab: int, eos: int) -> torch.Tensor:
    """Codec vocabulary mask: the last 1024 ids are control tokens except EOS (continuous.py:330-332)."""
    allowed = torch.ones(vocab, dtype=torch.bool)
    allowed[-1024:] = False
    allowed[eos] = True
    return allowed


def semantic(logits, uniforms, seen, steps, allowed, eos, *, penalty=1.05, min_steps=2, temperature=0.9,
             top_k=50, top_p=1.0) -> torch.Tensor:
    """Semantic-token sampling (continuous.py:365-370): repetition penalty on
    seen tokens, vocabulary mask, EOS blocked before `min_steps`, then categorical."""
    logits = logits.float()
    logits = torch.where(seen, torch.where(logits < 0, logits * penalty, logits / penalty), logits)
    logits = logits.masked_fill(~allowed, -float("inf"))
    logits[:, eos] = torch.where(steps < min_steps, -float("inf"), logits[:, eos])
    return categorical(logits, uniforms, temperature=temperature, top_k=top_k, top_p=top_p)


def sampling_graph_step(logits, uniforms, seen, steps, allowed, eos, **kw):
    """(tokens, seen | onehot(tokens)) as SamplingGraph.compute returns (sampling_graph.py:14-16)."""
    tokens = semantic(logits, uniforms, seen, steps, allowed, eos, **kw)
    return tokens, seen.scatter(1, tokens, True)


# ------------------------------------------------------------------ Philox4x32-10
_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(counter, key):
    """Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, SC'11), vectorised over rows.

    counter: uint32 [n, 4]; key: uint32 [n, 2] -> uint32 [n, 4].
    """
    c = np.asarray(counter, dtype=np.uint32).copy()
    k = np.asarray(key, dtype=np.uint32).copy()
    with np.errstate(over="ignore"):
        for _ in range(10):
            p0 = _M0 * c[:, 0].astype(np.uint64)
            p1 = _M1 * c[:, 2].astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & _MASK).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & _MASK).astype(np.uint32)
            c = np.stack([hi1 ^ c[:, 1] ^ k[:, 0], lo1, hi0 ^ c[:, 3] ^ k[:, 1], lo0], axis=1)
            k[:, 0] = k[:, 0] + _W0
            k[:, 1] = k[:, 1] + _W1
    return c


def philox_uniform(seed: int, offsets) -> np.ndarray:
    """u = (x0 >> 8) * 2^-24 of Philox(key=seed, counter={offset lo, offset hi, 0, 0})."""
    offsets = np.asarray(offsets, dtype=np.uint64)
    n = offsets.shape[0]
    counter = np.zeros((n, 4), dtype=np.uint32)
    counter[:, 0] = (offsets & _MASK).astype(np.uint32)
    counter[:, 1] = (offsets >> np.uint64(32)).astype(np.uint32)
    key = np.zeros((n, 2), dtype=np.uint32)
    key[:, 0] = np.uint32(seed & 0xFFFFFFFF)
    key[:, 1] = np.uint32((seed >> 32) & 0xFFFFFFFF)
    out = philox4x32_10(counter, key)
    return (out[:, 0] >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)


def philox_stream(seed: int, offset: int, count: int) -> np.ndarray:
    """Uniforms of q3t_philox_uniforms: element i = word i%4 of counter offset + i//4."""
    groups = (count + 3) // 4
    ctr = np.arange(groups, dtype=np.uint64) + np.uint64(offset)
    counter = np.zeros((groups, 4), dtype=np.uint32)
    counter[:, 0] = (ctr & _MASK).astype(np.uint32)
    counter[:, 1] = (ctr >> np.uint64(32)).astype(np.uint32)
    key = np.tile(np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], dtype=np.uint32), (groups, 1))
    words = philox4x32_10(counter, key).reshape(-1)[:count]
    return (words >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
