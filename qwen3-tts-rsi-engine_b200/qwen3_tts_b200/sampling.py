"""Seeded inverse-CDF sampling (sampling.py of the reference engine) on the GPU.

``categorical`` keeps the reference signature and adds ``top_p`` (default 1.0,
the reference's only setting). The draw is one fused kernel
(``q3t_sample``): temperature, top-k threshold (ties kept), softmax, optional
top-p, running CDF in vocabulary order, normalisation by its last entry and
the count of entries <= u. ``random_table`` is the reference's per-request CPU
uniform table and stays on the host generator so tables match bit for bit.
"""
from __future__ import annotations

import torch

from . import ops


def categorical(scores, uniform, *, temperature=0.9, top_k=50, top_p=1.0, triton_cdf=False):
    """scores [rows, vocab] (fp32 or bf16, CUDA), uniform [rows] fp32 -> tokens [rows, 1] int64."""
    del triton_cdf  # the CDF selection is always fused into the kernel
    if not isinstance(uniform, torch.Tensor) or uniform.ndim != 1:
        raise ValueError("Expected one uniform per row")
    return ops.sample(scores, uniforms=uniform.contiguous(), temperature=temperature, top_k=top_k, top_p=top_p)


def random_table(seed: int, steps: int) -> torch.Tensor:
    """[steps + 1, 16] uniforms from a CPU mt19937 generator seeded with `seed` (sampling.py:17-19)."""
    generator = torch.Generator(device="cpu").manual_seed(seed)
    return torch.rand(steps + 1, 16, generator=generator)
