"""Deterministic test inputs shared by the fixture generator and the tests.

Inputs are derived from Philox4x32-10 streams (oracle/sampling.py, pinned by
the Random123 known-answer vectors), so fixtures store only outputs.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle.sampling import philox_stream


def uniform(seed: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    return philox_stream(seed, 0, n).reshape(shape)


def normal(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    """Box-Muller normals (float32) from a Philox stream."""
    n = int(np.prod(shape))
    u = philox_stream(seed, 0, 2 * n).astype(np.float64)
    u1 = np.maximum(u[0::2], 1e-12)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u[1::2])
    return (z * scale).astype(np.float32).reshape(shape)


def bf16_scores(seed: int, rows: int, width: int, scale: float) -> torch.Tensor:
    """bf16-representable fp32 scores (the LM head emits bf16 logits)."""
    return torch.from_numpy(normal(seed, (rows, width), scale)).to(torch.bfloat16).float()
