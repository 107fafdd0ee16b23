"""A small Qwen3-style talker decoder with seeded weights, shared by the fixture
generator (which runs the reference's own PackedAttention / PackedMLP /
SlotGraph / PrefillGraph over it) and the CPU test that pins the oracle's
decoder (``oracle/decoder.py``) to those outputs.

Weights come from Philox streams (``inputs.normal``), so the fixture stores
only outputs. Geometry: the talker's head layout (16 query / 8 KV heads of
128) at a reduced width.
"""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

from tests.golden.inputs import normal

LAYERS, HIDDEN, FFN, VOCAB = 2, 256, 512, 96
Q_HEADS, KV_HEADS, HEAD_DIM = 16, 8, 128
EPS, THETA = 1e-6, 1_000_000.0

# decode step: 4 slots with ragged positions and rope deltas, two steps
SLOTS, CAPACITY = 4, 72
POSITIONS = [0, 5, 17, 63]
ROPE_DELTAS = [0, -3, 2, 5]
# padded prefill: 3 prompts of lengths 5, 8, 2 padded to 8 (a 4th all-padding row)
PREFILL_LENGTHS = [5, 8, 2]
PREFILL_BATCH, PREFILL_LEN = 4, 8


# code-predictor layer stack: step 0 runs two tokens at positions [0, 1] with a causal mask,
# steps 1.. one token each at position step + 1 (continuous.py:37-61)
PREDICTOR_BATCH, PREDICTOR_STEPS = 3, 4


def predictor_inputs(step: int) -> torch.Tensor:
    """Layer-stack inputs [PREDICTOR_BATCH, 2 if step == 0 else 1, HIDDEN] of predictor step `step`."""
    return torch.from_numpy(normal(950 + step, (PREDICTOR_BATCH, 2 if step == 0 else 1, HIDDEN)))


def config():
    from qwen3_tts_b200.config import TALKER
    return replace(TALKER, layers=LAYERS, hidden=HIDDEN, ffn=FFN, vocab=VOCAB, eps=EPS, theta=THETA)


def weights() -> dict:
    """Oracle-format fp32 weights (oracle/decoder.py): per-layer q/k/v/o, gate/up/down and norms,
    final norm and LM head."""
    seed = [500]

    def draw(shape, scale):
        seed[0] += 1
        return torch.from_numpy(normal(seed[0], shape, scale))

    def proj(out_f, in_f):
        return draw((out_f, in_f), in_f ** -0.5)

    def norm(n):
        return 1.0 + draw((n,), 0.1)

    layers = []
    for _ in range(LAYERS):
        layers.append({
            "input_norm": norm(HIDDEN),
            "q": proj(Q_HEADS * HEAD_DIM, HIDDEN), "k": proj(KV_HEADS * HEAD_DIM, HIDDEN),
            "v": proj(KV_HEADS * HEAD_DIM, HIDDEN),
            "q_norm": norm(HEAD_DIM), "k_norm": norm(HEAD_DIM),
            "o": proj(HIDDEN, Q_HEADS * HEAD_DIM),
            "post_norm": norm(HIDDEN),
            "gate": proj(FFN, HIDDEN), "up": proj(FFN, HIDDEN), "down": proj(HIDDEN, FFN),
        })
    return {"layers": layers, "norm": norm(HIDDEN), "head": proj(VOCAB, HIDDEN)}


def history(layer: int) -> tuple[torch.Tensor, torch.Tensor]:
    """KV arena contents [SLOTS, KV_HEADS, CAPACITY, HEAD_DIM] of `layer` before the first step:
    Philox normals below each slot's position, zeros from it on."""
    shape = (SLOTS, KV_HEADS, CAPACITY, HEAD_DIM)
    k = torch.from_numpy(normal(700 + 2 * layer, shape))
    v = torch.from_numpy(normal(701 + 2 * layer, shape))
    for b, p in enumerate(POSITIONS):
        k[b, :, p:] = 0
        v[b, :, p:] = 0
    return k, v


def step_inputs(step: int) -> torch.Tensor:
    """Decode inputs [SLOTS, HIDDEN] of step `step` (0 or 1)."""
    return torch.from_numpy(normal(800 + step, (SLOTS, HIDDEN)))


def prefill_inputs() -> torch.Tensor:
    """Right-padded prompt embeddings [PREFILL_BATCH, PREFILL_LEN, HIDDEN] (padding rows zero)."""
    x = torch.from_numpy(normal(900, (PREFILL_BATCH, PREFILL_LEN, HIDDEN)))
    for b in range(PREFILL_BATCH):
        n = PREFILL_LENGTHS[b] if b < len(PREFILL_LENGTHS) else 0
        x[b, n:] = 0
    return x


def prefill_mask() -> torch.Tensor:
    """[PREFILL_BATCH, PREFILL_LEN] long: 1 on real tokens; an all-padding row is all ones, as the
    reference's pad_prefill_batch appends dummy rows (prefill_graph.py:6-15)."""
    mask = torch.ones(PREFILL_BATCH, PREFILL_LEN, dtype=torch.long)
    for b, n in enumerate(PREFILL_LENGTHS):
        mask[b, n:] = 0
    return mask


def as_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().contiguous().numpy()
