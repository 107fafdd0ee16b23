"""The oracle's decoder layer against the reference's own decoder code.

`tests/golden/decoder.npz` holds the outputs of the reference's SlotGraph decode
step (continuous.py:172-198, with the codec head of continuous.py:613) and its
padded PrefillGraph (prefill_graph.py:31-50), run with the reference's
PackedAttention (packed_attention.py:37-85, text-only RoPE) and PackedMLP
(packed_mlp.py:19-27) installed over fp32 stand-in layers
(`tests/golden/make_golden.py`). The oracle (`oracle/decoder.py`, fp32 mode)
must reproduce them to fp32 accuracy on the same seeded weights and inputs:
the QKV split, the q/k norm before RoPE, the KV scatter at each slot's
position, the rope-delta offset, the causal and padding masks, the residual
structure, SwiGLU, the final norm and the head.
"""
from pathlib import Path

import numpy as np
import torch

from oracle import decoder as OD
from oracle.elementwise import rope_tables
from tests.golden import decoder_case as case

FIXTURE = np.load(Path(__file__).resolve().parent / "golden" / "decoder.npz")
# fp32 results of two implementations that order their sums differently
ATOL, RTOL = 2e-4, 2e-4


def _tables(positions):
    tables = OD.Tables(positions, case.HEAD_DIM, case.THETA)
    # the stand-in rotary runs in fp32 (the pinned step is fp32 end to end)
    tables.cos, tables.sin = rope_tables(positions, case.HEAD_DIM, case.THETA)
    return tables


def _close(got, want):
    np.testing.assert_allclose(got.numpy(), want, atol=ATOL * max(1.0, float(np.abs(want).max())), rtol=RTOL)


def test_decode_step_matches_reference_slot_graph():
    cfg, weights = case.config(), case.weights()
    cache = [case.history(layer) for layer in range(case.LAYERS)]
    positions = torch.tensor(case.POSITIONS)
    deltas = torch.tensor(case.ROPE_DELTAS)
    tables = _tables(case.CAPACITY + 8)
    for step in range(2):
        hidden, logits = OD.talker_decode_step(cfg, weights, case.step_inputs(step), positions + step, deltas,
                                               cache, tables, mode="fp32")
        _close(hidden, FIXTURE[f"decode_hidden_{step}"])
        _close(logits, FIXTURE[f"decode_logits_{step}"])
    # the KV arena after both steps: history untouched, each slot's two new rows in place
    _close(torch.stack([k for k, _ in cache]), FIXTURE["decode_keys"])
    _close(torch.stack([v for _, v in cache]), FIXTURE["decode_values"])


def test_padded_prefill_matches_reference_prefill_graph():
    cfg, weights = case.config(), case.weights()
    x = case.prefill_inputs()
    mask = case.prefill_mask()
    B, L = x.shape[:2]
    # real tokens attend to themselves and earlier real tokens; rotary position = token index
    rot = (mask.float().cumsum(-1) - 1).masked_fill(mask == 0, 1).long()
    pos = torch.arange(L).expand(B, L)
    cache = OD.new_cache(cfg, B, L)
    out = OD.decoder_forward(cfg, weights, x, rot, cache, pos, _tables(L + 1), mode="fp32")
    last = mask.sum(-1) - 1
    hidden = out[torch.arange(B), last]
    logits = hidden @ weights["head"].T
    real = len(case.PREFILL_LENGTHS)
    _close(hidden[:real], FIXTURE["prefill_hidden"][:real])
    _close(logits[:real], FIXTURE["prefill_logits"][:real])
    # K/V of every real token of every layer
    for layer, (k, v) in enumerate(cache):
        for b, n in enumerate(case.PREFILL_LENGTHS):
            _close(k[b, :, :n], FIXTURE["prefill_keys"][layer, b, :, :n])
            _close(v[b, :, :n], FIXTURE["prefill_values"][layer, b, :, :n])


def test_predictor_layer_stack_matches_reference_positions_and_masks():
    """Step 0: two tokens at positions [0, 1] under a causal mask; step s: one token at s + 1
    attending to everything cached (continuous.py:37-61), single-axis RoPE."""
    cfg, weights = case.config(), case.weights()
    B = case.PREDICTOR_BATCH
    cache = OD.new_cache(cfg, B, case.PREDICTOR_STEPS + 1)
    tables = _tables(case.PREDICTOR_STEPS + 2)
    for step in range(case.PREDICTOR_STEPS):
        pos = torch.tensor([[0, 1]]).expand(B, 2) if step == 0 else torch.full((B, 1), step + 1)
        out = OD.decoder_forward(cfg, weights, case.predictor_inputs(step), pos, cache, pos, tables, mode="fp32")
        _close(out, FIXTURE[f"predictor_hidden_{step}"])
