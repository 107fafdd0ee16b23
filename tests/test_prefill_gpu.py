"""Packed (ragged) talker prefill against the padded prefill and the CPU oracle.

The packed prefill runs the prompts end to end as one row set, each row at its own
(slot, position); the padded prefill (PrefillGraph, prefill_graph.py:31-50) pads every
prompt to the longest. Both must leave the same K/V in the arena slots and return the
same last-token hidden state and logits; the oracle (oracle/decoder.py, fp32) is the
truth for both.
"""
from dataclasses import replace

import pytest
import torch

from oracle import decoder as OD
from tests.golden.inputs import normal

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
LENGTHS = [37, 5, 129, 64, 1, 200]           # ragged, a single-token prompt, one past a power of two


def _setup(cuda, cfg, slots, capacity, seed):
    from qwen3_tts_b200.talker import SlotArena, rope_tables
    from qwen3_tts_b200.weights import decoder_weights, pack_decoder
    weights = decoder_weights(cfg, seed=seed)
    cos, sin = rope_tables(4096, cfg.head_dim, cfg.theta, cuda)
    return weights, pack_decoder(weights, cuda), SlotArena(cfg, slots, capacity, cuda), cos, sin


def _prompts(cfg, lengths, seed):
    return [torch.from_numpy(normal(seed + i, (n, cfg.hidden), 0.5)).to(BF16) for i, n in enumerate(lengths)]


def _run_packed(cuda, cfg, packed_w, arena, cos, sin, prompts, first_slot, requests, use_graph):
    from qwen3_tts_b200.batching import packed_rows, packed_tables, packed_units
    from qwen3_tts_b200.talker import PackedPrefill
    lengths = [p.shape[0] for p in prompts]
    rows = packed_rows(sum(lengths))
    graph = PackedPrefill(cfg, packed_w, arena, rows, requests, cos, sin)
    if use_graph:
        graph.capture()
    x = torch.cat(prompts)
    x = torch.cat([x, x[-1:].expand(rows - x.shape[0], -1)])
    row_slots, row_pos, last = packed_tables(lengths, first_slot, rows, requests)
    units = packed_units(lengths, first_slot, rows, requests)
    hidden, logits = graph.run(x.to(cuda), row_slots.to(cuda), row_pos.to(cuda), last.to(cuda), units.to(cuda))
    torch.cuda.synchronize()
    graph.close()
    return hidden[:len(prompts)].float().cpu(), logits[:len(prompts)].cpu()


def _rel(got, want):
    return float((got.float() - want.float()).norm() / want.float().norm())


@pytest.mark.parametrize("use_graph", [False, True])
def test_packed_prefill_matches_padded_prefill_at_full_width(cuda, use_graph):
    from qwen3_tts_b200.config import TALKER
    from qwen3_tts_b200.talker import TalkerPrefill
    cfg = replace(TALKER, layers=2)
    weights, packed_w, arena_a, cos, sin = _setup(cuda, cfg, 8, 256, seed=21)
    arena_b = type(arena_a)(cfg, 8, 256, cuda)
    prompts = _prompts(cfg, LENGTHS, 700)
    n, first = len(prompts), 1
    hidden, logits = _run_packed(cuda, cfg, packed_w, arena_b, cos, sin, prompts, first, 8, use_graph)

    padded = TalkerPrefill(cfg, packed_w, arena_a, 8, 256, cos, sin)
    if use_graph:
        padded.capture()
    x = torch.zeros(8, 256, cfg.hidden, dtype=BF16)
    for b, p in enumerate(prompts):
        x[b, :p.shape[0]] = p
    x[n:] = x[n - 1]
    lens = torch.tensor(LENGTHS + [LENGTHS[-1]] * (8 - n))
    slots = torch.tensor([first + min(b, n - 1) for b in range(8)])
    h_pad, l_pad = padded.run(x.to(cuda), lens.to(cuda), slots.to(cuda))
    torch.cuda.synchronize()
    padded.close()
    # identical kernels per row; only the split plans (summation order) differ, so the two
    # agree to bf16 rounding (one ulp is 2^-8 relative) carried through two layers
    torch.testing.assert_close(hidden, h_pad[:n].float().cpu(), atol=3e-2, rtol=3e-2)
    assert _rel(logits, l_pad[:n].cpu()) <= 1e-2
    for layer in range(cfg.layers):
        for b, length in enumerate(LENGTHS):
            for got, want in ((arena_b.keys[layer], arena_a.keys[layer]), (arena_b.values[layer],
                                                                           arena_a.values[layer])):
                torch.testing.assert_close(got[first + b, :, :length].float(), want[first + b, :, :length].float(),
                                           atol=3e-2, rtol=3e-2)
    # the slot before the packed prompts and the positions past each prompt are untouched
    assert not arena_b.packed[:, 0].any()
    for b, length in enumerate(LENGTHS):
        assert not arena_b.packed[:, first + b, :, length:].any()


def test_packed_prefill_matches_oracle(cuda):
    from qwen3_tts_b200.config import tiny_talker
    cfg = tiny_talker(layers=3)
    weights, packed_w, arena, cos, sin = _setup(cuda, cfg, 8, 256, seed=22)
    prompts = _prompts(cfg, LENGTHS, 800)
    hidden, logits = _run_packed(cuda, cfg, packed_w, arena, cos, sin, prompts, 2, 8, True)
    tables = OD.Tables(4096, cfg.head_dim, cfg.theta)
    for b, prompt in enumerate(prompts):
        length = prompt.shape[0]
        cache = OD.new_cache(cfg, 1, length)
        pos = torch.arange(length).view(1, length)
        out = OD.decoder_forward(cfg, weights, prompt.float().view(1, length, -1), pos, cache, pos, tables,
                                 mode="fp32")
        h_ref = out[0, -1]
        l_ref = h_ref @ weights["head"].float().T
        assert _rel(hidden[b], h_ref) <= 2e-2, b
        assert _rel(logits[b], l_ref) <= 2e-2, b
        for layer, (k, v) in enumerate(cache):
            assert _rel(arena.keys[layer][2 + b, :, :length].cpu(), k[0]) <= 2e-2, (b, layer)
            assert _rel(arena.values[layer][2 + b, :, :length].cpu(), v[0]) <= 2e-2, (b, layer)
