"""Talker decode step (28-layer stack on the slot arena) against the CPU oracle."""
import numpy as np
import pytest
import torch
from dataclasses import replace

from oracle import decoder as OD
from tests.golden.inputs import normal, uniform

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def prefill_arena(cfg, arena, cache, positions, seed):
    """Fill slots' KV history 0..pos-1 with the same random values on both sides."""
    for layer in range(cfg.layers):
        k = torch.from_numpy(normal(seed + 2 * layer, tuple(arena.keys[layer].shape))).to(BF16)
        v = torch.from_numpy(normal(seed + 2 * layer + 1, tuple(arena.keys[layer].shape))).to(BF16)
        for b, p in enumerate(positions):
            k[b, :, p:] = 0
            v[b, :, p:] = 0
        arena.keys[layer].copy_(k)
        arena.values[layer].copy_(v)
        cache[layer][0][:k.shape[0]].copy_(k.float())
        cache[layer][1][:k.shape[0]].copy_(v.float())


def run_case(cuda, cfg, batch, capacity, positions, seed=3, use_graph=True, context=None):
    from qwen3_tts_b200.talker import TalkerDecoder
    from qwen3_tts_b200.weights import decoder_weights
    weights = decoder_weights(cfg, seed=seed)
    engine = TalkerDecoder(cfg, weights, slots=batch, capacity=capacity, device=cuda, use_graphs=use_graph,
                           max_positions=4096)
    cache = OD.new_cache(cfg, batch, capacity)
    prefill_arena(cfg, engine.arena, cache, positions, 1000 + seed)
    embeds = torch.from_numpy(normal(seed + 50, (batch, cfg.hidden), 0.1)).to(BF16)
    pos = torch.tensor(positions, dtype=torch.long)
    delta = torch.tensor([0] * batch, dtype=torch.long)
    step = engine.step_for(batch, capacity if context is None else context)
    hidden, logits = step.run(embeds.to(cuda), pos.to(cuda), (pos + delta).to(cuda))
    torch.cuda.synchronize()
    tables = OD.Tables(4096, cfg.head_dim, cfg.theta)
    return engine, step, weights, cache, embeds, pos, delta, tables, hidden.cpu(), logits.cpu()


@pytest.mark.parametrize("use_graph", [False, True])
def test_tiny_talker_step_matches_oracle(cuda, use_graph):
    from qwen3_tts_b200.config import tiny_talker
    cfg = tiny_talker(layers=3)
    positions = [0, 5, 17, 63, 100]
    engine, step, weights, cache, embeds, pos, delta, tables, hidden, logits = run_case(
        cuda, cfg, 5, 128, positions, use_graph=use_graph)
    # bf16-emulating oracle: same rounding points, only accumulation order differs
    cache_b = [(k.clone(), v.clone()) for k, v in cache]
    h_ref, l_ref = OD.talker_decode_step(cfg, weights, embeds, pos, delta, cache_b, tables, mode="bf16f")
    torch.testing.assert_close(hidden.float(), h_ref, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(logits, l_ref, atol=2e-2, rtol=2e-2)
    # fp32 truth: logits within 1e-2 relative (normwise)
    h32, l32 = OD.talker_decode_step(cfg, weights, embeds, pos, delta, cache, tables, mode="fp32")
    assert float((logits - l32).norm() / l32.norm()) <= 1e-2
    # greedy ids bit-exact wherever the fp32 top-1/top-2 margin exceeds the logit error bound
    top2 = l32.topk(2, dim=-1).values
    margin = top2[:, 0] - top2[:, 1]
    decided = margin > 2 * (logits - l32).abs().max()
    assert torch.equal(logits.argmax(-1)[decided], l32.argmax(-1)[decided])
    # the KV written at each slot's position matches the oracle's
    for layer in range(cfg.layers):
        for b, p in enumerate(positions):
            torch.testing.assert_close(engine.arena.keys[layer][b, :, p].float().cpu(), cache_b[layer][0][b, :, p],
                                       atol=2e-2, rtol=2e-2)
            # V is the bf16 GEMM output: equal up to one bf16 rounding of a reordered fp32 sum
            torch.testing.assert_close(engine.arena.values[layer][b, :, p].float().cpu(),
                                       cache_b[layer][1][b, :, p], atol=1e-2, rtol=2 ** -7)
    engine.close()


def test_graph_replay_equals_eager_and_is_deterministic(cuda):
    from qwen3_tts_b200.config import tiny_talker
    cfg = tiny_talker(layers=2)
    positions = [3, 9, 40, 64]
    engine, step, *_rest, hidden, logits = run_case(cuda, cfg, 4, 96, positions, use_graph=True)
    eager = []
    for _ in range(2):
        step.compute()
        torch.cuda.synchronize()
        eager.append(step.logits.clone())
    for _ in range(2):
        step.graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(step.logits, eager[0])
    assert torch.equal(eager[0], eager[1])
    engine.close()


def test_full_width_talker_layers(cuda):
    """Real talker widths (hidden 2048, FFN 6144, vocab 3072) at reduced depth, C=32 ragged contexts."""
    from qwen3_tts_b200.config import TALKER
    cfg = replace(TALKER, layers=2)
    rng = uniform(77, (32,))
    positions = (64 + rng * (600 - 64)).astype(np.int64).tolist()
    engine, step, weights, cache, embeds, pos, delta, tables, hidden, logits = run_case(
        cuda, cfg, 32, 640, positions, seed=9)
    from qwen3_tts_b200 import ops
    assert ops.read_status(cuda) == 0
    h_ref, l_ref = OD.talker_decode_step(cfg, weights, embeds, pos, delta, cache, tables, mode="bf16f")
    # Logits within 1e-2 relative (normwise, ||diff||_2 / ||ref||_2); elementwise
    # the bf16 rounding chain of two full-width layers differs in a handful of
    # entries by a few bf16 ulps of the hidden state, so the max-abs bound is 6e-2.
    diff = (logits.float() - l_ref.float())
    assert float(diff.norm() / l_ref.float().norm()) <= 1e-2
    assert float(diff.abs().max()) <= 6e-2
    assert torch.isfinite(logits).all()
    engine.close()


def test_capacity_growth_preserves_history(cuda):
    from qwen3_tts_b200.config import tiny_talker
    from qwen3_tts_b200.talker import TalkerDecoder
    from qwen3_tts_b200.weights import decoder_weights
    cfg = tiny_talker(layers=1)
    engine = TalkerDecoder(cfg, decoder_weights(cfg, 1), slots=4, capacity=64, device=cuda, use_graphs=False,
                           max_positions=1024)
    engine.arena.packed.copy_(torch.from_numpy(normal(5, tuple(engine.arena.packed.shape))).to(BF16))
    before = engine.arena.packed.clone()
    engine.ensure_capacity(64)
    assert engine.arena.capacity == 128
    assert torch.equal(engine.arena.packed[:, :, :, :64], before)
    assert engine.arena.packed[:, :, :, 64:].eq(0).all()
    engine.close()
