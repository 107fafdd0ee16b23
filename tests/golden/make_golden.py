"""Generate the golden fixtures in this folder by running the REFERENCE engine.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py /path/to/qwen3-tts-rsi-engine

It imports the reference's own CPU-runnable modules (``qwen3_tts_engine``:
batching, sampling, continuous.SlotCache / ContinuousModel.semantic,
packed_kv, codec_code_buffer, request_views, codec_slots) and records their
outputs on seeded inputs. For the decoder it runs the reference's own
PackedAttention / PackedMLP (installed by the reference's install functions)
inside its SlotArena / SlotGraph decode step and its PrefillGraph, over small
stand-in decoder layers (``tests/qwen_tts_fakes.py``, which also stands in for
the four qwen-tts functions PackedAttention imports). The fixtures pin the CPU
oracle in ``oracle/``; nothing at test or bench time reads the reference
checkout.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE.parents[1] / "qwen3-tts-rsi-engine_b200"))
from tests.golden.inputs import bf16_scores, normal, uniform  # noqa: E402


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    from qwen3_tts_engine.batching import decode_batch_size
    from qwen3_tts_engine.codec_code_buffer import CodecCodeBuffer
    from qwen3_tts_engine.continuous import ContinuousModel, SlotCache
    from qwen3_tts_engine.packed_kv import copy_packed_prefix
    from qwen3_tts_engine.request_views import single_request_inputs
    from qwen3_tts_engine.sampling import categorical, random_table

    torch.set_num_threads(4)
    out: dict = {}
    arrays: dict = {}

    # ---- batching: every (slots, step, active)
    table = []
    for slots in [1, 2, 4, 8, 16, 32, 64]:
        for step in [0] + [x for x in [1, 2, 4, 8, 16, 32, 64] if x <= slots]:
            for active in range(1, slots + 1):
                table.append([slots, step, active, decode_batch_size(active, slots, step)])
    out["decode_batch_size"] = table

    # ---- random tables
    arrays["random_table_42"] = random_table(42, 100).numpy()
    arrays["random_table_7"] = random_table(7, 19).numpy()

    # ---- categorical on Philox-derived scores (talker width 3072, predictor width 2048)
    for seed, width in ((11, 3072), (12, 2048)):
        scores = bf16_scores(seed, 256, width, 3.0)
        uniforms = torch.from_numpy(uniform(seed + 100, (256,)))
        arrays[f"cat_tokens_{width}"] = categorical(scores, uniforms).numpy().astype(np.int16)
    boundary = torch.tensor([[-float("inf"), 0.0, -float("inf"), 0.0]]).repeat(3, 1)
    draws = torch.tensor([0.0, 0.5, 1.0 - torch.finfo(torch.float32).eps])
    out["cat_boundary"] = categorical(boundary, draws, top_k=2).flatten().tolist()

    # ---- semantic sampling (ContinuousModel.semantic unbound, as the reference probes do)
    eos, vocab = 2150, 3072
    allowed = torch.ones(vocab, dtype=torch.bool)
    allowed[-1024:] = False
    allowed[eos] = True
    state = SimpleNamespace(allowed=allowed, eos=eos, triton_cdf=False)
    logits = bf16_scores(21, 128, vocab, 2.0).to(torch.bfloat16)
    seen = torch.from_numpy(uniform(22, (128, vocab)) < 0.05)
    steps = torch.from_numpy((uniform(23, (128,)) * 5).astype(np.int64))
    uniforms = torch.from_numpy(uniform(24, (128,)))
    tokens = ContinuousModel.semantic(state, logits, uniforms, seen, steps)
    arrays["sem_tokens"] = tokens.numpy().astype(np.int16)

    # ---- SlotCache.update + SDPA on the packed slot table (fp32)
    g0 = torch.Generator().manual_seed(0)
    lens = torch.randint(1, 513, (8,), generator=g0)
    arena_k = torch.zeros(8, 8, 513, 128)
    arena_v = torch.zeros(8, 8, 513, 128)
    for b in range(8):
        n = int(lens[b])
        arena_k[b, :, :n] = torch.randn(8, n, 128, generator=g0)
        arena_v[b, :, :n] = torch.randn(8, n, 128, generator=g0)
    new_k = torch.randn(8, 8, 1, 128, generator=g0)
    new_v = torch.randn(8, 8, 1, 128, generator=g0)
    query = torch.randn(8, 16, 1, 128, generator=g0)
    arena = SimpleNamespace(capacity=513, native_kv_update=False, triton_kv_update=False,
                            keys=[arena_k], values=[arena_v])
    cache = SlotCache(arena, lens.clone(), 513, False)
    k_all, v_all = cache.update(new_k, new_v, 0, {})
    mask = torch.arange(513)[None, :] <= lens[:, None]
    attn = torch.nn.functional.scaled_dot_product_attention(query, k_all, v_all, mask[:, None, None, :],
                                                            enable_gqa=True)
    out["config1_lens"] = lens.tolist()
    out["config1_arena_k_sha256"] = sha(arena_k)
    out["config1_arena_v_sha256"] = sha(arena_v)
    arrays["config1_attention"] = attn.numpy()

    # ---- small SlotCache scatter (exact layout)
    keys = torch.from_numpy(normal(31, (4, 2, 64, 16)))
    values = torch.from_numpy(normal(32, (4, 2, 64, 16)))
    positions = torch.tensor([0, 63, 17, 1])
    nk = torch.from_numpy(normal(33, (4, 2, 1, 16)))
    nv = torch.from_numpy(normal(34, (4, 2, 1, 16)))
    small = SimpleNamespace(capacity=64, native_kv_update=False, triton_kv_update=False, keys=[keys], values=[values])
    SlotCache(small, positions, 64, False).update(nk, nv, 0, {})
    out["scatter_keys_sha256"] = sha(keys)
    out["scatter_values_sha256"] = sha(values)

    # ---- copy_packed_prefix
    target = torch.full((4, 5, 2, 7, 3), -7.0)
    source = torch.arange(4 * 3 * 2 * 5 * 6, dtype=torch.float32).view(4, 3, 2, 5, 6)[..., ::2]
    for row, slot, length in ((2, 3, 1), (0, 1, 5), (1, 4, 3)):
        copy_packed_prefix(target, source, slot, row=row, length=length)
    arrays["packed_prefix_target"] = target.numpy()

    # ---- codec code buffer ring
    buffer = CodecCodeBuffer(4, 16, "cpu")
    reads = []
    for tick in range(19):
        buffer.write(torch.arange(48).view(3, 16) + tick * 100, torch.tensor([tick, tick + 3, tick + 7]))
        if tick >= 7:
            reads.append(buffer.read([2, 0], [tick, tick - 7], 8).numpy())
    buffer.move(2, 0)
    reads.append(buffer.read([0], [18], 8).numpy()[:, :, :])
    arrays["code_buffer_reads"] = np.stack([r if r.shape[0] == 2 else np.concatenate([r, r]) for r in reads])

    # ---- request views
    gen = torch.Generator().manual_seed(42)
    st = SimpleNamespace(token=torch.tensor([[42]]), hidden=torch.randn(1, 1, 12, generator=gen),
                         uniforms=torch.rand(129, 16, generator=gen), trailing=torch.randn(1, 3, 12, generator=gen),
                         pad=torch.randn(1, 1, 12, generator=gen), seen=torch.zeros(1, 31, dtype=torch.bool),
                         frames=2, position=165, rope_delta=-13)
    views = single_request_inputs(st)
    arrays["views_draws"] = views.draws.numpy()
    arrays["views_text"] = views.text.numpy()
    arrays["views_uniforms"] = views.uniforms.numpy()
    out["views_integers"] = [int(views.positions[0]), int(views.rotary[0, 0, 0]), int(views.steps[0])]

    np.savez_compressed(HERE / "decode_path.npz", **arrays)
    (HERE / "decode_path.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", HERE / "decode_path.npz", HERE / "decode_path.json")
    codec_fixtures()
    decoder_fixtures()


TINY_CODEC = dict(codebooks=4, codebook_size=32, codebook_dim=8, semantic_codebooks=1, latent=12, hidden=8,
                  layers=2, heads=2, head_dim=4, ffn=16, window=6, eps=1e-5, theta=10000.0,
                  upsampling_ratios=(2,), upsample_rates=(2, 3), decoder_dim=8, layer_scale=0.1)
CODEC_SCHEDULE = {0: [2, 2, 4, 8, 4], 1: [1, 3, 8, 8]}


def codec_fixtures() -> None:
    """Run the reference's slot-indexed incremental codec (CodecSlots / CodecSlotGraph.compute,
    IncrementalCodec.run_module) over the oracle's stand-in decoder modules, two interleaved
    streams with ragged chunks, a slot move and a reset."""
    from qwen3_tts_engine.codec_slots import CodecSlotGraph, CodecSlots
    from oracle.codec import CodecDecoder, randomize
    from qwen3_tts_b200.config import CodecConfig

    cfg = CodecConfig(**TINY_CODEC)
    decoder = randomize(CodecDecoder(cfg), seed=5)
    slots = CodecSlots(decoder, 4)
    codes = {s: torch.from_numpy((uniform(60 + s, (1, cfg.codebooks, 20)) * cfg.codebook_size).astype(np.int64))
             for s in CODEC_SCHEDULE}
    slot_of = {0: 1, 1: 3}
    done = {0: 0, 1: 0}
    pcm = {0: [], 1: []}
    graphs = {}
    with torch.inference_mode():
        for step in range(max(len(v) for v in CODEC_SCHEDULE.values())):
            for stream, sched in CODEC_SCHEDULE.items():
                if step >= len(sched):
                    continue
                n = sched[step]
                graph = graphs.setdefault(n, CodecSlotGraph(slots, 1, n))
                graph.indices.copy_(torch.tensor([slot_of[stream]]))
                graph.codes.copy_(codes[stream][:, :, done[stream]:done[stream] + n])
                pcm[stream].append(graph.compute().clone())
                done[stream] += n
            if step == 1:  # compaction: stream 1 moves from slot 3 to slot 2 (CodecSlots.move)
                slots.move(3, 2)
                slot_of[1] = 2
        full = {s: decoder(codes[s]) for s in CODEC_SCHEDULE}
        # a reset slot decodes like a fresh stream
        slots.reset(slot_of[0])
        graph = graphs[4]
        graph.indices.copy_(torch.tensor([slot_of[0]]))
        graph.codes.copy_(codes[1][:, :, :4])
        fresh = graph.compute().clone()
    arrays = {f"codec_pcm_{s}": torch.cat(pcm[s], -1).numpy() for s in pcm}
    arrays.update({f"codec_full_{s}": full[s].numpy() for s in full})
    arrays["codec_fresh_after_reset"] = fresh.numpy()
    arrays["codec_frames"] = slots.frames.numpy()
    np.savez_compressed(HERE / "codec.npz", **arrays)
    print("wrote", HERE / "codec.npz")


def decoder_fixtures() -> None:
    """The talker decode step (SlotGraph.compute + codec_head, continuous.py:172-198, 612-613) and the
    padded batch prefill (PrefillGraph.compute, prefill_graph.py:31-50) run by the reference over
    fp32 stand-in layers with its PackedAttention (text-only RoPE, packed_attention.py:37-85) and
    PackedMLP (packed_mlp.py:19-27) installed."""
    from tests import qwen_tts_fakes as fakes
    from tests.golden import decoder_case as case
    fakes.install_modeling_stub()
    from qwen3_tts_engine.continuous import SlotArena, SlotGraph
    from qwen3_tts_engine.packed_attention import install_packed_attention
    from qwen3_tts_engine.packed_mlp import install_packed_mlp
    from qwen3_tts_engine.prefill_graph import PrefillGraph

    weights = case.weights()
    model = fakes.TalkerModel(case.LAYERS, case.HIDDEN, case.Q_HEADS, case.KV_HEADS, case.HEAD_DIM, case.FFN,
                              case.THETA)
    talker = fakes.Talker(model, case.VOCAB)
    fakes.load_oracle_weights(talker, weights)
    for layer in model.layers:
        layer.input_layernorm.variance_epsilon = case.EPS
        layer.post_attention_layernorm.variance_epsilon = case.EPS
        layer.self_attn.q_norm.variance_epsilon = case.EPS
        layer.self_attn.k_norm.variance_epsilon = case.EPS
    model.norm.variance_epsilon = case.EPS
    assert len(install_packed_attention(model, text_only_rope=True)) == case.LAYERS
    assert len(install_packed_mlp(model)) == case.LAYERS
    arrays = {}
    with torch.inference_mode():
        arena = SlotArena(model, case.SLOTS, case.CAPACITY)
        for layer in range(case.LAYERS):
            k, v = case.history(layer)
            arena.keys[layer].copy_(k)
            arena.values[layer].copy_(v)
        graph = SlotGraph(arena, case.SLOTS, case.CAPACITY)
        positions = torch.tensor(case.POSITIONS)
        deltas = torch.tensor(case.ROPE_DELTAS)
        for step in range(2):
            graph.inputs.copy_(case.step_inputs(step)[:, None])
            graph.positions.copy_(positions + step)
            graph.rotary.copy_((positions + step + deltas).view(1, -1, 1).expand(3, -1, 1))
            hidden = graph.compute()
            arrays[f"decode_hidden_{step}"] = case.as_numpy(hidden[:, 0])
            arrays[f"decode_logits_{step}"] = case.as_numpy(talker.codec_head(hidden[:, -1]).float())
        arrays["decode_keys"] = np.stack([case.as_numpy(k) for k in arena.keys])
        arrays["decode_values"] = np.stack([case.as_numpy(v) for v in arena.values])
        prefill = PrefillGraph(talker, case.PREFILL_BATCH, case.PREFILL_LEN)
        prefill.inputs.copy_(case.prefill_inputs())
        prefill.mask.copy_(case.prefill_mask())
        hidden, logits, cache = prefill.compute()
        arrays["prefill_hidden"] = case.as_numpy(hidden[:, 0])
        arrays["prefill_logits"] = case.as_numpy(logits)
        arrays["prefill_keys"] = np.stack([case.as_numpy(layer.keys) for layer in cache.layers])
        arrays["prefill_values"] = np.stack([case.as_numpy(layer.values) for layer in cache.layers])
        # the code predictor's layer stack over its 15-step position and mask pattern, with the
        # reference's PackedAttention on single-axis RoPE (continuous.py:37-61)
        from transformers.cache_utils import DynamicCache
        predictor = fakes.TalkerModel(case.LAYERS, case.HIDDEN, case.Q_HEADS, case.KV_HEADS, case.HEAD_DIM,
                                      case.FFN, case.THETA, talker=False)
        fakes.load_oracle_weights(fakes.Talker(predictor, case.VOCAB), weights)
        for layer in predictor.layers:
            for norm in (layer.input_layernorm, layer.post_attention_layernorm, layer.self_attn.q_norm,
                         layer.self_attn.k_norm):
                norm.variance_epsilon = case.EPS
        predictor.norm.variance_epsilon = case.EPS
        assert len(install_packed_attention(predictor)) == case.LAYERS
        assert len(install_packed_mlp(predictor)) == case.LAYERS
        cache = DynamicCache()
        mask = torch.zeros(1, 1, 2, 2)
        mask[..., 0, 1] = torch.finfo(torch.float32).min
        for step in range(case.PREDICTOR_STEPS):
            hidden = case.predictor_inputs(step)
            positions = torch.arange(2) if step == 0 else torch.tensor([step + 1])
            rotary = predictor.rotary_emb(hidden, positions[None].expand(hidden.shape[0], -1))
            for layer in predictor.layers:
                hidden = layer(hidden, attention_mask=mask if step == 0 else None, position_ids=positions[None],
                               past_key_values=cache, use_cache=True, cache_position=positions,
                               position_embeddings=rotary)[0]
            arrays[f"predictor_hidden_{step}"] = case.as_numpy(predictor.norm(hidden))
    np.savez_compressed(HERE / "decoder.npz", **arrays)
    print("wrote", HERE / "decoder.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/qwen3-tts-rsi-engine")
    main(sys.argv[1])
