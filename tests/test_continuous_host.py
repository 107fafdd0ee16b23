"""Host scheduling of ContinuousModel.tick with the device steps replaced by fakes (CPU).

Mirrors the reference's own host-logic tests (test_audio_transfer.py builds a
ContinuousModel with object.__new__ and a fake codec): the emission schedule
(continuous.py:636), stop/length reasons (continuous.py:637-641), grouping of
due slots by chunk length and codec batch (continuous.py:475-504), callback
order and bytes (continuous.py:528-539), result records and slot compaction by
moving the last slot (continuous.py:643-657), cancellation (continuous.py:544-556).
"""
import numpy as np
import pytest
import torch

from qwen3_tts_b200.continuous import ContinuousModel, EngineStats, RequestState

EOS = 2150


def fake_engine(tokens_by_id, codec_batch_size=2, incremental=True, context=72):
    model = object.__new__(ContinuousModel)
    model.device = torch.device("cpu")
    model.states = []
    model.max_slots, model.decode_bucket_step = 8, 0
    model.eos = EOS
    model.codec_chunk_frames = 8
    model.incremental_codec = incremental
    model.codec_batch_size = codec_batch_size
    model.context = context
    model.on_codes = None
    model.stats = EngineStats()
    model.calls = {"decode": [], "move": []}
    model.pipeline_audio = False
    model._inflight = None
    model._codec_free, model._codec_held = [], []

    def admit_batch(submissions):
        for identifier, payload in submissions:
            model.states.append(RequestState(identifier, payload, 10, 0, payload["max_new_tokens"]))

    def run_tick(count):
        assert count == len(model.states)
        return [tokens_by_id[s.identifier][s.frames] for s in model.states]

    def decode_group(indices, starts, length, rows=None):
        model.calls["decode"].append((list(indices), list(starts), length))
        rows = []
        for slot, start in zip(indices, starts):
            ident = model.states[slot].identifier
            base = ident if isinstance(ident, int) else 20 + ident[1]      # ("batch", i) from generate()
            frames = np.repeat(np.arange(start, start + length), 1920)
            rows.append(torch.from_numpy((base * 1000 + frames).astype(np.int16)))
        return torch.stack(rows)

    model.admit_batch = admit_batch
    model._run_tick = run_tick
    model._decode_group = decode_group
    model._move_slot = lambda source, destination: model.calls["move"].append((source, destination))
    return model


def pcm_of(ident, frames):
    return (ident * 1000 + np.repeat(np.arange(frames), 1920)).astype("<i2").tobytes()


def test_schedule_reasons_results_and_compaction():
    tokens = {1: [5] * 40, 2: [5, 5, 5, 5, EOS] + [5] * 40, 3: [7] * 40}
    model = fake_engine(tokens)
    emitted = []
    emit = lambda ident, pcm, rate: emitted.append((ident, len(pcm) // 3840, rate))
    payloads = {1: {"max_new_tokens": 12}, 2: {"max_new_tokens": 30}, 3: {"max_new_tokens": 20}}
    results = {}
    for tick in range(30):
        subs = [(i, payloads[i]) for i in (1, 2, 3)] if tick == 0 else []
        for ident, record in model.tick(subs, emit=emit):
            results[ident] = record
        if not model.states:
            break
    # request 2 sampled EOS at its fifth tick: 5 frames, "stop"; the others hit max_new_tokens - 1
    assert results[2]["finish_reason"] == "stop" and results[2]["codec_frames"] == 5
    assert results[1]["finish_reason"] == "length" and results[1]["codec_frames"] == 11
    assert results[3]["finish_reason"] == "length" and results[3]["codec_frames"] == 19
    for ident, record in results.items():
        assert record["pcm"] == pcm_of(ident, record["codec_frames"])
        assert record["sample_rate"] == 24000
    chunks = {i: [n for j, n, _ in emitted if j == i] for i in results}
    assert chunks[1] == [2, 2, 4, 3]
    assert chunks[2] == [2, 2, 1]
    assert chunks[3] == [2, 2, 4, 8, 3]
    # request 2 (slot 1 of 3) finished first: the last slot (2) moved into it
    assert model.calls["move"][0] == (2, 1)


def test_due_slots_group_by_length_and_codec_batch():
    tokens = {i: [5] * 40 for i in range(5)}
    model = fake_engine(tokens, codec_batch_size=2)
    model.tick([(i, {"max_new_tokens": 30}) for i in range(5)])
    model.tick()      # every request reaches 2 frames together: 5 due with length 2
    assert model.calls["decode"] == [([0, 1], [0, 0], 2), ([2, 3], [0, 0], 2), ([4], [0], 2)]


def test_cancellation_compacts_before_the_tick():
    tokens = {i: [5] * 40 for i in range(4)}
    model = fake_engine(tokens)
    model.tick([(i, {"max_new_tokens": 30}) for i in range(4)])
    model.tick(cancelled=[1])
    assert [s.identifier for s in model.states] == [0, 3, 2]
    assert model.calls["move"] == [(3, 1)]
    assert [s.frames for s in model.states] == [2, 2, 2]


def test_windowed_codec_decodes_left_context_and_skips_it():
    tokens = {0: [5] * 200}
    model = fake_engine(tokens, incremental=False, context=4)
    delivered = []
    model.tick([(0, {"max_new_tokens": 100})], emit=lambda i, pcm, r: delivered.append(pcm))
    for _ in range(15):
        model.tick(emit=lambda i, pcm, r: delivered.append(pcm))
    # emissions at 2, 4, 8, 16 frames: windows start at max(0, emitted - 4)
    assert model.calls["decode"] == [([0], [0], 2), ([0], [0], 4), ([0], [0], 8), ([0], [4], 12)]
    assert b"".join(delivered) == pcm_of(0, 16)


def test_tick_without_requests_is_a_no_op():
    model = fake_engine({})
    assert model.tick() == []


def test_engine_counters_follow_the_ticks():
    tokens = {1: [5] * 40, 2: [5, 5, EOS] + [5] * 40, 3: [5] * 40}
    model = fake_engine(tokens)
    model.tick([(1, {"max_new_tokens": 30}), (2, {"max_new_tokens": 30}), (3, {"max_new_tokens": 30})])
    model.tick(cancelled=[3])
    model.tick()                                  # request 2 draws EOS on its third frame
    stats = model.stats.as_dict()
    assert (stats["ticks"], stats["admitted"], stats["cancelled"], stats["finished"]) == (3, 3, 1, 1)
    assert stats["frames"] == 3 + 2 + 2 and stats["active"] == 2 and stats["batch"] == 2
    assert stats["tick_seconds"] >= stats["last_tick_ms"] / 1e3 > 0


@pytest.mark.parametrize("mode", ["timed", "nvtx"])
def test_phase_tracing_wraps_and_restores(mode):
    from qwen3_tts_b200.tracing import instrument
    tokens = {1: [5] * 40}
    model = fake_engine(tokens)
    originals = {name: vars(model).get(name) for name in ("admit_batch", "_run_tick", "_decode_group", "tick")}
    trace = instrument(model, mode)
    model.tick([(1, {"max_new_tokens": 30})], emit=lambda *a: None)
    model.tick(emit=lambda *a: None)
    assert trace.tick == 2
    if mode == "timed":
        phases = [(r["phase"], r["tick"]) for r in trace.records]
        assert ("admit", 0) in phases and ("tick_graph", 0) in phases and ("tick_graph", 1) in phases
        assert ("codec", 1) in phases          # the first chunk (2 frames) is due at the second tick
        summary = trace.summary()
        assert summary["tick_graph"]["calls"] == 2 and summary["tick_graph"]["seconds"] >= 0
    else:
        assert trace.records == []
    trace.remove()
    assert {name: vars(model).get(name) for name in originals} == originals
    with pytest.raises(ValueError):
        instrument(model, "perf")


def test_batch_generate_runs_every_payload_in_order():
    """CustomVoiceModel.generate's contract (model.py:58-129) over the continuous tick: results in
    payload order, chunks emitted under the payload index, more payloads than slots admitted as
    slots free up."""
    tokens = {("batch", i): [5] * (3 + 2 * i) + [EOS] + [5] * 40 for i in range(5)}
    model = fake_engine(tokens)
    model.max_slots = 2
    emitted = []
    payloads = [{"max_new_tokens": 30} for _ in range(5)]
    results = model.generate(payloads, emit=lambda index, pcm, rate: emitted.append((index, len(pcm) // 3840)))
    assert [r["finish_reason"] for r in results] == ["stop"] * 5
    assert [r["codec_frames"] for r in results] == [4, 6, 8, 10, 12]
    for index in range(5):
        assert sum(n for i, n in emitted if i == index) == results[index]["codec_frames"]
    assert not model.states
    model.states.append(RequestState("live", {}, 10, 0, 30))
    with pytest.raises(ValueError):
        model.generate(payloads)
