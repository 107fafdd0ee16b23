"""Multi-engine dispatcher on CPU: spawned engine processes running the scripted engine.

Covers routing to the least-loaded engine, per-engine caps, cancellation routing,
and host-side failure detection (an engine that raises, a process that exits, an
engine that stops making progress): the failed engine's requests finish with
finish_reason "error", the others are unaffected, and a fresh engine process
takes new requests. No GPU is involved.
"""
import time

import pytest

from qwen3_tts_b200.dispatcher import Dispatcher
from tests.fake_engine import chunk

FACTORY = "tests.fake_engine:FakeEngine"


def drive(dispatcher, submissions=(), cancelled=(), until=None, limit=15.0):
    """Tick until `until(results)` holds; returns (results, emitted chunks per id)."""
    results, chunks = {}, {}
    emit = lambda i, pcm, rate: chunks.setdefault(i, []).append(pcm)
    results.update(dict(dispatcher.tick(list(submissions), emit, list(cancelled))))
    deadline = time.monotonic() + limit
    while until is not None and not until(results) and time.monotonic() < deadline:
        results.update(dict(dispatcher.tick([], emit, [])))
    return results, chunks


@pytest.fixture()
def pair():
    d = Dispatcher(2, {}, per_engine=4, factory=FACTORY, devices=["cpu:0", "cpu:1"], start_timeout=120)
    yield d
    d.close()


def test_requests_spread_over_engines_and_complete(pair):
    subs = [(i, {"input": f"r{i}", "max_new_tokens": 4 + i}) for i in range(6)]
    results, chunks = drive(pair, subs, until=lambda r: len(r) == 6)
    assert sorted(results) == list(range(6))
    devices = [results[i]["device"] for i in range(6)]
    assert devices.count("cpu:0") == 3 and devices.count("cpu:1") == 3       # least-loaded routing
    for i in range(6):
        frames = 3 + i
        assert results[i]["finish_reason"] == "length" and results[i]["codec_frames"] == frames
        assert results[i]["pcm"] == b"".join(chunk(i, f) for f in range(frames))
        assert b"".join(chunks[i]) == results[i]["pcm"]
    assert pair.load() == [0, 0]


def test_per_engine_cap_and_cancellation(pair):
    subs = [(i, {"input": "x", "max_new_tokens": 200}) for i in range(8)]
    pair.tick(subs, None, [])
    assert pair.load() == [4, 4]
    with pytest.raises(RuntimeError):
        pair.tick([(99, {"input": "x", "max_new_tokens": 3})], None, [])
    pair.tick([], None, [0, 1, 2, 3, 4, 5, 6, 7])
    assert pair.load() == [0, 0]
    results, _ = drive(pair, [(10, {"input": "y", "max_new_tokens": 3})], until=lambda r: 10 in r)
    assert set(results) == {10}                         # cancelled requests never report


@pytest.mark.parametrize("failure", ["crash", "exit"])
def test_a_failed_engine_only_fails_its_own_requests(pair, failure):
    subs = [(0, {"input": "a", "max_new_tokens": 40}), (1, {"input": "b", "max_new_tokens": 40})]
    pair.tick(subs, None, [])
    owner_of_1 = pair.owner[1]
    pair.engines[owner_of_1].inbox.put(("submit", 2, {"input": failure, "max_new_tokens": 5}))
    pair.engines[owner_of_1].requests[2] = []
    pair.owner[2] = owner_of_1
    results, _ = drive(pair, until=lambda r: {0, 1, 2} <= set(r), limit=60)
    assert results[1]["finish_reason"] == "error" and results[2]["finish_reason"] == "error"
    assert results[0]["finish_reason"] == "length" and results[0]["codec_frames"] == 39
    # the replacement engine comes back and serves new work
    deadline = time.monotonic() + 120
    while not all(e.alive for e in pair.engines) and time.monotonic() < deadline:
        pair.tick([], None, [])
    assert all(e.alive for e in pair.engines)
    results, _ = drive(pair, [(3, {"input": "c", "max_new_tokens": 3}), (4, {"input": "d", "max_new_tokens": 3})],
                       until=lambda r: {3, 4} <= set(r))
    assert results[3]["finish_reason"] == results[4]["finish_reason"] == "length"


def test_a_stalled_engine_is_detected_by_the_watchdog():
    d = Dispatcher(1, {}, per_engine=2, factory=FACTORY, devices=["cpu:0"], start_timeout=120, stall_timeout=2.0,
                   restart=False)
    try:
        results, _ = drive(d, [(0, {"input": "hang", "max_new_tokens": 5})], until=lambda r: 0 in r, limit=30)
        assert results[0]["finish_reason"] == "error"
        assert d.load() == [None]
    finally:
        d.close()


def test_a_replacement_that_fails_to_start_is_not_started_again(tmp_path):
    d = Dispatcher(1, {"start_marker": str(tmp_path / "started")}, per_engine=2, factory=FACTORY,
                   devices=["cpu:0"], start_timeout=120)
    try:
        results, _ = drive(d, [(0, {"input": "crash", "max_new_tokens": 5})], until=lambda r: 0 in r, limit=30)
        assert results[0]["finish_reason"] == "error"
        first_replacement = d.engines[0].process
        deadline = time.monotonic() + 60
        while d.engines[0].starting and time.monotonic() < deadline:
            d.tick([], None, [])
        engine = d.engines[0]
        assert not engine.starting and not engine.alive and d.load() == [None]
        assert engine.process is first_replacement and not engine.process.is_alive()   # no second respawn
        for _ in range(20):
            d.tick([], None, [])
        assert d.engines[0].process is first_replacement
        with pytest.raises(RuntimeError, match="No engine has a free slot"):
            d.tick([(1, {"input": "x", "max_new_tokens": 3})], None, [])
    finally:
        d.close()


def test_result_pipe_yields_one_failure_per_engine_end():
    """An engine that reports its own failure and then closes its result pipe produces exactly
    one failure event (a second one would kill the replacement process); a pipe that closes
    without a goodbye produces one too, and only for an engine still marked alive."""
    import multiprocessing as mp
    from types import SimpleNamespace
    from qwen3_tts_b200.dispatcher import Dispatcher as D, Engine

    ctx = mp.get_context("spawn")

    def engine_with(messages, alive=True):
        reader, writer = ctx.Pipe(duplex=False)
        for message in messages:
            writer.send(message)
        writer.close()
        return Engine(rank=0, device="cpu:0", results=reader, alive=alive)

    holder = SimpleNamespace(engines=[engine_with([("tick", 0, [], []), ("failed", 0, "boom")])])
    events = D._poll(holder, 1.0)
    assert [e[0] for e in events] == ["tick", "failed"]
    assert holder.engines[0].results is None              # the closed pipe is dropped
    holder = SimpleNamespace(engines=[engine_with([])])   # exited without a word
    assert D._poll(holder, 1.0) == [("failed", 0, "result pipe closed")]
    holder = SimpleNamespace(engines=[engine_with([], alive=False)])
    assert D._poll(holder, 1.0) == []                     # already failed: no second failure
