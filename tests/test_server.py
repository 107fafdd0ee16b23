"""SpeechService over a continuous model (CPU, scripted engine): the HTTP/SSE contract of
the reference service (server.py:44-252; its tests test_server.py:11-227)."""
import asyncio
import base64
import json
import threading
from pathlib import Path
from types import SimpleNamespace

import pytest

aiohttp = pytest.importorskip("aiohttp")
from aiohttp import ClientSession, web  # noqa: E402

from qwen3_tts_b200.server import AudioChannel, SpeechService, normalize  # noqa: E402
from tests.fake_engine import FakeEngine, chunk  # noqa: E402


def options(**extra):
    base = dict(model=Path("unused"), device="cpu", queue_size=8, max_batch_size=4, streaming=True,
                continuous=True, prefill_per_tick=4, prefill_interval=1)
    base.update(extra)
    return SimpleNamespace(**base)


async def serve(service):
    app = web.Application()
    app.router.add_post("/speech", service.speech)
    app.router.add_get("/health", service.health)
    app.on_startup.append(service.start)
    app.on_cleanup.append(service.stop)
    runner = web.AppRunner(app)
    await runner.setup()
    site = web.TCPSite(runner, "127.0.0.1", 0)
    await site.start()
    return runner, f"http://127.0.0.1:{runner.addresses[0][1]}"


def events_of(text):
    return [json.loads(line[6:]) for line in text.splitlines() if line.startswith("data: ")]


def test_requests_are_validated_and_streamed_as_sse():
    owner = {}

    class Model(FakeEngine):
        def __init__(self, path, device):
            super().__init__(device)
            owner["thread"] = threading.get_ident()

        def tick(self, submissions, emit, cancelled):
            assert threading.get_ident() == owner["thread"]
            return super().tick(submissions, emit, cancelled)

    async def exercise():
        runner, url = await serve(SpeechService(options(), Model))
        try:
            async with ClientSession() as session:
                for bad in ([], {"input": ""}, {"input": "x", "max_new_tokens": 1}, {"input": "x", "seed": -1},
                            {"input": "x", "voice": "nobody"}, {"input": "x", "response_format": "wav"}):
                    async with session.post(url + "/speech", json=bad) as response:
                        assert response.status == 400
                async with session.post(url + "/speech", json={"input": "hello", "max_new_tokens": 5}) as response:
                    assert response.status == 200
                    events = events_of(await response.text())
                async with session.get(url + "/health") as response:
                    assert (await response.json())["status"] == "ready"
        finally:
            await runner.cleanup()
        kinds = [e["type"] for e in events]
        assert kinds[-1] == "speech.audio.done" and events[-1]["codec_frames"] == 4
        audio = b"".join(base64.b64decode(e["audio"]) for e in events if e["type"] == "speech.audio.delta")
        assert audio == b"".join(chunk(0, f) for f in range(4))   # streamed chunks + empty tail, no duplicates

    asyncio.run(asyncio.wait_for(exercise(), timeout=20))


def test_first_audio_arrives_before_the_request_finishes():
    released = threading.Event()

    class Model(FakeEngine):
        def __init__(self, path, device):
            super().__init__(device)

        def tick(self, submissions, emit, cancelled):
            out = super().tick(submissions, emit, cancelled)
            if out and not released.wait(timeout=5):
                raise RuntimeError("audio was held until completion")
            return out

    async def exercise():
        runner, url = await serve(SpeechService(options(), Model))
        try:
            async with ClientSession() as session:
                async with session.post(url + "/speech", json={"input": "x", "max_new_tokens": 4}) as response:
                    first = json.loads((await response.content.readline()).decode()[6:])
                    assert base64.b64decode(first["audio"]) == chunk(0, 0)
                    released.set()
                    rest = events_of(await response.text())
                    assert rest[-1]["type"] == "speech.audio.done"
        finally:
            released.set()
            await runner.cleanup()

    asyncio.run(asyncio.wait_for(exercise(), timeout=20))


def test_replacement_is_admitted_while_a_long_request_runs():
    log = []

    class Model(FakeEngine):
        def __init__(self, path, device):
            super().__init__(device)

        def tick(self, submissions, emit, cancelled):
            log.extend(("admit", p["input"]) for _, p in submissions)
            return super().tick(submissions, emit, cancelled)

    async def exercise():
        runner, url = await serve(SpeechService(options(max_batch_size=2), Model))
        try:
            async with ClientSession() as session:
                async def request(text, n):
                    async with session.post(url + "/speech", json={"input": text, "max_new_tokens": n}) as r:
                        assert "speech.audio.done" in await r.text()
                long = asyncio.create_task(request("long", 60))
                await request("short", 3)
                await request("replacement", 3)
                assert not long.done()
                await long
        finally:
            await runner.cleanup()
        admits = [entry[1] for entry in log if entry[0] == "admit"]
        assert sorted(admits) == ["long", "replacement", "short"]

    asyncio.run(asyncio.wait_for(exercise(), timeout=30))


def test_prefill_interval_batches_admission_and_cancellation_is_immediate():
    ticks = []

    async def exercise():
        loop = asyncio.get_running_loop()
        futures = [loop.create_future() for _ in range(3)]
        service = None
        queued = threading.Event()

        def enqueue_replacement():
            futures[1].cancel()
            service.queue.put_nowait(({"input": "replacement", "max_new_tokens": 3}, futures[2], AudioChannel(loop)))
            queued.set()

        class Model(FakeEngine):
            def __init__(self, path, device):
                super().__init__(device)
                self.step = 0

            def tick(self, submissions, emit, cancelled):
                ticks.append(([p["input"] for _, p in submissions], list(cancelled)))
                if self.step == 0:
                    loop.call_soon_threadsafe(enqueue_replacement)
                    assert queued.wait(2)
                self.step += 1
                return super().tick(submissions, None, cancelled)

        service = SpeechService(options(streaming=False, prefill_interval=4), Model)
        await service.start(None)
        try:
            for i, name in enumerate(["long", "cancel-me"]):
                service.queue.put_nowait(({"input": name, "max_new_tokens": 9}, futures[i], AudioChannel(loop)))
            await asyncio.wait_for(asyncio.gather(futures[0], futures[2]), timeout=10)
            await asyncio.wait_for(service.queue.join(), timeout=5)
        finally:
            await service.stop(None)
        assert futures[1].cancelled()
        assert ticks[0][0] == ["long", "cancel-me"]
        assert ticks[1][1] == [1]                              # cancellation on the very next tick
        assert all(not t[0] for t in ticks[1:4])               # no admission until tick 4
        assert ticks[4][0] == ["replacement"]

    asyncio.run(exercise())


def test_model_failure_fails_pending_requests_and_reports_unhealthy():
    class Model(FakeEngine):
        def __init__(self, path, device):
            super().__init__(device)

    async def exercise():
        service = SpeechService(options(), Model)
        runner, url = await serve(service)
        try:
            async with ClientSession() as session:
                async with session.post(url + "/speech", json={"input": "crash"}) as response:
                    events = events_of(await response.text())
                    assert events[-1]["type"] == "speech.audio.error"
                async with session.post(url + "/speech", json={"input": "x"}) as response:
                    assert response.status == 503
                async with session.get(url + "/health") as response:
                    assert response.status == 503
        finally:
            await runner.cleanup()

    asyncio.run(asyncio.wait_for(exercise(), timeout=20))


def test_normalize_keeps_token_ids_and_defaults():
    request = normalize({"input": "hi", "input_ids": [1, 2, 3]}, ["ryan"], ["english"])
    assert request["input_ids"] == [1, 2, 3] and request["seed"] == 42 and request["max_new_tokens"] == 2048
    with pytest.raises(ValueError):
        normalize({"input": "hi", "input_ids": [-1]}, ["ryan"], ["english"])


def test_audio_channel_hands_chunks_to_the_loop_without_a_round_trip():
    """emit() queues a base64-encoded chunk on the event loop without waiting for the loop (the
    owner thread never blocks on it while places are free); with `depth` chunks unread it waits
    for a place, and after its timeout marks the channel failed and drops later chunks."""
    import asyncio
    import base64
    import time
    loop = asyncio.new_event_loop()
    try:
        channel = AudioChannel(loop, depth=2, timeout=0.2)
        start = time.monotonic()
        channel.emit(b"ab", 24000)
        channel.emit(b"cde", 24000)   # the loop is not even running: no round trip
        assert time.monotonic() - start < 0.1
        channel.emit(b"fg", 24000)    # no free place: waits 0.2 s, then fails the channel
        assert channel.closed.is_set() and isinstance(channel.error, TimeoutError)
        channel.emit(b"hi", 24000)    # dropped

        async def drain():
            got = []
            while not channel.queue.empty():
                got.append(await channel.queue.get())
                channel.taken()
            return got
        got = loop.run_until_complete(drain())
        assert got == [(2, base64.b64encode(b"ab").decode(), 24000), (3, base64.b64encode(b"cde").decode(), 24000)]
    finally:
        loop.close()
