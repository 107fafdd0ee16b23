"""Request-level data parallelism: one engine process per GPU behind one tick interface.

Requests are independent (no cross-request state), so N GPUs serve N
independent ``ContinuousModel`` replicas with no collective on the data path.
``Dispatcher`` looks like a continuous model to ``SpeechService``
(``tick(submissions, emit, cancelled)``, ``speakers``, ``languages``,
``close``) and fans the work out:

* each new request goes to the live engine with the fewest requests in flight
  (ties: lowest rank), never above ``per_engine``;
* each engine process (``engine_main``) runs its own tick loop on its GPU and
  sends ONE message per tick over its own result pipe (the tick's audio deltas
  and finished records; a sender thread writes the pipe, so the GPU loop never
  blocks on the host side); the dispatcher waits on all pipes at once. A
  request's PCM crosses the process boundary once, as its deltas (the finished
  record carries no audio; the dispatcher reassembles it from the deltas it
  relayed);
* cancellations go to the engine that owns the request;
* failure detection is on the host: an engine that raises or whose process
  exits is marked dead, its in-flight requests complete with
  ``finish_reason "error"`` (the audio already streamed stays delivered), and
  a fresh process is started for that GPU; the other engines are unaffected.
  A replacement that fails or exits while starting is not started again: its
  GPU takes no more requests (logged).

Processes use the ``spawn`` start method (CUDA state is never forked).
"""
from __future__ import annotations

import importlib
import logging
import multiprocessing as mp
import queue as queue_mod
import threading
import time
from multiprocessing import connection as mp_connection
from dataclasses import dataclass, field

LOGGER = logging.getLogger(__name__)
SAMPLE_RATE = 24000


def _load(spec: str):
    module, _, attr = spec.partition(":")
    return getattr(importlib.import_module(module), attr)


class _PipeSender:
    """Engine side of a result pipe: messages are queued locally and written by a thread, so the
    engine's tick loop never waits for the dispatcher to read."""

    def __init__(self, conn):
        self.conn = conn
        self.queue: queue_mod.SimpleQueue = queue_mod.SimpleQueue()
        self.thread = threading.Thread(target=self._run, name="q3t-result-pipe", daemon=True)
        self.thread.start()

    def _run(self) -> None:
        while True:
            message = self.queue.get()
            if message is None:
                return
            try:
                self.conn.send(message)
            except (OSError, EOFError, BrokenPipeError):  # the dispatcher is gone
                return

    def put(self, message) -> None:
        self.queue.put(message)

    def close(self) -> None:
        """Flush every queued message, then close the pipe."""
        self.queue.put(None)
        self.thread.join(timeout=30)
        self.conn.close()


def engine_main(rank: int, device: str, kwargs: dict, inbox, result_conn, factory: str | None) -> None:
    """Engine process: build the model, then tick while requests are in flight. Each tick's
    events go to the dispatcher as one ("tick", rank, deltas, records) message."""
    outbox = _PipeSender(result_conn)
    try:
        if factory is None:
            from qwen3_tts_b200.continuous import ContinuousModel
            model = ContinuousModel(device=device, **kwargs)
        else:
            model = _load(factory)(device=device, **kwargs)
        outbox.put(("hello", rank, list(model.speakers), list(model.languages)))
    except Exception as error:  # the dispatcher sees the engine as dead
        outbox.put(("failed", rank, f"engine start failed: {error!r}"))
        outbox.close()
        return
    active: set = set()
    try:
        while True:
            submissions, cancelled, stop = [], [], False
            try:
                message = inbox.get(timeout=1.0) if not active else inbox.get_nowait()
                while True:
                    kind = message[0]
                    if kind == "submit":
                        submissions.append((message[1], message[2]))
                        active.add(message[1])
                    elif kind == "cancel":
                        cancelled.append(message[1])
                        active.discard(message[1])
                    elif kind == "stop":
                        stop = True
                    message = inbox.get_nowait()
            except queue_mod.Empty:
                pass
            if stop:
                break
            if not submissions and not cancelled and not active:
                continue
            deltas, records = [], []
            emit = lambda identifier, pcm, rate: deltas.append((identifier, pcm, rate))
            for identifier, output in model.tick(submissions, emit, cancelled):
                active.discard(identifier)
                # the audio already crossed as deltas: the record travels without its PCM
                records.append((identifier, {k: v for k, v in output.items() if k != "pcm"}))
            if deltas or records:
                outbox.put(("tick", rank, deltas, records))
    except Exception as error:
        LOGGER.exception("engine %d failed", rank)
        outbox.put(("failed", rank, repr(error)))
        outbox.close()
        return
    model.close()
    outbox.put(("closed", rank))
    outbox.close()


@dataclass
class Engine:
    rank: int
    device: str
    process: object = None
    inbox: object = None
    results: object = None                         # dispatcher end of the engine's result pipe
    alive: bool = False
    starting: bool = False                         # spawned, no "hello" yet
    requests: dict = field(default_factory=dict)   # identifier -> [frames delivered (bytes)]
    last_event: float = 0.0


class Dispatcher:
    def __init__(self, gpus: int, engine_kwargs: dict, per_engine: int, factory: str | None = None,
                 restart: bool = True, start_timeout: float = 600.0, devices=None, stall_timeout: float = 120.0):
        self.ctx = mp.get_context("spawn")
        self.kwargs, self.per_engine, self.factory, self.restart = engine_kwargs, per_engine, factory, restart
        self.stall_timeout = stall_timeout
        devices = devices or [f"cuda:{i}" for i in range(gpus)]
        self.engines = [Engine(rank, device) for rank, device in enumerate(devices)]
        self.speakers: list = []
        self.languages: list = []
        self.owner: dict = {}            # identifier -> rank
        self.pending_events: list = []
        for engine in self.engines:
            self._spawn(engine)
        self._wait_ready(start_timeout)

    @classmethod
    def start(cls, gpus: int, engine_kwargs: dict, per_engine: int, **options) -> "Dispatcher":
        return cls(gpus, engine_kwargs, per_engine, **options)

    # ------------------------------------------------------------------ processes
    def _spawn(self, engine: Engine) -> None:
        if engine.results is not None:
            engine.results.close()
        engine.inbox = self.ctx.Queue()
        reader, writer = self.ctx.Pipe(duplex=False)
        engine.results = reader
        engine.process = self.ctx.Process(target=engine_main, name=f"q3t-engine-{engine.rank}", daemon=True,
                                          args=(engine.rank, engine.device, self.kwargs, engine.inbox, writer,
                                                self.factory))
        engine.process.start()
        writer.close()  # the engine process holds the writing end
        engine.alive = False
        engine.starting = True

    def _poll(self, timeout: float) -> list:
        """Events from every engine's result pipe, waiting up to `timeout` for the first. A pipe
        whose engine is gone yields a ("failed", rank, reason) event."""
        pipes = {e.results: e for e in self.engines if e.results is not None}
        events: list = []
        for conn in mp_connection.wait(list(pipes), timeout=timeout):
            engine = pipes[conn]
            ended = False  # the engine said goodbye ("failed" / "closed") before its pipe closed
            try:
                while conn.poll():
                    event = conn.recv()
                    ended = ended or event[0] in ("failed", "closed")
                    events.append(event)
            except (EOFError, OSError):
                conn.close()
                engine.results = None
                if engine.alive and not ended:
                    events.append(("failed", engine.rank, "result pipe closed"))
        return events

    def _wait_ready(self, timeout: float) -> None:
        deadline = time.monotonic() + timeout
        while not all(e.alive for e in self.engines):
            remaining = deadline - time.monotonic()
            if remaining <= 0:
                raise RuntimeError("Engines did not start in time")
            events = self._poll(min(remaining, 1.0))
            if not events:
                for engine in self.engines:
                    if not engine.alive and not engine.process.is_alive():
                        raise RuntimeError(f"Engine {engine.rank} exited during start")
                continue
            for event in events:
                if event[0] == "hello":
                    engine = self.engines[event[1]]
                    engine.alive, engine.starting = True, False
                    self.speakers, self.languages = event[2], event[3]
                elif event[0] == "failed":
                    raise RuntimeError(event[2])
                else:
                    self.pending_events.append(event)

    # ------------------------------------------------------------------ routing
    def load(self) -> list:
        return [len(e.requests) if e.alive else None for e in self.engines]

    def _route(self, identifier, payload) -> None:
        live = [e for e in self.engines if e.alive and len(e.requests) < self.per_engine]
        if not live:
            raise RuntimeError("No engine has a free slot")
        engine = min(live, key=lambda e: (len(e.requests), e.rank))
        if not engine.requests:
            engine.last_event = time.monotonic()
        engine.requests[identifier] = []
        self.owner[identifier] = engine.rank
        engine.inbox.put(("submit", identifier, payload))

    def _fail_engine(self, engine: Engine, reason: str, outputs: list) -> None:
        LOGGER.error("engine %d lost: %s", engine.rank, reason)
        engine.alive = False
        for identifier, delivered in engine.requests.items():
            pcm = b"".join(delivered)
            outputs.append((identifier, {"pcm": pcm, "sample_rate": SAMPLE_RATE,
                                         "codec_frames": len(pcm) // (2 * 1920), "finish_reason": "error"}))
            self.owner.pop(identifier, None)
        engine.requests.clear()
        if engine.process is not None and engine.process.is_alive():
            engine.process.kill()
        if engine.process is not None:
            engine.process.join(timeout=5)
        if self.restart:
            self._spawn(engine)

    def _retire(self, engine: Engine, reason: str) -> None:
        """A replacement engine that failed while starting is not started again (a start that fails
        once, e.g. out of device memory, would fail in a loop): its device leaves the rotation."""
        LOGGER.error("engine %d could not start again (%s); its device takes no more requests", engine.rank, reason)
        engine.starting = False
        if engine.process is not None:
            engine.process.join(timeout=5)
            if engine.process.is_alive():
                engine.process.kill()
                engine.process.join(timeout=5)

    # ------------------------------------------------------------------ the continuous-model interface
    def tick(self, submissions=(), emit=None, cancelled=()):
        outputs: list = []
        for identifier in cancelled:
            rank = self.owner.pop(identifier, None)
            if rank is not None:
                self.engines[rank].requests.pop(identifier, None)
                self.engines[rank].inbox.put(("cancel", identifier))
        for identifier, payload in submissions:
            self._route(identifier, payload)
        in_flight = any(e.requests for e in self.engines)
        events = self.pending_events
        self.pending_events = []
        events += self._poll(0.0 if events else (0.05 if in_flight else 0.0005))
        now = time.monotonic()
        for event in events:
            kind, rank = event[0], event[1]
            engine = self.engines[rank]
            engine.last_event = now
            if kind == "tick":
                for identifier, pcm, rate in event[2]:
                    if identifier in engine.requests:
                        engine.requests[identifier].append(pcm)
                        if emit is not None:
                            emit(identifier, pcm, rate)
                for identifier, record in event[3]:
                    delivered = engine.requests.pop(identifier, None)
                    if delivered is not None:
                        self.owner.pop(identifier, None)
                        outputs.append((identifier, dict(record, pcm=b"".join(delivered))))
            elif kind == "failed":
                if engine.alive:
                    self._fail_engine(engine, event[2], outputs)
                elif engine.starting:
                    self._retire(engine, event[2])
            elif kind == "hello":
                engine.alive, engine.starting = True, False
        for engine in self.engines:
            if engine.alive and engine.process is not None and not engine.process.is_alive():
                self._fail_engine(engine, f"process exited with code {engine.process.exitcode}", outputs)
            elif engine.alive and engine.requests and now - engine.last_event > self.stall_timeout:
                self._fail_engine(engine, f"no progress for {self.stall_timeout:.0f} s", outputs)
            elif engine.starting and engine.process is not None and not engine.process.is_alive():
                self._retire(engine, f"process exited with code {engine.process.exitcode}")
        return outputs

    def close(self) -> None:
        for engine in self.engines:
            if engine.process is not None and engine.process.is_alive():
                engine.inbox.put(("stop",))
        deadline = time.monotonic() + 30
        while any(e.process is not None and e.process.is_alive() for e in self.engines) and time.monotonic() < deadline:
            self._poll(0.1)  # drain the pipes so that every engine can flush and exit
        for engine in self.engines:
            if engine.process is not None:
                engine.process.join(timeout=5)
                if engine.process.is_alive():
                    engine.process.kill()
                    engine.process.join(timeout=5)
            if engine.results is not None:
                engine.results.close()
                engine.results = None
