"""Streaming speech service over the continuous engine (SpeechService, server.py:44-252).

One model-owner thread does all device work; HTTP handlers never touch the
GPU. Requests arrive on ``POST /v1/audio/speech`` and are answered as
server-sent events:

* ``speech.audio.delta`` ``{audio: base64 PCM16LE, sample_rate, channels: 1}``
  (streamed chunks when ``streaming`` is on, then the not-yet-sent tail),
* ``speech.audio.done`` ``{finish_reason, codec_frames}``,
* ``speech.audio.error`` ``{error: {message}}`` if the request fails mid-stream.

Two scheduling modes, as in the reference: ``run`` groups queued requests into
micro-batches for a ``generate(payloads[, emit])`` model, and
``run_continuous`` drives ``tick(submissions, emit, cancelled)`` of a
continuous model, admitting up to ``prefill_per_tick`` new requests every
``prefill_interval`` ticks (cancellations are passed on every tick).

``model_factory(model_path, device)`` builds the model on the owner thread; the
dispatcher in ``dispatcher.py`` provides a factory that fronts one engine
process per GPU.
"""
from __future__ import annotations

import argparse
import asyncio
import base64
import json
import logging
import threading
from concurrent.futures import ThreadPoolExecutor
from functools import partial
from pathlib import Path

LOGGER = logging.getLogger(__name__)
MAX_INPUT_CHARS = 10000


class AudioChannel:
    """Bounded per-request audio queue fed from the model-owner thread.

    ``emit`` hands a chunk to the event loop without waiting for it (one
    ``call_soon_threadsafe``, no round trip), with the chunk already base64
    encoded on the emitting thread, so the loop only frames and writes events.
    At most ``depth`` chunks are queued: when the client falls behind, ``emit``
    blocks the owner thread for at most ``timeout`` (30 s) for a free place; a
    timeout or a closed loop marks the channel failed and later chunks are
    dropped."""

    def __init__(self, loop, depth: int = 16, timeout: float = 30.0):
        self.loop = loop
        self.queue: asyncio.Queue = asyncio.Queue()
        self.places = threading.Semaphore(depth)
        self.timeout = timeout
        self.closed = threading.Event()
        self.error = None

    def emit(self, pcm: bytes, sample_rate: int) -> None:
        if self.closed.is_set():
            return
        if not self.places.acquire(timeout=self.timeout):
            self.error = TimeoutError("client stopped reading audio")
            self.closed.set()
            return
        chunk = (len(pcm), base64.b64encode(pcm).decode(), sample_rate)
        try:
            self.loop.call_soon_threadsafe(self.queue.put_nowait, chunk)
        except RuntimeError as error:  # the loop is gone
            self.error = error
            self.closed.set()

    def taken(self) -> None:
        """The consumer took one chunk off the queue: one more may be queued."""
        self.places.release()

    def close(self) -> None:
        self.closed.set()
        while not self.queue.empty():
            self.queue.get_nowait()
            self.places.release()


def normalize(payload, speakers, languages) -> dict:
    """Validate one request body; raises ValueError/TypeError with the reason (HTTP 400)."""
    if not isinstance(payload, dict):
        raise ValueError("Request must be an object")
    text = payload.get("input")
    if not isinstance(text, str) or not text.strip():
        raise ValueError("Nonempty input text is required")
    if len(text) > MAX_INPUT_CHARS:
        raise ValueError(f"Input exceeds {MAX_INPUT_CHARS} characters")
    if payload.get("response_format", "pcm") != "pcm" or payload.get("stream_format", "sse") != "sse":
        raise ValueError("This endpoint requires PCM over SSE")
    request = {"input": text, "voice": str(payload.get("voice", "Ryan")).lower(),
               "language": str(payload.get("language", "English")).lower(),
               "instructions": payload.get("instructions", ""), "seed": payload.get("seed", 42),
               "max_new_tokens": payload.get("max_new_tokens", 2048)}
    if payload.get("input_ids") is not None:
        ids = payload["input_ids"]
        if not isinstance(ids, list) or not all(type(i) is int and i >= 0 for i in ids):
            raise ValueError("input_ids must be a list of non-negative integers")
        request["input_ids"] = ids
    if request["voice"] not in speakers or request["language"] not in languages:
        raise ValueError("Unsupported speaker or language")
    if not isinstance(request["instructions"], str):
        raise ValueError("Instructions must be text")
    if type(request["seed"]) is not int or not 0 <= request["seed"] < 2 ** 32:
        raise ValueError("Seed must be an unsigned 32-bit integer")
    if type(request["max_new_tokens"]) is not int or not 2 <= request["max_new_tokens"] <= 4096:
        raise ValueError("max_new_tokens must be an integer in [2,4096]")
    return request


def sse(event: dict) -> bytes:
    return ("data: " + json.dumps(event) + "\n\n").encode()


def delta(pcm: bytes, sample_rate: int, encoded: str | None = None) -> dict:
    audio = encoded if encoded is not None else base64.b64encode(pcm).decode()
    return {"type": "speech.audio.delta", "audio": audio, "sample_rate": sample_rate, "channels": 1}


def settle(future, channel, output) -> None:
    """Complete a request's future from the engine's result record (a failed audio channel wins)."""
    if future.done():
        return
    if channel.error is not None:
        future.set_exception(channel.error)
    else:
        future.set_result(output)


class OwnerThread:
    """The single thread that owns the model and does all device work (the engine is not
    thread-safe and CUDA graphs are replayed from one host thread)."""

    def __init__(self):
        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="model-owner")

    async def call(self, fn, *args, **kwargs):
        return await asyncio.get_running_loop().run_in_executor(self._pool, partial(fn, *args, **kwargs))

    def shutdown(self) -> None:
        self._pool.shutdown(wait=True, cancel_futures=True)


class RequestBook:
    """Requests admitted to a continuous model, keyed by the integer identifier the engine
    sees (0, 1, 2, ... in admission order). Every entry taken from the service queue is
    matched by exactly one ``task_done`` - when it is found cancelled before admission, when
    its cancellation is passed to the engine, when the engine returns its result, or when the
    engine fails - so ``queue.join()`` tracks requests still in flight."""

    def __init__(self, queue: asyncio.Queue, slots: int, budget: int, interval: int):
        self.queue, self.slots, self.budget, self.interval = queue, slots, budget, interval
        self.entries: dict = {}          # identifier -> (payload, future, channel)
        self.issued = 0                  # identifiers handed out
        self.ticks = 0

    def _admit(self, entry, into: list) -> None:
        payload, future, _ = entry
        if future.cancelled():           # the client left while the request was queued
            self.queue.task_done()
            return
        self.entries[self.issued] = entry
        into.append((self.issued, payload))
        self.issued += 1

    def withdraw_cancelled(self) -> list:
        """Identifiers whose clients went away; the engine drops them on the next tick."""
        gone = [ident for ident, (_, future, _) in self.entries.items() if future.cancelled()]
        for ident in gone:
            del self.entries[ident]
            self.queue.task_done()
        return gone

    async def next_admissions(self, withdrawn: list) -> list:
        """New requests for this tick: with nothing in flight, wait for one; then take queued
        requests up to the slot count and the per-tick budget, every `interval` ticks (at once
        when the engine is idle)."""
        fresh: list = []
        idle = not self.entries
        if idle and not withdrawn:
            self._admit(await self.queue.get(), fresh)
            if not fresh:
                return None              # it was cancelled while queued: look again
        if idle or fresh or self.ticks % self.interval == 0:
            while len(self.entries) < self.slots and len(fresh) < self.budget and not self.queue.empty():
                self._admit(self.queue.get_nowait(), fresh)
        return fresh

    def relay(self, streaming: bool):
        """The engine's emit callback: chunks go to the request's audio channel when streaming."""
        def emit(ident, pcm, rate):
            entry = self.entries.get(ident)
            if entry is not None and streaming:
                entry[2].emit(pcm, rate)
        return emit

    def finish(self, results) -> None:
        self.ticks += 1
        for ident, output in results:
            _, future, channel = self.entries.pop(ident)
            settle(future, channel, output)
            self.queue.task_done()

    def fail(self, error: Exception) -> None:
        for _, future, _ in self.entries.values():
            if not future.done():
                future.set_exception(error)
            self.queue.task_done()
        self.entries.clear()

    def abandon(self) -> None:
        for _, future, channel in self.entries.values():
            channel.close()
            future.cancel()


class SpeechService:
    """The HTTP/SSE service: handlers validate and queue requests; one worker task feeds
    them to the model on the owner thread, either as micro-batches (``generate``) or through
    the continuous ``tick`` loop (``--continuous``)."""

    def __init__(self, options, model_factory):
        self.options = options
        self.model_factory = model_factory
        self.queue: asyncio.Queue = asyncio.Queue(maxsize=options.queue_size)
        self.owner = OwnerThread()
        self.model = None
        self.worker = None
        self.failure = None

    @property
    def streaming(self) -> bool:
        return bool(getattr(self.options, "streaming", False))

    async def start(self, app) -> None:
        self.model = await self.owner.call(self.model_factory, str(self.options.model), self.options.device)
        continuous = getattr(self.options, "continuous", False)
        self.worker = asyncio.create_task(self.run_continuous() if continuous else self.run())

    async def stop(self, app) -> None:
        if self.worker is not None:
            self.worker.cancel()
            await asyncio.gather(self.worker, return_exceptions=True)
        if self.model is not None:
            await self.owner.call(self.model.close)
        self.owner.shutdown()

    # ------------------------------------------------------------------ micro-batch mode
    async def _collect_batch(self) -> list:
        batch = [await self.queue.get()]
        wait_ms = getattr(self.options, "batch_wait_ms", 0)
        if wait_ms:
            await asyncio.sleep(wait_ms / 1000)
        while len(batch) < self.options.max_batch_size and not self.queue.empty():
            batch.append(self.queue.get_nowait())
        return batch

    async def _generate(self, group: list) -> None:
        """One generate() call for requests sharing (seed, max_new_tokens); results in order."""
        emit = None
        if self.streaming:
            def emit(index, pcm, rate):
                group[index][2].emit(pcm, rate)
        try:
            outputs = await self.owner.call(self.model.generate, [payload for payload, _, _ in group],
                                            **({"emit": emit} if emit else {}))
            if len(outputs) != len(group):
                raise RuntimeError("Model batch output count mismatch")
        except Exception as error:
            LOGGER.exception("Model batch failed")
            for _, future, _ in group:
                if not future.done():
                    future.set_exception(error)
            return
        for (_, future, channel), output in zip(group, outputs):
            settle(future, channel, output)

    async def run(self) -> None:
        while True:
            batch = await self._collect_batch()
            groups: dict = {}
            for entry in batch:
                if not entry[1].cancelled():
                    groups.setdefault((entry[0]["seed"], entry[0]["max_new_tokens"]), []).append(entry)
            for group in groups.values():
                await self._generate(group)
            for _ in batch:
                self.queue.task_done()

    # ------------------------------------------------------------------ continuous mode
    async def run_continuous(self) -> None:
        book = RequestBook(self.queue, self.options.max_batch_size, getattr(self.options, "prefill_per_tick", 4),
                           getattr(self.options, "prefill_interval", 1))
        emit = book.relay(self.streaming)
        try:
            while True:
                withdrawn = book.withdraw_cancelled()
                fresh = await book.next_admissions(withdrawn)
                if fresh is None:
                    continue
                try:
                    results = await self.owner.call(self.model.tick, fresh, emit, withdrawn)
                except Exception as error:     # the engine is unusable: fail everything in flight
                    LOGGER.exception("Continuous model failed")
                    self.failure = error
                    book.fail(error)
                    return
                book.finish(results)
        except asyncio.CancelledError:
            book.abandon()
            raise

    # ------------------------------------------------------------------ HTTP
    async def health(self, incoming):
        from aiohttp import web
        state = "failed" if self.failure else "ready" if self.model else "starting"
        body = {"status": state, "queued": self.queue.qsize(), "backend": "b200",
                "audio_delivery": "codec-windows" if self.streaming else "complete-waveform"}
        stats = getattr(self.model, "stats", None)
        if hasattr(stats, "as_dict"):
            body["engine"] = stats.as_dict()
        return web.json_response(body, status=503 if self.failure else 200)

    async def _events(self, future, channel):
        """The SSE events of one request: streamed chunks while the request runs, then the
        tail of the final waveform the stream has not carried, then the done record."""
        sent = 0
        while self.streaming and not future.done():
            chunk = asyncio.ensure_future(channel.queue.get())
            try:
                await asyncio.wait((future, chunk), return_when=asyncio.FIRST_COMPLETED)
            finally:
                if not chunk.done():
                    chunk.cancel()
                    await asyncio.gather(chunk, return_exceptions=True)
            if chunk.done() and not chunk.cancelled():
                size, encoded, rate = chunk.result()
                channel.taken()
                sent += size
                yield delta(b"", rate, encoded)
        output = await future
        if sent > len(output["pcm"]):
            raise RuntimeError("Streaming output exceeded final waveform length")
        yield delta(output["pcm"][sent:], output["sample_rate"])
        yield {"type": "speech.audio.done", "finish_reason": output["finish_reason"],
               "codec_frames": output["codec_frames"]}

    async def speech(self, incoming):
        from aiohttp import web
        if self.failure is not None:
            return web.json_response({"error": "Model worker failed"}, status=503)
        try:
            request = normalize(await incoming.json(), self.model.speakers, self.model.languages)
        except (ValueError, TypeError) as error:
            return web.json_response({"error": str(error)}, status=400)
        loop = asyncio.get_running_loop()
        future, channel = loop.create_future(), AudioChannel(loop)
        try:
            self.queue.put_nowait((request, future, channel))
        except asyncio.QueueFull:
            return web.json_response({"error": "Request queue full"}, status=503)
        response = web.StreamResponse(headers={"Content-Type": "text/event-stream"})
        try:
            await response.prepare(incoming)
            async for event in self._events(future, channel):
                await response.write(sse(event))
        except asyncio.CancelledError:
            future.cancel()
            raise
        except ConnectionResetError:
            future.cancel()
        except Exception as error:
            await response.write(sse({"type": "speech.audio.error", "error": {"message": str(error)}}))
        finally:
            channel.close()
            if not future.done():
                future.cancel()
        return response


# Reference flags that choose between its NPU kernel variants or graph modes (server.py:265-309 of
# the reference). Every one of these paths is the single CUDA path here, so they are accepted, checked
# for the same combinations the reference rejects, passed to the engine as ignored flags, and do not
# change the computation.
VARIANT_FLAGS = ("talker_graph", "pack_qkv", "native_gqa", "text_only_rope", "triton_kv_update",
                 "triton_talker_rope", "bucket_kv", "valid_length_kv", "graph_embeddings", "fixed_predictor_rope",
                 "batch_audio_transfer", "reference_single", "graph_sampling", "triton_cdf", "direct_prompt",
                 "native_rope", "fused_residual", "cache_codec_constants", "codec_code_buffer", "triton_snake",
                 "cache_codec_codebooks", "pack_mlp", "fused_swiglu", "packed_kv_load", "single_request_views",
                 "batch_prefill", "graph_prefill", "native_kv_update")


def build_parser() -> argparse.ArgumentParser:
    """The reference's command line (server.py:258-311) plus ``--gpus`` and ``--seed``."""
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--model", type=Path, default=Path("random-init"),
                        help="checkpoint directory, or random-init for seeded weights")
    parser.add_argument("--device", default="cuda:0")
    parser.add_argument("--gpus", type=int, default=1, help="engine processes, one per GPU")
    parser.add_argument("--seed", type=int, default=0, help="random-init weight seed")
    parser.add_argument("--host", default="127.0.0.1")
    parser.add_argument("--port", type=int, default=8097)
    parser.add_argument("--max-batch-size", type=int, default=1, help="slots per engine (power of two)")
    parser.add_argument("--queue-size", type=int, default=128)
    parser.add_argument("--batch-wait-ms", type=float, default=0)
    parser.add_argument("--predictor-graph", nargs="?", const="step", choices=["step", "whole"])
    parser.add_argument("--streaming", action="store_true")
    parser.add_argument("--prewarm-codec", action="store_true")
    parser.add_argument("--prewarm-prefill", action="store_true")
    parser.add_argument("--codec-chunk-frames", type=int, choices=[8, 16], default=8)
    parser.add_argument("--bucket-prefill", action="store_true")
    parser.add_argument("--decode-bucket-step", type=int, default=0)
    parser.add_argument("--native-rope-scope", choices=["all", "talker", "predictor"], default="all")
    parser.add_argument("--rms-norm", choices=["native", "reference-rounding"])
    parser.add_argument("--codec-left-context", type=int, default=72)
    parser.add_argument("--codec-batch-size", type=int, choices=[1, 2, 4, 8], default=1)
    parser.add_argument("--continuous", action="store_true",
                        help="continuous admission through tick(); without it, micro-batches through generate()")
    parser.add_argument("--incremental-codec", action="store_true")
    parser.add_argument("--codec-streams", type=int, choices=[1, 2], default=1)
    parser.add_argument("--prefill-per-tick", type=int, default=4)
    parser.add_argument("--prefill-interval", type=int, default=1)
    parser.add_argument("--pipeline-audio", action="store_true",
                        help="decode each tick's audio on the codec lanes while the next tick runs")
    for flag in VARIANT_FLAGS:
        parser.add_argument("--" + flag.replace("_", "-"), action="store_true")
    return parser


def _rules(o) -> list:
    """(rejected, message) for the flag combinations the reference rejects (server.py:313-373)."""
    cont, incremental = o.continuous, o.incremental_codec
    needs_incremental = [(o.cache_codec_codebooks, "--cache-codec-codebooks"), (o.triton_snake, "--triton-snake"),
                         (o.codec_code_buffer, "--codec-code-buffer"),
                         (o.cache_codec_constants, "--cache-codec-constants"),
                         (o.codec_streams == 2, "--codec-streams 2"), (o.prewarm_codec, "--prewarm-codec")]
    needs_continuous = [(o.single_request_views, "--single-request-views"), (incremental, "--incremental-codec"),
                        (o.batch_prefill, "--batch-prefill"), (o.graph_prefill, "--graph-prefill"),
                        (o.triton_cdf, "--triton-cdf"), (o.graph_sampling, "--graph-sampling"),
                        (o.batch_audio_transfer, "--batch-audio-transfer"),
                        (bool(o.decode_bucket_step), "--decode-bucket-step"),
                        (o.fixed_predictor_rope, "--fixed-predictor-rope"), (o.graph_embeddings, "--graph-embeddings"),
                        (o.bucket_kv, "--bucket-kv"), (o.native_kv_update, "--native-kv-update")]
    return ([(not 1 <= o.prefill_interval <= 64 or (o.prefill_interval != 1 and not cont),
              "--prefill-interval must be 1..64 and requires --continuous when not 1"),
             (o.native_rope_scope != "all" and not o.native_rope, "--native-rope-scope requires --native-rope")]
            + [(used and not (cont and incremental), f"{name} requires --continuous --incremental-codec")
               for used, name in needs_incremental]
            + [(used and not cont, f"{name} requires --continuous") for used, name in needs_continuous]
            + [(o.fused_residual and o.rms_norm != "native", "--fused-residual requires --rms-norm native"),
               (o.packed_kv_load and not (cont and o.graph_prefill and not o.reference_single),
                "--packed-kv-load requires --continuous --graph-prefill without --reference-single"),
               (o.prewarm_prefill and (not o.graph_prefill or o.reference_single),
                "--prewarm-prefill requires --graph-prefill and excludes --reference-single"),
               (o.codec_chunk_frames != 8 and (not cont or not incremental or o.codec_code_buffer),
                "--codec-chunk-frames 16 requires continuous incremental codec without --codec-code-buffer"),
               (o.triton_talker_rope and not (cont and o.text_only_rope),
                "--triton-talker-rope requires --continuous --text-only-rope"),
               (o.triton_kv_update and not (cont and o.native_kv_update),
                "--triton-kv-update requires --continuous --native-kv-update"),
               (o.direct_prompt and (not cont or o.reference_single),
                "--direct-prompt requires continuous mode without reference-single"),
               (o.bucket_prefill and not o.graph_prefill, "--bucket-prefill requires --graph-prefill"),
               (o.valid_length_kv and (not cont or not o.native_gqa or o.reference_single),
                "--valid-length-kv requires continuous native GQA without reference-single"),
               (min(o.max_batch_size, o.queue_size) <= 0 or o.batch_wait_ms < 0 or o.codec_left_context < 0,
                "Invalid batch or queue settings"),
               (o.prefill_per_tick < 1 or (cont and o.max_batch_size & (o.max_batch_size - 1)),
                "Continuous slots must be a power of two and prefill budget must be positive"),
               (o.gpus < 1, "--gpus must be positive"),
               (o.gpus > 1 and not cont, "--gpus above 1 requires --continuous"),
               (o.pipeline_audio and not (cont and incremental),
                "--pipeline-audio requires --continuous --incremental-codec")])


def parse_options(argv=None):
    """Parse and cross-check the command line; errors exit through ``parser.error`` as the reference's do."""
    parser = build_parser()
    options = parser.parse_args(argv)
    for rejected, message in _rules(options):
        if rejected:
            parser.error(message)
    if options.decode_bucket_step:
        from .batching import decode_batch_size
        try:
            decode_batch_size(1, options.max_batch_size, options.decode_bucket_step)
        except ValueError as error:
            parser.error(str(error))
    return options


def engine_kwargs(options) -> dict:
    """ContinuousModel keyword arguments for the parsed command line."""
    # micro-batch mode (no --continuous) serves generate() batches of any size from a power-of-two arena
    slots = options.max_batch_size if options.continuous else 1 << (options.max_batch_size - 1).bit_length()
    kwargs = dict(max_slots=slots, codec_left_context=options.codec_left_context,
                  codec_batch_size=options.codec_batch_size, codec_chunk_frames=options.codec_chunk_frames,
                  incremental_codec=options.incremental_codec, codec_streams=options.codec_streams,
                  seed=options.seed, prewarm_codec=options.prewarm_codec, prewarm_prefill=options.prewarm_prefill,
                  bucket_prefill=options.bucket_prefill, decode_bucket_step=options.decode_bucket_step,
                  pipeline_audio=getattr(options, "pipeline_audio", False))
    kwargs.update({flag: getattr(options, flag) for flag in VARIANT_FLAGS if getattr(options, flag, False)})
    if getattr(options, "rms_norm", None):
        kwargs["rms_norm"] = options.rms_norm
    if str(options.model) != "random-init":   # a checkpoint directory (checkpoint.load_model)
        kwargs["model_path"] = str(options.model)
    return kwargs


def engine_factory(options):
    """Model factory for one GPU (``--gpus 1``) or the multi-GPU dispatcher."""
    kwargs = engine_kwargs(options)
    if options.gpus > 1:
        from .dispatcher import Dispatcher
        return lambda model, device: Dispatcher.start(options.gpus, kwargs, per_engine=options.max_batch_size)

    def build(model, device):
        from .continuous import ContinuousModel
        return ContinuousModel(device=device, **kwargs)
    return build


ROUTES = (("GET", "/health", "health"), ("POST", "/v1/audio/speech", "speech"))


def build_app(options):
    """The aiohttp application: the service's routes, model start-up and shutdown. The engine
    factory sees `max_batch_size` per engine; the service admits that many per GPU."""
    from aiohttp import web
    factory = engine_factory(argparse.Namespace(**vars(options)))
    options = argparse.Namespace(**vars(options))
    options.max_batch_size *= max(1, options.gpus)
    service = SpeechService(options, factory)
    app = web.Application(client_max_size=1024 * 1024)
    for method, path, handler in ROUTES:
        app.router.add_route(method, path, getattr(service, handler))
    app.on_startup.append(service.start)
    app.on_cleanup.append(service.stop)
    return app


def main(argv=None) -> None:
    from aiohttp import web
    options = parse_options(argv)
    logging.basicConfig(level=logging.INFO)
    app = build_app(options)
    web.run_app(app, host=options.host, port=options.port, handler_cancellation=True)


if __name__ == "__main__":
    main()
