"""Phase tracing for the continuous engine (the reference's tools/profile_continuous.py:23-39).

``instrument(model, mode)`` wraps the engine's phase methods on the instance
(prompt admission, the tick graph, audio emission, the codec call, the audio
copy to the host) and returns a ``Trace``; ``Trace.remove()`` puts the
original methods back.

* ``mode="nvtx"``: every call runs inside an NVTX range (and a torch profiler
  ``record_function``) named ``q3t/<phase>``, for ``ncu --nvtx`` filters or a
  timeline tool; nothing is timed here.
* ``mode="timed"``: the device is synchronised before and after each call and
  the host time is recorded per phase and tick (``Trace.records``,
  ``Trace.summary()``). The synchronisation serialises the phases, so these
  figures explain where a tick's time goes; they are never a throughput number.
"""
from __future__ import annotations

import functools
import time
from contextlib import ExitStack

import torch

PHASES = (("admit_batch", "admit"), ("_run_tick", "tick_graph"), ("emit_audio", "emit_audio"),
          ("_decode_group", "codec"), ("_to_host", "audio_to_host"))


class Trace:
    def __init__(self, model, mode: str):
        if mode not in ("nvtx", "timed"):
            raise ValueError("Trace mode must be 'nvtx' or 'timed'")
        self.model, self.mode = model, mode
        self.records: list[dict] = []
        self.tick = 0
        self._wrapped: list[tuple] = []      # (name, the instance attribute it replaced or None)

    def _sync(self) -> None:
        device = getattr(self.model, "device", None)
        if device is not None and torch.device(device).type == "cuda":
            torch.cuda.synchronize(device)

    def wrap(self, name: str, label: str) -> None:
        original = getattr(self.model, name)
        self._wrapped.append((name, vars(self.model).get(name)))

        @functools.wraps(original)
        def traced(*args, **kwargs):
            if self.mode == "timed":
                self._sync()
                start = time.perf_counter()
                result = original(*args, **kwargs)
                self._sync()
                self.records.append({"phase": label, "tick": self.tick, "seconds": time.perf_counter() - start})
                return result
            with ExitStack() as stack:
                stack.enter_context(torch.profiler.record_function("q3t/" + label))
                torch.cuda.nvtx.range_push("q3t/" + label)
                stack.callback(torch.cuda.nvtx.range_pop)
                return original(*args, **kwargs)

        setattr(self.model, name, traced)

    def summary(self) -> dict:
        """Per phase: calls, total seconds and mean milliseconds per call."""
        out: dict[str, dict] = {}
        for record in self.records:
            entry = out.setdefault(record["phase"], {"calls": 0, "seconds": 0.0})
            entry["calls"] += 1
            entry["seconds"] += record["seconds"]
        for entry in out.values():
            entry["mean_ms"] = entry["seconds"] / entry["calls"] * 1e3
        return out

    def remove(self) -> None:
        for name, previous in reversed(self._wrapped):
            if previous is not None:
                setattr(self.model, name, previous)
            elif name in vars(self.model):
                delattr(self.model, name)          # the class method shows through again
        self._wrapped.clear()


def instrument(model, mode: str = "nvtx") -> Trace:
    """Wrap the phases of `model` (an engine instance); the tick counter advances per ``tick``."""
    trace = Trace(model, mode)
    for name, label in PHASES:
        if hasattr(model, name):
            trace.wrap(name, label)
    original_tick = model.tick
    trace._wrapped.append(("tick", vars(model).get("tick")))

    @functools.wraps(original_tick)
    def tick(*args, **kwargs):
        try:
            return original_tick(*args, **kwargs)
        finally:
            trace.tick += 1

    model.tick = tick
    return trace
