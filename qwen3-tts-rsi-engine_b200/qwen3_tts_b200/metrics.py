"""Service metrics over per-request records (the reference's benchmark.summarize, benchmark.py:17-34).

A record holds ``success``, ``audio_seconds`` (delivered audio), ``elapsed_seconds``
(submission to completion) and ``ttfa_seconds`` (submission to the first nonempty
PCM chunk). Over the successful records:

* throughput = delivered audio seconds x codec frame rate / wall seconds (frames/s);
* TTFA p50 / p95 = percentiles of the first-audio times in ms, linearly
  interpolated between order statistics;
* RTF = the mean over requests of elapsed / audio seconds.

The run is ``INCONCLUSIVE`` (quality and server lifecycle are not evaluated
here) when every request succeeded and ``FAIL`` otherwise; a non-positive wall
time or frame rate raises ``ValueError``.
"""
from __future__ import annotations

import numpy as np


def summarize(records, wall_seconds: float, frame_rate: float) -> dict:
    if wall_seconds <= 0 or frame_rate <= 0:
        raise ValueError("Wall duration and frame rate must be positive")
    records = list(records)
    ok = [r for r in records if r["success"]]
    ttfa_ms = np.array([r["ttfa_seconds"] * 1000.0 for r in ok], dtype=np.float64)
    every = len(ok) == len(records)
    return {
        "requests": len(records),
        "successful_requests": len(ok),
        "failed_requests": len(records) - len(ok),
        "wall_seconds": wall_seconds,
        "throughput_frames_s": sum(r["audio_seconds"] for r in ok) * frame_rate / wall_seconds,
        "ttfa_p50_ms": float(np.percentile(ttfa_ms, 50)) if ok else None,
        "ttfa_p95_ms": float(np.percentile(ttfa_ms, 95)) if ok else None,
        "rtf_mean": float(np.mean([r["elapsed_seconds"] / r["audio_seconds"] for r in ok])) if ok else None,
        "request_completion_pass": bool(records) and every,
        "quality": "NOT_EVALUATED",
        "server_lifecycle": "NOT_EVALUATED",
        "status": "INCONCLUSIVE" if every else "FAIL",
    }
