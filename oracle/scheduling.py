"""Host-side scheduling rules of the reference (pure Python, exact).

TEST INFRASTRUCTURE ONLY (see the package docstring).
"""
from __future__ import annotations


def decode_batch_size(active: int, max_slots: int, step: int = 0) -> int:
    """Graph batch bucket for `active` requests (batching.py:4-11).

    Power-of-two bucket up to `step`; above it, the next multiple of `step`.
    """
    if not 1 <= active <= max_slots or max_slots & (max_slots - 1):
        raise ValueError("Active count must fit a positive power-of-two slot arena")
    if step < 0 or (step and (step & (step - 1) or step > max_slots)):
        raise ValueError("Decode bucket step must be zero or a power of two within the arena")
    if step == 0 or active <= step:
        bucket = 1
        while bucket < active:
            bucket <<= 1
        return bucket
    return -(-active // step) * step


def emission_target(emitted: int, chunk: int = 8) -> int:
    """Frame count at which the next audio chunk is due (continuous.py:636)."""
    if emitted == 0:
        return 2
    if emitted < 8:
        return emitted * 2
    return emitted + chunk


def context_bucket(required: int, capacity: int) -> int:
    """Talker attention context bucket with bucket_kv (continuous.py:605-606)."""
    bucket = 1
    while bucket < required:
        bucket <<= 1
    return min(capacity, max(64, bucket))


def codec_window(emitted: int, frames: int, context: int, incremental: bool):
    """(start, length, skip_samples) of the next codec call (continuous.py:481-484)."""
    start = emitted if incremental else max(0, emitted - context)
    return start, frames - start, (emitted - start) * 1920
