"""Decode graph batch bucket (batching.py:4-11 of the reference engine)."""
from __future__ import annotations


def decode_batch_size(active: int, max_slots: int, step: int = 0) -> int:
    """Power-of-two bucket up to `step`, then the next multiple of `step`.

    Raises ValueError unless 1 <= active <= max_slots, max_slots is a power of
    two, and step is 0 or a power of two no larger than max_slots.
    """
    if not 1 <= active <= max_slots or max_slots & (max_slots - 1):
        raise ValueError("Active count must fit a positive power-of-two slot arena")
    if step < 0 or (step and (step & (step - 1) or step > max_slots)):
        raise ValueError("Decode bucket step must be zero or a power of two within the arena")
    if not step or active <= step:
        return 1 << (active - 1).bit_length()
    return ((active + step - 1) // step) * step


def context_bucket(required: int, capacity: int) -> int:
    """Talker attention context with KV bucketing: next power of two >= required,
    at least 64, at most the arena capacity (continuous.py:605-606)."""
    return min(capacity, max(64, 1 << (required - 1).bit_length()))


def emission_target(emitted: int, chunk_frames: int = 8) -> int:
    """Frame count at which a request's next audio chunk is due (continuous.py:636):
    2 frames first, then doubling to 8, then every `chunk_frames`."""
    if emitted == 0:
        return 2
    return emitted * 2 if emitted < 8 else emitted + chunk_frames
