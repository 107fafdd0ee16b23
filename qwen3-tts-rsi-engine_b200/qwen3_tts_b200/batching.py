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


# Packed prefill: the attention's split plan counts rows x KV heads (8) below 65,536, and the
# 512-row buckets keep a packed group within 7,680 rows.
MAX_PACKED_ROWS = 7680


def packed_rows(total: int) -> int:
    """Row bucket of a packed prefill of `total` prompt rows: powers of two from 64 up to 512,
    then multiples of 512 (one captured graph per bucket, at most ~25% padding above 512)."""
    if total < 1:
        raise ValueError("A packed prefill needs at least one row")
    if total <= 512:
        return max(64, 1 << (total - 1).bit_length())
    return (total + 511) // 512 * 512


def packed_groups(lengths, max_rows: int) -> list:
    """Consecutive [start, end) groups of prompts whose lengths sum to at most `max_rows` (a
    longer prompt forms a group of its own)."""
    groups, start, rows = [], 0, 0
    for i, length in enumerate(lengths):
        if i > start and rows + length > max_rows:
            groups.append((start, i))
            start, rows = i, 0
        rows += length
    if lengths:
        groups.append((start, len(lengths)))
    return groups


def packed_tables(lengths, first_slot: int, rows: int, requests: int):
    """Row tables of a packed prefill (CPU int64): the arena slot and position of every packed
    row (prompt i occupies slot first_slot + i, positions 0..lengths[i]-1; rows past the real
    ones repeat the last real row) and the row index of each prompt's last token (entries past
    the prompts repeat the last one)."""
    import torch
    n, total = len(lengths), sum(lengths)
    if not 1 <= n <= requests or total > rows:
        raise ValueError("Packed prompts exceed the prefill's rows or requests")
    counts = torch.tensor(lengths, dtype=torch.long)
    row_slots = torch.repeat_interleave(torch.arange(first_slot, first_slot + n), counts)
    row_pos = torch.cat([torch.arange(length) for length in lengths])
    last = torch.cumsum(counts, 0) - 1
    pad = rows - total
    row_slots = torch.cat([row_slots, row_slots[-1:].expand(pad)])
    row_pos = torch.cat([row_pos, row_pos[-1:].expand(pad)])
    last = torch.cat([last, last[-1:].expand(requests - n)])
    return row_slots, row_pos, last


PREFILL_UNIT_ROWS = 64


def packed_unit_capacity(rows: int, requests: int) -> int:
    """Entries of the unit table of a packed prefill of `rows` rows and up to `requests`
    prompts: every prompt adds at most one partial 64-row unit, the padding rows one more."""
    return (rows + PREFILL_UNIT_ROWS - 1) // PREFILL_UNIT_ROWS + requests + 1


def packed_units(lengths, first_slot: int, rows: int, requests: int):
    """Unit table (CPU int32 [packed_unit_capacity(rows, requests), 4]) of the causal prefill
    attention: {first_row, count, keys, slot} per block of up to 64 consecutive rows of one
    prompt, keys = 1 + the block's last position; the padding rows past the prompts (copies
    of the last prompt's last row, packed_tables) form units of their own over that row's
    keys, so they compute exactly what it does. Units are ordered by decreasing key count
    (the longest causal spans start first); unused entries are zero."""
    import torch
    units, row = [], 0
    for i, length in enumerate(lengths):
        for start in range(0, length, PREFILL_UNIT_ROWS):
            count = min(PREFILL_UNIT_ROWS, length - start)
            units.append((row + start, count, start + count, first_slot + i))
        row += length
    total = row
    for start in range(total, rows, PREFILL_UNIT_ROWS):
        units.append((start, min(PREFILL_UNIT_ROWS, rows - start), lengths[-1], first_slot + len(lengths) - 1))
    capacity = packed_unit_capacity(rows, requests)
    if len(units) > capacity:
        raise ValueError("Packed prompts exceed the prefill's unit table")
    units.sort(key=lambda u: -u[2])
    table = torch.zeros(capacity, 4, dtype=torch.int32)
    if units:
        table[:len(units)] = torch.tensor(units, dtype=torch.int32)
    return table
