"""Slot-table KV arena and decode attention restated on the CPU.

TEST INFRASTRUCTURE ONLY (see the package docstring).
"""
from __future__ import annotations

import torch


def kv_write(keys, values, target_keys, target_values, positions) -> None:
    """target[b, h, positions[b], :] = source[b, h, 0, :] for K and V
    (kv_triton_ascend.py:25-36 `_write_row`; continuous.py:164-166 scatter)."""
    batch, heads, _, width = keys.shape
    for b in range(batch):
        p = int(positions[b])
        target_keys[b, :, p] = keys[b, :, 0]
        target_values[b, :, p] = values[b, :, 0]


def copy_packed_prefix(target, source, slot, row=0, length=None) -> None:
    """target[:, slot, :, :length] = source[:, row, :, :length] (packed_kv.py:31)."""
    length = source.shape[3] if length is None else length
    target[:, slot, :, :length] = source[:, row, :, :length]


def slot_move(buffers, source, destination) -> None:
    """Copy slot `source` over slot `destination` in every buffer (continuous.py:124-128)."""
    if source != destination:
        for buffer in buffers:
            buffer[destination] = buffer[source]


def grow(buffer, new_capacity: int, dim: int = 2):
    """Double-capacity copy of an arena buffer (continuous.py:359-363)."""
    shape = list(buffer.shape)
    shape[dim] = new_capacity
    out = torch.zeros(shape, dtype=buffer.dtype)
    index = [slice(None)] * buffer.ndim
    index[dim] = slice(0, buffer.shape[dim])
    out[tuple(index)] = buffer
    return out


def decode_attention(query, keys, values, positions, scale=None, rows_per_slot=1, window=0):
    """Query rows over their slot's keys, GQA.

    query [R, Hq, D], keys/values [slots, Hkv, cap, D] -> [R, Hq, D] (fp32).
    Row r reads slot r // rows_per_slot and sees keys lo..p, p = positions[r],
    lo = max(0, p - window + 1) with a sliding window (0 = none): the mask
    `indices <= positions` of SlotGraph.compute (continuous.py:191-192), the
    predictor's 2x2 causal first step (continuous.py:37-40) and the codec
    window `key > position - window` (codec_slots.py:73-77). Attention as
    torch SDPA with enable_gqa (scaled dot product, softmax, V).
    """
    batch, q_heads, dim = query.shape
    kv_heads = keys.shape[1]
    group = q_heads // kv_heads
    scale = dim ** -0.5 if scale is None else scale
    out = torch.empty(batch, q_heads, dim, dtype=torch.float32)
    for b in range(batch):
        p = int(positions[b])
        lo = max(0, p - window + 1) if window > 0 else 0
        slot = b // rows_per_slot
        k = keys[slot, :, lo:p + 1].float().repeat_interleave(group, dim=0)      # [Hq, n, D]
        v = values[slot, :, lo:p + 1].float().repeat_interleave(group, dim=0)
        s = torch.einsum("hd,hnd->hn", query[b].float(), k) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hn,hnd->hd", p, v)
    return out


def slot_cache_step(arena_keys, arena_values, new_keys, new_values, query, positions):
    """scatter one token per slot at `positions`, then attend
    over each slot's valid prefix (SlotCache.update continuous.py:152-169 +
    SDPA with the `indices <= positions` mask)."""
    kv_write(new_keys, new_values, arena_keys, arena_values, positions)
    return decode_attention(query, arena_keys, arena_values, positions)
