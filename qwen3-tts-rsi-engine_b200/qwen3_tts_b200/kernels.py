"""Reference-named kernel wrappers (the *_triton_ascend.py / packed_kv.py /
codec_row_scatter.py / cdf_triton_ascend.py entry points) over libq3t_b200.so.

Each keeps the reference signature, raises ValueError on invalid shapes,
dtypes, devices or aliasing before any launch, and enqueues on the current
CUDA stream without host synchronisation; data-dependent validity (positions,
indices) is the caller's contract as in the reference.
"""
from __future__ import annotations

from . import ops


def write(keys, values, target_keys, target_values, positions, row_tiled=False):
    """Paired single-token K/V scatter (kv_triton_ascend.py:39-64)."""
    del row_tiled  # one coalesced kernel serves both reference variants
    ops.kv_write(keys, values, target_keys, target_values, positions)


def rotary(hidden, cos, sin):
    """bf16-rounded rotate-half RoPE on BSND (rotary_triton_ascend.py:29-44)."""
    return ops.rotary(hidden, cos, sin)


def snake(hidden, alpha, inverse_beta, tiled=False):
    """SnakeBeta x + inv_beta * sin(alpha x)^2 on NCT rows (snake_triton_ascend.py:28-70)."""
    del tiled
    return ops.snake(hidden, alpha, inverse_beta)


def select(cdf, uniforms):
    """#{cdf / cdf[-1] <= u} per row (cdf_triton_ascend.py:20-36)."""
    return ops.cdf_select(cdf, uniforms)


def scatter_rows(target, indices, source):
    """target[indices[i]] = source[i] (codec_row_scatter.py:48-93)."""
    ops.scatter_rows(target, indices, source)


def copy_packed_prefix(target, source, slot, row=0, length=None):
    """target[:, slot, :, :length] = source[:, row, :, :length] (packed_kv.py:6-31)."""
    ops.copy_packed_prefix(target, source, slot, row=row, length=length)
