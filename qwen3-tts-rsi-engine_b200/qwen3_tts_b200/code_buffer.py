"""Per-slot ring of recent frame codes (CodecCodeBuffer, codec_code_buffer.py:5-31).

Frame f of slot s lives in row ``s * depth + f % depth`` of a
[slots, depth, codebooks] int64 device tensor. ``write`` and ``read`` are
single kernels from ``libq3t_b200.so``; ``move`` is the slot-compaction copy.
The reference fixes the depth at 8 frames; here it is a constructor argument
(default 8) so 16-frame codec chunks can use the same buffer.
"""
from __future__ import annotations

import torch

from . import ops


class CodecCodeBuffer:
    def __init__(self, slots: int, codebooks: int, device, depth: int = 8):
        if slots < 1 or codebooks < 1 or depth < 1:
            raise ValueError("Code buffer sizes must be positive")
        self.slots, self.codebooks, self.depth = slots, codebooks, depth
        self.data = torch.zeros(slots, depth, codebooks, dtype=torch.long, device=device)

    def write(self, codes: torch.Tensor, frame_indices: torch.Tensor) -> None:
        """Row i of `codes` [count, codebooks] goes to slot i at frame frame_indices[i]."""
        count = codes.shape[0]
        if (codes.ndim != 2 or codes.shape != (count, self.codebooks) or frame_indices.shape != (count,)
                or count > self.slots or count < 1 or codes.dtype != torch.long
                or frame_indices.dtype != torch.long or codes.device != self.data.device
                or frame_indices.device != self.data.device or codes.stride(1) != 1):
            raise ValueError("Code rows and frame indices must fit the slot arena")
        ops.code_ring_write(self.data, codes, frame_indices.contiguous())

    def read(self, slots, starts, length: int) -> torch.Tensor:
        """[len(slots), codebooks, length] codes of frames starts[i] .. starts[i] + length - 1."""
        slots, starts = list(slots), list(starts)
        if (not slots or len(slots) != len(starts) or not 1 <= length <= self.depth
                or min(slots) < 0 or max(slots) >= self.slots or min(starts) < 0):
            raise ValueError(f"Expected valid slots and a retained 1..{self.depth}-frame interval")
        table = torch.tensor([slots, starts], dtype=torch.long).to(self.data.device, non_blocking=True)
        return ops.code_ring_read(self.data, table[0], table[1], length)

    def read_device(self, indices: torch.Tensor, starts: torch.Tensor, length: int, out=None) -> torch.Tensor:
        """``read`` with device-resident slot and start vectors (no host upload)."""
        return ops.code_ring_read(self.data, indices, starts, length, out=out)

    def move(self, source: int, destination: int) -> None:
        if source != destination:
            ops.slot_move(self.data, source, destination)
