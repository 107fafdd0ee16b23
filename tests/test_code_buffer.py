"""Per-slot code ring (CodecCodeBuffer, codec_code_buffer.py:5-31 of the reference; its
tests/test_codec_code_buffer.py:7-32).

The expected history is kept in plain Python lists: frame f of a slot is the
codes written for it at f, and a read of ``length`` frames from ``start``
returns them as [codebooks, length] for each requested slot.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from qwen3_tts_b200.code_buffer import CodecCodeBuffer

FIXTURE = np.load(Path(__file__).resolve().parent / "golden" / "decode_path.npz")["code_buffer_reads"]


class ListRing:
    """CPU restatement of the ring (codec_code_buffer.py:5-31): frame f of slot s is row s * 8 + f % 8."""

    def __init__(self, slots, codebooks):
        self.rows = [[0] * codebooks for _ in range(slots * 8)]

    def write(self, codes, frames):
        for i, (row, frame) in enumerate(zip(codes.tolist(), frames.tolist())):
            self.rows[i * 8 + frame % 8] = row

    def read(self, slots, starts, length):
        return torch.tensor([[self.rows[s * 8 + (start + k) % 8] for k in range(length)]
                             for s, start in zip(slots, starts)]).transpose(1, 2)

    def move(self, source, destination):
        self.rows[destination * 8:destination * 8 + 8] = [list(r) for r in self.rows[source * 8:source * 8 + 8]]


def reference_sequence(buffer, to_device):
    """The write/read/move sequence tests/golden/make_golden.py ran on the reference's buffer."""
    reads = []
    for tick in range(19):
        buffer.write(to_device(torch.arange(48).view(3, 16) + tick * 100), to_device(torch.tensor([tick, tick + 3,
                                                                                                      tick + 7])))
        if tick >= 7:
            reads.append(buffer.read([2, 0], [tick, tick - 7], 8).cpu().numpy())
    buffer.move(2, 0)
    reads.append(buffer.read([0], [18], 8).cpu().numpy())
    return np.stack([r if r.shape[0] == 2 else np.concatenate([r, r]) for r in reads])


def test_ring_restatement_matches_the_reference_fixture():
    assert np.array_equal(reference_sequence(ListRing(4, 16), lambda t: t), FIXTURE)


@pytest.mark.gpu
def test_cuda_ring_matches_the_reference_fixture(cuda):
    assert np.array_equal(reference_sequence(CodecCodeBuffer(4, 16, cuda), lambda t: t.to(cuda)), FIXTURE)


@pytest.mark.parametrize("slots,starts,length", [([], [], 2), ([0], [0], 9), ([4], [0], 2), ([0], [-1], 2),
                                                  ([0, 1], [0], 2), ([0], [0], 0)])
def test_invalid_intervals_are_rejected_before_any_launch(slots, starts, length):
    with pytest.raises(ValueError):
        CodecCodeBuffer(4, 16, "cpu").read(slots, starts, length)


@pytest.mark.parametrize("codes,frames", [
    (torch.zeros(5, 16, dtype=torch.long), torch.zeros(5, dtype=torch.long)),      # more rows than slots
    (torch.zeros(2, 15, dtype=torch.long), torch.zeros(2, dtype=torch.long)),      # wrong codebook count
    (torch.zeros(2, 16, dtype=torch.long), torch.zeros(3, dtype=torch.long)),      # ragged frame indices
    (torch.zeros(2, 16, dtype=torch.int32), torch.zeros(2, dtype=torch.long)),     # dtype
])
def test_invalid_writes_are_rejected(codes, frames):
    with pytest.raises(ValueError):
        CodecCodeBuffer(4, 16, "cpu").write(codes, frames)


@pytest.mark.gpu
@pytest.mark.parametrize("depth", [8, 16])
def test_history_survives_wrap_ragged_progress_and_compaction(cuda, depth):
    buf = CodecCodeBuffer(4, 16, cuda, depth=depth)
    offsets = [0, 3, 7]                          # staggered admissions: slots at different frames
    history = [[] for _ in offsets]
    for tick in range(2 * depth + 3):
        codes = torch.arange(48).view(3, 16) + tick * 100
        buf.write(codes.to(cuda), torch.tensor([tick + o for o in offsets], device=cuda))
        for i in range(3):
            history[i].append(codes[i])
        if tick >= depth - 1:
            got = buf.read([2, 0], [tick + offsets[2] - (depth - 1), tick - (depth - 1)], depth).cpu()
            want = torch.stack([torch.stack(history[i][-depth:]).T for i in (2, 0)])
            assert torch.equal(got, want)
            short = buf.read([1], [tick + offsets[1] - 2], 3).cpu()
            assert torch.equal(short[0], torch.stack(history[1][-3:]).T)
    last = 2 * depth + 2
    buf.move(2, 0)
    got = buf.read([0], [last + offsets[2] - (depth - 1)], depth).cpu()
    assert torch.equal(got[0], torch.stack(history[2][-depth:]).T)
    # a reused slot starts again at frame 0: its fresh frames read back without stale rows
    for step in range(2):
        buf.write(torch.full((1, 16), 900 + step, device=cuda), torch.tensor([step], device=cuda))
    want = torch.stack([torch.full((16,), 900), torch.full((16,), 901)], -1)
    assert torch.equal(buf.read([0], [0], 2).cpu()[0], want)
    # device-resident indices give the same rows as the host-list read
    idx, starts = torch.tensor([1, 0], device=cuda), torch.tensor([last + offsets[1] - 1, 0], device=cuda)
    assert torch.equal(buf.read_device(idx, starts, 2).cpu(), buf.read([1, 0], [last + offsets[1] - 1, 0], 2).cpu())
