"""Argument checks that run on the host before any launch (packed_kv.py:6-31 of the reference;
its tests/test_packed_kv.py:45-81): every invalid slot, row, length, shape, dtype, device or
aliasing source raises ``ValueError`` from the argument checks themselves (matched by message,
so the later "Expected CUDA tensors" check cannot satisfy the test) and leaves the target as it was.
"""
import pytest
import torch

from qwen3_tts_b200 import kernels

ROWS = "valid packed KV row and prefix length"
PAIR = "independent compatible packed KV tensors"


def tensors():
    target = torch.arange(4 * 5 * 2 * 7 * 3, dtype=torch.float32).view(4, 5, 2, 7, 3)
    source = torch.arange(4 * 3 * 2 * 5 * 6, dtype=torch.float32).view(4, 3, 2, 5, 6)[..., ::2]
    return target, source


@pytest.mark.parametrize("slot,row,length", [(-1, 0, 1), (5, 0, 1), (0, 3, 1), (0, -1, 1), (0, 0, 0), (0, 0, 6),
                                             (True, 0, 1), (0, True, 1), (0, 0, True), (0, 0, 1.0)])
def test_invalid_bounds_cannot_write(slot, row, length):
    target, source = tensors()
    saved = target.clone()
    with pytest.raises(ValueError, match=ROWS):
        kernels.copy_packed_prefix(target, source, slot, row=row, length=length)
    assert torch.equal(target, saved)


@pytest.mark.parametrize("case", ["batch", "heads", "width", "dtype", "rank", "empty", "alias", "meta"])
def test_incompatible_or_aliasing_source_is_rejected(case):
    target, source = tensors()
    bad = {"batch": lambda: source[:3], "heads": lambda: source[:, :, :1], "width": lambda: source[..., :2],
           "dtype": lambda: source.double(), "rank": lambda: source[0], "empty": lambda: source[:, :0],
           "alias": lambda: target[:, :2], "meta": lambda: torch.empty_like(source, device="meta")}[case]()
    saved = target.clone()
    with pytest.raises(ValueError, match=PAIR):
        kernels.copy_packed_prefix(target, bad, 0, length=1)
    assert torch.equal(target, saved)


def test_valid_arguments_pass_the_checks_and_then_require_cuda():
    target, source = tensors()
    with pytest.raises(ValueError, match="Expected CUDA tensors"):
        kernels.copy_packed_prefix(target, source, 2, row=1, length=4)
