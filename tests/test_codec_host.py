"""Host-side contract of the slot codec (codec_slots.py:241-331 of the reference; its
tests/test_codec_streams.py:27-128): invalid or conflicting work is rejected before
any graph is captured or any group is submitted, group order and callbacks are kept,
and slot ranges are checked before any buffer is touched. No GPU: the codec object
is built without its device state and graph creation is replaced by a mock.
"""
from types import SimpleNamespace
from unittest.mock import Mock

import pytest
import torch

from qwen3_tts_b200.codec import CodecSlots, CodecState


def make_codec(streams=2):
    codec = object.__new__(CodecSlots)
    codec.slots, codec.max_chunk_frames, codec.stream_count = 8, 8, streams
    codec.cfg = SimpleNamespace(codebooks=16)
    codec.device = torch.device("cpu")
    codec._graph = Mock(side_effect=AssertionError("invalid work must not reach graph capture"))
    return codec


def codes(batch=2, length=2, dtype=torch.long):
    return torch.zeros(batch, 16, length, dtype=dtype)


@pytest.mark.parametrize("streams", [1, 2])
def test_cross_group_overlap_is_rejected_before_capture(streams):
    codec, callback = make_codec(streams), Mock()
    with pytest.raises(ValueError):
        codec.decode_groups([([0, 1], codes()), ([2, 0], codes())], on_output=callback)
    codec._graph.assert_not_called()
    callback.assert_not_called()


@pytest.mark.parametrize("streams", [1, 2])
@pytest.mark.parametrize("indices", [[], [1, 1], [-1, 2], [2, 8]])
def test_an_invalid_later_group_submits_nothing(streams, indices):
    codec = make_codec(streams)
    with pytest.raises(ValueError):
        codec.decode_groups([([0, 3], codes()), (indices, codes(max(1, len(indices))))])
    codec._graph.assert_not_called()


@pytest.mark.parametrize("bad", [codes(1), codes(length=9), codes(dtype=torch.float32),
                                 torch.zeros(2, 15, 2, dtype=torch.long), torch.zeros(2, 16, dtype=torch.long),
                                 codes(length=0)])
def test_invalid_code_shape_or_type_is_rejected_before_capture(bad):
    codec = make_codec()
    with pytest.raises(ValueError):
        codec.decode_groups([([0, 1], bad)])
    codec._graph.assert_not_called()


@pytest.mark.parametrize("streams", [1, 2])
def test_empty_work_needs_no_stream_or_capture(streams):
    codec = make_codec(streams)
    assert codec.decode_groups([]) == []
    codec._graph.assert_not_called()


def test_serial_groups_keep_order_and_hand_over_each_output():
    codec = make_codec(1)
    outputs = [(torch.tensor([17]), torch.tensor([1])), (torch.tensor([23]), torch.tensor([2]))]
    graph = Mock()
    graph.run.side_effect = outputs
    codec._graph = Mock(return_value=graph)
    callback = Mock()
    got = codec.decode_groups([([0, 1], codes()), ([4, 5], codes(length=3))], on_output=callback)
    assert got[0] is outputs[0] and got[1] is outputs[1]
    assert [c.args[0] for c in callback.call_args_list] == [0, 1]
    assert callback.call_args_list[0].args[1] is outputs[0]
    assert [c.args[:2] for c in codec._graph.call_args_list] == [(2, 2), (2, 3)]
    # the slot list reaches the graph as an index tensor in call order
    assert graph.run.call_args_list[1].args[0].tolist() == [4, 5]


def test_a_single_group_propagates_a_callback_failure():
    codec = make_codec(2)
    graph = Mock()
    graph.run.return_value = (torch.tensor([17]), torch.tensor([1]))
    codec._graph = Mock(return_value=graph)
    callback = Mock(side_effect=RuntimeError("consumer stopped"))
    with pytest.raises(RuntimeError, match="consumer stopped"):
        codec.decode_groups([([1, 6], codes())], callback)
    codec._graph.assert_called_once()


@pytest.mark.parametrize("start,count", [(-1, 2), (7, 2), (0, -1), (9, 0), (True, 1), (0, False), (1.0, 1)])
def test_invalid_slot_ranges_touch_nothing(start, count):
    state = object.__new__(CodecState)
    state.slots = 8
    state.frames = Mock(side_effect=AssertionError("no buffer may be touched"))
    with pytest.raises(ValueError):
        state.reset_range(start, count)


def test_an_empty_range_at_the_end_is_a_no_op():
    state = object.__new__(CodecState)
    state.slots = 8
    state.reset_range(8, 0)
    state.reset_range(0, 0)
