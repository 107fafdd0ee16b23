"""Property tests of the host scheduling rules against the oracle restatement (which the
golden fixtures pin to the reference, tests/test_oracle_golden.py): decode batch buckets
(batching.py:4-11), the audio emission schedule (continuous.py:636) and the KV context
bucket (continuous.py:605-606)."""
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import scheduling as OS
from qwen3_tts_b200.batching import (MAX_PACKED_ROWS, context_bucket, decode_batch_size, emission_target,
                                    packed_groups, packed_rows, packed_tables, packed_unit_capacity,
                                    packed_units)

POW2 = st.sampled_from([1, 2, 4, 8, 16, 32, 64, 128])


@settings(max_examples=400, deadline=None)
@given(slots=POW2, data=st.data())
def test_decode_bucket_fits_and_matches_the_oracle(slots, data):
    active = data.draw(st.integers(1, slots))
    step = data.draw(st.sampled_from([0] + [s for s in (1, 2, 4, 8, 16, 32, 64, 128) if s <= slots]))
    bucket = decode_batch_size(active, slots, step)
    assert bucket == OS.decode_batch_size(active, slots, step)
    assert active <= bucket <= slots
    if step == 0 or active <= step:
        assert bucket & (bucket - 1) == 0 and bucket < 2 * active
    else:
        assert bucket % step == 0 and bucket - active < step
    # buckets never shrink as more slots become active
    if active < slots:
        assert decode_batch_size(active + 1, slots, step) >= bucket


@settings(max_examples=200, deadline=None)
@given(chunk=st.sampled_from([8, 16]), frames=st.integers(1, 2048))
def test_emission_schedule_matches_the_oracle_and_bounds_chunks(chunk, frames):
    emitted, due = 0, []
    while emitted < frames:
        target = emission_target(emitted, chunk)
        assert target == OS.emission_target(emitted, chunk)
        assert target > emitted and target - emitted <= max(chunk, 8)
        emitted = min(target, frames)
        due.append(emitted)
    assert due[0] == min(2, frames) and due[-1] == frames
    assert all(b > a for a, b in zip(due, due[1:]))


@settings(max_examples=300, deadline=None)
@given(capacity=st.sampled_from([64, 128, 512, 1024, 4096]), data=st.data())
def test_context_bucket_covers_the_keys(capacity, data):
    required = data.draw(st.integers(1, capacity))
    bucket = context_bucket(required, capacity)
    assert bucket == OS.context_bucket(required, capacity)
    assert required <= bucket <= capacity and bucket >= min(64, capacity)
    assert bucket == capacity or bucket & (bucket - 1) == 0


@settings(max_examples=300, deadline=None)
@given(lengths=st.lists(st.integers(1, 600), min_size=1, max_size=64), max_rows=st.integers(256, MAX_PACKED_ROWS))
def test_packed_prefill_groups_and_tables_cover_every_prompt_once(lengths, max_rows):
    """Packed admission: consecutive groups within the row budget (a longer prompt alone), a
    row bucket that holds the group, and row tables that give every prompt's tokens their own
    slot and positions 0..n-1 with padding rows repeating the last real row."""
    groups = packed_groups(lengths, max_rows)
    assert groups[0][0] == 0 and groups[-1][1] == len(lengths)
    assert all(a[1] == b[0] for a, b in zip(groups, groups[1:]))
    first_slot = 3
    for start, end in groups:
        part = lengths[start:end]
        total = sum(part)
        assert total <= max_rows or end - start == 1
        if end < len(lengths):
            assert total + lengths[end] > max_rows             # greedy: the next prompt did not fit
        rows = packed_rows(total)
        assert total <= rows and (rows & (rows - 1) == 0 if rows <= 512 else rows % 512 == 0)
        assert rows <= max(64, 2 * total - 1) if total <= 512 else rows - total < 512
        slots, pos, last = packed_tables(part, first_slot, rows, 64)
        assert slots.shape == pos.shape == (rows,) and last.shape == (64,)
        offset = 0
        for i, n in enumerate(part):
            assert slots[offset:offset + n].tolist() == [first_slot + i] * n
            assert pos[offset:offset + n].tolist() == list(range(n))
            assert last[i] == offset + n - 1
            offset += n
        assert (slots[total:] == slots[total - 1]).all() and (pos[total:] == pos[total - 1]).all()
        assert (last[end - start:] == total - 1).all()


@settings(max_examples=300, deadline=None)
@given(lengths=st.lists(st.integers(1, 600), min_size=1, max_size=64))
def test_packed_prefill_units_cover_every_row_once(lengths):
    """Unit table of the causal prefill attention: every packed row (padding included) in
    exactly one unit of at most 64 consecutive rows of one slot, keys = 1 + the unit's last
    position, longest spans first, within the fixed table size."""
    rows = packed_rows(sum(lengths))
    first_slot = 2
    slots, pos, _ = packed_tables(lengths, first_slot, rows, 64)
    units = packed_units(lengths, first_slot, rows, 64)
    assert units.shape == (packed_unit_capacity(rows, 64), 4)
    used = units[units[:, 1] > 0]
    assert (units[len(used):] == 0).all()
    covered = []
    for first, count, keys, slot in used.tolist():
        assert 1 <= count <= 64
        span = range(first, first + count)
        assert all(int(slots[r]) == slot for r in span)
        assert keys == max(int(pos[r]) for r in span) + 1
        covered.extend(span)
    assert sorted(covered) == list(range(rows))
    assert used[:, 2].tolist() == sorted(used[:, 2].tolist(), reverse=True)
