"""Property tests of the host scheduling rules against the oracle restatement (which the
golden fixtures pin to the reference, tests/test_oracle_golden.py): decode batch buckets
(batching.py:4-11), the audio emission schedule (continuous.py:636) and the KV context
bucket (continuous.py:605-606)."""
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import scheduling as OS
from qwen3_tts_b200.batching import context_bucket, decode_batch_size, emission_target

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
