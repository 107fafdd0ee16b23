"""Service metrics: the reference's known answers (tests/test_benchmark.py:11-21 of the reference:
throughput 15 frames/s, RTF .75, TTFA p50 200 ms / p95 290 ms) and its failure contract."""
import pytest

from qwen3_tts_b200.metrics import summarize

ROWS = [{"success": True, "audio_seconds": 2, "elapsed_seconds": 1, "ttfa_seconds": .1},
        {"success": True, "audio_seconds": 4, "elapsed_seconds": 4, "ttfa_seconds": .3}]


def test_known_answers():
    result = summarize(ROWS, 5, 12.5)
    assert result["throughput_frames_s"] == 15
    assert result["rtf_mean"] == .75
    assert result["ttfa_p50_ms"] == pytest.approx(200)
    assert result["ttfa_p95_ms"] == pytest.approx(290)
    assert result["status"] == "INCONCLUSIVE" and result["request_completion_pass"]
    assert (result["requests"], result["successful_requests"], result["failed_requests"]) == (2, 2, 0)


def test_failed_requests_are_excluded_and_fail_the_run():
    rows = ROWS + [{"success": False, "audio_seconds": 0, "elapsed_seconds": 9, "ttfa_seconds": None}]
    result = summarize(rows, 5, 12.5)
    assert result["throughput_frames_s"] == 15 and result["rtf_mean"] == .75
    assert result["status"] == "FAIL" and not result["request_completion_pass"]
    assert result["failed_requests"] == 1
    none = summarize([rows[-1]], 5, 12.5)
    assert none["ttfa_p50_ms"] is None and none["rtf_mean"] is None and none["throughput_frames_s"] == 0


@pytest.mark.parametrize("wall,rate", [(0, 12.5), (-1, 12.5), (5, 0)])
def test_non_positive_wall_or_rate_raises(wall, rate):
    with pytest.raises(ValueError):
        summarize(ROWS, wall, rate)
