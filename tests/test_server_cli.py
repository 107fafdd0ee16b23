"""Server command line: the reference's flags parse (server.py:258-311 of the reference), the
combinations it rejects are rejected the same way (server.py:313-373), and the parsed options
reach the engine constructor. No GPU and no model: only parsing and the keyword mapping."""
import pytest

from qwen3_tts_b200.server import VARIANT_FLAGS, engine_kwargs, parse_options

# the flag set of the reference's measured continuous configuration (its frozen serving argv)
MEASURED = ("--port 8099 --continuous --streaming --pack-qkv --max-batch-size 64 --codec-left-context 72 "
            "--codec-batch-size 4 --incremental-codec --pack-mlp --native-kv-update --batch-prefill "
            "--prefill-per-tick 64 --text-only-rope --prewarm-codec --native-gqa --graph-embeddings --graph-prefill "
            "--rms-norm native --fused-swiglu --native-rope --graph-sampling --native-rope-scope predictor "
            "--triton-snake --cache-codec-codebooks --triton-kv-update --triton-talker-rope --prewarm-prefill "
            "--bucket-prefill --direct-prompt").split()


def test_measured_reference_argv_parses_and_reaches_the_engine():
    options = parse_options(MEASURED)
    assert options.continuous and options.streaming and options.prefill_per_tick == 64
    kwargs = engine_kwargs(options)
    assert kwargs["max_slots"] == 64 and kwargs["codec_batch_size"] == 4 and kwargs["codec_left_context"] == 72
    assert kwargs["incremental_codec"] and kwargs["prewarm_codec"] and kwargs["prewarm_prefill"]
    assert kwargs["bucket_prefill"] and kwargs["codec_streams"] == 1 and kwargs["rms_norm"] == "native"
    assert kwargs["pack_qkv"] and kwargs["triton_snake"] and kwargs["direct_prompt"]
    assert "model_path" not in kwargs            # random-init unless --model names a checkpoint


def test_defaults_and_checkpoint_path():
    options = parse_options([])
    assert not options.continuous                 # micro-batches through generate(), as the reference
    kwargs = engine_kwargs(options)
    assert kwargs["max_slots"] == 1 and kwargs["codec_batch_size"] == 1 and not kwargs["incremental_codec"]
    assert not any(flag in kwargs for flag in VARIANT_FLAGS)
    assert engine_kwargs(parse_options(["--model", "/models/cv"]))["model_path"] == "/models/cv"
    # a micro-batch size that is not a power of two runs on the next power-of-two arena
    assert engine_kwargs(parse_options(["--max-batch-size", "3"]))["max_slots"] == 4
    assert engine_kwargs(parse_options(["--continuous", "--max-batch-size", "16"]))["max_slots"] == 16


C = "--continuous "


@pytest.mark.parametrize("argv", [
    "--prefill-interval 0", C + "--prefill-interval 65", "--prefill-interval 4", C + "--native-rope-scope talker",
    C + "--codec-streams 2", C + "--triton-snake", C + "--codec-code-buffer", C + "--cache-codec-constants",
    C + "--cache-codec-codebooks", C + "--prewarm-codec", "--incremental-codec --prewarm-codec",
    "--fused-residual", "--fused-residual --rms-norm reference-rounding",
    C + "--packed-kv-load", C + "--packed-kv-load --graph-prefill --reference-single", C + "--prewarm-prefill",
    C + "--codec-chunk-frames 16", C + "--codec-chunk-frames 16 --incremental-codec --codec-code-buffer",
    C + "--triton-talker-rope", C + "--triton-kv-update", C + "--direct-prompt --reference-single", "--direct-prompt",
    C + "--bucket-prefill", C + "--valid-length-kv", C + "--valid-length-kv --native-gqa --reference-single",
    "--max-batch-size 0", "--queue-size 0", "--batch-wait-ms -1", "--codec-left-context -1", "--prefill-per-tick 0",
    C + "--max-batch-size 48", C + "--max-batch-size 64 --decode-bucket-step 7", "--decode-bucket-step 8",
    "--codec-batch-size 3", "--gpus 0", "--gpus 2", "--incremental-codec", "--graph-prefill", "--batch-prefill",
    "--graph-sampling", "--triton-cdf", "--native-kv-update", "--single-request-views", "--bucket-kv",
    "--graph-embeddings", "--fixed-predictor-rope", "--batch-audio-transfer"])
def test_rejected_combinations_exit(argv, capsys):
    with pytest.raises(SystemExit) as info:
        parse_options(argv.split())
    assert info.value.code == 2


@pytest.mark.parametrize("argv", [
    C + "--codec-streams 2 --incremental-codec", C + "--codec-chunk-frames 16 --incremental-codec",
    "--fused-residual --rms-norm native", C + "--prewarm-prefill --graph-prefill",
    C + "--bucket-prefill --graph-prefill", C + "--valid-length-kv --native-gqa",
    C + "--max-batch-size 64 --decode-bucket-step 8", C + "--triton-talker-rope --text-only-rope",
    C + "--triton-kv-update --native-kv-update", "--max-batch-size 3 --batch-wait-ms 5",
    C + "--gpus 2 --max-batch-size 32"])
def test_accepted_combinations(argv):
    parse_options(argv.split())
