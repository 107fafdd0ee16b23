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
    kwargs = engine_kwargs(options)
    assert kwargs["max_slots"] == 1 and kwargs["codec_batch_size"] == 1 and not kwargs["incremental_codec"]
    assert not any(flag in kwargs for flag in VARIANT_FLAGS)
    assert engine_kwargs(parse_options(["--model", "/models/cv"]))["model_path"] == "/models/cv"


@pytest.mark.parametrize("argv", [
    "--prefill-interval 0", "--prefill-interval 65", "--native-rope-scope talker",
    "--codec-streams 2", "--triton-snake", "--codec-code-buffer", "--cache-codec-constants",
    "--cache-codec-codebooks", "--prewarm-codec", "--fused-residual", "--fused-residual --rms-norm reference-rounding",
    "--packed-kv-load", "--packed-kv-load --graph-prefill --reference-single", "--prewarm-prefill",
    "--codec-chunk-frames 16", "--codec-chunk-frames 16 --incremental-codec --codec-code-buffer",
    "--triton-talker-rope", "--triton-kv-update", "--direct-prompt --reference-single", "--bucket-prefill",
    "--valid-length-kv", "--valid-length-kv --native-gqa --reference-single", "--max-batch-size 0",
    "--queue-size 0", "--batch-wait-ms -1", "--codec-left-context -1", "--prefill-per-tick 0",
    "--max-batch-size 48", "--max-batch-size 64 --decode-bucket-step 7", "--codec-batch-size 3",
    "--gpus 0"])
def test_rejected_combinations_exit(argv, capsys):
    with pytest.raises(SystemExit) as info:
        parse_options(argv.split())
    assert info.value.code == 2


@pytest.mark.parametrize("argv", [
    "--codec-streams 2 --incremental-codec", "--codec-chunk-frames 16 --incremental-codec",
    "--fused-residual --rms-norm native", "--prewarm-prefill --graph-prefill", "--bucket-prefill --graph-prefill",
    "--valid-length-kv --native-gqa", "--max-batch-size 64 --decode-bucket-step 8",
    "--triton-talker-rope --text-only-rope", "--triton-kv-update --native-kv-update"])
def test_accepted_combinations(argv):
    parse_options(argv.split())
