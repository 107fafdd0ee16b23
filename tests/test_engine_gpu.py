"""End-to-end engine (ContinuousModel.tick) against the teacher-forced CPU oracle.

Reduced widths (talker/predictor hidden 256, 2 layers each, text vocab 1024,
codec hidden 128) with the real head geometry, vocabularies (3072 / 2048),
16 codebooks, 1920 samples per frame and the real emission schedule. Greedy
sampling (top-k 1) for both samplers so every draw has one answer:

* every draw of the engine is the oracle's best-scoring token (gap 0) or a near
  tie within 5e-2 of it (bf16 rounding may flip those), and >= 90 % are exact;
* the audio of every request, concatenated from its emitted chunks, is within
  SNR >= 40 dB of the oracle codec on the same codes;
* chunk boundaries follow the schedule 2, 4, 8, then every 8 frames; results
  carry the concatenated PCM, the frame count and the finish reason;
* admission mid-flight and cancellation (slot compaction) keep every other
  request's state intact (their draws keep matching the oracle).
"""
import math
from collections import defaultdict
from dataclasses import replace

import numpy as np
import pytest
import torch

from oracle import codec as OC
from oracle import engine as OE
from oracle import prompt as OP
from oracle.sampling import random_table

pytestmark = pytest.mark.gpu


def snr_db(ref, got):
    ref, got = np.asarray(ref, dtype=np.float64), np.asarray(got, dtype=np.float64)
    return 10 * math.log10(float((ref ** 2).sum()) / max(float(((got - ref) ** 2).sum()), 1e-30))


def configs():
    from qwen3_tts_b200.config import CodecConfig, tiny_predictor, tiny_prompt, tiny_talker
    codec = CodecConfig(codebooks=16, codebook_size=2048, codebook_dim=64, semantic_codebooks=1, latent=128,
                        hidden=128, layers=2, heads=2, head_dim=64, ffn=256, window=72, upsampling_ratios=(2, 2),
                        upsample_rates=(8, 5, 4, 3), decoder_dim=256, layer_scale=0.1)
    return tiny_talker(2), tiny_predictor(2), tiny_prompt(256), codec


PAYLOADS = {
    "a": dict(input_ids=list(range(40, 45)), voice="voice_a", language="english", instructions="",
              max_new_tokens=12, seed=101),
    "b": dict(input_ids=list(range(300, 317)), voice="voice_b", language="auto", instructions="",
              max_new_tokens=19, seed=202),
    "c": dict(input="hello from the slot arena", voice="voice_a", language="chinese", instructions="",
              max_new_tokens=27, seed=303),
    "d": dict(input_ids=[7, 8, 9], voice="voice_b", language="korean", instructions="",
              max_new_tokens=10, seed=404),
    "e": dict(input_ids=list(range(500, 530)), voice="voice_a", language="english", instructions="",
              max_new_tokens=30, seed=505),
}


@pytest.mark.parametrize("packed", [True, False])
def test_engine_ticks_match_teacher_forced_oracle(cuda, packed):
    from qwen3_tts_b200 import prompt as P
    from qwen3_tts_b200.continuous import ContinuousModel
    from qwen3_tts_b200.weights import decoder_weights
    tcfg, pcfg, prcfg, ccfg = configs()
    tw = decoder_weights(tcfg, 11, "cpu")
    pw = decoder_weights(pcfg, 12, "cpu")
    prw = P.prompt_weights(prcfg, 13, "cpu")
    decoder = OC.randomize(OC.CodecDecoder(ccfg), seed=14)
    engine = ContinuousModel(None, cuda, max_slots=4, initial_capacity=64, talker_config=tcfg,
                             predictor_config=pcfg, codec_config=ccfg, prompt_config=prcfg,
                             weights={"talker": tw, "predictor": pw, "prompt": prw}, codec_decoder=decoder,
                             top_k=1, subtalker_top_k=1, max_frames=64, packed_prefill=packed)
    log = defaultdict(list)
    engine.on_codes = lambda ident, frame, codes, token: log[ident].append((frame, codes, token))
    chunks = defaultdict(list)
    results = {}
    schedule = {0: ["a", "b", "c"], 4: ["d"], 9: ["e"]}
    cancel = {7: ["b"]}
    for tick in range(64):
        submissions = [(name, PAYLOADS[name]) for name in schedule.get(tick, [])]
        out = engine.tick(submissions, emit=lambda ident, pcm, rate: chunks[ident].append((pcm, rate)),
                          cancelled=cancel.get(tick, ()))
        results.update(dict(out))
        if not engine.states and tick > 9:
            break
    engine.close()

    assert set(results) == {"a", "c", "d", "e"}            # "b" was cancelled
    for name, result in results.items():
        payload = PAYLOADS[name]
        assert result["finish_reason"] in ("length", "stop")
        if result["finish_reason"] == "length":
            assert result["codec_frames"] == payload["max_new_tokens"] - 1
        assert result["sample_rate"] == 24000
        pcm = b"".join(c for c, _ in chunks[name])
        assert result["pcm"] == pcm
        assert len(pcm) == result["codec_frames"] * 1920 * 2
        # chunk schedule: due at 2, 4, 8, 16, 24, ... frames (or the final frame)
        ends = np.cumsum([len(c) // (1920 * 2) for c, _ in chunks[name]]).tolist()
        expected, emitted = [], 0
        while emitted < result["codec_frames"]:
            emitted = min(2 if emitted == 0 else emitted * 2 if emitted < 8 else emitted + 8, result["codec_frames"])
            expected.append(emitted)
        assert ends == expected, (name, ends, expected)

    # teacher-forced oracle over every request's frames (including the cancelled one)
    table_codec = tw["embedding"].float()
    gaps, labels = [], []
    for name, frames in log.items():
        payload = PAYLOADS[name]
        ids = P.text_ids(prcfg, payload)
        tags = P.codec_tags(prcfg, payload["voice"], payload["language"])
        built = OP.build(prcfg, prw, table_codec, ids, tags)
        oracle = OE.RequestOracle(tcfg, pcfg, tw, pw, built["inputs_embeds"], built["tts_pad_embed"],
                                  random_table(payload["seed"], payload["max_new_tokens"]), capacity=256)
        assert [f for f, _, _ in frames] == list(range(len(frames)))
        oracle.first(frames[0][1][0])
        for frame, codes, token in frames:
            oracle.frame(codes, token)
        gaps.extend(oracle.gaps)
        labels.extend((name,) + label for label in oracle.labels)
        if name in results:
            codes = torch.tensor([c for _, c, _ in frames]).T[None]          # [1, 16, frames]
            ref = OC.IncrementalOracle(decoder).decode(codes, OC.IncrementalOracle(decoder).new_state())
            ref = (np.clip(ref[0, 0].numpy(), -1, 1) * 32767).astype(np.int16)
            got = np.frombuffer(results[name]["pcm"], dtype="<i2")
            assert got.shape == ref.shape
            assert snr_db(ref, got) >= 40.0, name
    gaps = np.array(gaps)
    worst = [(float(gaps[i]),) + labels[i] for i in np.argsort(-gaps)[:12] if gaps[i] > 0]
    assert np.all(gaps <= 5e-2), worst
    assert (gaps == 0).mean() >= 0.9, (float((gaps == 0).mean()), worst)


def test_engine_prompt_matches_oracle(cuda):
    """Direct prompt preparation (text projection GEMMs + codec prefix) against the oracle."""
    from qwen3_tts_b200 import prompt as P
    from qwen3_tts_b200.weights import decoder_weights
    tcfg, _, prcfg, _ = configs()
    tw = decoder_weights(tcfg, 21, "cpu")
    prw = P.prompt_weights(prcfg, 22, "cpu")
    builder = P.CustomVoicePrompt(prcfg, prw, tw["embedding"].to(cuda), cuda)
    for payload in PAYLOADS.values():
        for extra in ({}, {"instruction_ids": [11, 12, 13, 14]}):
            payload = dict(payload, **extra)
            got = builder.build(payload)
            ids = P.text_ids(prcfg, payload)
            tags = P.codec_tags(prcfg, payload["voice"], payload["language"])
            ref = OP.build(prcfg, prw, tw["embedding"].float(), ids, tags, instruction_ids=extra.get("instruction_ids"))
            inputs = got["inputs_embeds"][0].float().cpu()
            assert inputs.shape == ref["inputs_embeds"].shape
            torch.testing.assert_close(inputs, ref["inputs_embeds"], atol=2e-2, rtol=2e-2)
            torch.testing.assert_close(got["tts_pad_embed"][0, 0].float().cpu(), ref["tts_pad_embed"], atol=1e-2,
                                       rtol=1e-2)
    with pytest.raises(ValueError):
        builder.build(dict(PAYLOADS["a"], voice="nobody"))
    with pytest.raises(ValueError):
        builder.build(dict(PAYLOADS["a"], language="klingon"))
    # the batched builder (one projection for every request): same rows, packed end to end
    payloads = [dict(p, **extra) for p in PAYLOADS.values() for extra in ({}, {"instruction_ids": [11, 12, 13, 14]})]
    packed, prompts = builder.build_many(payloads)
    offset = 0
    for payload, prompt in zip(payloads, prompts):
        single = builder.build(payload)["inputs_embeds"][0]
        inputs = prompt["inputs_embeds"][0]
        assert inputs.shape == single.shape and prompt["max_new_tokens"] == payload["max_new_tokens"]
        assert inputs.data_ptr() == packed[offset].data_ptr()
        offset += inputs.shape[0]
        ids = P.text_ids(prcfg, payload)
        tags = P.codec_tags(prcfg, payload["voice"], payload["language"])
        ref = OP.build(prcfg, prw, tw["embedding"].float(), ids, tags, instruction_ids=payload.get("instruction_ids"))
        torch.testing.assert_close(inputs.float().cpu(), ref["inputs_embeds"], atol=2e-2, rtol=2e-2)
        torch.testing.assert_close(inputs.float(), single.float(), atol=1e-2, rtol=1e-2)
    assert offset == packed.shape[0]


def test_engine_from_checkpoint_matches_engine_from_weights(cuda, tmp_path):
    """``ContinuousModel(model_path=...)`` over a safetensors checkpoint (sharded talker/predictor/
    prompt file, config.json, codec under speech_tokenizer/) reads the geometry and weights the
    weight-dict engine is given: the same codes, tokens and PCM, bit for bit."""
    from qwen3_tts_b200 import checkpoint as C
    from qwen3_tts_b200 import prompt as P
    from qwen3_tts_b200.codec_weights import random_codec
    from qwen3_tts_b200.continuous import ContinuousModel
    from qwen3_tts_b200.weights import decoder_weights
    tcfg, pcfg, prcfg, ccfg = configs()
    tw, pw = decoder_weights(tcfg, 31, "cpu"), decoder_weights(pcfg, 32, "cpu")
    prw, codec = P.prompt_weights(prcfg, 33, "cpu"), random_codec(ccfg, 34)
    C.save_model(tmp_path, tw, pw, prw, tcfg, pcfg, prcfg, shards=2)
    C.save_codec(tmp_path / "speech_tokenizer", codec)
    common = dict(max_slots=4, initial_capacity=64, codec_config=ccfg, prompt_config=prcfg, top_k=1,
                  subtalker_top_k=1, max_frames=64)
    sources = [dict(talker_config=tcfg, predictor_config=pcfg, weights={"talker": tw, "predictor": pw, "prompt": prw},
                    codec_decoder=codec), dict(model_path=str(tmp_path))]
    runs = []
    for source in sources:
        engine = ContinuousModel(device=cuda, **common, **source)
        assert engine.talker_config == tcfg and engine.predictor_config == pcfg
        log, chunks, results = defaultdict(list), defaultdict(list), {}
        engine.on_codes = lambda ident, frame, codes, token: log[ident].append((frame, codes, token))
        for tick in range(48):
            submissions = [(name, PAYLOADS[name]) for name in (("a", "c", "d") if tick == 0 else ())]
            out = engine.tick(submissions, emit=lambda ident, pcm, rate: chunks[ident].append(pcm))
            results.update(dict(out))
            if not engine.states and tick > 0:
                break
        engine.close()
        assert set(results) == {"a", "c", "d"}
        runs.append((dict(log), dict(chunks), results))
    assert runs[0] == runs[1]
