"""pipeline_audio: the codec chunks a tick makes due are decoded on the codec lanes while the
next tick's graph runs, and delivered by that next tick. Against the engine without it, on the
same requests, weights and schedule (admission mid-flight, a cancellation, ragged lengths):
every result and every emitted chunk is bit-identical; results arrive one tick later.
"""
from collections import defaultdict

import pytest
import torch

from oracle import codec as OC
from tests.test_engine_gpu import PAYLOADS, configs

pytestmark = pytest.mark.gpu


def run(cuda, pipeline, streams):
    from qwen3_tts_b200 import prompt as P
    from qwen3_tts_b200.continuous import ContinuousModel
    from qwen3_tts_b200.weights import decoder_weights
    tcfg, pcfg, prcfg, ccfg = configs()
    engine = ContinuousModel(None, cuda, max_slots=4, initial_capacity=64, talker_config=tcfg, predictor_config=pcfg,
                             codec_config=ccfg, prompt_config=prcfg,
                             weights={"talker": decoder_weights(tcfg, 11, "cpu"),
                                      "predictor": decoder_weights(pcfg, 12, "cpu"),
                                      "prompt": P.prompt_weights(prcfg, 13, "cpu")},
                             codec_decoder=OC.randomize(OC.CodecDecoder(ccfg), seed=14), top_k=1, subtalker_top_k=1,
                             max_frames=64, codec_batch_size=2, codec_streams=streams, pipeline_audio=pipeline)
    schedule = {0: ["a", "b", "c"], 4: ["d"], 9: ["e"]}
    cancel = {7: ["b"]}
    chunks, results, finished_at = defaultdict(list), {}, {}
    for tick in range(80):
        out = engine.tick([(n, PAYLOADS[n]) for n in schedule.get(tick, [])],
                          emit=lambda ident, pcm, rate: chunks[ident].append(pcm), cancelled=cancel.get(tick, ()))
        for ident, result in out:
            results[ident] = result
            finished_at[ident] = tick
        if tick > 9 and not engine.states and engine._inflight is None:
            break
    engine.close()
    return results, chunks, finished_at


def test_pipelined_audio_matches_the_synchronous_engine(cuda):
    base, base_chunks, base_at = run(cuda, False, 1)
    piped, piped_chunks, piped_at = run(cuda, True, 2)
    assert set(base) == set(piped) == {"a", "c", "d", "e"}
    for ident in base:
        assert piped[ident] == base[ident], ident
        assert piped_chunks[ident] == base_chunks[ident], ident
        assert b"".join(piped_chunks[ident]) == piped[ident]["pcm"]
        assert piped_at[ident] == base_at[ident] + 1
    # one lane of its own when the codec has a single stream
    single, single_chunks, _ = run(cuda, True, 1)
    assert single == base
    assert all(single_chunks[ident] == base_chunks[ident] for ident in base)
