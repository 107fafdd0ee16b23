"""The codec oracle reproduces the reference's slot-indexed incremental codec.

Fixtures come from the reference's CodecSlots / CodecSlotGraph.compute run on
the oracle's stand-in decoder modules (tests/golden/make_golden.py): two
interleaved streams with ragged chunks, a slot move and a reset.
"""
from pathlib import Path

import numpy as np
import torch

from oracle.codec import CodecDecoder, IncrementalOracle, randomize
from tests.golden.inputs import uniform

GOLDEN = Path(__file__).resolve().parent / "golden"
TINY_CODEC = dict(codebooks=4, codebook_size=32, codebook_dim=8, semantic_codebooks=1, latent=12, hidden=8,
                  layers=2, heads=2, head_dim=4, ffn=16, window=6, eps=1e-5, theta=10000.0,
                  upsampling_ratios=(2,), upsample_rates=(2, 3), decoder_dim=8, layer_scale=0.1)
SCHEDULE = {0: [2, 2, 4, 8, 4], 1: [1, 3, 8, 8]}


def tiny_decoder():
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "qwen3-tts-rsi-engine_b200"))
    from qwen3_tts_b200.config import CodecConfig
    cfg = CodecConfig(**TINY_CODEC)
    return cfg, randomize(CodecDecoder(cfg), seed=5)


def test_incremental_oracle_matches_reference_slot_codec():
    fx = np.load(GOLDEN / "codec.npz")
    cfg, decoder = tiny_decoder()
    oracle = IncrementalOracle(decoder)
    codes = {s: torch.from_numpy((uniform(60 + s, (1, cfg.codebooks, 20)) * cfg.codebook_size).astype(np.int64))
             for s in SCHEDULE}
    states = {s: oracle.new_state() for s in SCHEDULE}
    done = {s: 0 for s in SCHEDULE}
    pcm = {s: [] for s in SCHEDULE}
    for step in range(5):
        for stream, sched in SCHEDULE.items():
            if step < len(sched):
                n = sched[step]
                pcm[stream].append(oracle.decode(codes[stream][:, :, done[stream]:done[stream] + n], states[stream]))
                done[stream] += n
    for s in SCHEDULE:
        got = torch.cat(pcm[s], -1)
        torch.testing.assert_close(got, torch.from_numpy(fx[f"codec_pcm_{s}"]), atol=1e-6, rtol=1e-5)
        # chunked streaming equals the full-sequence decoder
        torch.testing.assert_close(got, torch.from_numpy(fx[f"codec_full_{s}"]), atol=1e-6, rtol=1e-5)
    fresh = oracle.decode(codes[1][:, :, :4], oracle.new_state())
    torch.testing.assert_close(fresh, torch.from_numpy(fx["codec_fresh_after_reset"]), atol=1e-6, rtol=1e-5)
