"""Incremental codec on the GPU against the CPU oracle (fp32) on identical codes.

Bar: PCM within SNR >= 40 dB of the reference codec on
identical codes; here the reference codec is the pinned oracle (the
reference's own slot logic over the stand-in modules, tests/test_codec_oracle.py).
"""
import math

import numpy as np
import pytest
import torch

from oracle import codec as OC
from tests.golden.inputs import uniform

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def snr_db(ref, got):
    ref, got = ref.double(), got.double()
    ref, got = ref.detach(), got.detach()
    return 10 * math.log10(float((ref ** 2).sum()) / max(float(((got - ref) ** 2).sum()), 1e-30))


def small_cfg():
    from qwen3_tts_b200.config import CodecConfig
    # real upsampling and window, reduced widths: 16 codebooks, window 72, hidden 128, 2 layers
    return CodecConfig(codebooks=16, codebook_size=256, codebook_dim=64, semantic_codebooks=1, latent=128,
                       hidden=128, layers=2, heads=2, head_dim=64, ffn=256, window=72,
                       upsampling_ratios=(2, 2), upsample_rates=(8, 5, 4, 3), decoder_dim=256, layer_scale=0.1)


def build(cfg, cuda, slots, seed=7):
    from qwen3_tts_b200.codec import CodecSlots, pack_codec
    decoder = OC.randomize(OC.CodecDecoder(cfg), seed=seed)
    engine = CodecSlots(cfg, pack_codec(decoder, cuda), slots, cuda, max_chunk_frames=8, use_graphs=True)
    return decoder, engine


def test_codec_streams_match_oracle(cuda):
    from qwen3_tts_b200 import ops
    cfg = small_cfg()
    assert cfg.head_dim * cfg.heads == cfg.hidden
    decoder, engine = build(cfg, cuda, slots=6)
    oracle = OC.IncrementalOracle(decoder)
    n_frames = 20
    codes = {s: torch.from_numpy((uniform(200 + s, (1, cfg.codebooks, n_frames)) * cfg.codebook_size)
                                 .astype(np.int64)) for s in range(3)}
    slot_of = {0: 4, 1: 1, 2: 5}
    schedule = [[2, 1, 4], [2, 3, 4], [4, 4, 4], [8, 4, 8], [4, 8]]  # chunk per stream per tick
    done = {s: 0 for s in codes}
    gpu_pcm = {s: [] for s in codes}
    for tick in schedule:
        groups = {}
        for s, n in enumerate(tick):
            if done[s] + n <= n_frames:
                groups.setdefault(n, []).append(s)
        for n, streams in groups.items():
            idx = [slot_of[s] for s in streams]
            chunk = torch.cat([codes[s][:, :, done[s]:done[s] + n] for s in streams]).to(cuda)
            wave, pcm = engine.decode(idx, chunk)
            for i, s in enumerate(streams):
                gpu_pcm[s].append(wave[i].cpu())
                done[s] += n
    torch.cuda.synchronize()
    assert ops.read_status(cuda) == 0
    for s in codes:
        got = torch.cat(gpu_pcm[s])
        ref = decoder(codes[s][:, :, :done[s]])[0, 0]
        assert got.shape == ref.shape
        assert torch.isfinite(got).all()
        snr = snr_db(ref, got)
        assert snr >= 40.0, f"stream {s}: SNR {snr:.1f} dB"
    engine.close()


def test_codec_move_reset_and_pcm16(cuda):
    cfg = small_cfg()
    decoder, engine = build(cfg, cuda, slots=4, seed=9)
    codes = torch.from_numpy((uniform(300, (1, cfg.codebooks, 12)) * cfg.codebook_size).astype(np.int64))
    w1, _ = engine.decode([2], codes[:, :, :4].to(cuda))
    engine.move(2, 0)                      # compaction keeps the stream's state
    w2, pcm = engine.decode([0], codes[:, :, 4:12].to(cuda))
    ref = decoder(codes)[0, 0]
    got = torch.cat([w1[0].cpu(), w2[0].cpu()])
    assert snr_db(ref, got) >= 40.0
    # on-device PCM16 equals the reference's host conversion of the same waveform
    wave = w2[0].cpu().numpy()
    expect = (np.clip(wave, -1, 1) * 32767).astype("<i2")
    assert np.array_equal(pcm[0].cpu().numpy(), expect)
    engine.reset(0)                        # a reset slot decodes like a fresh stream
    w3, _ = engine.decode([0], codes[:, :, :4].to(cuda))
    assert torch.allclose(w3[0].cpu(), w1[0].cpu(), atol=1e-6)
    with pytest.raises(ValueError):
        engine.decode([0, 0], torch.cat([codes[:, :, :2]] * 2).to(cuda))
    with pytest.raises(ValueError):
        engine.decode([0], codes[:, :, :9].to(cuda))
    engine.close()


def test_codec_two_lanes_match_one_lane(cuda):
    """codec_streams=2 (codec_slots.py:279-305): the groups of one decode_groups call run on two
    alternating streams with per-lane graphs; the audio and the per-slot state equal the
    one-stream decode bit for bit, and a reset after the call is ordered after the lanes."""
    from qwen3_tts_b200.codec import CodecSlots, pack_codec
    cfg = small_cfg()
    decoder = OC.randomize(OC.CodecDecoder(cfg), seed=11)
    packed = pack_codec(decoder, cuda)
    one = CodecSlots(cfg, packed, 6, cuda, max_chunk_frames=8, streams=1)
    two = CodecSlots(cfg, packed, 6, cuda, max_chunk_frames=8, streams=2)
    gen = torch.Generator().manual_seed(5)
    for chunk in range(3):
        groups = [([0, 3], 4), ([5], 2), ([1, 2], 4), ([4], 8)]
        calls = [(idx, torch.randint(0, cfg.codebook_size, (len(idx), cfg.codebooks, n), generator=gen).to(cuda))
                 for idx, n in groups]
        out1 = one.decode_groups(calls)
        out2 = two.decode_groups(calls)
        for (w1, p1), (w2, p2) in zip(out1, out2):
            assert torch.equal(w1, w2) and torch.equal(p1, p2)
    two.reset(5)
    one.reset(5)
    for a, b in zip(one.state.buffers, two.state.buffers):
        assert torch.equal(a, b)
    one.close()
    two.close()
