"""The codec's sliding-window KV ring past its wrap point (codec_slots.py:160-163, 73-77 of the reference).

The codec keeps each layer's keys in a 128-row ring (position p in row p % 128)
and attends over the last 72 positions. Shorter tests stay below the wrap; these
run positions up to 300:

* the attention kernel over a ring arena equals the fp32 oracle over the same
  keys laid out linearly (rows outside the window hold a poison value);
* two interleaved codec streams of 150 frames, in chunks of 2, 2, 4, 8, ... as
  the reference's slot-codec probes schedule them, stay within SNR >= 40 dB of
  the full-sequence oracle decode.
"""

import numpy as np
import pytest
import torch

from oracle import kv as KV
from tests.golden.inputs import uniform

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def test_ring_arena_attention_matches_the_linear_oracle(cuda):
    from qwen3_tts_b200 import ops
    positions = [0, 71, 72, 127, 128, 200, 255, 256, 300]
    slots, heads, dim, ring, window = len(positions), 8, 64, 128, 72
    g = torch.Generator().manual_seed(5)
    lin_k = torch.randn(slots, heads, 301, dim, generator=g).to(BF16)
    lin_v = torch.randn(slots, heads, 301, dim, generator=g).to(BF16)
    ring_k = torch.full((slots, heads, ring, dim), 100.0).to(BF16)     # poison: never inside a window
    ring_v = torch.full((slots, heads, ring, dim), 100.0).to(BF16)
    for s, p in enumerate(positions):
        for q in range(max(0, p - ring + 1), p + 1):
            ring_k[s, :, q % ring] = lin_k[s, :, q]
            ring_v[s, :, q % ring] = lin_v[s, :, q]
    query = torch.randn(slots, heads, dim, generator=g).to(BF16)
    pos = torch.tensor(positions)
    ref = KV.decode_attention(query, lin_k, lin_v, pos, window=window)
    got = ops.decode_attention(query.to(cuda), ring_k.to(cuda), ring_v.to(cuda), pos.to(cuda), context=ring,
                               window=window, ring=ring)
    torch.testing.assert_close(got.cpu().float(), ref, atol=2e-2, rtol=0)
    assert ops.read_status(cuda) == 0


def test_long_interleaved_streams_cross_the_ring(cuda):
    from qwen3_tts_b200 import ops
    from tests.test_codec_gpu import build, small_cfg, snr_db
    cfg = small_cfg()
    decoder, engine = build(cfg, cuda, slots=3, seed=13)
    frames = 150
    codes = {s: torch.from_numpy((uniform(400 + s, (1, cfg.codebooks, frames)) * cfg.codebook_size)
                                 .astype(np.int64)) for s in (0, 1)}
    slot_of = {0: 2, 1: 0}
    chunks = {0: [2, 2, 4] + [8] * 17 + [6], 1: [4, 4] + [8] * 17 + [6]}
    assert all(sum(c) == frames for c in chunks.values())
    done, waves = {0: 0, 1: 0}, {0: [], 1: []}
    for tick in range(max(len(c) for c in chunks.values())):
        groups = {}
        for s, sched in chunks.items():
            if tick < len(sched):
                groups.setdefault(sched[tick], []).append(s)
        for n, streams in groups.items():
            batch = torch.cat([codes[s][:, :, done[s]:done[s] + n] for s in streams]).to(cuda)
            wave, _ = engine.decode([slot_of[s] for s in streams], batch)
            for i, s in enumerate(streams):
                waves[s].append(wave[i].cpu())
                done[s] += n
    torch.cuda.synchronize()
    assert ops.read_status(cuda) == 0
    for s in codes:
        with torch.no_grad():
            ref = decoder(codes[s])[0, 0]
        got = torch.cat(waves[s])
        assert got.shape == ref.shape
        assert snr_db(ref, got) >= 40.0, s
        # the tail after the wrap (frames 128..149) on its own
        tail = slice(128 * 1920, None)
        assert snr_db(ref[tail], got[tail]) >= 40.0, s
    engine.close()
