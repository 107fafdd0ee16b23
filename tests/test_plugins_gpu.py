"""Module-replacement plugins on the CUDA kernels against fp32 torch stand-ins of the qwen-tts modules.

Every plugin installed (native RMSNorm, packed attention, packed MLP, fused residual
decoder) on a 2-layer bf16 decoder with the talker head geometry (16 q / 8 kv heads x
128, hidden 256, FFN 512); the reference is the same module tree run in fp32 before
installation. Bar: normwise relative error <= 3e-2 (bf16 weights/activations through
two layers), and a decode step that reads its keys from a ragged slot arena.
"""
import copy

import pytest
import torch

from tests import qwen_tts_fakes as Q

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def rel(got, ref):
    return float((got.float() - ref.float()).norm() / ref.float().norm())


def install_all(model, text_only_rope):
    from qwen3_tts_b200.fused_decoder import install_fused_decoders
    from qwen3_tts_b200.operators import install_rms_norms
    from qwen3_tts_b200.packed_attention import install_packed_attention
    from qwen3_tts_b200.packed_mlp import install_packed_mlp
    return (install_rms_norms(model, "native") + install_packed_attention(model, text_only_rope=text_only_rope)
            + install_packed_mlp(model) + install_fused_decoders(model))


def test_rms_norm_modes_match_the_module(cuda):
    from qwen3_tts_b200.operators import CudaRMSNorm
    norm = Q.randomize(Q.Qwen3TTSRMSNorm(256), 2).to(cuda, BF16)
    x = torch.randn(7, 3, 256, generator=torch.Generator().manual_seed(3)).to(cuda, BF16)
    ref = norm(x.float())                      # fp32 normalisation, bf16 weight
    for mode in ("native", "reference-rounding"):
        got = CudaRMSNorm(norm, mode)(x)
        assert got.dtype == BF16 and got.shape == x.shape
        torch.testing.assert_close(got.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("talker", [False, True])
def test_plugged_decoder_prefill_and_decode_match_fp32(cuda, talker):
    reference = Q.randomize(Q.TinyDecoder(layers=2, talker=talker), 11).to(cuda)
    plugged = copy.deepcopy(reference).to(BF16)
    restore = install_all(plugged, text_only_rope=talker)
    g = torch.Generator().manual_seed(12)
    x = torch.randn(2, 6, 256, generator=g).to(cuda)
    pos = torch.arange(6, device=cuda).repeat(2, 1)
    with torch.no_grad():
        full = reference(x, pos)
        cache = Q.ConcatCache()
        prefill = plugged(x[:, :5].to(BF16), pos[:, :5], cache)
        step = plugged(x[:, 5:].to(BF16), pos[:, 5:], cache)
    assert rel(prefill, full[:, :5]) <= 3e-2
    assert rel(step, full[:, 5:]) <= 3e-2
    from qwen3_tts_b200.operators import restore_modules
    restore_modules(restore)
    assert type(plugged.layers[0]).__name__.startswith("Qwen3TTS")


def test_decode_over_a_ragged_slot_arena(cuda):
    reference = Q.randomize(Q.TinyDecoder(layers=2), 21).to(cuda)
    plugged = copy.deepcopy(reference).to(BF16)
    install_all(plugged, text_only_rope=False)
    g = torch.Generator().manual_seed(22)
    positions = torch.tensor([4, 9, 2], device=cuda)
    keys = [(0.5 * torch.randn(3, 8, 16, 128, generator=g)).to(cuda) for _ in range(2)]
    values = [torch.randn(3, 8, 16, 128, generator=g).to(cuda) for _ in range(2)]
    x = torch.randn(3, 1, 256, generator=g).to(cuda)
    with torch.no_grad():
        ref = reference(x, positions[:, None], Q.SlotCache([k.clone() for k in keys], [v.clone() for v in values],
                                                           positions))
        arena = Q.SlotCache([k.to(BF16) for k in keys], [v.to(BF16) for v in values], positions)
        got = plugged(x.to(BF16), positions[:, None], arena)
    for row in range(3):
        assert rel(got[row], ref[row]) <= 3e-2, row
    # the new keys landed at each row's own position
    assert arena.arena_keys[0][1, :, 9].abs().sum() > 0
