"""Module-replacement plugins (host side, no GPU): the reference's install functions
(packed_attention.py:88-95, packed_mlp.py:30-37, operators.py:26-38,
fused_decoder.py:40-47) match children by class name, return (parent, name, original)
in visiting order, and ``restore_modules`` puts every original back; constructors
raise the reference's ``ValueError``s.
"""
import pytest
import torch

from qwen3_tts_b200.fused_decoder import FusedResidualDecoder, install_fused_decoders
from qwen3_tts_b200.operators import CudaRMSNorm, install_rms_norms, restore_modules
from qwen3_tts_b200.packed_attention import PackedAttention, install_packed_attention
from qwen3_tts_b200.packed_mlp import PackedMLP, install_packed_mlp
from tests import qwen_tts_fakes as Q


def model(talker=True):
    return Q.randomize(Q.TinyDecoder(layers=2, talker=talker), 1).to(torch.bfloat16)


def test_install_and_restore_every_plugin():
    m = model()
    originals = {name: mod for name, mod in m.named_modules()}
    norms = install_rms_norms(m, "native")
    attention = install_packed_attention(m, text_only_rope=True)
    mlps = install_packed_mlp(m)
    layers = install_fused_decoders(m)
    # 2 layers x (input, post, q, k) + the final norm; 2 attentions; 2 MLPs; 2 layers
    assert (len(norms), len(attention), len(mlps), len(layers)) == (9, 2, 2, 2)
    assert all(type(original).__name__ == "Qwen3TTSRMSNorm" for _, _, original in norms)
    assert all(isinstance(m.layers[i], FusedResidualDecoder) for i in range(2))
    assert isinstance(m.layers[0].reference.self_attn, PackedAttention)
    assert isinstance(m.layers[1].reference.mlp, PackedMLP)
    assert isinstance(m.norm, CudaRMSNorm) and m.norm.mode == "native"
    assert [type(o).__name__ for _, _, o in attention] == ["Qwen3TTSTalkerAttention"] * 2
    for replacements in (layers, mlps, attention, norms):
        restore_modules(replacements)
    assert {name: mod for name, mod in m.named_modules()} == originals


def test_restore_runs_in_reverse_order():
    m = model()
    first = install_rms_norms(m)
    second = install_rms_norms(m)            # wraps the wrappers
    assert isinstance(m.norm, CudaRMSNorm) and isinstance(m.norm.reference, CudaRMSNorm)
    restore_modules(first + second)
    assert isinstance(m.norm, Q.Qwen3TTSRMSNorm)


def test_matching_is_by_class_name_only():
    class Qwen3TTSRMSNormLike(Q.Qwen3TTSRMSNorm):
        pass
    m = torch.nn.Sequential(Qwen3TTSRMSNormLike(8), Q.Qwen3TTSRMSNorm(8))
    replaced = install_rms_norms(m)
    assert [name for _, name, _ in replaced] == ["1"]


def test_constructor_contracts():
    with pytest.raises(ValueError):
        install_rms_norms(model(), mode="fast")
    with pytest.raises(ValueError):     # talker attention needs identical position axes
        install_packed_attention(model(talker=True))
    with pytest.raises(ValueError):
        install_packed_attention(model(talker=False), native_rope_scope="decoder")
    assert len(install_packed_attention(model(talker=False))) == 2
    gelu = Q.Qwen3TTSTalkerTextMLP(64, 128, act="gelu")
    with pytest.raises(ValueError, match="SiLU"):
        PackedMLP(gelu.to(torch.bfloat16))
    biased = Q.Qwen3TTSTalkerTextMLP(64, 128, bias=True)
    with pytest.raises(ValueError, match="bias-free"):
        PackedMLP(biased.to(torch.bfloat16))
    with pytest.raises(ValueError, match="native RMSNorm"):
        install_fused_decoders(model())
    m = model()
    install_rms_norms(m, "reference-rounding")
    with pytest.raises(ValueError, match="native RMSNorm"):
        install_fused_decoders(m)


def test_packed_weights_follow_the_reference_layout():
    attention = Q.randomize(Q.Qwen3TTSAttention(64, 4, 2, 16, bias=True), 3).to(torch.bfloat16)
    packed = PackedAttention(attention)
    assert packed.sizes == [64, 32, 32]
    assert torch.equal(packed.weight, torch.cat([attention.q_proj.weight, attention.k_proj.weight,
                                                 attention.v_proj.weight]))
    assert torch.equal(packed.bias, torch.cat([attention.q_proj.bias, attention.k_proj.bias, attention.v_proj.bias]))
    mlp = Q.randomize(Q.Qwen3TTSTalkerTextMLP(64, 128), 4).to(torch.bfloat16)
    tiles = PackedMLP(mlp).weight.view(2, 2, 64, 64)        # [group, gate|up, 64 rows, hidden]
    assert torch.equal(tiles[:, 0].reshape(128, 64), mlp.gate_proj.weight)
    assert torch.equal(tiles[:, 1].reshape(128, 64), mlp.up_proj.weight)


def test_fake_reference_cache_paths_agree():
    """The fp32 stand-ins the GPU tests compare against: prefill + decode through the concatenating
    cache equals one pass over the whole sequence."""
    m = Q.randomize(Q.TinyDecoder(layers=2, talker=False), 5)
    x = torch.randn(2, 6, 256, generator=torch.Generator().manual_seed(6))
    pos = torch.arange(6).repeat(2, 1)
    full = m(x, pos)
    cache = Q.ConcatCache()
    m(x[:, :5], pos[:, :5], cache)
    step = m(x[:, 5:], pos[:, 5:], cache)
    torch.testing.assert_close(step, full[:, 5:], atol=1e-4, rtol=1e-4)
