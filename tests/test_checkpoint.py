"""Safetensors checkpoint loading (host side, no GPU).

The loader reads the qwen-tts CustomVoice names (``talker.model.layers.{i}...``,
``talker.codec_head.weight`` found by suffix as tools/probe_sampling_head.py:44-46
does, ``talker.code_predictor.*``, ``talker.text_projection.*``) and the
config.json ids the reference reads (custom_voice_prompt.py:30-50, model.py:72).
No real checkpoint is available here, so the tests write checkpoints in that
layout from seeded weights and check that every tensor and config field comes
back exactly, and that malformed files fail with ``ValueError`` before any
tensor is read.
"""
import json
from dataclasses import replace

import pytest
import torch

from qwen3_tts_b200 import checkpoint as C
from qwen3_tts_b200 import prompt as P
from qwen3_tts_b200.config import tiny_predictor, tiny_prompt, tiny_talker
from qwen3_tts_b200.weights import decoder_weights

safetensors = pytest.importorskip("safetensors.torch")


def model(dialect=True):
    tcfg, pcfg = tiny_talker(2), tiny_predictor(2)
    prcfg = tiny_prompt(256)
    if dialect:
        prcfg = replace(prcfg, languages=prcfg.languages + (("beijing_dialect", 2074),),
                        dialects=(("voice_b", "beijing_dialect"),))
    return tcfg, pcfg, prcfg, decoder_weights(tcfg, 1), decoder_weights(pcfg, 2), P.prompt_weights(prcfg, 3)


def assert_same(a, b):
    if isinstance(a, dict):
        assert a.keys() == b.keys()
        for k in a:
            assert_same(a[k], b[k])
    elif isinstance(a, list):
        assert len(a) == len(b)
        for x, y in zip(a, b):
            assert_same(x, y)
    else:
        assert a.dtype == b.dtype and torch.equal(a, b)


@pytest.mark.parametrize("shards", [1, 3])
def test_model_round_trip(tmp_path, shards):
    tcfg, pcfg, prcfg, tw, pw, prw = model()
    C.save_model(tmp_path, tw, pw, prw, tcfg, pcfg, prcfg, shards=shards)
    if shards > 1:
        assert (tmp_path / "model.safetensors.index.json").exists()
        assert not (tmp_path / "model.safetensors").exists()
    loaded = C.load_model(tmp_path, prompt_base=tiny_prompt(256))
    assert loaded["talker_config"] == tcfg
    assert loaded["predictor_config"] == pcfg
    assert loaded["prompt_config"] == prcfg
    assert_same(loaded["weights"], {"talker": tw, "predictor": pw, "prompt": prw})


def test_outer_prefix_and_identity_projection(tmp_path):
    """A wrapper prefix before ``talker.`` is found through the head suffix; a predictor as wide
    as the talker without ``small_to_mtp_projection`` gets an identity projection."""
    tcfg, pcfg, prcfg, tw, pw, prw = model(dialect=False)
    tensors = C.model_state_dict(tw, pw, prw, prefix="wrapper.model.talker.")
    for key in [k for k in tensors if "small_to_mtp_projection" in k]:
        del tensors[key]
    safetensors.save_file(tensors, str(tmp_path / "model.safetensors"))
    loaded = C.load_model(tmp_path, prompt_base=prcfg)
    assert loaded["talker_config"].layers == 2 and loaded["predictor_config"].groups == 15
    assert torch.equal(loaded["weights"]["predictor"]["proj"], torch.eye(pcfg.hidden, dtype=torch.bfloat16))
    assert not loaded["weights"]["predictor"]["proj_bias"].any()
    assert_same(loaded["weights"]["talker"], tw)


def test_config_ids_from_json(tmp_path):
    """Prompt ids, language/speaker tables (a one-element spk_id list included) and the EOS id
    come from config.json; chat-template ids stay those of the base prompt config."""
    tcfg, pcfg, prcfg, tw, pw, prw = model(dialect=False)
    C.save_model(tmp_path, tw, pw, prw, tcfg, pcfg, prcfg)
    config = json.loads((tmp_path / "config.json").read_text())
    config["tts_pad_token_id"] = 1010
    tc = config["talker_config"]
    tc.update(codec_eos_token_id=2151, codec_pad_id=2140, spk_id={"Vivian": [3005], "Ryan": 3006},
              spk_is_dialect={"vivian": False, "ryan": "sichuan_dialect"},
              codec_language_id={"English": 2050, "Chinese": 2055, "sichuan_dialect": 2062})
    (tmp_path / "config.json").write_text(json.dumps(config))
    got = C.load_model(tmp_path, prompt_base=prcfg)
    pr = got["prompt_config"]
    assert got["talker_config"].eos == 2151
    assert pr.tts_pad == 1010 and pr.codec_pad == 2140 and pr.im_start == prcfg.im_start
    assert pr.speaker_ids == {"vivian": 3005, "ryan": 3006}
    assert pr.language_ids == {"english": 2050, "chinese": 2055, "sichuan_dialect": 2062}
    # the dialect speaker's Chinese/auto prompt carries the dialect's language id
    assert P.codec_tags(pr, "Ryan", "auto")[2] == 2062
    assert P.codec_tags(pr, "Vivian", "chinese")[2] == 2055


def _write(tmp_path, tensors, config=None):
    safetensors.save_file(tensors, str(tmp_path / "model.safetensors"))
    if config is not None:
        (tmp_path / "config.json").write_text(json.dumps(config))


@pytest.mark.parametrize("case", ["two_heads", "missing", "shape", "projection", "speaker_range", "no_file"])
def test_malformed_checkpoints_raise(tmp_path, case):
    tcfg, pcfg, prcfg, tw, pw, prw = model(dialect=False)
    tensors = C.model_state_dict(tw, pw, prw)
    config = C.model_config_json(tcfg, pcfg, prcfg)
    message = {"two_heads": "Expected one talker output head", "missing": "talker.model.layers.1.self_attn.k_norm",
               "shape": "talker.model.layers.1.mlp.down_proj.weight", "projection": "small_to_mtp_projection",
               "speaker_range": "outside the talker vocabulary", "no_file": "No model.safetensors"}[case]
    if case == "two_heads":
        tensors["other.talker.codec_head.weight"] = tensors["talker.codec_head.weight"].clone()
    elif case == "missing":
        del tensors["talker.model.layers.1.self_attn.k_norm.weight"]
    elif case == "shape":
        tensors["talker.model.layers.1.mlp.down_proj.weight"] = torch.zeros(tcfg.hidden, tcfg.ffn + 64,
                                                                            dtype=torch.bfloat16)
    elif case == "speaker_range":
        config["talker_config"]["spk_id"] = {"voice_a": 4000}
    if case not in ("no_file", "projection"):
        _write(tmp_path, tensors, config)
    if case == "projection":   # a talker wider than the predictor, without the projection
        t512 = replace(tcfg, hidden=512)
        tensors = C.model_state_dict(decoder_weights(t512, 4), decoder_weights(replace(pcfg, talker_hidden=512), 5),
                                     P.prompt_weights(replace(prcfg, hidden=512), 6))
        for key in [k for k in tensors if "small_to_mtp_projection" in k]:
            del tensors[key]
        _write(tmp_path, tensors)
    with pytest.raises(ValueError, match=message):
        C.load_model(tmp_path, prompt_base=prcfg)


def test_codec_round_trip_and_module_names(tmp_path):
    """The codec tree written by ``save_codec`` reads back exactly; a torch module state dict in
    the same attribute layout (RVQ layers stored as ``_layers``, under an outer prefix) loads into
    the same tree."""
    from oracle import codec as OC
    from qwen3_tts_b200.codec_weights import random_codec
    from tests.test_engine_gpu import configs
    ccfg = configs()[3]
    tree = random_codec(ccfg, 7)
    C.save_codec(tmp_path / "a", tree)
    back = C.load_codec(tmp_path / "a", ccfg)
    assert_same(C.codec_state_dict(back), C.codec_state_dict(tree))

    module = OC.randomize(OC.CodecDecoder(ccfg), seed=8)
    raw = {"decoder." + k: v.detach().contiguous() for k, v in module.state_dict().items()}
    assert any("._layers." in k for k in raw)
    (tmp_path / "b").mkdir()
    safetensors.save_file(raw, str(tmp_path / "b" / "model.safetensors"))
    loaded = C.load_codec(tmp_path / "b", ccfg)
    assert_same(C.codec_state_dict(loaded), C.codec_state_dict(module))


def test_codec_shape_mismatch_raises(tmp_path):
    from qwen3_tts_b200.codec_weights import random_codec
    from tests.test_engine_gpu import configs
    ccfg = configs()[3]
    tensors = C.codec_state_dict(random_codec(ccfg, 7))
    tensors["pre_transformer.layers.1.q_proj.weight"] = torch.zeros(3, 3)
    safetensors.save_file({k: v.contiguous() for k, v in tensors.items()}, str(tmp_path / "model.safetensors"))
    with pytest.raises(ValueError, match="pre_transformer.layers.1.q_proj.weight"):
        C.load_codec(tmp_path, ccfg)


# ------------------------------------------------------------------ names from the module tree
class _Bag(torch.nn.Module):
    def __init__(self, **children):
        super().__init__()
        for name, child in children.items():
            setattr(self, name, child)


def _model_tree(tcfg, pcfg, prcfg):
    """A stand-in for the qwen-tts CustomVoice model as the reference drives it
    (model.py:18-34 ``wrapper.model.talker``): ``talker.model.layers`` / ``.norm`` (prefill_graph.py:34-44),
    ``talker.get_input_embeddings()`` and ``talker.code_predictor.get_input_embeddings()[i]``
    (continuous.py:584-590), ``talker.codec_head`` (continuous.py:458, 613), ``talker.text_projection`` over
    ``talker.get_text_embeddings()`` (custom_voice_prompt.py:38-63), decoder layers with the attribute names
    the reference's PackedAttention / PackedMLP / FusedResidualDecoder read (q_proj, k_proj, v_proj,
    o_proj, q_norm, k_norm, gate_proj, up_proj, down_proj, input_layernorm, post_attention_layernorm).
    Names the reference never spells out (text_projection.linear_fc1/2, code_predictor.lm_head,
    small_to_mtp_projection) are qwen-tts's own."""
    from tests.qwen_tts_fakes import Qwen3TTSDecoderLayer, Qwen3TTSRMSNorm, Qwen3TTSTalkerDecoderLayer, randomize
    from torch import nn

    def layers(kind, cfg):
        return nn.ModuleList([kind(cfg.hidden, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, layer_idx=i)
                              for i in range(cfg.layers)])

    predictor = _Bag(model=_Bag(layers=layers(Qwen3TTSDecoderLayer, pcfg), norm=Qwen3TTSRMSNorm(pcfg.hidden),
                                codec_embedding=nn.ModuleList([nn.Embedding(pcfg.vocab, tcfg.hidden)
                                                               for _ in range(pcfg.groups)])),
                     lm_head=nn.ModuleList([nn.Linear(pcfg.hidden, pcfg.vocab, bias=False)
                                            for _ in range(pcfg.groups)]),
                     small_to_mtp_projection=nn.Linear(tcfg.hidden, pcfg.hidden))
    predictor.get_input_embeddings = lambda: predictor.model.codec_embedding
    talker = _Bag(model=_Bag(layers=layers(Qwen3TTSTalkerDecoderLayer, tcfg), norm=Qwen3TTSRMSNorm(tcfg.hidden),
                             codec_embedding=nn.Embedding(tcfg.vocab, tcfg.hidden),
                             text_embedding=nn.Embedding(prcfg.text_vocab, prcfg.text_hidden)),
                  text_projection=_Bag(linear_fc1=nn.Linear(prcfg.text_hidden, prcfg.text_hidden),
                                       linear_fc2=nn.Linear(prcfg.text_hidden, prcfg.hidden)),
                  codec_head=nn.Linear(tcfg.hidden, tcfg.vocab, bias=False), code_predictor=predictor)
    talker.get_input_embeddings = lambda: talker.model.codec_embedding
    talker.get_text_embeddings = lambda: talker.model.text_embedding
    model = _Bag(talker=talker)
    randomize(model, seed=9)
    return model


def test_checkpoint_named_by_the_reference_module_tree_loads(tmp_path):
    """A checkpoint whose keys are the state_dict of the module tree the reference walks (not this
    module's own writer) loads, and every logical tensor is the module parameter it names."""
    tcfg, pcfg, prcfg, *_ = model(dialect=False)
    tree = _model_tree(tcfg, pcfg, prcfg)
    state = {k: v.detach().to(torch.bfloat16).contiguous() for k, v in tree.state_dict().items()}
    assert sum(k.endswith("talker.codec_head.weight") for k in state) == 1    # the probe's lookup
    safetensors.save_file(state, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps(C.model_config_json(tcfg, pcfg, prcfg)))
    loaded = C.load_model(tmp_path, prompt_base=tiny_prompt(256))
    assert loaded["talker_config"] == tcfg and loaded["predictor_config"] == pcfg
    talker, code_predictor = tree.talker, tree.talker.code_predictor
    w = loaded["weights"]
    bf = lambda p: p.detach().to(torch.bfloat16)     # noqa: E731
    for logical, tree_layers in ((w["talker"]["layers"], talker.model.layers),
                                 (w["predictor"]["layers"], code_predictor.model.layers)):
        for got, layer in zip(logical, tree_layers):
            attn, mlp = layer.self_attn, layer.mlp
            pairs = {"q": attn.q_proj, "k": attn.k_proj, "v": attn.v_proj, "o": attn.o_proj, "q_norm": attn.q_norm,
                     "k_norm": attn.k_norm, "input_norm": layer.input_layernorm,
                     "post_norm": layer.post_attention_layernorm, "gate": mlp.gate_proj, "up": mlp.up_proj,
                     "down": mlp.down_proj}
            for key, module in pairs.items():
                assert torch.equal(got[key], bf(module.weight)), key
    assert torch.equal(w["talker"]["head"], bf(talker.codec_head.weight))
    assert torch.equal(w["talker"]["embedding"], bf(talker.get_input_embeddings().weight))
    assert torch.equal(w["talker"]["norm"], bf(talker.model.norm.weight))
    for j in range(pcfg.groups):
        assert torch.equal(w["predictor"]["embeddings"][j], bf(code_predictor.get_input_embeddings()[j].weight))
        assert torch.equal(w["predictor"]["heads"][j], bf(code_predictor.lm_head[j].weight))
    assert torch.equal(w["predictor"]["proj"], bf(code_predictor.small_to_mtp_projection.weight))
    assert torch.equal(w["prompt"]["text_embedding"], bf(talker.get_text_embeddings().weight))
    assert torch.equal(w["prompt"]["fc2_bias"], bf(talker.text_projection.linear_fc2.bias))
