"""Safetensors checkpoint loading for the talker, code predictor, prompt projection and codec.

The reference builds its model with ``Qwen3TTSModel.from_pretrained`` from the
qwen-tts 0.1.1 CustomVoice checkpoint (model.py:18-21) and reads tensors of
that checkpoint directly by name when it needs them
(tools/probe_sampling_head.py:43-49: ``safe_open(<model>/model.safetensors)``,
the talker output head found as the one key ending in
``talker.codec_head.weight``). This module reads the same files into the
logical weight dicts that ``weights.pack_decoder``, ``prompt.CustomVoicePrompt``
and ``codec.pack_codec`` lay out for the kernels.

Names. The talker prefix ``P`` is whatever precedes ``codec_head.weight`` in
the single key ending ``talker.codec_head.weight`` (so an outer wrapper prefix
is tolerated, as in the reference probe). Under it:

* talker decoder ``P model.layers.{i}.`` + Qwen3 layer names
  (``input_layernorm``, ``self_attn.{q,k,v,o}_proj``, ``self_attn.{q,k}_norm``,
  ``post_attention_layernorm``, ``mlp.{gate,up,down}_proj``), ``P model.norm``,
  codec embedding ``P model.codec_embedding``, head ``P codec_head``;
* prompt ``P model.text_embedding``, ``P text_projection.linear_fc{1,2}``
  (weights and biases);
* code predictor ``P code_predictor.model.layers.{i}.`` (same layer names),
  ``.model.norm``, embeddings ``.model.codec_embedding.{j}``, heads
  ``.lm_head.{j}``, input projection ``.small_to_mtp_projection`` (absent when
  the predictor is as wide as the talker: identity).

These are the module attribute paths of the qwen-tts model tree the reference
drives (``talker.model``, ``talker.text_projection``, ``talker.codec_head``,
``talker.code_predictor``; continuous.py:584-613, custom_voice_prompt.py:38-63).
Geometry (layers, widths, heads, vocabularies) is read off the tensor shapes;
``config.json`` supplies what shapes cannot: norm epsilon and RoPE base
(``talker_config.rms_norm_eps`` / ``rope_theta``, the same under
``talker_config.code_predictor_config``), the EOS id
(``talker_config.codec_eos_token_id``, model.py:72) and the prompt ids
(``tts_{bos,eos,pad}_token_id``; ``talker_config.codec_*_id``,
``codec_language_id``, ``spk_id``, ``spk_is_dialect``;
custom_voice_prompt.py:30-50). Every missing tensor or shape mismatch raises
``ValueError`` naming the tensor, before anything is copied to the device.

The codec (``speech_tokenizer/model.safetensors``) is read into the module
tree ``pack_codec`` walks: the key of every tensor is its attribute path in
that tree (``quantizer.rvq_first.vq.layers.0._codebook.embedding_sum``,
``pre_transformer.layers.3.q_proj.weight``, ``decoder.1.block.2.conv1.conv.weight``
...), under whatever prefix precedes the one key ending in
``pre_conv.conv.weight``; ``_layers`` is accepted for ``vq.layers``.
"""
from __future__ import annotations

import json
from dataclasses import replace
from pathlib import Path
from types import SimpleNamespace as NS

import torch

from .config import CODEC, PREDICTOR, PROMPT, TALKER, CodecConfig, PredictorConfig, PromptConfig, TalkerConfig

BF16 = torch.bfloat16

# logical layer tensor -> checkpoint name under "<decoder>.layers.{i}."
LAYER_NAMES = {
    "input_norm": "input_layernorm.weight",
    "q": "self_attn.q_proj.weight",
    "k": "self_attn.k_proj.weight",
    "v": "self_attn.v_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "o": "self_attn.o_proj.weight",
    "post_norm": "post_attention_layernorm.weight",
    "gate": "mlp.gate_proj.weight",
    "up": "mlp.up_proj.weight",
    "down": "mlp.down_proj.weight",
}
HEAD_SUFFIX = "talker.codec_head.weight"
CODEC_ANCHOR = "pre_conv.conv.weight"


class Checkpoint:
    """Lazy reader over one safetensors file, a directory holding ``model.safetensors``,
    or a sharded directory (``model.safetensors.index.json`` -> ``weight_map``)."""

    def __init__(self, path, name: str = "model.safetensors"):
        from safetensors import safe_open  # noqa: F401  (fail here, before any work, if absent)
        path = Path(path)
        self.config = {}
        if path.is_dir():
            root = path
            index = root / f"{name}.index.json"
            if index.exists():
                weight_map = json.loads(index.read_text())["weight_map"]
                self._where = {key: root / shard for key, shard in weight_map.items()}
            elif (root / name).exists():
                self._where = None
                self._single = root / name
            else:
                raise ValueError(f"No {name} (or {name}.index.json) in {root}")
            config = root / "config.json"
            if config.exists():
                self.config = json.loads(config.read_text())
        elif path.exists():
            self._where, self._single = None, path
        else:
            raise ValueError(f"Checkpoint not found: {path}")
        self._handles = {}
        if self._where is None:
            self._keys = set(self._handle(self._single).keys())
        else:
            self._keys = set(self._where)

    def _handle(self, file: Path):
        handle = self._handles.get(file)
        if handle is None:
            from safetensors import safe_open
            if not file.exists():
                raise ValueError(f"Checkpoint shard missing: {file}")
            handle = safe_open(str(file), framework="pt", device="cpu")
            self._handles[file] = handle
        return handle

    def keys(self) -> set:
        return self._keys

    def close(self) -> None:
        """Release the open file handles (tensors already read stay valid)."""
        self._handles.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __contains__(self, key: str) -> bool:
        return key in self._keys

    def shape(self, key: str) -> tuple:
        self._require(key)
        return tuple(self._handle(self._file(key)).get_slice(key).get_shape())

    def get(self, key: str, shape=None) -> torch.Tensor:
        self._require(key)
        if shape is not None and self.shape(key) != tuple(shape):
            raise ValueError(f"Checkpoint tensor {key} has shape {self.shape(key)}, expected {tuple(shape)}")
        return self._handle(self._file(key)).get_tensor(key)

    def _file(self, key: str) -> Path:
        return self._single if self._where is None else self._where[key]

    def _require(self, key: str) -> None:
        if key not in self._keys:
            raise ValueError(f"Checkpoint tensor missing: {key}")

    def prefix(self, suffix: str, what: str) -> str:
        names = [key for key in self._keys if key.endswith(suffix)]
        if len(names) != 1:
            raise ValueError(f"Expected one {what} ({suffix}), got {sorted(names)}")
        return names[0][:-len(suffix)]


def _count(ckpt: Checkpoint, pattern: str) -> int:
    n = 0
    while pattern.format(n) in ckpt:
        n += 1
    return n


def _decoder_geometry(ckpt: Checkpoint, base: str) -> dict:
    layers = _count(ckpt, base + "layers.{}." + LAYER_NAMES["input_norm"])
    if layers == 0:
        raise ValueError(f"Checkpoint has no decoder layers under {base}layers.")
    first = base + "layers.0."
    hidden = ckpt.shape(first + LAYER_NAMES["input_norm"])[0]
    head_dim = ckpt.shape(first + LAYER_NAMES["q_norm"])[0]
    q_rows = ckpt.shape(first + LAYER_NAMES["q"])[0]
    kv_rows = ckpt.shape(first + LAYER_NAMES["k"])[0]
    if q_rows % head_dim or kv_rows % head_dim:
        raise ValueError(f"Projection rows of {first} are not multiples of head_dim {head_dim}")
    return dict(layers=layers, hidden=hidden, head_dim=head_dim, q_heads=q_rows // head_dim,
                kv_heads=kv_rows // head_dim, ffn=ckpt.shape(first + LAYER_NAMES["gate"])[0])


def _layer_shapes(cfg) -> dict:
    return {"input_norm": (cfg.hidden,), "q": (cfg.q_width, cfg.hidden), "k": (cfg.kv_width, cfg.hidden),
            "v": (cfg.kv_width, cfg.hidden), "q_norm": (cfg.head_dim,), "k_norm": (cfg.head_dim,),
            "o": (cfg.hidden, cfg.q_width), "post_norm": (cfg.hidden,), "gate": (cfg.ffn, cfg.hidden),
            "up": (cfg.ffn, cfg.hidden), "down": (cfg.hidden, cfg.ffn)}


def _layers(ckpt: Checkpoint, base: str, cfg, device, dtype) -> list:
    return [{name: ckpt.get(f"{base}layers.{i}.{key}").to(device=device, dtype=dtype)
             for name, key in LAYER_NAMES.items()} for i in range(cfg.layers)]


def _float(section: dict, key: str, default: float) -> float:
    value = section.get(key)
    return default if value is None else float(value)


def read_configs(ckpt: Checkpoint, prompt_base: PromptConfig = PROMPT) -> tuple:
    """(TalkerConfig, PredictorConfig, PromptConfig) from tensor shapes plus config.json.

    The chat-template ids (``im_start``, ``assistant``, ...) belong to the text tokenizer, not
    to config.json: they are kept from ``prompt_base``."""
    prefix = ckpt.prefix(HEAD_SUFFIX, "talker output head") + "talker."
    top = ckpt.config
    tc = top.get("talker_config") or {}
    pc = tc.get("code_predictor_config") or top.get("code_predictor_config") or {}
    geometry = _decoder_geometry(ckpt, prefix + "model.")
    vocab = ckpt.shape(prefix + "codec_head.weight")[0]
    pp = prefix + "code_predictor."
    groups = _count(ckpt, pp + "lm_head.{}.weight")
    if groups == 0:
        raise ValueError(f"Checkpoint has no code predictor heads under {pp}lm_head.")
    talker = TalkerConfig(**geometry, vocab=vocab, eps=_float(tc, "rms_norm_eps", TALKER.eps),
                          theta=_float(tc, "rope_theta", TALKER.theta),
                          eos=int(tc.get("codec_eos_token_id", TALKER.eos)), codebooks=groups + 1)
    pgeometry = _decoder_geometry(ckpt, pp + "model.")
    predictor = PredictorConfig(**pgeometry, vocab=ckpt.shape(pp + "lm_head.0.weight")[0],
                                eps=_float(pc, "rms_norm_eps", PREDICTOR.eps),
                                theta=_float(pc, "rope_theta", PREDICTOR.theta), groups=groups,
                                talker_hidden=talker.hidden)
    text_vocab, text_hidden = ckpt.shape(prefix + "model.text_embedding.weight")
    prompt = replace(prompt_base, text_vocab=text_vocab, text_hidden=text_hidden, hidden=talker.hidden)
    ids = {"tts_pad": top.get("tts_pad_token_id"), "tts_bos": top.get("tts_bos_token_id"),
           "tts_eos": top.get("tts_eos_token_id"), "codec_pad": tc.get("codec_pad_id"),
           "codec_bos": tc.get("codec_bos_id"), "codec_think": tc.get("codec_think_id"),
           "codec_nothink": tc.get("codec_nothink_id"), "codec_think_bos": tc.get("codec_think_bos_id"),
           "codec_think_eos": tc.get("codec_think_eos_id")}
    prompt = replace(prompt, **{k: int(v) for k, v in ids.items() if v is not None})
    if tc.get("codec_language_id"):
        prompt = replace(prompt, languages=tuple((k.lower(), int(v)) for k, v in tc["codec_language_id"].items()))
    if tc.get("spk_id"):
        prompt = replace(prompt, speakers=tuple((k.lower(), _speaker_id(k, v)) for k, v in tc["spk_id"].items()))
    if tc.get("spk_is_dialect"):
        prompt = replace(prompt, dialects=tuple((k.lower(), v) for k, v in tc["spk_is_dialect"].items()
                                                if v is not False))
    for name, value in [(n, getattr(prompt, n)) for n in ("codec_pad", "codec_bos", "codec_think", "codec_nothink",
                                                          "codec_think_bos", "codec_think_eos")] + \
            [(f"speaker {k}", v) for k, v in prompt.speakers] + [(f"language {k}", v) for k, v in prompt.languages]:
        if not 0 <= value < vocab:
            raise ValueError(f"Codec id of {name} ({value}) is outside the talker vocabulary {vocab}")
    return talker, predictor, prompt


def _speaker_id(name, value) -> int:
    if isinstance(value, (list, tuple)):
        if len(value) != 1:
            raise ValueError(f"Speaker {name} has {len(value)} codec ids; one is supported")
        value = value[0]
    return int(value)


def load_model(path, device="cpu", dtype=BF16, prompt_base: PromptConfig = PROMPT) -> dict:
    """Read talker, predictor and prompt weights (plus their configs) from a checkpoint.

    Returns ``{"talker_config", "predictor_config", "prompt_config", "weights": {"talker",
    "predictor", "prompt"}}`` with the weight dicts in the layout of ``weights.decoder_weights``
    and ``prompt.prompt_weights``; all shapes are checked before the first tensor is read.
    """
    if not isinstance(path, Checkpoint):
        with Checkpoint(path) as ckpt:
            return load_model(ckpt, device, dtype, prompt_base)
    ckpt = path
    tcfg, pcfg, prcfg = read_configs(ckpt, prompt_base)
    prefix = ckpt.prefix(HEAD_SUFFIX, "talker output head") + "talker."
    pp = prefix + "code_predictor."
    proj = pp + "small_to_mtp_projection."
    expected = {prefix + "model.norm.weight": (tcfg.hidden,),
                prefix + "codec_head.weight": (tcfg.vocab, tcfg.hidden),
                prefix + "model.codec_embedding.weight": (tcfg.vocab, tcfg.hidden),
                pp + "model.norm.weight": (pcfg.hidden,),
                prefix + "text_projection.linear_fc1.weight": (prcfg.text_hidden, prcfg.text_hidden),
                prefix + "text_projection.linear_fc1.bias": (prcfg.text_hidden,),
                prefix + "text_projection.linear_fc2.weight": (prcfg.hidden, prcfg.text_hidden),
                prefix + "text_projection.linear_fc2.bias": (prcfg.hidden,)}
    for base, cfg in ((prefix + "model.", tcfg), (pp + "model.", pcfg)):
        for i in range(cfg.layers):
            for name, shape in _layer_shapes(cfg).items():
                expected[f"{base}layers.{i}.{LAYER_NAMES[name]}"] = shape
    for j in range(pcfg.groups):
        expected[f"{pp}lm_head.{j}.weight"] = (pcfg.vocab, pcfg.hidden)
        expected[f"{pp}model.codec_embedding.{j}.weight"] = (pcfg.vocab, tcfg.hidden)
    if proj + "weight" in ckpt:
        expected[proj + "weight"] = (pcfg.hidden, tcfg.hidden)
        expected[proj + "bias"] = (pcfg.hidden,)
    elif pcfg.hidden != tcfg.hidden:
        raise ValueError(f"Checkpoint tensor missing: {proj}weight (predictor {pcfg.hidden} wide, talker "
                         f"{tcfg.hidden})")
    for key, shape in expected.items():
        if ckpt.shape(key) != shape:
            raise ValueError(f"Checkpoint tensor {key} has shape {ckpt.shape(key)}, expected {shape}")

    def get(key):
        return ckpt.get(key).to(device=device, dtype=dtype)

    talker = {"layers": _layers(ckpt, prefix + "model.", tcfg, device, dtype), "norm": get(prefix + "model.norm.weight"),
              "head": get(prefix + "codec_head.weight"), "embedding": get(prefix + "model.codec_embedding.weight")}
    predictor = {"layers": _layers(ckpt, pp + "model.", pcfg, device, dtype), "norm": get(pp + "model.norm.weight"),
                 "heads": torch.stack([get(f"{pp}lm_head.{j}.weight") for j in range(pcfg.groups)]),
                 "embeddings": torch.stack([get(f"{pp}model.codec_embedding.{j}.weight")
                                            for j in range(pcfg.groups)])}
    if proj + "weight" in ckpt:
        predictor["proj"], predictor["proj_bias"] = get(proj + "weight"), get(proj + "bias")
    else:
        predictor["proj"] = torch.eye(pcfg.hidden, device=device, dtype=dtype)
        predictor["proj_bias"] = torch.zeros(pcfg.hidden, device=device, dtype=dtype)
    tp = prefix + "text_projection."
    prompt = {"text_embedding": get(prefix + "model.text_embedding.weight"),
              "fc1": get(tp + "linear_fc1.weight"), "fc1_bias": get(tp + "linear_fc1.bias"),
              "fc2": get(tp + "linear_fc2.weight"), "fc2_bias": get(tp + "linear_fc2.bias")}
    return {"talker_config": tcfg, "predictor_config": pcfg, "prompt_config": prcfg,
            "weights": {"talker": talker, "predictor": predictor, "prompt": prompt}}


def model_state_dict(talker: dict, predictor: dict, prompt: dict, prefix: str = "talker.") -> dict:
    """The inverse of ``load_model``: checkpoint names -> tensors (for conversion and tests)."""
    out = {}
    for base, weights in ((prefix + "model.", talker), (prefix + "code_predictor.model.", predictor)):
        for i, layer in enumerate(weights["layers"]):
            for name, key in LAYER_NAMES.items():
                out[f"{base}layers.{i}.{key}"] = layer[name]
        out[base + "norm.weight"] = weights["norm"]
    out[prefix + "codec_head.weight"] = talker["head"]
    out[prefix + "model.codec_embedding.weight"] = talker["embedding"]
    pp = prefix + "code_predictor."
    for j in range(predictor["heads"].shape[0]):
        out[f"{pp}lm_head.{j}.weight"] = predictor["heads"][j]
        out[f"{pp}model.codec_embedding.{j}.weight"] = predictor["embeddings"][j]
    out[pp + "small_to_mtp_projection.weight"] = predictor["proj"]
    out[pp + "small_to_mtp_projection.bias"] = predictor["proj_bias"]
    out[prefix + "model.text_embedding.weight"] = prompt["text_embedding"]
    tp = prefix + "text_projection."
    out[tp + "linear_fc1.weight"], out[tp + "linear_fc1.bias"] = prompt["fc1"], prompt["fc1_bias"]
    out[tp + "linear_fc2.weight"], out[tp + "linear_fc2.bias"] = prompt["fc2"], prompt["fc2_bias"]
    return {k: _owned(v) for k, v in out.items()}


def _owned(tensor: torch.Tensor) -> torch.Tensor:
    """A CPU tensor that owns its storage (safetensors refuses tensors that share one)."""
    t = tensor.detach().to("cpu").contiguous()
    return t if t.untyped_storage().nbytes() == t.numel() * t.element_size() else t.clone()


def model_config_json(talker: TalkerConfig, predictor: PredictorConfig, prompt: PromptConfig) -> dict:
    """The config.json fields ``read_configs`` reads, for a checkpoint this module writes."""
    return {"tts_pad_token_id": prompt.tts_pad, "tts_bos_token_id": prompt.tts_bos, "tts_eos_token_id": prompt.tts_eos,
            "talker_config": {
                "rms_norm_eps": talker.eps, "rope_theta": talker.theta, "codec_eos_token_id": talker.eos,
                "codec_pad_id": prompt.codec_pad, "codec_bos_id": prompt.codec_bos,
                "codec_think_id": prompt.codec_think, "codec_nothink_id": prompt.codec_nothink,
                "codec_think_bos_id": prompt.codec_think_bos, "codec_think_eos_id": prompt.codec_think_eos,
                "codec_language_id": dict(prompt.languages), "spk_id": dict(prompt.speakers),
                "spk_is_dialect": {name: dict(prompt.dialects).get(name, False) for name, _ in prompt.speakers},
                "code_predictor_config": {"rms_norm_eps": predictor.eps, "rope_theta": predictor.theta}}}


def save_model(directory, talker: dict, predictor: dict, prompt: dict, talker_config: TalkerConfig,
               predictor_config: PredictorConfig, prompt_config: PromptConfig, shards: int = 1) -> None:
    """Write ``model.safetensors`` (or ``shards`` files plus the index) and ``config.json``."""
    from safetensors.torch import save_file
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    tensors = model_state_dict(talker, predictor, prompt)
    if shards <= 1:
        save_file(tensors, str(directory / "model.safetensors"))
    else:
        names = sorted(tensors)
        weight_map = {}
        for s in range(shards):
            part = names[s::shards]
            file = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
            save_file({k: tensors[k] for k in part}, str(directory / file))
            weight_map.update({k: file for k in part})
        (directory / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    (directory / "config.json").write_text(json.dumps(model_config_json(talker_config, predictor_config,
                                                                        prompt_config), indent=1))


# ---------------------------------------------------------------------------------------------- codec
def _leaves(node, path: str = ""):
    """(attribute path, parent, attribute or index) of every tensor in a codec module tree."""
    if isinstance(node, (list, tuple)):
        for i, child in enumerate(node):
            yield from _leaves_child(child, path, i, node)
    elif isinstance(node, NS):
        for name, child in vars(node).items():
            if name != "cfg":
                yield from _leaves_child(child, path, name, node)


def _leaves_child(child, path, name, parent):
    key = f"{path}.{name}" if path else str(name)
    if isinstance(child, torch.Tensor):
        yield key, parent, name
    else:
        yield from _leaves(child, key)


def codec_state_dict(decoder) -> dict:
    """Attribute path -> tensor for a codec tree (``codec_weights.random_codec`` layout) or any
    torch module whose ``state_dict`` uses the same paths."""
    if isinstance(decoder, torch.nn.Module):
        return {k.replace("._layers.", ".vq.layers."): v.detach().cpu().contiguous()
                for k, v in decoder.state_dict().items()}
    return {key: parent[name] if isinstance(parent, (list, tuple)) else getattr(parent, name)
            for key, parent, name in _leaves(decoder)}


def load_codec(path, cfg: CodecConfig = CODEC):
    """A codec module tree for ``codec.pack_codec`` from a safetensors file or directory
    (``model.safetensors`` there), with every tensor's shape checked against ``cfg``."""
    from .codec_weights import codec_template
    if not isinstance(path, Checkpoint):
        with Checkpoint(path) as ckpt:
            return load_codec(ckpt, cfg)
    ckpt = path
    prefix = ckpt.prefix(CODEC_ANCHOR, "codec pre-conv")
    tree = codec_template(cfg)
    for key, parent, name in list(_leaves(tree)):
        slot = parent[name] if isinstance(parent, list) else getattr(parent, name)
        stored = prefix + key
        if stored not in ckpt:
            stored = prefix + key.replace(".vq.layers.", "._layers.")
        tensor = ckpt.get(stored, tuple(slot.shape)).to(torch.float32)
        if isinstance(parent, list):
            parent[name] = tensor
        else:
            setattr(parent, name, tensor)
    return tree


def save_codec(path, decoder) -> None:
    from safetensors.torch import save_file
    path = Path(path)
    if path.suffix != ".safetensors":
        path.mkdir(parents=True, exist_ok=True)
        path = path / "model.safetensors"
    save_file({k: v.float().contiguous() for k, v in codec_state_dict(decoder).items()}, str(path))
