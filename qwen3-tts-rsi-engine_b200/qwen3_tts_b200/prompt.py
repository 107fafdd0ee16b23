"""Direct CustomVoice prompt preparation on the GPU (custom_voice_prompt.py:13-70).

The prompt is assembled from three embedding sources:

* text ids (role tokens, the text, the instruction) -> ``text_embedding`` ->
  ``text_projection`` (fc1 + SiLU, fc2): one gather kernel and two tcgen05
  GEMMs (the SiLU runs in the fc1 epilogue);
* the tts special ids (bos, eos, pad), projected the same way once and cached;
* codec control ids (think tags, language, speaker, codec pad/bos) from the
  talker's codec embedding, cached per (speaker, language).

Layout of one prompt (rows of width ``hidden``), as the reference builds it:
``[instruction] + role(3) + prefix(n_codec - 1) + (text + tts_eos) + codec_pad
+ (tts_pad + codec_bos)``, where prefix row i is ``tts_pad`` (``tts_bos`` for
the last) plus codec row i. The trailing text hidden and the pad embedding are
both ``tts_pad`` (non-streaming mode).

There are no tokenizer files in this build: a payload supplies ``input_ids``
(text token ids) directly, or ``input`` text that is mapped byte-wise (UTF-8
bytes as ids) as a deterministic stand-in.
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .config import PromptConfig

BF16 = torch.bfloat16

# Sampling settings the engine implements natively (continuous.py:388-393).
SUPPORTED_SAMPLING = {"do_sample": True, "top_k": 50, "top_p": 1.0, "temperature": 0.9,
                      "repetition_penalty": 1.05, "subtalker_dosample": True, "subtalker_top_k": 50,
                      "subtalker_top_p": 1.0, "subtalker_temperature": 0.9}


def prompt_weights(cfg: PromptConfig, seed: int, device="cpu") -> dict:
    """Seeded N(0, 0.02) text embedding and text_projection (weights and biases)."""
    g = torch.Generator(device=torch.device(device)).manual_seed(seed)

    def normal(*shape):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 0.02).to(BF16)

    return {"text_embedding": normal(cfg.text_vocab, cfg.text_hidden),
            "fc1": normal(cfg.text_hidden, cfg.text_hidden), "fc1_bias": normal(cfg.text_hidden),
            "fc2": normal(cfg.hidden, cfg.text_hidden), "fc2_bias": normal(cfg.hidden)}


def text_ids(cfg: PromptConfig, payload: dict, key: str = "input", ids_key: str = "input_ids") -> list:
    if payload.get(ids_key) is not None:
        ids = [int(i) for i in payload[ids_key]]
    else:
        ids = list(str(payload.get(key, "")).encode("utf-8"))
    if any(not 0 <= i < cfg.text_vocab for i in ids):
        raise ValueError("Text token id outside the text vocabulary")
    return ids


def assistant_ids(cfg: PromptConfig, ids: list) -> list:
    """Chat template around the text: 3 role ids first, 5 template ids last."""
    return [cfg.im_start, cfg.assistant, cfg.newline] + ids + [cfg.im_end, cfg.newline, cfg.im_start,
                                                                cfg.assistant, cfg.newline]


def instruct_ids(cfg: PromptConfig, ids: list) -> list:
    return [cfg.im_start, cfg.user, cfg.newline] + ids + [cfg.im_end, cfg.newline]


def codec_tags(cfg: PromptConfig, speaker: str, language: str) -> list:
    """Codec control ids of the prefix: think tags (+ language), speaker, codec pad, codec bos."""
    speakers, languages = cfg.speaker_ids, cfg.language_ids
    if speaker.lower() not in speakers:
        raise ValueError(f"Unsupported speaker: {speaker}")
    if language.lower() != "auto" and language.lower() not in languages:
        raise ValueError(f"Unsupported language: {language}")
    language_id = None if language.lower() == "auto" else languages[language.lower()]
    dialect = dict(cfg.dialects).get(speaker.lower(), False)
    if language.lower() in ("chinese", "auto") and dialect is not False:
        language_id = languages[dialect]
    tags = ([cfg.codec_nothink, cfg.codec_think_bos, cfg.codec_think_eos] if language_id is None
            else [cfg.codec_think, cfg.codec_think_bos, language_id, cfg.codec_think_eos])
    return tags + [speakers[speaker.lower()], cfg.codec_pad, cfg.codec_bos]


class CustomVoicePrompt:
    """Builds ``inputs_embeds`` [1, L, hidden] bf16 for one request on the device."""

    def __init__(self, cfg: PromptConfig, weights: dict, codec_embedding: torch.Tensor, device):
        self.cfg = cfg
        self.device = torch.device(device)
        dev = lambda t: t.to(device=self.device, dtype=BF16).contiguous()
        self.table = dev(weights["text_embedding"])
        self.fc1, self.fc1_bias = ops.pack_tiles(dev(weights["fc1"])), dev(weights["fc1_bias"])
        self.fc2, self.fc2_bias = ops.pack_tiles(dev(weights["fc2"])), dev(weights["fc2_bias"])
        self.codec_embedding = codec_embedding
        self.special = None
        self.prefixes: dict = {}

    def project(self, ids: list) -> torch.Tensor:
        """text_projection(text_embedding(ids)) -> [len(ids), hidden] bf16."""
        index = torch.tensor(ids, dtype=torch.long).to(self.device, non_blocking=True)
        x = ops.embedding(index, self.table)
        h = ops.linear(x, self.fc1, self.fc1_bias, epilogue=_lib.EPI_SILU)
        return ops.linear(h, self.fc2, self.fc2_bias)

    def _ones(self, length: int) -> torch.Tensor:
        """[1, length] int64 ones (a view of one cached device row)."""
        if getattr(self, "_mask", None) is None or self._mask.shape[1] < length:
            self._mask = torch.ones(1, max(length, 4096), dtype=torch.long, device=self.device)
        return self._mask[:, :length]

    def codec(self, ids: list) -> torch.Tensor:
        index = torch.tensor(ids, dtype=torch.long).to(self.device, non_blocking=True)
        return ops.embedding(index, self.codec_embedding)

    def _prefix(self, speaker: str, language: str):
        tags = codec_tags(self.cfg, speaker, language)
        key = tuple(tags)
        if key not in self.prefixes:
            bos, _eos, pad = self.special
            codec = self.codec(tags)                       # [n, hidden]
            n = codec.shape[0]
            text_side = torch.cat((pad.expand(n - 2, -1), bos), 0)
            prefix = text_side + codec[:-1]               # bf16 adds, as the reference's tensors round
            self.prefixes[key] = (prefix, codec[-2:-1], pad + codec[-1:])
        return self.prefixes[key]

    @torch.inference_mode()
    def build(self, payload: dict) -> dict:
        cfg = self.cfg
        if self.special is None:
            self.special = self.project([cfg.tts_bos, cfg.tts_eos, cfg.tts_pad]).split(1, 0)
        bos, eos, pad = self.special
        prefix, codec_pad, final_bos = self._prefix(payload["voice"], payload["language"])
        ids = assistant_ids(cfg, text_ids(cfg, payload))
        parts = []
        instruction = payload.get("instructions") or payload.get("instruction_ids")
        if instruction:
            parts.append(self.project(instruct_ids(cfg, text_ids(cfg, payload, "instructions", "instruction_ids"))))
        role_and_text = self.project(ids)                  # one projection for role + text + template
        parts.append(role_and_text[:3])
        parts.append(prefix)
        parts.append(torch.cat((role_and_text[3:-5], eos), 0) + codec_pad)
        parts.append(final_bos)
        inputs = torch.cat(parts, 0).unsqueeze(0)
        result = dict(SUPPORTED_SAMPLING)
        result.update(max_new_tokens=int(payload["max_new_tokens"]), inputs_embeds=inputs,
                      attention_mask=torch.ones(inputs.shape[:2], dtype=torch.long, device=self.device),
                      trailing_text_hidden=pad.clone().unsqueeze(0), tts_pad_embed=pad.clone().unsqueeze(0))
        return result

    @torch.inference_mode()
    def build_many(self, payloads) -> tuple:
        """build() for several requests with ONE text projection (one gather, two GEMMs) over
        every request's ids and one concatenation: returns the prompts' rows packed end to end
        [sum of lengths, hidden] bf16 and, per request, build()'s dict whose ``inputs_embeds``
        is a view of its rows. The codec pad row added to the text rows is the same embedding
        for every request (the last two codec tags are always codec_pad, codec_bos)."""
        cfg = self.cfg
        if self.special is None:
            self.special = self.project([cfg.tts_bos, cfg.tts_eos, cfg.tts_pad]).split(1, 0)
        _bos, eos, pad = self.special
        plans, ids_all = [], []
        for payload in payloads:
            prefix, codec_pad, final_bos = self._prefix(payload["voice"], payload["language"])
            ids = assistant_ids(cfg, text_ids(cfg, payload))
            instruction = payload.get("instructions") or payload.get("instruction_ids")
            inst = instruct_ids(cfg, text_ids(cfg, payload, "instructions", "instruction_ids")) if instruction else []
            plans.append((len(ids_all), len(inst), len(ids), prefix, codec_pad, final_bos))
            ids_all.extend(inst)
            ids_all.extend(ids)
        projected = self.project(ids_all)
        codec_pad = plans[0][4]
        shifted = projected + codec_pad                    # text rows + codec pad, bf16 adds
        eos_pad = eos + codec_pad
        parts, lengths = [], []
        for start, n_inst, n_ids, prefix, _pad, final_bos in plans:
            t0 = start + n_inst
            rows = [projected[start:t0]] if n_inst else []
            rows += [projected[t0:t0 + 3], prefix, shifted[t0 + 3:t0 + n_ids - 5], eos_pad, final_bos]
            parts.extend(rows)
            lengths.append(sum(r.shape[0] for r in rows))
        packed = torch.cat(parts, 0)
        prompts, offset = [], 0
        trailing = pad.unsqueeze(0)
        for payload, length in zip(payloads, lengths):
            result = dict(SUPPORTED_SAMPLING)
            result.update(max_new_tokens=int(payload["max_new_tokens"]),
                          inputs_embeds=packed[offset:offset + length].unsqueeze(0),
                          attention_mask=self._ones(length), trailing_text_hidden=trailing,
                          tts_pad_embed=trailing)
            prompts.append(result)
            offset += length
        return packed, prompts

