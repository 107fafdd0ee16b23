"""CustomVoice prompt assembly restated on the CPU (custom_voice_prompt.py:23-70).

TEST INFRASTRUCTURE ONLY (see the package docstring).

``text_projection`` is the qwen-tts ResizeMLP the reference calls
(fc1 -> SiLU -> fc2, both with bias; custom_voice_prompt.py:37-38, 61-66);
its internals belong to qwen-tts==0.1.1 (absent here), so this part is
unpinned. The assembly order and the bf16 additions follow
custom_voice_prompt.py:43-66 exactly.
"""
from __future__ import annotations

import torch

from .elementwise import bf


def project(weights: dict, ids, mode: str = "bf16") -> torch.Tensor:
    """text_projection(text_embedding(ids)) -> [n, hidden] fp32 (bf16-valued in bf16 mode)."""
    x = weights["text_embedding"][torch.as_tensor(ids, dtype=torch.long)].float()
    h = x @ weights["fc1"].float().T + weights["fc1_bias"].float()
    if mode == "bf16":
        h = bf(torch.nn.functional.silu(bf(h)))
        return bf(h @ weights["fc2"].float().T + weights["fc2_bias"].float())
    h = torch.nn.functional.silu(h)
    return h @ weights["fc2"].float().T + weights["fc2_bias"].float()


def build(cfg, weights: dict, codec_embedding: torch.Tensor, text_ids, speaker_tags, instruction_ids=None,
          mode: str = "bf16") -> dict:
    """inputs_embeds [L, hidden], trailing_text_hidden / tts_pad_embed [hidden].

    text_ids: the text's token ids; speaker_tags: codec control ids
    (think tags [+ language], speaker, codec pad, codec bos)."""
    add = (lambda a, b: bf(a + b)) if mode == "bf16" else (lambda a, b: a + b)
    bos, eos, pad = project(weights, [cfg.tts_bos, cfg.tts_eos, cfg.tts_pad], mode)
    codec = codec_embedding[torch.as_tensor(speaker_tags, dtype=torch.long)].float()
    n = codec.shape[0]
    text_side = torch.cat((pad.expand(n - 2, -1), bos[None]), 0)
    prefix = add(text_side, codec[:-1])
    codec_pad, final_bos = codec[-2], add(pad, codec[-1])
    ids = [cfg.im_start, cfg.assistant, cfg.newline] + list(text_ids) + [cfg.im_end, cfg.newline, cfg.im_start,
                                                                        cfg.assistant, cfg.newline]
    parts = []
    if instruction_ids:
        parts.append(project(weights, [cfg.im_start, cfg.user, cfg.newline] + list(instruction_ids)
                             + [cfg.im_end, cfg.newline], mode))
    projected = project(weights, ids, mode)
    parts.append(projected[:3])
    parts.append(prefix)
    parts.append(add(torch.cat((projected[3:-5], eos[None]), 0), codec_pad[None]))
    parts.append(final_bos[None])
    return {"inputs_embeds": torch.cat(parts, 0), "trailing_text_hidden": pad.clone(), "tts_pad_embed": pad.clone()}
