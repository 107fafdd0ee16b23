"""Residual-add + post-attention RMSNorm fusion for decoder layers (fused_decoder.py:1-47 of the reference).

``install_fused_decoders(model, reference_single)`` replaces every child whose
class is named ``Qwen3TTSTalkerDecoderLayer`` or ``Qwen3TTSDecoderLayer`` by
``FusedResidualDecoder`` and returns the ``(parent, name, original)`` list for
``operators.restore_modules``. As in the reference, the layer's
post-attention norm must already run in ``'native'`` mode (``install_rms_norms``
with ``mode='native'``), because the fused kernel normalises the unrounded fp32
sum (``q3t_add_rms_norm``, one kernel for residual = attention + hidden and its
RMSNorm); the constructor raises ``ValueError`` otherwise. The layer's own
input norm, attention and MLP modules run unchanged.
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .operators import replace_children


class FusedResidualDecoder(torch.nn.Module):
    def __init__(self, reference, reference_single=False):
        super().__init__()
        self.reference = reference
        self.reference_single = reference_single
        if hasattr(reference, "attention_type"):
            self.attention_type = reference.attention_type
        if getattr(reference.post_attention_layernorm, "mode", None) != "native":
            raise ValueError("Residual fusion requires native RMSNorm")

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                output_attentions=False, use_cache=False, cache_position=None, position_embeddings=None, **kwargs):
        layer = self.reference
        arguments = dict(attention_mask=attention_mask, position_ids=position_ids, past_key_values=past_key_values,
                         output_attentions=output_attentions, use_cache=use_cache, cache_position=cache_position,
                         position_embeddings=position_embeddings, **kwargs)
        if self.reference_single and hidden_states.shape[0] == 1:
            return layer(hidden_states, **arguments)
        attended, weights = layer.self_attn(hidden_states=layer.input_layernorm(hidden_states), **arguments)
        norm = layer.post_attention_layernorm
        normalized, residual = ops.add_rms_norm(attended.contiguous(), hidden_states.contiguous(),
                                                norm.weight.detach(), norm.variance_epsilon, _lib.NORM_NATIVE)
        output = residual + layer.mlp(normalized)
        return (output, weights) if output_attentions else (output,)


def install_fused_decoders(model, reference_single=False) -> list:
    return replace_children(model, ("Qwen3TTSTalkerDecoderLayer", "Qwen3TTSDecoderLayer"),
                            lambda child: FusedResidualDecoder(child, reference_single))
