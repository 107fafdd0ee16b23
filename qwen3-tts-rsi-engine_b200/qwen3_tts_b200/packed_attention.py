"""Packed Q/K/V attention module on the CUDA kernels (packed_attention.py:11-95 of the reference).

``install_packed_attention(model, ...)`` replaces every child whose class is
named ``Qwen3TTSTalkerAttention`` or ``Qwen3TTSAttention`` by ``PackedAttention``
and returns the ``(parent, name, original)`` list for ``operators.restore_modules``.
The keyword flags are the reference's; those that choose between its NPU
kernels (``native_gqa``, ``native_rope``, ``triton_talker_rope``) are validated
as the reference validates them and otherwise do not change the computation:
there is one CUDA path.

Forward, per call with hidden states [B, S, hidden]:

1. Q|K|V in one tcgen05 GEMM over the concatenated weights (q, k, v row order
   and split sizes as packed_attention.py:14-22), bias if the projections have one;
2. q_norm / k_norm through the wrapped module's own norm modules (``CudaRMSNorm``
   once ``install_rms_norms`` has run) on [B, S, heads, head_dim];
3. rotate-half RoPE with bf16 rounding (``q3t_rotary``), cos/sin [B, S, D]; for the
   talker's multimodal attention the first position axis is used, which requires
   identical CustomVoice axes (``text_only_rope=True``; the constructor raises
   otherwise, as the reference does for its native rotary paths);
4. the cache update through ``past_key_values.update`` (any cache with the HF
   ``update(key, value, layer_idx, kwargs)`` contract, e.g. the slot cache);
5. attention: with no mask, or a decode step whose cache reports
   ``actual_seq_lengths_kv``, the split-KV decode kernel (``q3t_decode_attention``)
   over the returned [B, kv_heads, L, D] keys, query row s of batch b seeing keys
   0 .. L - S + s (or length - 1); a call with an explicit mask (padded batches)
   uses torch's scaled-dot-product attention with that mask;
6. o_proj as a tcgen05 GEMM. Attention weights are not returned (None).
"""
from __future__ import annotations

import torch

from . import ops
from .operators import replace_children

CLASS_NAMES = ("Qwen3TTSTalkerAttention", "Qwen3TTSAttention")


class PackedAttention(torch.nn.Module):
    def __init__(self, reference, native_gqa=False, text_only_rope=False, reference_single=False, native_rope=False,
                 native_rope_scope="all", triton_talker_rope=False):
        super().__init__()
        if native_rope_scope not in ("all", "talker", "predictor"):
            raise ValueError("Native rotary scope must be all, talker or predictor")
        self.reference = reference
        self.multimodal = type(reference).__name__ == "Qwen3TTSTalkerAttention"
        if self.multimodal and not text_only_rope:
            raise ValueError("CUDA rotary requires identical CustomVoice position axes (text_only_rope=True)")
        projections = [reference.q_proj, reference.k_proj, reference.v_proj]
        self.sizes = [p.out_features for p in projections]
        weight = torch.cat([p.weight.detach() for p in projections], dim=0)
        if weight.dtype != torch.bfloat16:
            raise ValueError("Packed attention expects BF16 projections")
        self.weight = torch.nn.Parameter(weight.contiguous(), requires_grad=False)
        self.bias = None
        if projections[0].bias is not None:
            self.bias = torch.nn.Parameter(torch.cat([p.bias.detach() for p in projections]).contiguous(),
                                           requires_grad=False)
        self.native_gqa, self.native_rope, self.triton_talker_rope = native_gqa, native_rope, triton_talker_rope
        self.native_rope_scope, self.text_only_rope = native_rope_scope, text_only_rope
        self.reference_single = reference_single

    def forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None, cache_position=None,
                **kwargs):
        ref = self.reference
        if self.reference_single and hidden_states.shape[0] == 1:
            return ref(hidden_states, position_embeddings, attention_mask, past_key_values=past_key_values,
                       cache_position=cache_position, **kwargs)
        batch, length = hidden_states.shape[:2]
        d = ref.head_dim
        qkv = ops.linear(hidden_states.contiguous(), self.weight, self.bias)
        query, key, value = qkv.split(self.sizes, dim=-1)
        query = ref.q_norm(query.reshape(batch, length, -1, d))
        key = ref.k_norm(key.reshape(batch, length, -1, d))
        cos, sin = position_embeddings
        if self.multimodal:
            cos, sin = cos[0], sin[0]
        cos = cos.to(torch.bfloat16).expand(batch, length, d).contiguous()
        sin = sin.to(torch.bfloat16).expand(batch, length, d).contiguous()
        query = ops.rotary(query.contiguous(), cos, sin).transpose(1, 2)
        key = ops.rotary(key.contiguous(), cos, sin).transpose(1, 2)
        value = value.reshape(batch, length, -1, d).transpose(1, 2)
        if past_key_values is not None:
            key, value = past_key_values.update(key, value, ref.layer_idx,
                                                {"sin": sin, "cos": cos, "cache_position": cache_position})
        lengths = getattr(past_key_values, "actual_seq_lengths_kv", None)
        window = getattr(ref, "sliding_window", None) or 0
        if attention_mask is None or (lengths is not None and length == 1):
            keys, values = key.contiguous(), value.contiguous()
            visible = keys.shape[2]
            if visible < 64:   # one whole 64-key tile per (slot, head); positions never reach the padding
                keys = torch.nn.functional.pad(keys, (0, 0, 0, 64 - visible))
                values = torch.nn.functional.pad(values, (0, 0, 0, 64 - visible))
            rows = query.transpose(1, 2).reshape(batch * length, -1, d).contiguous()
            if lengths is not None and length == 1:
                positions = torch.as_tensor(lengths, dtype=torch.int64).to(keys.device) - 1
            else:
                positions = (torch.arange(length, device=keys.device) + (visible - length)).repeat(batch)
            out = ops.decode_attention(rows, keys, values, positions, rows_per_slot=length, scale=ref.scaling,
                                       window=window)
            out = out.reshape(batch, length, -1)
        else:
            mask = attention_mask
            out = torch.nn.functional.scaled_dot_product_attention(
                query, key, value, attn_mask=mask, scale=ref.scaling, enable_gqa=True)
            out = out.transpose(1, 2).reshape(batch, length, -1)
        o = ref.o_proj
        return ops.linear(out.contiguous(), o.weight.detach(), None if o.bias is None else o.bias.detach()), None


def install_packed_attention(model, native_gqa=False, text_only_rope=False, reference_single=False, native_rope=False,
                             native_rope_scope="all", triton_talker_rope=False) -> list:
    return replace_children(model, CLASS_NAMES, lambda child: PackedAttention(
        child, native_gqa=native_gqa, text_only_rope=text_only_rope, reference_single=reference_single,
        native_rope=native_rope, native_rope_scope=native_rope_scope, triton_talker_rope=triton_talker_rope))
