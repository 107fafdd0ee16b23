"""Packed gate/up MLP module on the CUDA kernels (packed_mlp.py:5-37 of the reference).

``install_packed_mlp(model, fused, reference_single)`` replaces every child whose
class is named ``Qwen3TTSTalkerTextMLP`` by ``PackedMLP`` and returns the
``(parent, name, original)`` list for ``operators.restore_modules``. The
reference's checks are kept (SiLU activation, bias-free gate/up projections,
``ValueError`` otherwise). Forward: one tcgen05 GEMM over the gate and up rows
interleaved per 64-row group with SiLU(gate) * up in its epilogue
(``Q3T_EPI_SWIGLU_PAIRED``), then the down projection as a second GEMM. ``fused``
chose between the reference's two SwiGLU forms on the NPU; here both run the
same fused epilogue.
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .operators import replace_children
from .weights import interleave_gate_up


class PackedMLP(torch.nn.Module):
    def __init__(self, reference, fused=False, reference_single=False):
        super().__init__()
        if reference.config.hidden_act != "silu":
            raise ValueError("Packed MLP requires the SiLU activation")
        if reference.gate_proj.bias is not None or reference.up_proj.bias is not None:
            raise ValueError("Packed MLP expects bias-free projections")
        gate, up = reference.gate_proj.weight.detach(), reference.up_proj.weight.detach()
        if gate.dtype != torch.bfloat16 or up.dtype != torch.bfloat16:
            raise ValueError("Packed MLP expects BF16 projections")
        self.reference = reference
        self.weight = torch.nn.Parameter(interleave_gate_up(gate, up), requires_grad=False)
        self.down_proj = reference.down_proj
        self.fused = fused
        self.reference_single = reference_single

    def forward(self, hidden):
        if self.reference_single and hidden.shape[0] == 1:
            return self.reference(hidden)
        act = ops.linear(hidden.contiguous(), self.weight, epilogue=_lib.EPI_SWIGLU_PAIRED)
        down = self.down_proj
        return ops.linear(act, down.weight.detach(), None if down.bias is None else down.bias.detach())


def install_packed_mlp(model, fused=False, reference_single=False) -> list:
    return replace_children(model, ("Qwen3TTSTalkerTextMLP",),
                            lambda child: PackedMLP(child, fused=fused, reference_single=reference_single))
