"""RMSNorm module replacement on the CUDA kernels (operators.py:6-38 of the reference).

``install_rms_norms(model, mode, reference_single)`` swaps every child module
whose class is named ``Qwen3TTSRMSNorm`` for ``CudaRMSNorm`` and returns the
``(parent, name, original)`` list that ``restore_modules`` undoes (in reverse
order), as the reference's plugin functions do. ``mode`` keeps the reference's
two roundings: ``'reference-rounding'`` normalises in fp32, rounds to bf16 and
then multiplies by the weight in bf16; ``'native'`` applies the weight before
the single rounding (``q3t_rms_norm`` modes 0 and 1).
"""
from __future__ import annotations

import torch

from . import _lib, ops

MODES = {"reference-rounding": _lib.NORM_REFERENCE, "native": _lib.NORM_NATIVE}


class CudaRMSNorm(torch.nn.Module):
    def __init__(self, reference, mode="reference-rounding", reference_single=False):
        super().__init__()
        if mode not in MODES:
            raise ValueError("RMSNorm mode must be 'reference-rounding' or 'native'")
        self.reference = reference
        self.reference_single = reference_single
        self.weight = reference.weight
        self.variance_epsilon = reference.variance_epsilon
        self.mode = mode

    def forward(self, inputs):
        if self.reference_single and inputs.shape[0] == 1:
            return self.reference(inputs)
        if inputs.dtype != torch.bfloat16 or self.weight.dtype != torch.bfloat16:
            raise ValueError("CUDA RMSNorm expects BF16 inputs and weight")
        return ops.rms_norm(inputs.contiguous(), self.weight.detach(), self.variance_epsilon, MODES[self.mode])


def replace_children(model, class_names, build) -> list:
    """Replace every child whose class name is in `class_names` by build(child); return the
    (parent, name, original) list in visiting order."""
    replacements = []
    for parent in list(model.modules()):
        for name, child in list(parent.named_children()):
            if type(child).__name__ in class_names:
                replacements.append((parent, name, child))
                setattr(parent, name, build(child))
    return replacements


def install_rms_norms(model, mode="reference-rounding", reference_single=False) -> list:
    if mode not in MODES:
        raise ValueError("RMSNorm mode must be 'reference-rounding' or 'native'")
    return replace_children(model, ("Qwen3TTSRMSNorm",), lambda child: CudaRMSNorm(child, mode, reference_single))


def restore_modules(replacements) -> None:
    for parent, name, original in reversed(replacements):
        setattr(parent, name, original)
