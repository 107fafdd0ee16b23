"""Read-only one-request views (request_views.py:6-49 of the reference engine).

With device-resident slot state the tick graph gathers every row on the GPU,
so this view is only the reference's B=1 contract: borrowed tensors plus one
upload of the three integers (position, rotary position, step)."""
from __future__ import annotations

from typing import NamedTuple


class SingleRequestInputs(NamedTuple):
    tokens: object
    hidden: object
    draws: object
    text: object
    uniforms: object
    seen: object
    positions: object
    rotary: object
    steps: object


def single_request_inputs(state):
    """Views of one RequestState-like object (fields token, hidden, uniforms, trailing, pad,
    seen, frames, position, rope_delta); raises ValueError if the frame has no current and
    next uniform row."""
    import torch

    frame = state.frames
    if type(frame) is not int or not 0 <= frame < state.uniforms.shape[0] - 1:
        raise ValueError("Expected a frame with current and next uniform rows")
    integers = torch.tensor([state.position, state.position + state.rope_delta, frame + 1],
                            device=state.token.device, dtype=torch.long)
    text = state.trailing[:, frame:frame + 1] if frame < state.trailing.shape[1] else state.pad
    return SingleRequestInputs(state.token, state.hidden, state.uniforms[frame:frame + 1], text,
                               state.uniforms[frame + 1:frame + 2, 0], state.seen, integers[:1],
                               integers[1:2].view(1, 1, 1).expand(3, -1, -1), integers[2:3])
