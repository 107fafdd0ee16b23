"""One-request views (request_views.py:18-49 of the reference; its tests/test_request_views.py:51-127).

The expected tuple is written out per field from the reference contract: token,
hidden and seen are the state's own tensors; draws = uniforms row ``frame``;
text = trailing column ``frame`` while the text lasts, else the pad row; the
next uniform = uniforms[frame + 1, 0]; then position, rotary position (3 x 1 x 1
broadcast) and step = frame + 1 as int64 tensors sharing one storage.
"""
import subprocess
import sys
from types import SimpleNamespace
from unittest.mock import patch

import pytest
import torch

from qwen3_tts_b200.request_views import single_request_inputs


def make_state(dtype=torch.bfloat16, strided=False, seed=42):
    step = 2 if strided else 1
    g = torch.Generator().manual_seed(seed)
    uniforms = torch.zeros(129, 16 * step)
    uniforms[:, ::step] = torch.rand(129, 16, generator=g)
    return SimpleNamespace(
        token=torch.tensor([[seed]]),
        hidden=torch.randn(1, 1, 12 * step, generator=g).to(dtype)[..., ::step],
        uniforms=uniforms[:, ::step],
        trailing=torch.randn(1, 3, 12 * step, generator=g).to(dtype)[..., ::step],
        pad=torch.randn(1, 1, 12 * step, generator=g).to(dtype)[..., ::step],
        seen=torch.zeros(1, 31 * step, dtype=torch.bool)[:, ::step],
        frames=0, position=123 + seed, rope_delta={17: -13, 42: 0, 43: 17}[seed])


def expected(state):
    f = state.frames
    text = state.trailing[:, f:f + 1] if f < state.trailing.shape[1] else state.pad
    return (state.token, state.hidden, state.uniforms[f:f + 1], text, state.uniforms[f + 1:f + 2, 0],
            state.seen, torch.tensor([state.position]),
            torch.full((3, 1, 1), state.position + state.rope_delta), torch.tensor([f + 1]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("strided", [False, True])
@pytest.mark.parametrize("seed", [17, 42, 43])
def test_boundary_frames_match_contract(dtype, strided, seed):
    state = make_state(dtype, strided, seed)
    before = {k: getattr(state, k).clone() for k in ("token", "hidden", "uniforms", "trailing", "pad", "seen")}
    for frame in (0, 1, 2, 7, 63, 127):
        state.frames = frame
        got = single_request_inputs(state)
        want = expected(state)
        assert len(got) == len(want) == 9
        for a, b in zip(got, want):
            assert a.shape == b.shape and a.dtype == b.dtype and torch.equal(a, b)
    for k, v in before.items():   # the views never write their sources
        assert torch.equal(getattr(state, k), v)


def test_views_borrow_sources_and_copies_stay_owned():
    state = make_state(strided=True)
    views = single_request_inputs(state)
    assert views.tokens is state.token and views.hidden is state.hidden and views.seen is state.seen
    owned = [x.clone() for x in views]
    state.hidden.add_(3)
    state.uniforms.add_(0.01)
    state.seen.fill_(True)
    state.frames, state.position = 7, state.position + 7
    single_request_inputs(state)
    assert torch.equal(views.hidden, state.hidden)          # borrowed: sees the change
    assert torch.equal(views.draws, state.uniforms[:1])
    assert not torch.equal(owned[1], state.hidden)         # owned copies keep the old values


def test_integers_share_one_storage_and_broadcast():
    state = make_state()
    state.position, state.rope_delta = 1 << 40, -(1 << 35)
    views = single_request_inputs(state)
    ints = (views.positions, views.rotary, views.steps)
    assert len({x.untyped_storage().data_ptr() for x in ints}) == 1
    assert all(x.dtype == torch.long for x in ints)
    assert views.rotary.shape == (3, 1, 1)
    assert views.rotary.flatten().tolist() == [state.position + state.rope_delta] * 3
    assert views.positions.item() == state.position and views.steps.item() == 1


def test_invalid_frames_raise_before_any_upload():
    state = make_state()
    with patch("torch.tensor") as upload:
        for frame in (-1, 128, True, 1.0):
            state.frames = frame
            with pytest.raises(ValueError):
                single_request_inputs(state)
        upload.assert_not_called()


def test_module_imports_without_torch():
    code = ("import builtins, sys\n"
            "real = builtins.__import__\n"
            "def guard(name, *a, **k):\n"
            "    if name.split('.')[0] in ('torch', 'numpy'):\n"
            "        raise ImportError(name)\n"
            "    return real(name, *a, **k)\n"
            "builtins.__import__ = guard\n"
            "import importlib.util\n"
            "spec = importlib.util.spec_from_file_location('rv', sys.argv[1])\n"
            "module = importlib.util.module_from_spec(spec); spec.loader.exec_module(module)\n"
            "print(module.single_request_inputs.__name__)\n")
    import qwen3_tts_b200.request_views as rv
    out = subprocess.run([sys.executable, "-c", code, rv.__file__], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "single_request_inputs"


def test_views_match_the_reference_fixture():
    """The state tests/golden/make_golden.py gave the reference's single_request_inputs."""
    from pathlib import Path
    import json
    import numpy as np
    golden = Path(__file__).resolve().parent / "golden"
    arrays = np.load(golden / "decode_path.npz")
    meta = json.loads((golden / "decode_path.json").read_text())
    g = torch.Generator().manual_seed(42)
    state = SimpleNamespace(token=torch.tensor([[42]]), hidden=torch.randn(1, 1, 12, generator=g),
                            uniforms=torch.rand(129, 16, generator=g), trailing=torch.randn(1, 3, 12, generator=g),
                            pad=torch.randn(1, 1, 12, generator=g), seen=torch.zeros(1, 31, dtype=torch.bool),
                            frames=2, position=165, rope_delta=-13)
    views = single_request_inputs(state)
    assert np.array_equal(views.draws.numpy(), arrays["views_draws"])
    assert np.array_equal(views.text.numpy(), arrays["views_text"])
    assert np.array_equal(views.uniforms.numpy(), arrays["views_uniforms"])
    assert [int(views.positions[0]), int(views.rotary[0, 0, 0]), int(views.steps[0])] == meta["views_integers"]
