"""The allocation-free attention entry point matches the workspace entry point.

`q3t_decode_attention_noalloc` serves callers that cannot allocate device
memory (a runtime with a fixed pre-reserved pool, a foreign-language host with
no CUDA allocator): its split-KV scratch is a fixed 4 MiB device array inside
the library instead of a caller workspace. This test calls both entry points
through the C ABI on the same inputs, twice in a row with different positions
(the array keeps the previous call's contents, so the second call checks that
stale tickets and partials do not leak), and compares the outputs within the
attention tolerance used by the other parity tests (2e-2 absolute on bf16).

The file name sorts last so a run that stops at its first failure has already
run every other test.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def _call_both(lib, q, k, v, pos, context):
    from qwen3_tts_b200 import ops
    rows, q_heads, head_dim = q.shape
    slots, kv_heads, capacity, _ = k.shape
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(4, dtype=torch.int32, device=q.device)
    ref = torch.empty_like(q)
    need = ops.decode_attention_workspace_bytes(rows, q_heads, head_dim, context)
    workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
    rc = lib.q3t_decode_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), ref.data_ptr(), rows, 1,
                                  None, 0, q_heads, kv_heads, head_dim, slots, capacity, context, 0,
                                  head_dim ** -0.5,
                                  workspace.data_ptr(), workspace.numel(), status.data_ptr(), stream)
    assert rc == 0
    out = torch.full_like(q, float("nan"))
    rc = lib.q3t_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), out.data_ptr(),
                                          rows, 1, q_heads, kv_heads, head_dim, capacity, context, 0,
                                          head_dim ** -0.5, status.data_ptr(), stream)
    assert rc == 0, lib.q3t_last_error()
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    return ref, out


def test_noalloc_attention_matches_workspace_entry_point_twice(cuda):
    from qwen3_tts_b200 import _lib
    lib = _lib.load()
    gen = torch.Generator(device="cpu").manual_seed(1234)
    slots, kv_heads, q_heads, head_dim, capacity = 32, 8, 16, 128, 2304
    k = torch.randn(slots, kv_heads, capacity, head_dim, generator=gen).to(BF16).to(cuda)
    v = torch.randn(slots, kv_heads, capacity, head_dim, generator=gen).to(BF16).to(cuda)
    q = torch.randn(slots, q_heads, head_dim, generator=gen).to(BF16).to(cuda)
    first = torch.randint(0, capacity, (slots,), generator=gen)
    second = torch.randint(0, 300, (slots,), generator=gen)  # fewer chunks: stale state must not leak
    for positions in (first, second):
        ref, out = _call_both(lib, q, k, v, positions.to(cuda), capacity)
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=0)


def test_noalloc_attention_rejects_oversized_calls_before_launch(cuda):
    from qwen3_tts_b200 import _lib
    lib = _lib.load()
    rows, kv_heads, q_heads, head_dim, capacity = 2048, 16, 16, 128, 8
    k = torch.zeros(rows, kv_heads, capacity, head_dim, dtype=BF16, device=cuda)
    q = torch.zeros(rows, q_heads, head_dim, dtype=BF16, device=cuda)
    out = torch.zeros_like(q)
    pos = torch.zeros(rows, dtype=torch.long, device=cuda)
    rc = lib.q3t_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), k.data_ptr(), pos.data_ptr(), out.data_ptr(),
                                          rows, 1, q_heads, kv_heads, head_dim, capacity, capacity, 0, 0.088, None,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.Q3T_ESPACE
    assert "static scratch" in lib.q3t_last_error().decode()
