"""The allocation-free attention entry point matches the workspace entry point.

`q3t_decode_attention_noalloc` serves callers that cannot allocate device
memory (a runtime with a fixed pre-reserved pool, a foreign-language host with
no CUDA allocator): its split-KV scratch is a fixed 4 MiB device array inside
the library instead of a caller workspace. This test calls both entry points
through the C ABI on the same inputs, twice in a row, and compares the outputs
within the attention tolerance used by the other parity tests (2e-2 absolute on
bf16).

The array keeps the previous call's contents, so the second call must reuse it
for real: the first call spreads contexts over the whole arena (up to five
512-key chunks per row, so rows merge partials through tickets), the second
uses contexts of 600-1499 keys (two or three chunks per row, still merging, but
over a smaller range of partial slots) — stale tickets or partials of the first
call would corrupt it.

The file name sorts last so a run that stops at its first failure has already
run every other test.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def _noalloc(lib, q, k, v, pos, out, context, rows_per_slot=1, arena_slots=None, status=None):
    rows, q_heads, head_dim = q.shape
    slots, kv_heads, capacity, _ = k.shape
    return lib.q3t_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), out.data_ptr(),
                                            rows, rows_per_slot, q_heads, kv_heads, head_dim,
                                            slots if arena_slots is None else arena_slots, capacity, context, 0,
                                            head_dim ** -0.5, None if status is None else status.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)


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
    rc = _noalloc(lib, q, k, v, pos, out, context, status=status)
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
    # 32 rows x 8 heads over 2304 keys: 512-key chunks, five per full row
    first = torch.randint(0, capacity, (slots,), generator=gen)
    first[0] = capacity - 1                                   # at least one row spans every chunk
    second = torch.randint(600, 1500, (slots,), generator=gen)  # 2-3 chunks: merges over fewer partial slots
    for positions in (first, second):
        ref, out = _call_both(lib, q, k, v, positions.to(cuda), capacity)
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=0)


def test_noalloc_attention_rejects_oversized_calls_before_launch(cuda):
    from qwen3_tts_b200 import _lib
    lib = _lib.load()
    # too many tickets: 2048 rows x 16 kv heads > 16384
    rows, kv_heads, q_heads, head_dim, capacity = 2048, 16, 16, 128, 8
    k = torch.zeros(rows, kv_heads, capacity, head_dim, dtype=BF16, device=cuda)
    q = torch.zeros(rows, q_heads, head_dim, dtype=BF16, device=cuda)
    out = torch.zeros_like(q)
    pos = torch.zeros(rows, dtype=torch.long, device=cuda)
    assert _noalloc(lib, q, k, k, pos, out, capacity) == _lib.Q3T_ESPACE
    assert "static scratch" in lib.q3t_last_error().decode()
    # tickets fit (16 x 8 = 128) but the partials do not: 64 chunks of 512 keys x 128 tickets
    # x 2 x 130 floats = 8.5 MB > 4 MiB
    rows, kv_heads, capacity = 16, 8, 32768
    k = torch.zeros(rows, kv_heads, capacity, head_dim, dtype=BF16, device=cuda)
    q = torch.zeros(rows, q_heads, head_dim, dtype=BF16, device=cuda)
    out = torch.zeros_like(q)
    pos = torch.full((rows,), capacity - 1, dtype=torch.long, device=cuda)
    assert _noalloc(lib, q, k, k, pos, out, capacity) == _lib.Q3T_ESPACE
    assert "partial bytes" in lib.q3t_last_error().decode()


def test_noalloc_attention_rejects_rows_beyond_the_arena(cuda):
    from qwen3_tts_b200 import _lib
    lib = _lib.load()
    k = torch.zeros(4, 8, 64, 128, dtype=BF16, device=cuda)
    q = torch.zeros(8, 16, 128, dtype=BF16, device=cuda)
    out = torch.zeros_like(q)
    pos = torch.zeros(8, dtype=torch.long, device=cuda)
    # 8 query rows, one per slot, but the arena holds 4 slots
    assert _noalloc(lib, q, k, k, pos, out, 64) == _lib.Q3T_EINVAL
    assert "arena slots" in lib.q3t_last_error().decode()
    # two rows per slot fit
    assert _noalloc(lib, q, k, k, pos, out, 64, rows_per_slot=2) == 0, lib.q3t_last_error()
    torch.cuda.synchronize()
