"""Parity of each CUDA kernel (through the C ABI) with the CPU oracle.

Integer / copy / index work is compared bit-exactly. Floating-point kernels
state their tolerance next to the assertion.
"""
import math

import numpy as np
import pytest
import torch

from oracle import elementwise as E
from oracle import kv as KV
from oracle import sampling as S
from tests.golden.inputs import bf16_scores, normal, uniform

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


@pytest.fixture(scope="module")
def ops(cuda):
    from qwen3_tts_b200 import ops as _ops
    return _ops


def rnd(seed, shape, scale=1.0, dtype=torch.float32):
    return torch.from_numpy(normal(seed, shape, scale)).to(dtype)


def assert_status_clean(ops, dev):
    assert ops.read_status(dev) == 0


# ------------------------------------------------------------------ KV arena
@pytest.mark.parametrize("dtype", [BF16, torch.float32])
@pytest.mark.parametrize("strided", [False, True])
def test_kv_write_exact(ops, cuda, dtype, strided):
    B, H, S_, D = 6, 8, 97, 128
    arena_k = rnd(1, (B, H, S_, D), dtype=dtype)
    arena_v = rnd(2, (B, H, S_, D), dtype=dtype)
    if strided:  # K/V as views of one packed QKV projection [B, 1, (16+8+8)*D]
        packed = rnd(3, (B, 1, 32 * D), dtype=dtype)
        k = packed[..., 16 * D:24 * D].view(B, 1, H, D).transpose(1, 2)
        v = packed[..., 24 * D:].view(B, 1, H, D).transpose(1, 2)
    else:
        k, v = rnd(4, (B, H, 1, D), dtype=dtype), rnd(5, (B, H, 1, D), dtype=dtype)
    pos = torch.tensor([0, 96, 13, 1, 50, 95])
    ek, ev = arena_k.clone(), arena_v.clone()
    KV.kv_write(k, v, ek, ev, pos)
    gk, gv = arena_k.to(cuda), arena_v.to(cuda)
    ops.kv_write(k.to(cuda), v.to(cuda), gk, gv, pos.to(cuda))
    assert torch.equal(gk.cpu(), ek) and torch.equal(gv.cpu(), ev)
    assert_status_clean(ops, cuda)


def test_kv_write_out_of_range_position_is_skipped_and_flagged(ops, cuda):
    arena = torch.zeros(2, 2, 8, 16, dtype=BF16, device=cuda)
    k = torch.ones(2, 2, 1, 16, dtype=BF16, device=cuda)
    ops.kv_write(k, k, arena, arena.clone(), torch.tensor([3, 8], device=cuda))
    assert arena[0, :, 3].eq(1).all() and arena[1].eq(0).all()
    assert ops.read_status(cuda) & 8


def test_kv_write_rejects_bad_layout_before_launch(ops, cuda):
    arena = torch.zeros(2, 2, 8, 16, dtype=BF16, device=cuda)
    k = torch.ones(2, 2, 1, 16, dtype=BF16, device=cuda)
    with pytest.raises(ValueError):
        ops.kv_write(k, k, arena, arena, torch.tensor([1, 2], dtype=torch.int32, device=cuda))
    with pytest.raises(ValueError):
        ops.kv_write(k, k[:, :1], arena, arena, torch.tensor([1, 2], device=cuda))


@pytest.mark.parametrize("dtype", [BF16, torch.float32, torch.int64])
def test_copy_packed_prefix_exact(ops, cuda, dtype):
    target = torch.full((4, 5, 2, 7, 3), -7).to(dtype)
    source = torch.arange(4 * 3 * 2 * 5 * 6).view(4, 3, 2, 5, 6).to(dtype)[..., ::2]
    gt, gs = target.to(cuda), source.to(cuda)
    for row, slot, length in ((2, 3, 1), (0, 1, 5), (1, 4, 3)):
        KV.copy_packed_prefix(target, source, slot, row=row, length=length)
        ops.copy_packed_prefix(gt, gs, slot, row=row, length=length)
    assert torch.equal(gt.cpu(), target)
    saved = gt.clone()
    for slot, row, length in ((-1, 0, 1), (5, 0, 1), (0, 3, 1), (0, 0, 0), (0, 0, 6), (True, 0, 1)):
        with pytest.raises(ValueError):
            ops.copy_packed_prefix(gt, gs, slot, row=row, length=length)
    assert torch.equal(gt, saved)


def test_slot_move_zero_and_growth_exact(ops, cuda):
    packed = rnd(7, (6, 4, 2, 33, 16), dtype=BF16)
    g = packed.to(cuda)
    ops.slot_move(g, 3, 1, dim=1)
    packed[:, 1] = packed[:, 3]
    assert torch.equal(g.cpu(), packed)
    ops.slot_zero(g, 2, 2, dim=1)
    packed[:, 2:4] = 0
    assert torch.equal(g.cpu(), packed)
    big = torch.zeros(6, 4, 2, 66, 16, dtype=BF16, device=cuda)
    ops.copy_prefix_along(big, g, dim=3)
    assert torch.equal(big[:, :, :, :33].cpu(), packed) and big[:, :, :, 33:].eq(0).all()
    frames = torch.arange(8, device=cuda)
    ops.slot_move(frames, 7, 0)
    assert frames.tolist() == [7, 1, 2, 3, 4, 5, 6, 7]


# ------------------------------------------------------------------ elementwise
@pytest.mark.parametrize("mode", ["reference", "native"])
@pytest.mark.parametrize("width", [128, 1024, 2048])
def test_rms_norm(ops, cuda, mode, width):
    from qwen3_tts_b200 import _lib
    x = rnd(8, (37, width), 2.0, BF16)
    w = (1 + rnd(9, (width,), 0.1)).to(BF16)
    ref = E.rms_norm(x, w, 1e-6, mode)
    out = ops.rms_norm(x.to(cuda), w.to(cuda), 1e-6, _lib.NORM_REFERENCE if mode == "reference" else _lib.NORM_NATIVE)
    # bf16 output; the fp32 sum-of-squares order differs -> at most one bf16 ulp
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=0, rtol=2 ** -7)
    assert (out.cpu().float() == ref.float()).float().mean() > 0.97


def test_add_rms_norm(ops, cuda):
    a, h = rnd(10, (9, 2048), 1.0, BF16), rnd(11, (9, 2048), 1.0, BF16)
    w = (1 + rnd(12, (2048,), 0.1)).to(BF16)
    for mode in ("native", "reference"):
        from qwen3_tts_b200 import _lib
        ref_n, ref_r = E.add_rms_norm(a, h, w, 1e-6, mode)
        n, r = ops.add_rms_norm(a.to(cuda), h.to(cuda), w.to(cuda), 1e-6,
                                _lib.NORM_NATIVE if mode == "native" else _lib.NORM_REFERENCE)
        assert torch.equal(r.cpu().float(), ref_r)
        torch.testing.assert_close(n.cpu().float(), ref_n.float(), atol=0, rtol=2 ** -7)


@pytest.mark.parametrize("heads,width", [(16, 128), (8, 128), (8, 64)])
def test_rotary_bit_exact(ops, cuda, heads, width):
    x = rnd(13, (3, 5, heads, width), 1.0, BF16)
    phase = rnd(14, (3, 5, width // 2), 3.0).repeat(1, 1, 2)
    cos, sin = phase.cos().to(BF16), phase.sin().to(BF16)
    ref = E.rotary_bf16(x, cos, sin)
    out = ops.rotary(x.to(cuda), cos.to(cuda), sin.to(cuda))
    assert torch.equal(out.cpu(), ref)  # products and sums of bf16 are exact in fp32
    with pytest.raises(ValueError):
        ops.rotary(x.to(cuda)[..., :3, :], cos.to(cuda), sin.to(cuda))


def test_swiglu(ops, cuda):
    packed = rnd(15, (33, 2 * 6144), 2.0, BF16)
    ref = E.swiglu(packed)
    out = ops.swiglu(packed.to(cuda))
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=1e-6, rtol=2 ** -7)


@pytest.mark.parametrize("dtype", [BF16, torch.float32])
@pytest.mark.parametrize("shape", [(4, 1536, 32), (4, 96, 15360), (1, 16, 2)])
def test_snake(ops, cuda, dtype, shape):
    x = rnd(16, shape, 2.0, dtype)
    alpha = torch.from_numpy(0.5 + uniform(17, (shape[1],)))
    inv = 1.0 / (torch.exp(rnd(18, (shape[1],), 0.3)) + 1e-9)
    ref = E.snake(x, alpha, inv)
    out = ops.snake(x.to(cuda), alpha.to(cuda), inv.to(cuda))
    if dtype == BF16:
        # sinf vs the CPU sin may differ by an ulp before the bf16 rounding
        torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2 ** -8, rtol=2 ** -7)
        assert (out.cpu().float() == ref.float()).float().mean() > 0.99
    else:
        torch.testing.assert_close(out.cpu(), ref, atol=1e-5, rtol=1e-5)


def test_scatter_rows_exact(ops, cuda):
    target = rnd(19, (8, 3, 5, 4), dtype=BF16)
    source_full = rnd(20, (3, 3, 10, 4), dtype=BF16)
    source = source_full[:, :, ::2]  # strided
    idx = torch.tensor([6, 0, 3])
    ref = target.clone()
    E.scatter_rows(ref, idx, source)
    g = target.to(cuda)
    ops.scatter_rows(g, idx.to(cuda), source_full.to(cuda)[:, :, ::2])
    assert torch.equal(g.cpu(), ref)
    frames = torch.zeros(8, dtype=torch.long, device=cuda)
    ops.scatter_rows(frames, torch.tensor([2, 5], device=cuda), torch.tensor([7, 9], device=cuda))
    assert frames.tolist() == [0, 0, 7, 0, 0, 9, 0, 0]
    with pytest.raises(ValueError):
        ops.scatter_rows(g, idx.to(cuda), g[:3])  # aliasing source


def test_frame_embed_and_embedding_exact(ops, cuda):
    first = rnd(21, (3072, 256), 0.02, BF16)
    groups = rnd(22, (15, 2048, 256), 0.02, BF16)
    codes = torch.cat([torch.from_numpy((uniform(23, (9, 1)) * 3072).astype(np.int64)),
                       torch.from_numpy((uniform(24, (9, 15)) * 2048).astype(np.int64))], dim=1)
    text = rnd(25, (9, 256), 0.05, BF16)
    ref = E.frame_embed(codes, first, groups, text)
    out = ops.frame_embed(codes.to(cuda), first.to(cuda), groups.to(cuda), text.to(cuda))
    assert torch.equal(out.cpu(), ref)
    emb = ops.embedding(codes[:, 0].contiguous().to(cuda), first.to(cuda))
    assert torch.equal(emb.cpu(), first[codes[:, 0]])


# ------------------------------------------------------------------ GEMM
def torch_linear(x, w, bias=None):
    y = x.float() @ w.float().T
    return y if bias is None else y + bias.float()


@pytest.mark.parametrize("rows", [1, 7, 16, 32, 33, 64, 100, 256, 300])
@pytest.mark.parametrize("k,n", [(2048, 4096), (2048, 2048), (6144, 2048), (1024, 2048), (96, 200)])
def test_linear_store_bf16(ops, cuda, rows, k, n):
    x = rnd(30 + rows, (rows, k), 1.0, BF16)
    w = rnd(31 + n, (n, k), 0.02, BF16)
    ref = torch_linear(x, w)
    out = ops.linear(x.to(cuda), w.to(cuda))
    # bf16 output of an fp32-accumulated dot product: one bf16 rounding plus order effects
    torch.testing.assert_close(out.cpu().float(), ref, atol=2e-3 * math.sqrt(k / 64), rtol=1e-2)
    assert_status_clean(ops, cuda)


@pytest.mark.parametrize("rows,k,n", [(1, 2048, 4096), (32, 2048, 12288), (33, 6144, 2048), (64, 96, 200),
                                      (300, 1024, 2048)])
def test_linear_tiled_weights_equal_row_major(ops, cuda, rows, k, n):
    from qwen3_tts_b200 import _lib
    x = rnd(35, (rows, k), 1.0, BF16).to(cuda)
    w = rnd(36, (n, k), 0.02, BF16).to(cuda)
    tiled = ops.pack_tiles(w)
    ref = ops.linear(x, w, out_dtype=torch.float32)
    got = ops.linear(x, tiled, out_dtype=torch.float32)
    assert torch.equal(got, ref)  # same tiles, same MMA order: bit-identical
    if n % 128 == 0:
        got = ops.linear(x, tiled, epilogue=_lib.EPI_SWIGLU_PAIRED)
        assert torch.equal(got, ops.linear(x, w, epilogue=_lib.EPI_SWIGLU_PAIRED))


def test_linear_fp32_bias_residual_and_strided_input(ops, cuda):
    from qwen3_tts_b200 import _lib
    rows, k, n = 24, 2048, 3072
    base = rnd(40, (rows, k + 64), 1.0, BF16)
    x = base[:, 32:32 + k]  # row stride k+64, 64-byte offset
    w = rnd(41, (n, k), 0.02, BF16)
    b = rnd(42, (n,), 0.1, BF16)
    out = ops.linear(base.to(cuda)[:, 32:32 + k], w.to(cuda), b.to(cuda), out_dtype=torch.float32)
    ref = torch_linear(x, w, b)
    torch.testing.assert_close(out.cpu(), ref, atol=3e-3, rtol=1e-2)
    res = rnd(43, (rows, n), 1.0, BF16)
    out = ops.linear(x.contiguous().to(cuda), w.to(cuda), epilogue=_lib.EPI_RESIDUAL, residual=res.to(cuda))
    ref = (res.float() + torch_linear(x, w).to(BF16).float()).to(BF16)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("rows,k,n", [(32, 1024, 4096), (5000, 192, 192), (7680, 96, 96)])
def test_linear_inplace_residual_and_l2_prefetch(ops, cuda, rows, k, n):
    """In-place residual epilogue (out aliases the residual, as the codec's residual units and the
    decoder's O/down projections run it) against the fp32 reference, and q3t_linear_ex
    (next weights pulled into L2) bit-identical to the plain GEMM, with and without the row norm."""
    from qwen3_tts_b200 import _lib
    x = rnd(60 + rows, (rows, k), 1.0, BF16)
    w = rnd(61, (n, k), 0.02, BF16)
    res = rnd(62, (rows, n), 1.0, BF16)
    ref = (res.float() + torch_linear(x, w).to(BF16).float()).to(BF16)
    xd, wd, nxt = x.to(cuda), ops.pack_tiles(w.to(cuda)), ops.pack_tiles(rnd(63, (2048, 1024), 0.02, BF16).to(cuda))
    y = res.to(cuda)
    ops.linear(xd, wd, out=y, epilogue=_lib.EPI_RESIDUAL, residual=y)
    torch.testing.assert_close(y.cpu().float(), ref.float(), atol=2e-2, rtol=1e-2)
    y2 = res.to(cuda)
    ops.linear(xd, wd, out=y2, epilogue=_lib.EPI_RESIDUAL, residual=y2, prefetch=nxt)
    assert torch.equal(y, y2)
    a = ops.linear(xd, wd, out_dtype=torch.float32, row_norm_eps=1e-6)
    b = ops.linear(xd, wd, out_dtype=torch.float32, row_norm_eps=1e-6, prefetch=nxt)
    assert torch.equal(a, b)
    assert_status_clean(ops, cuda)


@pytest.mark.parametrize("batch,frames,C,N,taps,dil,reverse", [
    (2, 40, 128, 256, 7, 3, False), (3, 300, 96, 96, 7, 9, False), (2, 64, 192, 384, 2, 1, True),
    (1, 5, 512, 1024, 3, 1, False), (4, 700, 16, 1, 7, 1, False), (2, 1100, 32, 64, 7, 1, False)])
def test_conv_linear_matches_gather_then_linear(ops, cuda, batch, frames, C, N, taps, dil, reverse):
    """Implicit-GEMM causal conv (q3t_conv_pad + q3t_conv_linear: tap-shifted 3-D TMA rows of the
    padded buffer, channels zero-padded to 64 per tap) against im2col (q3t_conv_gather) + GEMM, with
    per-slot histories, SnakeBeta on the input, and the STORE / RESIDUAL / SNAKE epilogues."""
    from qwen3_tts_b200 import _lib
    H = (taps - 1) * dil
    x = rnd(80 + frames, (batch * frames, C), 1.0, BF16).to(cuda)
    hist = rnd(81, (batch + 2, H, C), 1.0, BF16).to(cuda)
    slots = torch.tensor(list(range(batch + 1, 0, -1))[:batch], dtype=torch.long, device=cuda)
    alpha = (0.5 + torch.rand(C, generator=torch.Generator().manual_seed(82))).to(cuda)
    inv = (0.5 + torch.rand(C, generator=torch.Generator().manual_seed(83))).to(cuda)
    w = rnd(84, (N, taps * C), 0.05, BF16).to(cuda)
    bias = rnd(85, (N,), 0.1, BF16).to(cuda)
    col = ops.conv_gather(x, batch, frames, taps=taps, dilation=dil, reverse=reverse, history=hist, slots=slots,
                          alpha=alpha, inverse_beta=inv)
    ref32 = col.float() @ w.float().T + bias.float()
    xs = ops.conv_pad(x, batch, frames, history=hist, slots=slots, alpha=alpha, inverse_beta=inv)
    tiles = ops.conv_weight_tiles(w, taps)
    got = ops.conv_linear(xs, batch, frames, H, tiles, taps=taps, dilation=dil, reverse=reverse, bias=bias)
    k = taps * C
    torch.testing.assert_close(got.float(), ref32, atol=2e-3 * math.sqrt(k / 64) + 1e-2, rtol=1e-2)
    res = rnd(86, (batch * frames, N), 1.0, BF16).to(cuda)
    y = res.clone()
    ops.conv_linear(xs, batch, frames, H, tiles, taps=taps, dilation=dil, reverse=reverse, bias=bias, out=y,
                    epilogue=_lib.EPI_RESIDUAL, residual=y)
    assert torch.equal(y, (res.float() + got.float()).to(BF16))
    a2 = (0.5 + torch.rand(N, generator=torch.Generator().manual_seed(87))).to(cuda)
    i2 = (0.5 + torch.rand(N, generator=torch.Generator().manual_seed(88))).to(cuda)
    snaked = ops.conv_linear(xs, batch, frames, H, tiles, taps=taps, dilation=dil, reverse=reverse, bias=bias,
                             epilogue=_lib.EPI_SNAKE, snake=(a2, i2))
    if N % 8 == 0:  # the same SnakeBeta applied by the gather to the stored conv output
        assert torch.equal(snaked, ops.conv_gather(got, batch, frames, taps=1, alpha=a2, inverse_beta=i2))
    assert_status_clean(ops, cuda)


@pytest.mark.parametrize("rows", [1, 32, 64, 130])
def test_linear_paired_swiglu(ops, cuda, rows):
    from qwen3_tts_b200 import _lib
    from qwen3_tts_b200.weights import interleave_gate_up
    k, f = 2048, 6144
    x = rnd(50, (rows, k), 1.0, BF16)
    gate, up = rnd(51, (f, k), 0.02, BF16), rnd(52, (f, k), 0.02, BF16)
    packed = interleave_gate_up(gate, up)
    out = ops.linear(x.to(cuda), packed.to(cuda), epilogue=_lib.EPI_SWIGLU_PAIRED)
    g = torch_linear(x, gate).to(BF16)
    u = torch_linear(x, up).to(BF16)
    ref = E.swiglu(torch.cat([g, u], dim=-1))
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=1e-2, rtol=2e-2)


def _prefill_reference(q, k, v, positions, units, scale):
    """fp32 causal attention of every row a unit covers over keys 0..positions[r] of its slot."""
    out = {}
    qf, kf, vf = q.float(), k.float(), v.float()
    group = q.shape[1] // k.shape[1]
    for first, count, keys, slot in units.tolist():
        for r in range(first, first + count):
            p = int(positions[r])
            kk = kf[slot, :, :p + 1].repeat_interleave(group, 0)      # [Hq, p+1, D]
            vv = vf[slot, :, :p + 1].repeat_interleave(group, 0)
            w = torch.softmax((kk @ qf[r].unsqueeze(-1)).squeeze(-1) * scale, -1)
            out[r] = (w.unsqueeze(-1) * vv).sum(1)
    return out


@pytest.mark.parametrize("lengths", [[1], [5, 64, 65, 200], [129, 3, 300, 17]])
def test_prefill_attention_matches_fp32_causal_reference(ops, cuda, lengths):
    """The tcgen05 causal prefill attention (64-row query tiles x 64-key blocks, S and PV in
    TMEM, online softmax, MN-major V operand) over a packed unit table: ragged prompts in
    scattered slots, a single-token prompt, spans across 1..5 key blocks, and padding rows that
    repeat the last row."""
    from qwen3_tts_b200.batching import packed_rows, packed_tables, packed_units
    slots, kvh, cap, D = 6, 8, 320, 128
    total = sum(lengths)
    rows = packed_rows(total)
    k = rnd(300, (slots, kvh, cap, D), 1.0, BF16)
    v = rnd(301, (slots, kvh, cap, D), 1.0, BF16)
    q = rnd(302, (rows, 2 * kvh, D), 1.0, BF16)
    first_slot = 1
    _, positions, _ = packed_tables(lengths, first_slot, rows, 8)
    units = packed_units(lengths, first_slot, rows, 8)
    out = torch.full((rows, 2 * kvh, D), float("nan"), dtype=BF16, device=cuda)
    ops.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), positions.to(cuda), units.to(cuda), out=out)
    got = out.cpu().float()
    ref = _prefill_reference(q, k, v, positions, units, D ** -0.5)
    assert sorted(ref) == list(range(rows))           # every packed row, padding included
    want = torch.stack([ref[r] for r in range(rows)])
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)
    assert_status_clean(ops, cuda)


def test_prefill_attention_skips_units_out_of_range(ops, cuda):
    """A unit whose slot lies outside the arena is skipped with the bad-index status bit; the
    valid units of the same call still run."""
    k = rnd(310, (2, 8, 64, 128), 1.0, BF16).to(cuda)
    q = rnd(311, (64, 16, 128), 1.0, BF16).to(cuda)
    positions = torch.arange(64, dtype=torch.long, device=cuda) % 32
    units = torch.tensor([[0, 32, 32, 0], [32, 32, 32, 7], [0, 0, 0, 0]], dtype=torch.int32, device=cuda)
    out = torch.zeros(64, 16, 128, dtype=BF16, device=cuda)
    ops.read_status(cuda, clear=True)
    ops.prefill_attention(q, k, k, positions, units, out=out)
    status = ops.read_status(cuda, clear=True)
    assert status & ops.STATUS_BAD_INDEX
    assert out[:32].abs().sum() > 0 and not out[32:].any()


def _kernels_launched(fn):
    """Names of the CUDA kernels `fn` launches (torch profiler, CUPTI)."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}


@pytest.mark.parametrize("rows,k,n,epi", [(2085, 2048, 4096, "store"), (4096, 2048, 2048, "residual"),
                                          (1500, 2048, 12288, "swiglu"), (3000, 1000, 2000, "bias"),
                                          (2560, 6144, 2048, "scaled")])
def test_linear_wide_tiles_match_fp32_and_the_split_k_kernel(ops, cuda, rows, k, n, epi):
    """Prefill-sized row counts run the persistent 128 x 256 wide-tile kernel (two TMEM
    accumulators, 64-row TMA-stored chunks): ragged last row tile, K and N off the tile grid
    (zero-filled loads, clipped stores), an in-place residual, paired SwiGLU, bias and the
    scaled residual, against the fp32 reference and the split-K kernel (Q3T_LINEAR_NARROW)."""
    from qwen3_tts_b200 import _lib
    from qwen3_tts_b200.weights import interleave_gate_up
    x = rnd(90 + rows, (rows, k), 1.0, BF16)
    bias = scale = residual = None
    epilogue = _lib.EPI_STORE
    if epi == "swiglu":
        gate, up = rnd(91, (n // 2, k), 0.02, BF16), rnd(92, (n // 2, k), 0.02, BF16)
        w = interleave_gate_up(gate, up)
        ref = E.swiglu(torch.cat([torch_linear(x, gate).to(BF16), torch_linear(x, up).to(BF16)], dim=-1)).float()
        epilogue = _lib.EPI_SWIGLU_PAIRED
    else:
        w = rnd(93, (n, k), 0.02, BF16)
        acc = torch_linear(x, w)
        if epi == "bias":
            bias = rnd(94, (n,), 0.5, BF16)
            acc = acc + bias.float()
        ref = acc.to(BF16).float()
        if epi in ("residual", "scaled"):
            residual = rnd(95, (rows, n), 1.0, BF16)
            epilogue = _lib.EPI_RESIDUAL
            if epi == "scaled":
                scale = rnd(96, (n,), 0.5, BF16)
                ref = (scale.float() * ref).to(BF16).float()
                epilogue = _lib.EPI_RESIDUAL_SCALED
            ref = (residual.float() + ref).to(BF16).float()
    tiles = ops.pack_tiles(w.to(cuda))
    dev = lambda t: None if t is None else t.to(cuda)

    def run(narrow):
        # the residual epilogue runs in place (out aliases the residual), as the decoder layers do
        out = residual.clone().to(cuda) if epi == "residual" else None
        res = out if epi == "residual" else dev(residual)
        return ops.linear(x.to(cuda), tiles, dev(bias), out=out, epilogue=epilogue, residual=res, scale=dev(scale),
                          narrow=narrow)

    names = _kernels_launched(lambda: run(False))
    assert any("linear_wide_kernel" in name for name in names), names
    wide = run(False)
    narrow = run(True)
    torch.testing.assert_close(wide.cpu().float(), ref, atol=2e-2, rtol=2e-2)
    # same bf16 operands and fp32 accumulation; the two kernels differ at most by one rounding
    torch.testing.assert_close(wide.float(), narrow.float(), atol=1e-2, rtol=1e-2)
    assert_status_clean(ops, cuda)


@pytest.mark.parametrize("rows,k,n", [(1, 2048, 4096), (32, 2048, 4096), (32, 2048, 12288), (64, 1024, 2048),
                                      (100, 2048, 640), (300, 256, 1024)])
def test_linear_rownorm_equals_rmsnorm_then_linear(ops, cuda, rows, k, n):
    """The folded RMSNorm GEMM (norm weight premultiplied, row RMS taken from the streamed
    activation tiles, summed over the split-K cluster in rank order) against the fp32
    reference rsqrt(mean(x^2)+eps) * (x @ bf16(W*w)^T), for one-CTA and clustered splits,
    BN 16..256, and the STORE / RESIDUAL / paired-SwiGLU epilogues."""
    from qwen3_tts_b200 import _lib
    from qwen3_tts_b200.weights import fold_norm
    eps = 1e-6
    x = rnd(70 + rows, (rows, k), 1.0, BF16)
    w = rnd(71, (n, k), 0.02, BF16)
    g = (1.0 + rnd(72, (k,), 0.1, torch.float32)).to(BF16)
    folded = fold_norm(w, g)
    r = 1.0 / torch.sqrt(x.float().pow(2).mean(-1, keepdim=True) + eps)
    prod = (x.float() @ folded.float().T) * r
    out = ops.linear(x.to(cuda), ops.pack_tiles(folded.to(cuda)), row_norm_eps=eps)
    # bf16 output of an fp32-accumulated, fp32-scaled dot product: one rounding plus order effects
    torch.testing.assert_close(out.cpu().float(), prod, atol=2e-3 * math.sqrt(k / 64), rtol=1e-2)
    res = rnd(73, (rows, n), 1.0, BF16)
    out = ops.linear(x.to(cuda), folded.to(cuda), epilogue=_lib.EPI_RESIDUAL, residual=res.to(cuda), row_norm_eps=eps)
    ref = (res.float() + prod.to(BF16).float()).to(BF16)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-2, rtol=1e-2)
    if n % 128 == 0:
        out = ops.linear(x.to(cuda), folded.to(cuda), epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=eps)
        gate = prod.view(rows, n // 128, 2, 64)[:, :, 0].reshape(rows, n // 2).to(BF16)
        up = prod.view(rows, n // 128, 2, 64)[:, :, 1].reshape(rows, n // 2).to(BF16)
        ref = E.swiglu(torch.cat([gate, up], dim=-1))
        torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-2, rtol=2e-2)
    assert_status_clean(ops, cuda)


@pytest.mark.parametrize("rows,q_heads,kv_heads,head_dim,capacity,norms", [
    (32, 16, 8, 128, 2304, True), (5, 16, 8, 128, 128, True), (7, 8, 8, 128, 640, False), (4, 4, 2, 64, 300, True),
    (64, 16, 8, 128, 17, True)])
def test_fused_qkv_attention_equals_separate_kernels(ops, cuda, rows, q_heads, kv_heads, head_dim, capacity, norms):
    """q3t_decode_attention_qkv (q/k norm + RoPE + KV write inside the attention kernel)
    against q3t_qk_norm_rope_kv followed by q3t_decode_attention: the same per-op bf16
    rounding, so the outputs and the arena rows written are bit-identical."""
    from qwen3_tts_b200.talker import rope_tables
    gen = torch.Generator().manual_seed(rows * 7 + head_dim)
    width = (q_heads + 2 * kv_heads) * head_dim
    qkv = torch.randn(rows, width + 64, generator=gen).to(BF16).to(cuda)[:, :width]   # strided rows
    keys = torch.randn(rows, kv_heads, capacity, head_dim, generator=gen).to(BF16).to(cuda)
    values = torch.randn(rows, kv_heads, capacity, head_dim, generator=gen).to(BF16).to(cuda)
    positions = torch.randint(0, capacity, (rows,), generator=gen).to(cuda)
    positions[0] = 0
    positions[-1] = capacity - 1
    rotary = (positions + 3).contiguous()
    qn = (1 + 0.1 * torch.randn(head_dim, generator=gen)).to(BF16).to(cuda) if norms else None
    kn = (1 + 0.1 * torch.randn(head_dim, generator=gen)).to(BF16).to(cuda) if norms else None
    cos, sin = rope_tables(capacity + 8, head_dim, 1e6, cuda)
    k1, v1 = keys.clone(), values.clone()
    q = ops.qk_norm_rope_kv(qkv, qn, kn, 1e-6, cos, sin, rotary, positions, k1, v1, q_heads=q_heads,
                            kv_heads=kv_heads, head_dim=head_dim)
    ref = ops.decode_attention(q, k1, v1, positions, context=capacity)
    k2, v2 = keys.clone(), values.clone()
    got = ops.decode_attention_qkv(qkv, qn, kn, 1e-6, cos, sin, rotary, k2, v2, positions, q_heads=q_heads,
                                   kv_heads=kv_heads, head_dim=head_dim, context=capacity)
    torch.cuda.synchronize()
    assert torch.equal(k2, k1) and torch.equal(v2, v1)
    assert torch.equal(got, ref)
    # the L2 prefetch hint of q3t_decode_attention_qkv_ex (two weight ranges, one of them
    # tiled) changes nothing that the kernel computes or writes
    pf_a = torch.randn(3000, 64, generator=gen).to(BF16).to(cuda)
    pf_b = ops.pack_tiles(torch.randn(256, 128, generator=gen).to(BF16).to(cuda))
    k3, v3 = keys.clone(), values.clone()
    hinted = ops.decode_attention_qkv(qkv, qn, kn, 1e-6, cos, sin, rotary, k3, v3, positions, q_heads=q_heads,
                                      kv_heads=kv_heads, head_dim=head_dim, context=capacity, prefetch=(pf_a, pf_b))
    torch.cuda.synchronize()
    assert torch.equal(k3, k1) and torch.equal(v3, v1)
    assert torch.equal(hinted, ref)
    with pytest.raises(ValueError):
        ops.decode_attention_qkv(qkv, qn, kn, 1e-6, cos, sin, rotary, k3, v3, positions, q_heads=q_heads,
                                 kv_heads=kv_heads, head_dim=head_dim, context=capacity,
                                 prefetch=(pf_a, pf_a, pf_a))
    assert_status_clean(ops, cuda)


def test_attention_plan_changes_the_split_not_the_result(ops, cuda):
    """q3t_attention_plan writes a per-batch chunk size (one wave of resident CTAs) into the
    workspace; the decode attention then splits the keys differently, which only changes the
    fp32 merge order of the chunk partials (bf16 outputs within one rounding), and writes the
    same K/V rows."""
    from qwen3_tts_b200.talker import rope_tables
    rows, q_heads, kv_heads, head_dim, capacity = 32, 16, 8, 128, 4096
    gen = torch.Generator().manual_seed(91)
    width = (q_heads + 2 * kv_heads) * head_dim
    qkv = torch.randn(rows, width, generator=gen).to(BF16).to(cuda)
    keys = torch.randn(rows, kv_heads, capacity, head_dim, generator=gen).to(BF16).to(cuda)
    values = torch.randn(rows, kv_heads, capacity, head_dim, generator=gen).to(BF16).to(cuda)
    positions = torch.randint(64, 2049, (rows,), generator=gen).to(cuda)
    qn = (1 + 0.1 * torch.randn(head_dim, generator=gen)).to(BF16).to(cuda)
    kn = (1 + 0.1 * torch.randn(head_dim, generator=gen)).to(BF16).to(cuda)
    cos, sin = rope_tables(capacity, head_dim, 1e6, cuda)
    ws = torch.zeros(ops.decode_attention_workspace_bytes(rows, q_heads, head_dim, capacity), dtype=torch.uint8,
                     device=cuda)
    k0, v0 = keys.clone(), values.clone()
    base = ops.decode_attention_qkv(qkv, qn, kn, 1e-6, cos, sin, positions, k0, v0, positions, q_heads=q_heads,
                                    kv_heads=kv_heads, head_dim=head_dim, context=capacity, workspace=ws)
    ops.attention_plan(positions, ws, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim, context=capacity)
    planned = int(ws.view(torch.int32)[65535].item())
    assert planned >= 512 and planned % 64 == 0 and planned <= 2 * capacity
    k1, v1 = keys.clone(), values.clone()
    got = ops.decode_attention_qkv(qkv, qn, kn, 1e-6, cos, sin, positions, k1, v1, positions, q_heads=q_heads,
                                   kv_heads=kv_heads, head_dim=head_dim, context=capacity, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(k1, k0) and torch.equal(v1, v0)
    torch.testing.assert_close(got.float(), base.float(), atol=1e-2, rtol=1e-2)
    assert_status_clean(ops, cuda)


def test_linear_graph_replay_is_deterministic(ops, cuda):
    x = rnd(60, (32, 2048), 1.0, BF16).to(cuda)
    w = rnd(61, (6144, 2048), 0.02, BF16).to(cuda)
    out = torch.empty(32, 6144, dtype=BF16, device=cuda)
    ops.linear(x, w, out=out)
    first = out.clone()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.linear(x, w, out=out)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(graph, stream=s):
        ops.linear(x, w, out=out)
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, first)
    graph.reset()


def test_linear_rejects_bad_arguments(ops, cuda):
    from qwen3_tts_b200 import _lib
    x = torch.zeros(4, 100, dtype=BF16, device=cuda)
    w = torch.zeros(128, 100, dtype=BF16, device=cuda)
    with pytest.raises(ValueError):
        ops.linear(x, w)  # in_features not a multiple of 8
    with pytest.raises(ValueError):
        ops.linear(torch.zeros(4, 64, dtype=BF16, device=cuda), torch.zeros(100, 64, dtype=BF16, device=cuda),
                   epilogue=_lib.EPI_SWIGLU_PAIRED)


# ------------------------------------------------------------------ attention
def attention_case(cuda, B, Hq, Hkv, D, cap, positions, seed):
    keys = rnd(seed, (B, Hkv, cap, D), 1.0, BF16)
    values = rnd(seed + 1, (B, Hkv, cap, D), 1.0, BF16)
    q = rnd(seed + 2, (B, Hq, D), 1.0, BF16)
    pos = torch.tensor(positions)
    ref = KV.decode_attention(q, keys, values, pos)
    return ref, (q.to(cuda), keys.to(cuda), values.to(cuda), pos.to(cuda))


def test_decode_attention_config1(ops, cuda):
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(1, 513, (8,), generator=g)
    ref, args = attention_case(cuda, 8, 16, 8, 128, 513, lens.tolist(), 70)
    out = ops.decode_attention(*args)
    # bf16 output vs fp32 oracle on the same bf16 inputs (north-star bar 2e-2)
    torch.testing.assert_close(out.cpu().float(), ref, atol=2e-2, rtol=0)
    assert (out.cpu().float() - ref).abs().max() < 1e-2
    assert_status_clean(ops, cuda)


@pytest.mark.parametrize("B,Hq,Hkv,D,cap", [(32, 16, 8, 128, 2304), (64, 16, 8, 128, 1024), (3, 8, 8, 64, 143),
                                            (5, 16, 8, 128, 16), (2, 16, 8, 64, 300), (64, 16, 8, 128, 17),
                                            (7, 8, 8, 64, 64)])
def test_decode_attention_ragged(ops, cuda, B, Hq, Hkv, D, cap):
    """Ragged positions against the fp32 oracle; contexts of one 64-key tile (16, 17 - the code
    predictor's - and 64) take the one-stage kernel (four CTAs per SM), longer ones the two-stage."""
    pos = (uniform(80 + B, (B,)) * cap).astype(np.int64).clip(0, cap - 1)
    pos[0] = 0
    pos[-1] = cap - 1
    ref, args = attention_case(cuda, B, Hq, Hkv, D, cap, pos.tolist(), 90 + B)
    out = ops.decode_attention(*args)
    torch.testing.assert_close(out.cpu().float(), ref, atol=2e-2, rtol=0)
    # smaller context bucket: positions must stay below it
    ctx = int(pos.max()) + 1
    out2 = ops.decode_attention(*args, context=ctx)
    torch.testing.assert_close(out2.cpu().float(), ref, atol=2e-2, rtol=0)


def test_decode_attention_ignores_poisoned_tail(ops, cuda):
    ref, (q, k, v, pos) = attention_case(cuda, 4, 16, 8, 128, 200, [5, 63, 64, 130], 100)
    for b, p in enumerate(pos.tolist()):
        k[b, :, p + 1:] = float("nan")
        v[b, :, p + 1:] = float("inf")
    out = ops.decode_attention(q, k, v, pos)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.cpu().float(), ref, atol=2e-2, rtol=0)


def test_decode_attention_rows_per_slot_and_window(ops, cuda):
    # predictor first step: 2 query rows per slot at positions (0, 1) - a 2x2 causal mask
    B, Hq, Hkv, D, cap = 6, 16, 8, 128, 16
    keys = rnd(110, (B, Hkv, cap, D), 1.0, BF16)
    values = rnd(111, (B, Hkv, cap, D), 1.0, BF16)
    q = rnd(112, (2 * B, Hq, D), 1.0, BF16)
    pos = torch.tensor([0, 1] * B)
    ref = KV.decode_attention(q, keys, values, pos, rows_per_slot=2)
    out = ops.decode_attention(q.to(cuda), keys.to(cuda), values.to(cuda), pos.to(cuda), rows_per_slot=2)
    torch.testing.assert_close(out.cpu().float(), ref, atol=2e-2, rtol=0)
    # codec transformer: head_dim 64, 8 heads, sliding window 72 over a long history
    B, H, D, cap = 4, 8, 64, 300
    keys = rnd(113, (B, H, cap, D), 1.0, BF16)
    values = rnd(114, (B, H, cap, D), 1.0, BF16)
    q = rnd(115, (B * 3, H, D), 1.0, BF16)
    pos = torch.tensor([0, 50, 71, 72, 140, 299, 5, 100, 200, 71, 72, 73])
    ref = KV.decode_attention(q, keys, values, pos, rows_per_slot=3, window=72)
    out = ops.decode_attention(q.to(cuda), keys.to(cuda), values.to(cuda), pos.to(cuda), rows_per_slot=3, window=72)
    torch.testing.assert_close(out.cpu().float(), ref, atol=2e-2, rtol=0)


# ------------------------------------------------------------------ sampling
def boundary_free(tokens_a, tokens_b, limit=1):
    return int((tokens_a != tokens_b).sum()) <= limit


@pytest.mark.parametrize("seed,width", [(11, 3072), (12, 2048)])
def test_categorical_matches_oracle(ops, cuda, seed, width):
    scores = bf16_scores(seed, 256, width, 3.0)
    u = torch.from_numpy(uniform(seed + 100, (256,)))
    ref = S.categorical(scores, u)
    got = ops.sample(scores.to(cuda), uniforms=u.to(cuda)).cpu()
    # identical CDFs up to fp32 rounding of exp/sum order: a draw can flip only
    # when u lies within ~1e-6 of a CDF step (expected count << 1 here)
    assert boundary_free(got, ref)


def test_sample_boundary_cases(ops, cuda):
    scores = torch.tensor([[-float("inf"), 0.0, -float("inf"), 0.0]]).repeat(3, 1)
    draws = torch.tensor([0.0, 0.5, 1.0 - torch.finfo(torch.float32).eps])
    got = ops.sample(scores.to(cuda), uniforms=draws.to(cuda), top_k=2, temperature=0.9).flatten().tolist()
    assert got == [1, 3, 3]


def test_sample_frequencies_and_permutation_equivariance(ops, cuda):
    """p = (1/4, 3/4) over 10000 table draws: id 1 three times in four, equal to the oracle draw
    for draw, and permuting rows permutes the tokens."""
    draws = S.random_table(42, 1000).flatten()[:10000]
    scores = torch.tensor([[0.0, 1.0986122886681098]]).repeat(len(draws), 1)
    got = ops.sample(scores.to(cuda), uniforms=draws.to(cuda), temperature=1.0, top_k=2).flatten().cpu()
    ref = S.categorical(scores, draws, temperature=1.0, top_k=2).flatten()
    assert abs(got.float().mean().item() - 0.75) < 0.02
    assert boundary_free(got, ref)
    order = torch.randperm(len(draws), generator=torch.Generator().manual_seed(123))
    permuted = ops.sample(scores[order].to(cuda), uniforms=draws[order].to(cuda), temperature=1.0,
                          top_k=2).flatten().cpu()
    assert torch.equal(permuted, got[order])


def test_semantic_sampling_and_seen_update(ops, cuda):
    vocab, eos = 3072, 2150
    logits = bf16_scores(21, 128, vocab, 2.0).to(BF16)
    seen = torch.from_numpy(uniform(22, (128, vocab)) < 0.05)
    steps = torch.from_numpy((uniform(23, (128,)) * 5).astype(np.int64))
    u = torch.from_numpy(uniform(24, (128,)))
    allowed = S.allowed_mask(vocab, eos)
    ref_tokens, ref_seen = S.sampling_graph_step(logits, u, seen, steps, allowed, eos)
    seen_out = torch.empty(128, vocab, dtype=torch.bool, device=cuda)
    got = ops.sample(logits.to(cuda), uniforms=u.to(cuda), seen=seen.to(cuda), allowed=allowed.to(cuda),
                     steps=steps.to(cuda), eos=eos, seen_out=seen_out)
    assert boundary_free(got.cpu(), ref_tokens)
    same = (got.cpu() == ref_tokens).flatten()
    assert torch.equal(seen_out.cpu()[same], ref_seen[same])
    # EOS is never drawn before step 2 and masked ids never drawn
    assert not ((got.cpu().flatten() == eos) & (steps < 2)).any()
    assert allowed[got.cpu().flatten()].all()


def test_top_p_and_philox(ops, cuda):
    scores = bf16_scores(33, 64, 2048, 3.0)
    offsets = torch.arange(64, dtype=torch.int64) * 16 + 5
    seed = 0x1234_5678_9ABC
    u = torch.from_numpy(S.philox_uniform(seed, offsets.numpy()))
    ref = S.categorical(scores, u, top_p=0.95)
    got = ops.sample(scores.to(cuda), seed=seed, philox_offsets=offsets.to(cuda), top_p=0.95).cpu()
    assert boundary_free(got, ref)
    stream = ops.philox_uniforms(seed, 7, 1001, cuda).cpu().numpy()
    assert np.array_equal(stream, S.philox_stream(seed, 7, 1001))


def test_cdf_select_exact(ops, cuda):
    p = torch.from_numpy(uniform(34, (32, 2048))) ** 4
    cdf = p.cumsum(-1)
    u = torch.from_numpy(uniform(35, (32,)))
    ref = S.cdf_select(cdf, u)
    assert torch.equal(ops.cdf_select(cdf.to(cuda), u.to(cuda)).cpu(), ref)
    # plateau boundaries +-1 ulp (probe_cdf_tail semantics)
    cdf = torch.tensor([[0.0, 0.25, 0.25, 0.5, 1.0]] * 3)
    u = torch.tensor([0.25, np.nextafter(np.float32(0.25), np.float32(0)), np.nextafter(np.float32(0.25), np.float32(1))],
                     dtype=torch.float32)
    assert torch.equal(ops.cdf_select(cdf.to(cuda), u.to(cuda)).cpu(), S.cdf_select(cdf, u))
