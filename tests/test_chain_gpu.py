"""q3t_linear_chain (persistent chain of dependent projections) against the per-projection
tcgen05 GEMM (q3t_linear / q3t_linear_rownorm) and a plain PyTorch fp32 reference.

The chain splits K differently from the single GEMM (stream-K pieces reduced in
contributor order), so bf16 outputs may differ from q3t_linear by one rounding of
a reordered fp32 sum: compared within 2 bf16 ulps of the output scale; against the
fp32 reference of the same bf16 operands within 1e-2 relative (normwise), the
bar the engine's logits are held to. Repeated launches on one workspace (graph
replays, chains of different shapes) must give bit-identical results: the
counters reset themselves and the reduction order is fixed.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


def _weights(gen, out_f, in_f, device):
    from qwen3_tts_b200 import ops
    w = (torch.randn(out_f, in_f, generator=gen) * in_f ** -0.5).to(BF16).to(device)
    return w, ops.pack_tiles(w)


def _fp32(x, w, eps=None):
    x32, w32 = x.float(), w.float()
    y = x32 @ w32.T
    if eps is not None:
        y = y * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return y


def _close(got, want, ulps=2):
    scale = want.float().abs().max().clamp(min=1e-3)
    assert (got.float() - want.float()).abs().max() <= ulps * 2 ** -7 * scale


def _rel(got, want):
    return float((got.float() - want.float()).norm() / want.float().norm().clamp(min=1e-12))


@pytest.mark.parametrize("rows", [1, 7, 16, 33, 64])
def test_single_stage_epilogues_match_linear(cuda, rows):
    from qwen3_tts_b200 import _lib, ops
    gen = torch.Generator().manual_seed(rows)
    ws = ops.linear_chain_workspace(rows, cuda)
    x = torch.randn(rows, 2048, generator=gen).to(BF16).to(cuda)
    res = torch.randn(rows, 2048, generator=gen).to(BF16).to(cuda)
    w, wt = _weights(gen, 2048, 2048, cuda)
    # STORE with the folded row norm
    ref = ops.linear(x, wt, row_norm_eps=1e-6)
    got = torch.empty_like(ref)
    ops.linear_chain([{"x": x, "weight": wt, "out": got, "row_norm_eps": 1e-6}], ws)
    _close(got, ref)
    assert _rel(got, _fp32(x, w, 1e-6)) < 1e-2
    # RESIDUAL
    ref = ops.linear(x, wt, out=res.clone(), epilogue=_lib.EPI_RESIDUAL, residual=res)
    got = res.clone()
    ops.linear_chain([{"x": x, "weight": wt, "out": got, "epilogue": _lib.EPI_RESIDUAL, "residual": got}], ws)
    _close(got, ref)
    # fp32 STORE (codebook head), 2048 outputs from 1024 inputs
    w2, wt2 = _weights(gen, 2048, 1024, cuda)
    x2 = x[:, :1024].contiguous()
    ref = ops.linear(x2, wt2, out_dtype=torch.float32, row_norm_eps=1e-6)
    got = torch.empty_like(ref)
    ops.linear_chain([{"x": x2, "weight": wt2, "out": got, "row_norm_eps": 1e-6}], ws)
    _close(got, ref)
    # paired SwiGLU with the folded row norm (gate/up interleaved per 128-row tile)
    w3, wt3 = _weights(gen, 2 * 3072, 2048, cuda)
    ref = ops.linear(x, wt3, epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=1e-6)
    got = torch.empty_like(ref)
    ops.linear_chain([{"x": x, "weight": wt3, "out": got, "epilogue": _lib.EPI_SWIGLU_PAIRED,
                       "row_norm_eps": 1e-6}], ws)
    _close(got, ref)
    torch.cuda.synchronize()
    assert ops.read_status(cuda) == 0


def _layer(gen, hidden, heads_width, ffn, qkv_width, device):
    from qwen3_tts_b200 import ops
    from qwen3_tts_b200.weights import PackedLayer
    o, ot = _weights(gen, hidden, heads_width, device)
    gu, gut = _weights(gen, 2 * ffn, hidden, device)
    down, downt = _weights(gen, hidden, ffn, device)
    qkv, qkvt = _weights(gen, qkv_width, hidden, device)
    layer = PackedLayer(input_norm=None, qkv=qkvt, q_norm=None, k_norm=None, o=ot, post_norm=None, gate_up=gut,
                        down=downt, folded=True)
    return layer, (o, gu, down, qkv)


@pytest.mark.parametrize("geometry", ["talker", "predictor"])
@pytest.mark.parametrize("rows", [5, 32, 64])
def test_layer_chain_matches_separate_gemms(cuda, geometry, rows):
    """O (+residual) -> gate/up (norm, SwiGLU) -> down (+residual) -> next QKV (norm)."""
    from qwen3_tts_b200 import _lib, ops
    from qwen3_tts_b200.talker import mlp_stages, qkv_stage
    hidden, ffn = (2048, 6144) if geometry == "talker" else (1024, 3072)
    gen = torch.Generator().manual_seed(11 + rows)
    layer, (o, gu, down, qkv_w) = _layer(gen, hidden, 2048, ffn, 4096, cuda)
    nxt = type(layer)(**{**layer.__dict__})
    attn = torch.randn(rows, 2048, generator=gen).to(BF16).to(cuda)
    x0 = torch.randn(rows, hidden, generator=gen).to(BF16).to(cuda)
    eps = 1e-6
    # separate launches
    h_ref = ops.linear(attn, layer.o, out=torch.empty_like(x0), epilogue=_lib.EPI_RESIDUAL, residual=x0)
    act_ref = ops.linear(h_ref, layer.gate_up, epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=eps)
    h2_ref = ops.linear(act_ref, layer.down, out=h_ref.clone(), epilogue=_lib.EPI_RESIDUAL, residual=h_ref)
    qkv_ref = ops.linear(h2_ref, nxt.qkv, row_norm_eps=eps)
    # one chain
    ws = ops.linear_chain_workspace(rows, cuda)
    h = torch.empty_like(x0)
    act = torch.empty(rows, ffn, dtype=BF16, device=cuda)
    qkv = torch.empty(rows, 4096, dtype=BF16, device=cuda)
    stages = mlp_stages(attn, x0, layer, h, act, eps) + [qkv_stage(h, nxt, qkv, eps, depends=2)]
    outs = []
    for _ in range(3):   # repeated launches on one workspace: counters reset, results bit-identical
        ops.linear_chain(stages, ws)
        torch.cuda.synchronize()
        outs.append((h.clone(), act.clone(), qkv.clone()))
    assert ops.read_status(cuda) == 0
    for later in outs[1:]:
        for a, b in zip(outs[0], later):
            assert torch.equal(a, b)
    h, act, qkv = outs[0]
    # the chain's stages against the separate GEMMs fed the chain's own intermediate values
    _close(act, ops.linear(ops.linear(attn, layer.o, out=torch.empty_like(x0), epilogue=_lib.EPI_RESIDUAL,
                                      residual=x0), layer.gate_up, epilogue=_lib.EPI_SWIGLU_PAIRED,
                           row_norm_eps=eps), ulps=4)
    _close(qkv, ops.linear(h, nxt.qkv, row_norm_eps=eps))
    # and end to end against the separate launches (intermediate roundings may differ by an ulp)
    assert _rel(h, h2_ref) < 1e-2 and _rel(qkv, qkv_ref) < 1e-2
    # fp32 reference of the final projection from the chain's own h
    assert _rel(qkv, _fp32(h, qkv_w, eps)) < 1e-2


def test_chain_in_a_cuda_graph_replays_and_mixed_shapes_share_a_workspace(cuda):
    from qwen3_tts_b200 import _lib, ops
    gen = torch.Generator().manual_seed(5)
    rows = 24
    ws = ops.linear_chain_workspace(rows, cuda)
    x = torch.randn(rows, 1024, generator=gen).to(BF16).to(cuda)
    _, a = _weights(gen, 3072, 1024, cuda)
    _, b = _weights(gen, 1024, 3072, cuda)
    _, c = _weights(gen, 2048, 1024, cuda)
    y = torch.empty(rows, 3072, dtype=BF16, device=cuda)
    z = torch.empty(rows, 1024, dtype=BF16, device=cuda)
    logits = torch.empty(rows, 2048, dtype=torch.float32, device=cuda)
    long = [{"x": x, "weight": a, "out": y, "row_norm_eps": 1e-6, "depends": -1},
            {"x": y, "weight": b, "out": z, "depends": 0},
            {"x": z, "weight": c, "out": logits, "row_norm_eps": 1e-6, "depends": 1}]
    short = [{"x": x, "weight": c, "out": logits, "depends": -1}]
    ops.linear_chain(long, ws)
    torch.cuda.synchronize()
    expect = logits.clone()
    ops.linear_chain(short, ws)
    torch.cuda.synchronize()
    expect_short = logits.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.linear_chain(long, ws)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        ops.linear_chain(long, ws)
    for _ in range(4):
        logits.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(logits, expect)
        ops.linear_chain(short, ws)
        torch.cuda.synchronize()
        assert torch.equal(logits, expect_short)
    graph.reset()
    assert ops.read_status(cuda) == 0
    # the fp32 path of the last stage matches its separate GEMM
    _close(expect, ops.linear(ops.linear(ops.linear(x, a, row_norm_eps=1e-6), b), c, out_dtype=torch.float32,
                              row_norm_eps=1e-6), ulps=4)
