"""Talker decode step on the slot-table KV arena, captured as CUDA graphs.

Mirrors ``SlotArena`` / ``SlotGraph`` of the reference (continuous.py:97-229):
one KV arena holds every slot's keys and values, a decode step runs the whole
28-layer stack for a bucket of slots, and one CUDA graph is captured per
(batch bucket, context bucket) with static input buffers, so any slot
assignment replays the same graph (positions live in device buffers).

Per layer the step launches five kernels, all from ``libq3t_b200.so``:
QKV GEMM (input RMSNorm folded in) -> ragged GQA attention (q/k norm, RoPE
and the KV write fused in) -> O GEMM (+ residual) -> gate/up GEMM
(post-attention RMSNorm folded in, + SwiGLU) -> down GEMM (+ residual); then
the final norm and the LM head (fp32 logits). With unfolded weights the two
norms, and with ``fused_attention=False`` the q/k kernel, run separately.
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .batching import packed_unit_capacity
from .config import DecoderConfig
from .weights import pack_decoder

BF16 = torch.bfloat16
# Run each layer's projections as one persistent q3t_linear_chain launch where the shape allows.
CHAIN_PROJECTIONS = False
# Which kernels pull later projections' weights into L2 in the decode step: "none", "gemm" (each
# GEMM the next GEMM's) or "attention" (the attention kernel O and gate/up, O down, gate/up the
# next QKV). Measured on the 28-layer step (64 / 32 slots): none 2.96 / 1.94 ms, gemm 2.98 /
# 1.94 ms, attention 3.16 / 2.08 ms - the weight streams already run near the HBM rate and the
# prefetch only adds traffic.
PREFETCH_PLAN = "none"


def rope_tables(positions: int, dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Default RoPE cos/sin [positions, dim] in bf16 (fp32 angles, duplicated halves)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    freqs = torch.arange(positions, dtype=torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(BF16).to(device), emb.sin().to(BF16).to(device)


def qkv_stage(x, layer, out, eps, depends):
    """Chain stage: the packed QKV projection with the input RMSNorm folded in."""
    return {"x": x, "weight": layer.qkv, "out": out, "row_norm_eps": eps, "depends": depends}


def mlp_stages(attn, residual, layer, h, act, eps):
    """Chain stages after an attention: h = residual + O(attn); act = SwiGLU(gate/up(norm(h)));
    h = h + down(act) (PackedAttention.o_proj, packed_attention.py:85; PackedMLP, packed_mlp.py:19-27)."""
    return [
        {"x": attn, "weight": layer.o, "out": h, "epilogue": _lib.EPI_RESIDUAL, "residual": residual, "depends": -1},
        {"x": h, "weight": layer.gate_up, "out": act, "epilogue": _lib.EPI_SWIGLU_PAIRED, "row_norm_eps": eps,
         "depends": 0},
        {"x": act, "weight": layer.down, "out": h, "epilogue": _lib.EPI_RESIDUAL, "residual": h, "depends": 1},
    ]


class SlotArena:
    """Per-layer K/V for every slot in one packed allocation [2L, slots, kv_heads, capacity, head_dim].

    ``keys[i]`` / ``values[i]`` are views of layer i (continuous.py:97-116 with packed_kv).
    """

    def __init__(self, cfg: DecoderConfig, slots: int, capacity: int, device):
        self.cfg = cfg
        self.slots = slots
        self.capacity = capacity
        self.device = torch.device(device)
        self.packed = torch.zeros((cfg.layers * 2, slots, cfg.kv_heads, capacity, cfg.head_dim), dtype=BF16,
                                  device=self.device)
        self.keys = list(self.packed[:cfg.layers].unbind(0))
        self.values = list(self.packed[cfg.layers:].unbind(0))

    def load_packed(self, slot: int, source: torch.Tensor, row: int = 0, length=None) -> None:
        """Copy one prefilled request prefix [2L, rows, kv, len, D] into `slot` (packed_kv.py:6)."""
        ops.copy_packed_prefix(self.packed, source, slot, row=row, length=length)

    def load(self, slot: int, keys: list, values: list, row: int = 0, length=None) -> None:
        """Per-layer prefix copy from [rows, kv, len, D] caches (continuous.py:118-122)."""
        source = torch.stack(list(keys) + list(values))
        self.load_packed(slot, source, row=row, length=length)

    def move(self, source: int, destination: int) -> None:
        """Slot compaction: copy `source` over `destination` in every layer (continuous.py:124-128)."""
        if source != destination:
            ops.slot_move(self.packed, source, destination, dim=1)

    def grown(self, capacity: int) -> "SlotArena":
        """A new arena of larger capacity holding this arena's contents (continuous.py:353-363)."""
        arena = SlotArena(self.cfg, self.slots, capacity, self.device)
        ops.copy_prefix_along(arena.packed, self.packed, dim=3)
        return arena


class TalkerStep:
    """Static-buffer decode step for `batch` slots attending over `context` keys."""

    def __init__(self, cfg: DecoderConfig, weights: dict, arena: SlotArena, batch: int, context: int, cos, sin,
                 norm_mode: int = _lib.NORM_REFERENCE, fused_attention: bool = True):
        if not 1 <= context <= arena.capacity:
            raise ValueError("Attention context must fit the KV arena")
        if batch > arena.slots:
            raise ValueError("Decode batch exceeds the slot arena")
        self.cfg, self.w, self.arena = cfg, weights, arena
        self.batch, self.context = batch, context
        self.cos, self.sin = cos, sin
        self.norm_mode = norm_mode
        self.fused_attention = fused_attention   # q/k norm, RoPE and KV write inside the attention kernel
        self.prefetch_plan = PREFETCH_PLAN       # see PREFETCH_PLAN
        self.prefetch_weights = PREFETCH_PLAN != "none"
        dev = arena.device
        B, H = batch, cfg.hidden
        self.inputs = torch.zeros(B, H, dtype=BF16, device=dev)
        self.positions = torch.zeros(B, dtype=torch.long, device=dev)
        self.rotary = torch.zeros(B, dtype=torch.long, device=dev)
        self.h = torch.zeros(B, H, dtype=BF16, device=dev)
        self.xn = torch.zeros(B, H, dtype=BF16, device=dev)
        self.qkv = torch.zeros(B, cfg.qkv_width, dtype=BF16, device=dev)
        self.q = torch.zeros(B, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.attn = torch.zeros(B, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.act = torch.zeros(B, cfg.ffn, dtype=BF16, device=dev)
        self.hidden = torch.zeros(B, H, dtype=BF16, device=dev)
        self.logits = torch.zeros(B, cfg.vocab, dtype=torch.float32, device=dev)
        gemms = [(H, cfg.qkv_width), (cfg.q_width, H), (H, 2 * cfg.ffn), (cfg.ffn, H), (H, cfg.vocab)]
        need = max(ops.linear_workspace_bytes(B, k, n) for k, n in gemms)
        self.ws_linear = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
        need = ops.decode_attention_workspace_bytes(B, cfg.q_heads, cfg.head_dim, context)
        self.ws_attn = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
        self.status = ops.status_word(dev)
        # Projections between two attentions run as one persistent chain launch (q3t_linear_chain):
        # needs folded norms, tiled weights and at most 64 rows
        self.use_chain = (CHAIN_PROJECTIONS and B <= 64 and fused_attention and weights["layers"][0].folded
                          and isinstance(weights["layers"][0].qkv, ops.TiledWeight))
        self.ws_chain = ops.linear_chain_workspace(B, dev) if self.use_chain else None
        self.graph = None
        self.output = (self.hidden, self.logits)

    # ---------------------------------------------------------------- one eager pass
    def compute(self) -> None:
        if self.use_chain:
            self._compute_chained()
            return
        cfg, w, B = self.cfg, self.w, self.batch
        lw = ops.linear
        res_in = self.inputs
        layers = w["layers"]
        # split-KV chunks sized once per step for this batch's contexts (all layers share them)
        ops.attention_plan(self.positions, self.ws_attn, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads,
                           head_dim=cfg.head_dim, context=self.context)
        # weights of later GEMMs are pulled into L2 ahead of use
        pf = (lambda t: t) if self.prefetch_weights else (lambda t: None)
        by_attention = self.prefetch_plan == "attention" and self.fused_attention
        for i, layer in enumerate(layers):
            following = layers[i + 1].qkv if i + 1 < len(layers) else w["head"]
            after_qkv = None if by_attention else pf(layer.o)
            if layer.folded:
                lw(res_in, layer.qkv, out=self.qkv, row_norm_eps=cfg.eps, prefetch=after_qkv)
            else:
                ops.rms_norm(res_in, layer.input_norm, cfg.eps, self.norm_mode, out=self.xn)
                lw(self.xn, layer.qkv, out=self.qkv, workspace=self.ws_linear, prefetch=after_qkv)
            if self.fused_attention:
                ops.decode_attention_qkv(self.qkv, layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin,
                                         self.rotary, self.arena.keys[i], self.arena.values[i], self.positions,
                                         q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                                         context=self.context, out=self.attn, workspace=self.ws_attn,
                                         prefetch=(pf(layer.o), pf(layer.gate_up)) if by_attention else ())
            else:
                ops.qk_norm_rope_kv(self.qkv, layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin, self.rotary,
                                    self.positions, self.arena.keys[i], self.arena.values[i], q_heads=cfg.q_heads,
                                    kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, query_out=self.q)
                ops.decode_attention(self.q, self.arena.keys[i], self.arena.values[i], self.positions,
                                     context=self.context, out=self.attn, workspace=self.ws_attn)
            lw(self.attn.view(B, cfg.q_width), layer.o, out=self.h, epilogue=_lib.EPI_RESIDUAL, residual=res_in,
               workspace=self.ws_linear, prefetch=pf(layer.down if by_attention else layer.gate_up))
            after_gate_up = pf(following if by_attention else layer.down)
            if layer.folded:
                lw(self.h, layer.gate_up, out=self.act, epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=cfg.eps,
                   prefetch=after_gate_up)
            else:
                ops.rms_norm(self.h, layer.post_norm, cfg.eps, self.norm_mode, out=self.xn)
                lw(self.xn, layer.gate_up, out=self.act, epilogue=_lib.EPI_SWIGLU_PAIRED, workspace=self.ws_linear,
                   prefetch=after_gate_up)
            lw(self.act, layer.down, out=self.h, epilogue=_lib.EPI_RESIDUAL, residual=self.h,
               workspace=self.ws_linear, prefetch=None if by_attention else pf(following))
            res_in = self.h
        ops.rms_norm(res_in, w["norm"], cfg.eps, self.norm_mode, out=self.hidden)
        lw(self.hidden, w["head"], out=self.logits, workspace=self.ws_linear)

    def _compute_chained(self) -> None:
        """The step with each layer's O, gate/up, down and the next layer's QKV as one
        q3t_linear_chain launch: per layer one attention kernel and one chain kernel."""
        cfg, w, B = self.cfg, self.w, self.batch
        layers = w["layers"]
        ops.attention_plan(self.positions, self.ws_attn, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads,
                           head_dim=cfg.head_dim, context=self.context)
        ops.linear_chain([qkv_stage(self.inputs, layers[0], self.qkv, cfg.eps, depends=-1)], self.ws_chain)
        res_in = self.inputs
        for i, layer in enumerate(layers):
            ops.decode_attention_qkv(self.qkv, layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin,
                                     self.rotary, self.arena.keys[i], self.arena.values[i], self.positions,
                                     q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                                     context=self.context, out=self.attn, workspace=self.ws_attn)
            stages = mlp_stages(self.attn.view(B, cfg.q_width), res_in, layer, self.h, self.act, cfg.eps)
            if i + 1 < len(layers):
                stages.append(qkv_stage(self.h, layers[i + 1], self.qkv, cfg.eps, depends=2))
            ops.linear_chain(stages, self.ws_chain)
            res_in = self.h
        ops.rms_norm(res_in, w["norm"], cfg.eps, self.norm_mode, out=self.hidden)
        ops.linear(self.hidden, w["head"], out=self.logits, workspace=self.ws_linear)

    def launches_per_step(self) -> int:
        if self.use_chain:
            return 2 * self.cfg.layers + 4

        per_layer = (6 if self.w["layers"][0].folded else 8) - (1 if self.fused_attention else 0)
        return per_layer * self.cfg.layers + 3

    # ---------------------------------------------------------------- graph capture / replay
    @torch.inference_mode()
    def capture(self, warmup: int = 3) -> None:
        """Warm up on a side stream, then capture (continuous.py:200-216).

        Warm-up really runs, so the KV entries it writes (position 0 of the
        first `batch` slots) are saved before and restored after.
        """
        saved = [(k[:self.batch, :, 0].clone(), v[:self.batch, :, 0].clone())
                 for k, v in zip(self.arena.keys, self.arena.values)]
        self.positions.zero_()
        self.rotary.zero_()
        stream = torch.cuda.Stream(device=self.inputs.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.compute()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.compute()
        torch.cuda.synchronize()
        for layer, (k, v) in enumerate(saved):
            self.arena.keys[layer][:self.batch, :, 0].copy_(k)
            self.arena.values[layer][:self.batch, :, 0].copy_(v)

    @torch.inference_mode()
    def run(self, inputs, positions, rotary, clone: bool = True):
        """Copy inputs into the static buffers, replay, return (hidden, logits)."""
        self.inputs.copy_(inputs)
        self.positions.copy_(positions)
        self.rotary.copy_(rotary)
        if self.graph is None:
            self.compute()
        else:
            self.graph.replay()
        if clone:
            return self.hidden.clone(), self.logits.clone()
        return self.hidden, self.logits

    def close(self) -> None:
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None


class TalkerPrefill:
    """Batched padded prefill straight into arena slots (PrefillGraph, prefill_graph.py:18-78).

    ``batch`` prompts padded to ``length`` run the full causal stack; row
    (b, t) writes its K/V at position t of arena slot ``slots[b]`` and attends
    keys 0..t of that slot. Returns the final-norm hidden state and fp32 logits
    of each prompt's last real token (continuous.py:455-458)."""

    def __init__(self, cfg: DecoderConfig, weights: dict, arena: SlotArena, batch: int, length: int, cos, sin,
                 norm_mode: int = _lib.NORM_REFERENCE):
        if length > arena.capacity:
            raise ValueError("Prompt longer than the KV arena")
        self.cfg, self.w, self.arena = cfg, weights, arena
        self.batch, self.length = batch, length
        self.cos, self.sin, self.norm_mode = cos, sin, norm_mode
        dev = arena.device
        R, H = batch * length, cfg.hidden
        self.inputs = torch.zeros(R, H, dtype=BF16, device=dev)
        self.slots = torch.zeros(batch, dtype=torch.long, device=dev)
        self.last = torch.zeros(batch, dtype=torch.long, device=dev)          # row index b*L + len_b - 1
        self.positions = torch.arange(length, device=dev).repeat(batch).contiguous()
        self.h = torch.zeros(R, H, dtype=BF16, device=dev)
        self.xn = torch.zeros(R, H, dtype=BF16, device=dev)
        self.qkv = torch.zeros(R, cfg.qkv_width, dtype=BF16, device=dev)
        self.q = torch.zeros(R, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.attn = torch.zeros(R, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.act = torch.zeros(R, cfg.ffn, dtype=BF16, device=dev)
        self.hidden = torch.zeros(batch, H, dtype=BF16, device=dev)
        self.logits = torch.zeros(batch, cfg.vocab, dtype=torch.float32, device=dev)
        need = ops.decode_attention_workspace_bytes(R, cfg.q_heads, cfg.head_dim, length)
        self.ws_attn = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
        self.status = ops.status_word(dev)
        self.graph = None

    def compute(self) -> None:
        cfg, w, R, L = self.cfg, self.w, self.batch * self.length, self.length
        res_in = self.inputs
        for i, layer in enumerate(w["layers"]):
            if layer.folded:
                ops.linear(res_in, layer.qkv, out=self.qkv, row_norm_eps=cfg.eps)
            else:
                ops.rms_norm(res_in, layer.input_norm, cfg.eps, self.norm_mode, out=self.xn)
                ops.linear(self.xn, layer.qkv, out=self.qkv)
            ops.qk_norm_rope_kv(self.qkv, layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin, self.positions,
                                self.positions, self.arena.keys[i], self.arena.values[i], q_heads=cfg.q_heads,
                                kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, length=L, query_out=self.q,
                                slots=self.slots)
            ops.decode_attention(self.q, self.arena.keys[i], self.arena.values[i], self.positions, context=L,
                                 rows_per_slot=L, slots=self.slots, out=self.attn, workspace=self.ws_attn)
            ops.linear(self.attn.view(R, cfg.q_width), layer.o, out=self.h, epilogue=_lib.EPI_RESIDUAL,
                       residual=res_in)
            if layer.folded:
                ops.linear(self.h, layer.gate_up, out=self.act, epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=cfg.eps)
            else:
                ops.rms_norm(self.h, layer.post_norm, cfg.eps, self.norm_mode, out=self.xn)
                ops.linear(self.xn, layer.gate_up, out=self.act, epilogue=_lib.EPI_SWIGLU_PAIRED)
            ops.linear(self.act, layer.down, out=self.h, epilogue=_lib.EPI_RESIDUAL, residual=self.h)
            res_in = self.h
        ops.embedding(self.last, self.h, out=self.xn[:self.batch])       # last real row of each prompt
        ops.rms_norm(self.xn[:self.batch], w["norm"], cfg.eps, self.norm_mode, out=self.hidden)
        ops.linear(self.hidden, w["head"], out=self.logits)

    @torch.inference_mode()
    def capture(self, warmup: int = 2) -> None:
        """Capture after warm-up; warm-up writes only to scratch slot rows that are
        restored (slots default to 0..batch-1; their first `length` positions are saved)."""
        saved = self.arena.packed[:, :self.batch, :, :self.length].clone()
        self.slots.copy_(torch.arange(self.batch, device=self.slots.device))
        self.last.copy_(torch.arange(self.batch, device=self.last.device) * self.length + self.length - 1)
        stream = torch.cuda.Stream(device=self.inputs.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.compute()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.compute()
        torch.cuda.synchronize()
        self.arena.packed[:, :self.batch, :, :self.length].copy_(saved)

    @torch.inference_mode()
    def run(self, embeds, lengths, slots):
        """embeds [batch, length, H] (right-padded), lengths [batch], slots [batch] -> (hidden, logits)."""
        self.inputs.copy_(embeds.reshape(self.batch * self.length, -1))
        self.slots.copy_(slots)
        self.last.copy_(torch.arange(self.batch, device=self.last.device) * self.length + lengths - 1)
        if self.graph is None:
            self.compute()
        else:
            self.graph.replay()
        return self.hidden.clone(), self.logits.clone()

    def close(self) -> None:
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None


class PackedPrefill:
    """Batched prefill of several prompts packed end to end, without padding to the longest
    (PrefillGraph, prefill_graph.py:18-78, computes the same causal stack over padded rows).

    Row r of the `rows` packed rows belongs to arena slot ``row_slots[r]`` at position
    ``row_pos[r]`` (0 .. its prompt length - 1): it writes its K/V there and attends keys
    0..row_pos[r] of that slot, so every prompt sees only itself. The attention runs as
    causal 64-row query tiles on the tensor cores (ops.prefill_attention over the unit table
    of batching.packed_units). Rows past the real ones repeat the last real row (same slot,
    position and input, and units of their own: identical K/V writes). Returns the
    final-norm hidden state and fp32 logits of each prompt's last token (``last`` holds
    their row indices; up to `requests` prompts)."""

    def __init__(self, cfg: DecoderConfig, weights: dict, arena: SlotArena, rows: int, requests: int, cos, sin,
                 norm_mode: int = _lib.NORM_REFERENCE):
        if rows > arena.capacity * arena.slots:
            raise ValueError("Packed prefill longer than the KV arena")
        self.cfg, self.w, self.arena = cfg, weights, arena
        self.rows, self.requests = rows, requests
        self.cos, self.sin, self.norm_mode = cos, sin, norm_mode
        dev = arena.device
        R, H = rows, cfg.hidden
        self.inputs = torch.zeros(R, H, dtype=BF16, device=dev)
        self.row_slots = torch.zeros(R, dtype=torch.long, device=dev)
        self.row_pos = torch.zeros(R, dtype=torch.long, device=dev)
        self.last = torch.zeros(requests, dtype=torch.long, device=dev)
        self.units = torch.zeros(packed_unit_capacity(rows, requests), 4, dtype=torch.int32, device=dev)
        self.h = torch.zeros(R, H, dtype=BF16, device=dev)
        self.xn = torch.zeros(R, H, dtype=BF16, device=dev)
        self.qkv = torch.zeros(R, cfg.qkv_width, dtype=BF16, device=dev)
        self.q = torch.zeros(R, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.attn = torch.zeros(R, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.act = torch.zeros(R, cfg.ffn, dtype=BF16, device=dev)
        self.gathered = torch.zeros(requests, H, dtype=BF16, device=dev)
        self.hidden = torch.zeros(requests, H, dtype=BF16, device=dev)
        self.logits = torch.zeros(requests, cfg.vocab, dtype=torch.float32, device=dev)
        self.status = ops.status_word(dev)
        # From a thousand rows on, the projections run the wide-tile kernel, which takes no folded
        # RMSNorm: the norm runs as its own pass with a unit weight (the norm weight stays
        # folded into the projection weights), x -> bf16(x * rsqrt(mean(x^2) + eps)).
        self.unit = torch.ones(H, dtype=BF16, device=dev) if rows >= 1024 else None
        self.graph = None

    def _norm_linear(self, x, layer, weight, out, **kw) -> None:
        cfg = self.cfg
        if not layer.folded:
            ops.rms_norm(x, layer.input_norm if weight is layer.qkv else layer.post_norm, cfg.eps, self.norm_mode,
                         out=self.xn)
            ops.linear(self.xn, weight, out=out, **kw)
        elif self.unit is not None:
            ops.rms_norm(x, self.unit, cfg.eps, self.norm_mode, out=self.xn)
            ops.linear(self.xn, weight, out=out, **kw)
        else:
            ops.linear(x, weight, out=out, row_norm_eps=cfg.eps, **kw)

    def compute(self) -> None:
        cfg, w, R = self.cfg, self.w, self.rows
        res_in = self.inputs
        for i, layer in enumerate(w["layers"]):
            self._norm_linear(res_in, layer, layer.qkv, self.qkv)
            ops.qk_norm_rope_kv(self.qkv, layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin, self.row_pos,
                                self.row_pos, self.arena.keys[i], self.arena.values[i], q_heads=cfg.q_heads,
                                kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, length=1, query_out=self.q,
                                slots=self.row_slots)
            ops.prefill_attention(self.q, self.arena.keys[i], self.arena.values[i], self.row_pos, self.units,
                                  out=self.attn)
            ops.linear(self.attn.view(R, cfg.q_width), layer.o, out=self.h, epilogue=_lib.EPI_RESIDUAL,
                       residual=res_in)
            self._norm_linear(self.h, layer, layer.gate_up, self.act, epilogue=_lib.EPI_SWIGLU_PAIRED)
            ops.linear(self.act, layer.down, out=self.h, epilogue=_lib.EPI_RESIDUAL, residual=self.h)
            res_in = self.h
        ops.embedding(self.last, self.h, out=self.gathered)       # last row of each prompt
        ops.rms_norm(self.gathered, w["norm"], cfg.eps, self.norm_mode, out=self.hidden)
        ops.linear(self.hidden, w["head"], out=self.logits)

    @torch.inference_mode()
    def capture(self, warmup: int = 2) -> None:
        """Capture after warm-up; warm-up runs every row as position 0 of slot 0, whose first
        position is saved and restored."""
        saved = self.arena.packed[:, :1, :, :1].clone()
        self.row_slots.zero_()
        self.row_pos.zero_()
        self.last.zero_()
        self.units.zero_()
        starts = torch.arange(0, self.rows, 64, dtype=torch.int32)
        self.units[:len(starts)] = torch.stack([starts, (self.rows - starts).clamp(max=64), torch.ones_like(starts),
                                                torch.zeros_like(starts)], 1).to(self.units.device)
        stream = torch.cuda.Stream(device=self.inputs.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.compute()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.compute()
        torch.cuda.synchronize()
        self.arena.packed[:, :1, :, :1].copy_(saved)

    @torch.inference_mode()
    def run(self, packed, row_slots, row_pos, last, units):
        """packed [rows, H] (padding rows repeat the last real row), row_slots / row_pos [rows],
        last [requests], units (batching.packed_units) -> (hidden, logits) of the `requests`
        prompts."""
        self.inputs.copy_(packed)
        self.row_slots.copy_(row_slots)
        self.row_pos.copy_(row_pos)
        self.last.copy_(last)
        self.units.copy_(units)
        if self.graph is None:
            self.compute()
        else:
            self.graph.replay()
        return self.hidden.clone(), self.logits.clone()

    def close(self) -> None:
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None


class TalkerDecoder:
    """Talker weights, arena and per-bucket step graphs."""

    def __init__(self, cfg: DecoderConfig, weights: dict, slots: int, capacity: int, device, packed: bool = False,
                 use_graphs: bool = True, max_positions: int = 1 << 15):
        self.cfg = cfg
        self.device = torch.device(device)
        self.weights = weights if packed else pack_decoder(weights, self.device)
        self.arena = SlotArena(cfg, slots, capacity, self.device)
        self.cos, self.sin = rope_tables(max_positions, cfg.head_dim, cfg.theta, self.device)
        self.use_graphs = use_graphs
        self.graphs: dict[tuple[int, int], TalkerStep] = {}

    def ensure_capacity(self, required: int) -> None:
        """Grow the arena by doubling when `required` does not fit (continuous.py:353-363)."""
        if required < self.arena.capacity:
            return
        for graph in self.graphs.values():
            graph.close()
        self.graphs.clear()
        new = max(self.arena.capacity * 2, 1 << int(required).bit_length())
        self.arena = self.arena.grown(new)

    def step_for(self, batch: int, context: int) -> TalkerStep:
        key = (batch, context)
        step = self.graphs.get(key)
        if step is None:
            step = TalkerStep(self.cfg, self.weights, self.arena, batch, context, self.cos, self.sin)
            if self.use_graphs:
                step.capture()
            self.graphs[key] = step
        return step

    def close(self) -> None:
        for graph in self.graphs.values():
            graph.close()
        self.graphs.clear()
