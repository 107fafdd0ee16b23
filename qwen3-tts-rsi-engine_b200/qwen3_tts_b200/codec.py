"""Incremental 12.5 Hz codec on the GPU with slot-indexed streaming state.

Mirrors ``CodecSlots`` / ``CodecSlotGraph`` (codec_slots.py:42-338) and the
state rules of ``IncrementalCodec.run_module`` (incremental_codec.py:51-116):
every stream owns a slot; a decode call takes a group of slots (unique) and
their new codes [batch, codebooks, frames], and per slot the engine keeps

* causal-conv histories (the last (kernel-1)*dilation input frames),
* the transposed convs' overlap as their last input frame (the reference
  keeps the equivalent output tail minus bias),
* the sliding-window transformer's keys/values in a 128-row ring per layer
  (positions are absolute frame indices; the window of 72 sees 71 history keys),
* the frame counter.

Activations are time-major [batch * frames, channels] bf16. Each causal
convolution is ``q3t_conv_pad`` (the slot's history then the new frames, with
the preceding SnakeBeta applied, written once) followed by the implicit tcgen05
GEMM ``q3t_conv_linear``, whose activation tiles are tap-shifted rows of that
buffer (no im2col copy); a transposed conv of stride r is one such GEMM over
[x[t] | x[t-1]] whose r * C_out outputs per input frame are the upsampled
sequence. A residual unit's second SnakeBeta runs in the epilogue of its
dilated conv, so its 1x1 conv reads that output directly. One CUDA graph is
captured per (batch, frames) key.
"""
from __future__ import annotations

import math

import torch

from . import _lib, ops
from .config import CodecConfig
from .talker import rope_tables
from .weights import fold_norm, interleave_gate_up

BF16 = torch.bfloat16
RING = 128
F32 = torch.float32


# ---------------------------------------------------------------------- weights
def _snake(module, device):
    alpha = torch.exp(module.alpha.detach().float()).to(device).contiguous()
    inv = (1.0 / (torch.exp(module.beta.detach().float()) + module.no_div_by_zero)).to(device).contiguous()
    return alpha, inv


def _conv(module, device):
    """Causal Conv1d [C_out, C_in, k] -> GEMM weight [C_out, k*C_in] (K ordered (tap, channel))."""
    w = module.conv.weight.detach()
    c_out, c_in, k = w.shape
    weight = w.permute(0, 2, 1).reshape(c_out, k * c_in).to(device=device, dtype=BF16).contiguous()
    bias = module.conv.bias.detach().to(device=device, dtype=BF16).contiguous() if module.conv.bias is not None else None
    return {"w": weight, "tiles": ops.conv_weight_tiles(weight, k) if k > 1 else None, "b": bias, "k": k,
            "d": module.conv.dilation[0], "pad": module.padding, "c_in": c_in, "c_out": c_out}


def _tconv(module, device):
    """ConvTranspose1d [C_in, C_out, 2r or r] of stride r -> GEMM weight [r*C_out, taps*C_in].

    Output row (frame t, phase j) = b + W[:, :, j]^T x[t] (+ W[:, :, j+r]^T x[t-1] when the kernel is 2r)."""
    w = module.conv.weight.detach()
    c_in, c_out, k = w.shape
    r = module.conv.stride[0]
    taps = k // r
    rows = []
    for j in range(r):
        rows.append(torch.cat([w[:, :, j + m * r].T for m in range(taps)], dim=1))  # [C_out, taps*C_in]
    weight = torch.cat(rows, dim=0).to(device=device, dtype=BF16).contiguous()
    bias = module.conv.bias.detach().repeat(r).to(device=device, dtype=BF16).contiguous()
    return {"w": weight, "tiles": ops.conv_weight_tiles(weight, taps) if taps > 1 else None, "b": bias, "r": r,
            "taps": taps, "c_in": c_in, "c_out": c_out}


def _linear(module, device):
    b = module.bias.detach().to(device=device, dtype=BF16).contiguous() if module.bias is not None else None
    return module.weight.detach().to(device=device, dtype=BF16).contiguous(), b


def pack_codec(decoder, device) -> dict:
    """Device layouts of a tokenizer-v2 decoder module stack (see oracle/codec.py for the modules)."""
    cfg = decoder.cfg
    dev = torch.device(device)
    q = decoder.quantizer
    tables = []
    for group in (q.rvq_first, q.rvq_rest):
        for layer in group.vq.layers:
            book = layer._codebook
            tables.append(book.embedding_sum / book.cluster_usage.clamp(min=book.epsilon)[:, None])
    w_first = q.rvq_first.output_proj.weight.detach()[:, :, 0]
    w_rest = q.rvq_rest.output_proj.weight.detach()[:, :, 0]
    packed = {
        "rvq_tables": torch.stack(tables).to(device=dev, dtype=BF16).contiguous(),
        "rvq_proj": torch.cat([w_first, w_rest], dim=1).to(device=dev, dtype=BF16).contiguous(),
        "pre_conv": _conv(decoder.pre_conv, dev),
    }
    tr = decoder.pre_transformer
    layers = []
    for layer in tr.layers:
        input_norm = layer.input_layernorm.weight.detach().to(dev, BF16).contiguous()
        post_norm = layer.post_attention_layernorm.weight.detach().to(dev, BF16).contiguous()
        qkv = torch.cat([layer.q_proj.weight, layer.k_proj.weight, layer.v_proj.weight]).detach().to(dev, BF16)
        gate_up = interleave_gate_up(layer.gate_proj.weight.detach(), layer.up_proj.weight.detach()).to(dev, BF16)
        layers.append({
            "input_norm": input_norm,
            # the RMSNorm weights are folded into the projections that follow them;
            # the GEMMs apply the row RMS themselves (q3t_linear_rownorm)
            "qkv": fold_norm(qkv, input_norm).contiguous(),
            "o": layer.o_proj.weight.detach().to(dev, BF16).contiguous(),
            "attn_scale": layer.attn_scale.detach().to(dev, BF16).contiguous(),
            "post_norm": post_norm,
            "gate_up": fold_norm(gate_up, post_norm).contiguous(),
            "down": layer.down_proj.weight.detach().to(dev, BF16).contiguous(),
            "mlp_scale": layer.mlp_scale.detach().to(dev, BF16).contiguous(),
        })
    packed["transformer"] = {
        "input_proj": _linear(tr.input_proj, dev), "layers": layers,
        "norm": tr.norm.weight.detach().to(dev, BF16).contiguous(), "output_proj": _linear(tr.output_proj, dev),
    }
    ups = []
    for tconv, block in decoder.upsample:
        ups.append({
            "tconv": _tconv(tconv, dev),
            "dw_w": block.dwconv.conv.weight.detach()[:, 0, :].float().to(dev).contiguous(),
            "dw_b": block.dwconv.conv.bias.detach().float().to(dev).contiguous(),
            "ln_w": block.norm.weight.detach().float().to(dev).contiguous(),
            "ln_b": block.norm.bias.detach().float().to(dev).contiguous(),
            "ln_eps": block.norm.eps,
            "pw1": _linear(block.pwconv1, dev), "pw2": _linear(block.pwconv2, dev),
            "gamma": block.gamma.detach().to(dev, BF16).contiguous(),
        })
    packed["upsample"] = ups
    blocks = []
    mods = list(decoder.decoder)
    packed["conv0"] = _conv(mods[0], dev)
    for blk in mods[1:-2]:
        snake, tconv, *units = blk.block
        blocks.append({
            "snake": _snake(snake, dev), "tconv": _tconv(tconv, dev),
            "units": [{"snake1": _snake(u.act1, dev), "conv1": _conv(u.conv1, dev),
                       "snake2": _snake(u.act2, dev), "conv2": _conv(u.conv2, dev)} for u in units],
        })
    packed["blocks"] = blocks
    packed["final_snake"] = _snake(mods[-2], dev)
    packed["final_conv"] = _conv(mods[-1], dev)
    return packed


# ---------------------------------------------------------------------- state
class CodecState:
    """Per-slot streaming state of every stream (CodecSlots buffers, codec_slots.py:171-189)."""

    def __init__(self, cfg: CodecConfig, packed: dict, slots: int, device):
        self.cfg, self.slots = cfg, slots
        dev = torch.device(device)
        self.frames = torch.zeros(slots, dtype=torch.long, device=dev)
        L = cfg.layers
        self.kv = torch.zeros(2 * L, slots, cfg.heads, RING, cfg.head_dim, dtype=BF16, device=dev)
        self.histories: dict[str, torch.Tensor] = {}

        def hist(name, frames, channels):
            self.histories[name] = torch.zeros(slots, frames, channels, dtype=BF16, device=dev)

        hist("pre_conv", packed["pre_conv"]["pad"], packed["pre_conv"]["c_in"])
        for i, up in enumerate(packed["upsample"]):
            hist(f"up{i}.dw", 6, up["tconv"]["c_out"])
        hist("conv0", packed["conv0"]["pad"], packed["conv0"]["c_in"])
        for i, blk in enumerate(packed["blocks"]):
            hist(f"b{i}.tconv", blk["tconv"]["taps"] - 1, blk["tconv"]["c_in"])
            for u, unit in enumerate(blk["units"]):
                hist(f"b{i}.u{u}.conv1", unit["conv1"]["pad"], unit["conv1"]["c_in"])
        hist("final", packed["final_conv"]["pad"], packed["final_conv"]["c_in"])
        self.buffers = [self.frames, self.kv] + list(self.histories.values())

    def reset(self, slot: int) -> None:
        self.reset_range(slot, 1)

    def reset_range(self, start: int, count: int) -> None:
        """Clear newly admitted contiguous slots (codec_slots.py:313-325)."""
        if type(start) is not int or type(count) is not int or start < 0 or count < 0 or start + count > self.slots:
            raise ValueError("Expected a valid contiguous Codec slot range")
        if count:
            ops.slot_zero(self.frames, start, count)
            ops.slot_zero(self.kv, start, count, dim=1)
            for h in self.histories.values():
                ops.slot_zero(h, start, count)

    def move(self, source: int, destination: int) -> None:
        """Slot compaction (codec_slots.py:328-331)."""
        if source != destination:
            ops.slot_move(self.frames, source, destination)
            ops.slot_move(self.kv, source, destination, dim=1)
            for h in self.histories.values():
                ops.slot_move(h, source, destination)


# ---------------------------------------------------------------------- one (batch, frames) step
class CodecStep:
    """Static buffers and the kernel sequence of one decode call shape."""

    def __init__(self, cfg: CodecConfig, packed: dict, state: CodecState, batch: int, frames: int, cos, sin):
        self.cfg, self.p, self.state = cfg, packed, state
        self.batch, self.frames = batch, frames
        self.cos, self.sin = cos, sin
        dev = state.frames.device
        B, T = batch, frames
        self.indices = torch.zeros(B, dtype=torch.long, device=dev)
        self.codes = torch.zeros(B, cfg.codebooks, T, dtype=torch.long, device=dev)
        self.rot = torch.zeros(B * T, dtype=torch.long, device=dev)
        self.cache = torch.zeros(B * T, dtype=torch.long, device=dev)
        self.buf: dict[str, torch.Tensor] = {}
        self.samples = T * cfg.samples_per_frame
        self.wave = torch.zeros(B, self.samples, dtype=F32, device=dev)
        self.pcm = torch.zeros(B, self.samples, dtype=torch.int16, device=dev)
        self.status = ops.status_word(dev)
        self.ws_attn = None
        self.graph = None
        self.launches = 0          # this library's kernels per replay (counted at capture)
        self.replays = 0
        self._allocate(dev)

    def _b(self, name, rows, cols):
        t = self.buf.get(name)
        if t is None or t.shape != (rows, cols):
            t = torch.zeros(rows, cols, dtype=BF16, device=self.indices.device)
            self.buf[name] = t
        return t

    def _xs(self, hist_name, rows, channels):
        """Padded conv input [batch * (history + frames), channels] for the conv with history `hist_name`."""
        H = self.state.histories[hist_name].shape[1]
        return self._b(hist_name + ".xs", self.batch * H + rows, channels)

    def _allocate(self, dev):
        cfg, p, B, T = self.cfg, self.p, self.batch, self.frames
        R = B * T
        self._b("rvq", R, 2 * cfg.codebook_dim)
        self._b("x0", R, cfg.codebook_dim)
        self._xs("pre_conv", R, cfg.codebook_dim)
        self._b("lat", R, cfg.latent)
        self._b("h", R, cfg.hidden)
        self._b("xn", R, cfg.hidden)
        self._b("qkv", R, 3 * cfg.heads * cfg.head_dim)
        self._b("q", R, cfg.heads * cfg.head_dim)
        self._b("attn", R, cfg.heads * cfg.head_dim)
        self._b("act", R, cfg.ffn)
        need = ops.decode_attention_workspace_bytes(R, cfg.heads, cfg.head_dim, RING)
        self.ws_attn = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
        rows = R
        for i, up in enumerate(p["upsample"]):
            rows *= up["tconv"]["r"]
            C = up["tconv"]["c_out"]
            self._b(f"up{i}", rows, C)
            self._b(f"up{i}.ln", rows, C)
            self._b(f"up{i}.pw1", rows, 4 * C)
        self._xs("conv0", rows, p["conv0"]["c_in"])
        self._b("d0", rows, p["conv0"]["c_out"])
        for i, blk in enumerate(p["blocks"]):
            t = blk["tconv"]
            self._xs(f"b{i}.tconv", rows, t["c_in"])
            rows *= t["r"]
            C = t["c_out"]
            self._b(f"b{i}.y", rows, C)
            for u in range(len(blk["units"])):
                self._xs(f"b{i}.u{u}.conv1", rows, C)
            self._b(f"b{i}.col1", rows, C)
        self._xs("final", rows, p["final_conv"]["c_in"])
        self._b("out", rows, 1)

    # ------------------------------------------------------------------ kernels of one call
    def _conv(self, x, rows_in, conv, hist_name, *, snake=None, out=None, epilogue=_lib.EPI_STORE, residual=None,
              out_snake=None, reverse=False):
        """Causal conv (or, with `reverse`, the [x[t] | x[t-1]] transposed conv) of x with the slot
        histories: pad (+ SnakeBeta) -> history update -> implicit GEMM."""
        B, T = self.batch, rows_in // self.batch
        hist = self.state.histories[hist_name]
        alpha, inv = snake if snake is not None else (None, None)
        xs = self.buf[hist_name + ".xs"]
        ops.conv_pad(x, B, T, history=hist, slots=self.indices, alpha=alpha, inverse_beta=inv, out=xs)
        ops.conv_history(x, B, T, hist, slots=self.indices)
        taps = conv["taps"] if reverse else conv["k"]
        ops.conv_linear(xs, B, T, hist.shape[1], conv["tiles"], taps=taps, dilation=1 if reverse else conv["d"],
                        reverse=reverse, bias=conv["b"], out=out, epilogue=epilogue, residual=residual,
                        snake=out_snake)

    def compute(self) -> None:
        cfg, p, st, b = self.cfg, self.p, self.state, self.buf
        B, T = self.batch, self.frames
        R = B * T
        # RVQ dequantisation and the pre-transformer causal conv
        ops.rvq_gather(self.codes, p["rvq_tables"], cfg.semantic_codebooks, out=b["rvq"])
        ops.linear(b["rvq"], p["rvq_proj"], out=b["x0"])
        self._conv(b["x0"], R, p["pre_conv"], "pre_conv", out=b["lat"])
        # sliding-window transformer
        tr = p["transformer"]
        ops.linear(b["lat"], *tr["input_proj"], out=b["h"])
        ops.codec_positions(st.frames, self.indices, B, T, RING, self.rot, self.cache, advance=True)
        L = cfg.layers
        for i, layer in enumerate(tr["layers"]):
            keys, values = st.kv[i], st.kv[L + i]
            ops.linear(b["h"], layer["qkv"], out=b["qkv"], row_norm_eps=cfg.eps)
            q = ops.qk_norm_rope_kv(b["qkv"], None, None, cfg.eps, self.cos, self.sin, self.rot, self.cache, keys,
                                    values, q_heads=cfg.heads, kv_heads=cfg.heads, head_dim=cfg.head_dim, length=T,
                                    query_out=b["q"].view(R, cfg.heads, cfg.head_dim), slots=self.indices)
            ops.decode_attention(q, keys, values, self.rot, context=RING, rows_per_slot=T, window=cfg.window,
                                 slots=self.indices, ring=RING, out=b["attn"].view(R, cfg.heads, cfg.head_dim),
                                 workspace=self.ws_attn)
            ops.linear(b["attn"], layer["o"], out=b["h"], epilogue=_lib.EPI_RESIDUAL_SCALED, residual=b["h"],
                       scale=layer["attn_scale"])
            ops.linear(b["h"], layer["gate_up"], out=b["act"], epilogue=_lib.EPI_SWIGLU_PAIRED,
                       row_norm_eps=cfg.eps)
            ops.linear(b["act"], layer["down"], out=b["h"], epilogue=_lib.EPI_RESIDUAL_SCALED, residual=b["h"],
                       scale=layer["mlp_scale"])
        ops.rms_norm(b["h"], tr["norm"], cfg.eps, out=b["xn"])
        ops.linear(b["xn"], *tr["output_proj"], out=b["lat"])
        # upsampling: transposed conv (kernel == stride) + ConvNeXt
        x, rows = b["lat"], R
        for i, up in enumerate(p["upsample"]):
            t = up["tconv"]
            y = b[f"up{i}"]
            ops.linear(x, t["w"], t["b"], out=y.view(rows, t["r"] * t["c_out"]))
            rows *= t["r"]
            ops.dwconv_layernorm(y, B, rows // B, st.histories[f"up{i}.dw"], self.indices, up["dw_w"], up["dw_b"],
                                 up["ln_w"], up["ln_b"], up["ln_eps"], out=b[f"up{i}.ln"])
            ops.conv_history(y, B, rows // B, st.histories[f"up{i}.dw"], slots=self.indices)
            ops.linear(b[f"up{i}.ln"], *up["pw1"], out=b[f"up{i}.pw1"], epilogue=_lib.EPI_GELU)
            ops.linear(b[f"up{i}.pw1"], *up["pw2"], out=y, epilogue=_lib.EPI_RESIDUAL_SCALED, residual=y,
                       scale=up["gamma"])
            x = y
        # decoder: causal conv, 4 blocks (Snake -> transposed conv -> 3 residual units), Snake, conv
        self._conv(x, rows, p["conv0"], "conv0", out=b["d0"])
        x = b["d0"]
        for i, blk in enumerate(p["blocks"]):
            t = blk["tconv"]
            y = b[f"b{i}.y"]
            self._conv(x, rows, t, f"b{i}.tconv", snake=blk["snake"], out=y.view(rows, t["r"] * t["c_out"]),
                       reverse=True)
            rows *= t["r"]
            for u, unit in enumerate(blk["units"]):
                # dilated conv with the unit's second SnakeBeta in its epilogue, then the 1x1 conv + residual
                self._conv(y, rows, unit["conv1"], f"b{i}.u{u}.conv1", snake=unit["snake1"], out=b[f"b{i}.col1"],
                           epilogue=_lib.EPI_SNAKE, out_snake=unit["snake2"])
                ops.linear(b[f"b{i}.col1"], unit["conv2"]["w"], unit["conv2"]["b"], out=y,
                           epilogue=_lib.EPI_RESIDUAL, residual=y)
            x = y
        self._conv(x, rows, p["final_conv"], "final", snake=p["final_snake"], out=b["out"])
        ops.pcm16(b["out"], wave=self.wave, pcm=self.pcm)

    @torch.inference_mode()
    def capture(self, warmup: int = 2) -> None:
        """Warm up and capture; the state rows the warm-up touches are saved and restored
        (codec_slots.py:101-121)."""
        self.indices.copy_(torch.arange(self.batch, device=self.indices.device))
        saved = [buf.index_select(0 if buf.dim() == 1 or buf is not self.state.kv else 1, self.indices).clone()
                 for buf in self.state.buffers]
        stream = torch.cuda.Stream(device=self.indices.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.compute()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        before = _lib.launch_count()
        with torch.cuda.graph(self.graph, stream=stream):
            self.compute()
        self.launches = _lib.launch_count() - before     # this library's kernels per replay
        torch.cuda.synchronize()
        for buf, original in zip(self.state.buffers, saved):
            buf.index_copy_(0 if buf is not self.state.kv else 1, self.indices, original)

    @torch.inference_mode()
    def run(self, indices, codes, clone: bool = True):
        # slot indices from pinned host memory, asynchronously: a pageable or blocking copy would
        # make the host wait for everything queued on this stream (the tick the decode follows)
        if not isinstance(indices, torch.Tensor):
            indices = torch.tensor(indices, dtype=torch.long, pin_memory=True)
        self.indices.copy_(indices, non_blocking=True)
        self.codes.copy_(codes)
        if self.graph is None:
            self.compute()
        else:
            self.graph.replay()
            self.replays += 1
        return (self.wave.clone(), self.pcm.clone()) if clone else (self.wave, self.pcm)

    def close(self) -> None:
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None


class CodecSlots:
    """Slot-indexed incremental codec (codec_slots.py:133-338 surface)."""

    def __init__(self, cfg: CodecConfig, packed: dict, slots: int, device, max_chunk_frames: int = 8,
                 use_graphs: bool = True, max_positions: int = 1 << 14, streams: int = 1):
        if slots < 1:
            raise ValueError("Codec slots must be positive")
        if streams not in (1, 2):
            raise ValueError("Codec streams must be 1 or 2")
        if not 1 <= max_chunk_frames <= RING - cfg.window:
            raise ValueError("Codec maximum chunk must fit the KV ring")
        self.cfg, self.packed, self.slots = cfg, packed, slots
        self.device = torch.device(device)
        self.max_chunk_frames = max_chunk_frames
        self.state = CodecState(cfg, packed, slots, self.device)
        self.cos, self.sin = rope_tables(max_positions, cfg.head_dim, cfg.theta, self.device)
        self.use_graphs = use_graphs
        self.graphs: dict[tuple, CodecStep] = {}
        # Two lanes (codec_slots.py:279-305): groups of one call alternate between two streams,
        # each lane with its own graphs and buffers, fenced before decode_groups returns.
        self.stream_count = streams
        self.lanes = [torch.cuda.Stream(device=self.device) for _ in range(streams)] if streams == 2 else []

    def _graph(self, batch: int, length: int, lane: int = 0) -> CodecStep:
        key = (batch, length) if self.stream_count == 1 else (batch, length, lane)
        step = self.graphs.get(key)
        if step is None:
            step = CodecStep(self.cfg, self.packed, self.state, batch, length, self.cos, self.sin)
            if self.use_graphs:
                step.capture()
            self.graphs[key] = step
        return step

    def _validate(self, indices, codes) -> None:
        if (not indices or len(set(indices)) != len(indices) or min(indices) < 0 or max(indices) >= self.slots
                or codes.ndim != 3 or codes.shape[0] != len(indices) or codes.shape[1] != self.cfg.codebooks
                or not 1 <= codes.shape[-1] <= self.max_chunk_frames or codes.device != self.device
                or codes.dtype != torch.long):
            raise ValueError(f"Expected unique valid slots and [batch, codebooks, 1..{self.max_chunk_frames}] codes")

    def prewarm(self, max_batch: int) -> None:
        if not 1 <= max_batch <= self.slots:
            raise ValueError("Codec warmup batch must fit the slot arena")
        for batch in range(1, max_batch + 1):
            for length in range(1, self.max_chunk_frames + 1):
                for lane in range(self.stream_count):
                    self._graph(batch, length, lane)

    def decode(self, indices, codes, lane: int = 0):
        """Decode new codes of the given slots -> (wave fp32 [b, len*1920], pcm16 [b, len*1920])."""
        indices = list(indices)
        self._validate(indices, codes)
        # the slot list as a pinned host tensor: the graph uploads it without waiting on the stream
        slots = torch.tensor(indices, dtype=torch.long, pin_memory=torch.cuda.is_available())
        return self._graph(len(indices), codes.shape[-1], lane).run(slots, codes)

    def decode_groups(self, groups, on_output=None):
        """Decode several (indices, codes) groups (codec_slots.py:241-305 surface); the groups'
        slots are disjoint. With one stream they are enqueued in order on the current stream;
        with two, group i runs on lane i % 2 after the current stream's pending work, and the
        current stream waits for both lanes before this returns (so resets and moves that
        follow are ordered after the decodes). `on_output(i, output)` gets each (wave, pcm).
        Every group is checked (slots in range, unique within and across groups, code shape and
        type) before the first one is submitted, so an invalid later group launches nothing."""
        groups = [(list(indices), codes) for indices, codes in groups]
        claimed = set()
        for indices, codes in groups:
            self._validate(indices, codes)
            if claimed.intersection(indices):
                raise ValueError("Codec groups must use disjoint slots")
            claimed.update(indices)
        if self.stream_count == 1 or len(groups) < 2:
            outputs = []
            for index, (indices, codes) in enumerate(groups):
                outputs.append(self.decode(indices, codes))
                if on_output is not None:
                    on_output(index, outputs[-1])
            return outputs
        producer = torch.cuda.current_stream(self.device)
        for lane in self.lanes:
            lane.wait_stream(producer)
        outputs = []
        try:
            for index, (indices, codes) in enumerate(groups):
                lane = self.lanes[index % 2]
                with torch.cuda.stream(lane):
                    codes.record_stream(lane)
                    outputs.append(self.decode(indices, codes, lane=index % 2))
        finally:
            for lane in self.lanes:
                producer.wait_stream(lane)
        for index, (wave, pcm) in enumerate(outputs):
            wave.record_stream(producer)
            pcm.record_stream(producer)
            if on_output is not None:
                on_output(index, (wave, pcm))
        return outputs

    def reset(self, slot: int) -> None:
        self.state.reset(slot)

    def reset_range(self, start: int, count: int) -> None:
        self.state.reset_range(start, count)

    def move(self, source: int, destination: int) -> None:
        self.state.move(source, destination)

    def close(self) -> None:
        for step in self.graphs.values():
            step.close()
        self.graphs.clear()


class CodecGraph:
    """Windowed (non-incremental) decode of whole code windows (codec_graph.py:10-29).

    ``decode(codes [b, codebooks, T])`` returns the audio of all T frames decoded
    from a fresh stream, as the reference's full-sequence decoder call does. The
    causal decoder's output for a window equals that of an incremental decode of
    the same frames from zeroed state, so the window runs through a private
    CodecSlots arena of `max_batch` slots: the slots are reset, then the frames
    go through in chunks of up to `chunk` frames (one captured graph per
    (batch, chunk length)) and the chunk outputs are concatenated."""

    def __init__(self, cfg: CodecConfig, packed: dict, device, max_batch: int = 4, chunk: int = 56,
                 use_graphs: bool = True):
        self.slots = CodecSlots(cfg, packed, max_batch, device, max_chunk_frames=chunk, use_graphs=use_graphs)
        self.chunk = chunk
        self.captures = self.slots.graphs

    @torch.inference_mode()
    def decode(self, codes: torch.Tensor):
        batch, _, frames = codes.shape
        if not 1 <= batch <= self.slots.slots or frames < 1:
            raise ValueError("Window batch must fit the codec graph arena")
        self.slots.reset_range(0, batch)
        indices = list(range(batch))
        waves, pcms = [], []
        for start in range(0, frames, self.chunk):
            wave, pcm = self.slots.decode(indices, codes[..., start:start + self.chunk].contiguous())
            waves.append(wave)
            pcms.append(pcm)
        return torch.cat(waves, -1), torch.cat(pcms, -1)

    def close(self) -> None:
        self.slots.close()
