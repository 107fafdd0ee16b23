#!/usr/bin/env python
"""Benchmark of the B200 Qwen3-TTS decode path.

One "step" is one talker decode step for a continuous batch of 32 slots:
the 28-layer Qwen3 talker (hidden 2048, 16q/8kv x 128, FFN 6144, vocab 3072,
random-init N(0, 0.02) weights from a seed) on the slot-table KV arena with
ragged contexts U[64, 2048], greedy next-token selection, and the next
step's input embedding, replayed as one CUDA graph. Every 16 steps a few
slots are evicted and re-admitted with new seeded contexts. Each step emits
one codec frame per slot, so throughput is reported as frames/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs one independent engine replica per GPU (request-level data
parallelism: no collective on the data path); rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen3-tts-rsi-engine_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "codec frames/s (talker decode step, C=32)"
UNIT = "frames/s"
SLOTS = 32
CAPACITY = 4096
ADMIT_EVERY = 16
ADMIT_SLOTS = 4


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=40)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--layers", type=int, default=28, help="talker depth (28 = the benchmarked model)")
    p.add_argument("--slots", type=int, default=SLOTS,
                   help="step workload: concurrent slots (32 = BASELINE config 2; 64 = the C=64 roofline target)")
    p.add_argument("--op-costs", action="store_true",
                   help="print the in-graph cost of each talker-layer op (28 chained launches per op) and exit")
    p.add_argument("--workload", choices=["step", "serving", "predictor", "codec"], default="step",
                   help="step: BASELINE config 2 (default); serving: BASELINE config 5, end-to-end ContinuousModel")
    p.add_argument("--concurrency", type=int, default=32, help="serving: requests in flight (closed loop)")
    p.add_argument("--requests", type=int, default=128, help="serving: synthetic requests per timed pass")
    p.add_argument("--batch", type=int, default=64, help="predictor / codec: rows or streams (BASELINE configs 3, 4)")
    p.add_argument("--codec-streams", type=int, default=1, choices=[1, 2],
                   help="serving: codec decode lanes (ContinuousModel codec_streams)")
    p.add_argument("--frames", type=int, default=200, help="predictor: timed frames (BASELINE config 3)")
    return p.parse_args()


# ---------------------------------------------------------------------- distributed plumbing
class Dist:
    def __init__(self, backend: str):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.enabled = self.world > 1
        if self.enabled:
            import datetime
            import torch.distributed as dist
            kwargs = {}
            if backend == "nccl":  # one GPU per rank, bound before the group forms
                torch.cuda.set_device(self.local)
                kwargs["device_id"] = torch.device("cuda", self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kwargs)

    def barrier(self):
        if self.enabled:
            import torch.distributed as dist
            dist.barrier()

    def max(self, value: float) -> float:
        if not self.enabled:
            return value
        import torch.distributed as dist
        t = torch.tensor([value], dtype=torch.float64,
                         device="cuda" if dist.get_backend() == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.enabled:
            import torch.distributed as dist
            dist.destroy_process_group()


# ---------------------------------------------------------------------- workload
class Workload:
    """Seeded ragged contexts and the eviction/admission schedule."""

    def __init__(self, seed: int, slots: int = None):
        self.g = torch.Generator().manual_seed(seed)
        self.slots = slots = SLOTS if slots is None else slots
        self.positions = torch.randint(64, 2049, (slots,), generator=self.g)

    def admit(self):
        """Evict ADMIT_SLOTS seeded slots and admit new requests with fresh contexts."""
        slots = torch.randperm(self.slots, generator=self.g)[:ADMIT_SLOTS]
        fresh = torch.randint(64, 2049, (ADMIT_SLOTS,), generator=self.g)
        return slots, fresh


# ---------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons every 10 ms through NVML (read-only), so that a
    timed region of a tenth of a second still gets several samples."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.stop_flag = None
        self.thread = None
        self.max_mhz = None

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.index]) if visible else self.index
            handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            return
        self.stop_flag = threading.Event()

        def loop():
            while not self.stop_flag.is_set():
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                    reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                    power = pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                    self.samples.append((sm, reasons, power))
                except Exception:
                    pass
                self.stop_flag.wait(0.01)

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def stop(self):
        if self.thread is None:
            return None
        self.stop_flag.set()
        self.thread.join(timeout=2)
        if not self.samples:
            return None
        active = set()
        for _, bits, _ in self.samples:
            for name, bit in self.REASONS.items():
                if bits & bit:
                    active.add(name)
        return {"sm_mhz": float(np.median([s[0] for s in self.samples])), "sm_max_mhz": float(self.max_mhz),
                "reasons": sorted(active), "power_w_max": max(s[2] for s in self.samples),
                "samples": len(self.samples)}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu traffic summary under profiles/
    (a `| kernel | bytes | ...` table row), if present."""
    path = ROOT / "profiles" / "traffic.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        cells = [c.strip() for c in line.strip().strip("|").split("|")]
        if len(cells) >= 2 and cells[0] == kernel and cells[1].isdigit():
            return int(cells[1])
    return None


# ---------------------------------------------------------------------- CPU baseline (oracle)
def cpu_decode_sample(cfg, positions, steps: int, sample_layers: int, seed: int, threads=(None,)):
    """Time the oracle's fp32 talker layers on the host cores for `steps` steps.

    Bounded sample: `sample_layers` of the 28 layers at full widths and the
    real ragged contexts; the per-step time is scaled by 28 / sample_layers.
    Runs once per entry of `threads` (None = every host core) and returns
    [(seconds per step, threads used)] in that order.
    """
    from dataclasses import replace

    from oracle import decoder as OD
    from qwen3_tts_b200.weights import decoder_weights

    small = replace(cfg, layers=sample_layers)
    weights = decoder_weights(small, seed, device="cpu", dtype=torch.bfloat16)
    for layer in weights["layers"]:
        for key in list(layer):
            layer[key] = layer[key].float()
    cap = int(positions.max()) + steps + 2
    tables = OD.Tables(cap + 1, cfg.head_dim, cfg.theta)
    h = torch.randn(len(positions), 1, cfg.hidden) * 0.1
    results = []
    for count in threads:
        torch.set_num_threads(count or os.cpu_count() or 1)
        cache = OD.new_cache(small, len(positions), cap)
        pos = positions.clone().view(-1, 1)
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            x = h
            for w, (ck, cv) in zip(weights["layers"], cache):
                x = OD.layer_forward(small, w, x, pos, ck, cv, pos, tables, "fp32")
            times.append(time.perf_counter() - t0)
            pos = pos + 1
        results.append((float(np.median(times)) * (cfg.layers / sample_layers), torch.get_num_threads()))
    torch.set_num_threads(os.cpu_count() or 1)
    return results


# ---------------------------------------------------------------------- B200 arm
def run_b200(args, dist: Dist):
    from qwen3_tts_b200 import _lib, ops
    from qwen3_tts_b200.config import TALKER
    from dataclasses import replace
    from qwen3_tts_b200.talker import TalkerDecoder
    from qwen3_tts_b200.weights import decoder_weights

    cfg = TALKER if args.layers == TALKER.layers else replace(TALKER, layers=args.layers)
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    work = Workload(args.seed + dist.rank)
    weights = decoder_weights(cfg, seed=args.seed, device=dev)
    engine = TalkerDecoder(cfg, weights, slots=SLOTS, capacity=CAPACITY, device=dev, use_graphs=False)
    del weights
    step = engine.step_for(SLOTS, CAPACITY)
    table = engine.weights["embedding"]
    tokens = torch.zeros(SLOTS, 1, dtype=torch.long, device=dev)
    zero_u = torch.zeros(SLOTS, dtype=torch.float32, device=dev)
    step.positions.copy_(work.positions.to(dev))
    step.rotary.copy_(work.positions.to(dev))
    step.inputs.copy_((torch.randn(SLOTS, cfg.hidden, device=dev) * 0.05).to(torch.bfloat16))

    def tick():
        step.compute()
        ops.sample(step.logits, uniforms=zero_u, top_k=1, temperature=1.0, tokens=tokens)  # greedy
        ops.embedding(tokens.view(-1), table, out=step.inputs)
        ops.advance(step.positions)
        ops.advance(step.rotary)

    # count our kernels per step (eager pass), then capture the step as one graph
    before = _lib.launch_count()
    tick()
    torch.cuda.synchronize()
    launches_per_step = _lib.launch_count() - before
    saved = step.positions.clone(), step.rotary.clone()
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(2):
            tick()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        tick()
    torch.cuda.synchronize()
    step.positions.copy_(saved[0])
    step.rotary.copy_(saved[1])

    # the eviction/admission schedule is drawn up front and kept on the device, so an
    # admission inside the timed region is two device-side scatters (no host sync)
    schedule = [work.admit() for _ in range(max(1, args.steps // ADMIT_EVERY + 1))]
    adm_slots = torch.stack([s for s, _ in schedule]).to(dev)
    adm_fresh = torch.stack([f for _, f in schedule]).to(dev)

    def admit(i):
        if i and i % ADMIT_EVERY == 0:
            k = i // ADMIT_EVERY - 1
            step.positions.index_copy_(0, adm_slots[k], adm_fresh[k])
            step.rotary.index_copy_(0, adm_slots[k], adm_fresh[k])

    for i in range(args.warmup):
        graph.replay()
    # keep replaying (untimed) for ~0.5 s so the clocks are at their loaded steady state
    t_end = time.perf_counter() + 0.5
    while time.perf_counter() < t_end:
        graph.replay()
        torch.cuda.synchronize()
    step.positions.copy_(work.positions.to(dev) + args.warmup)
    step.rotary.copy_(work.positions.to(dev) + args.warmup)
    torch.cuda.synchronize()
    positions_at_start = step.positions.cpu()

    clocks = ClockSampler(dev.index)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        admit(i)
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    elapsed_ms = dist.max(start.elapsed_time(end))
    clock_info = clocks.stop()
    status = ops.read_status(dev)

    # ---- end to end through the public step API: pinned host inputs in, token ids out, every step
    host_in = torch.empty(SLOTS, cfg.hidden, dtype=torch.bfloat16).pin_memory()
    host_in.copy_((torch.randn(SLOTS, cfg.hidden) * 0.05).to(torch.bfloat16))
    host_pos = work.positions.clone().pin_memory()
    host_tok = torch.empty(SLOTS, 1, dtype=torch.long).pin_memory()
    step_g = engine.step_for(SLOTS, CAPACITY)
    step_g.positions.copy_(host_pos.to(dev))
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step_g.compute()
        ops.sample(step_g.logits, uniforms=zero_u, top_k=1, temperature=1.0, tokens=tokens)
    torch.cuda.current_stream().wait_stream(stream)
    with torch.cuda.graph(e2e_graph, stream=stream):
        step_g.compute()
        ops.sample(step_g.logits, uniforms=zero_u, top_k=1, temperature=1.0, tokens=tokens)
    torch.cuda.synchronize()
    e2e_steps = max(4, args.steps // 2)
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        step_g.inputs.copy_(host_in, non_blocking=True)
        step_g.positions.copy_(host_pos, non_blocking=True)
        step_g.rotary.copy_(host_pos, non_blocking=True)
        e2e_graph.replay()
        host_tok.copy_(tokens, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        host_pos += 1
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = dist.max(e0.elapsed_time(e1))
    h2d = host_in.numel() * 2 + host_pos.numel() * 8 * 2
    d2h = host_tok.numel() * 8
    if os.environ.get("Q3T_BENCH_DIAG"):
        for name, g in (("tick_graph", graph), ("step_graph", e2e_graph)):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                g.replay()
            b.record()
            torch.cuda.synchronize()
            print(json.dumps({"diag": name, "ms_per_replay": a.elapsed_time(b) / args.steps}), file=sys.stderr)

    # ---- roofline of the dominant kernels, timed alone with L2 flushed between launches
    kernels = kernel_rooflines(cfg, engine, step, positions_at_start, dev)
    result = {
        "elapsed_ms": elapsed_ms, "launches_per_step": launches_per_step, "status": status,
        "clocks": clock_info, "e2e_ms": e2e_ms, "e2e_steps": e2e_steps, "h2d": h2d, "d2h": d2h,
        "kernels": kernels, "positions": positions_at_start, "cfg": cfg,
    }
    graph.reset()
    e2e_graph.reset()
    engine.close()
    return result


def attention_in_graph(cfg, engine, step, pos, replays=5):
    """Seconds per launch of the decode attention as the step runs it: one CUDA graph of
    cfg.layers back-to-back launches over the layers' K/V (programmatic dependent launch,
    the step's chunk plan), timed with CUDA events on the replay stream."""
    from qwen3_tts_b200 import ops

    def chain():
        for i in range(cfg.layers):
            ops.decode_attention(step.q, engine.arena.keys[i], engine.arena.values[i], pos, context=step.context,
                                 out=step.attn, workspace=step.ws_attn)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        chain()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        chain()
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(replays):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    graph.reset()
    return a.elapsed_time(b) / 1e3 / (replays * cfg.layers)


def kernel_rooflines(cfg, engine, step, positions, dev):
    from qwen3_tts_b200 import _lib, ops
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    B = SLOTS
    layer = engine.weights["layers"][0]
    pos = positions.to(dev)

    def timed(fn, reps=10):
        total = 0.0
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            total += a.elapsed_time(b)
        return total / reps / 1e3  # seconds per launch

    kv_bytes = int(((positions + 1).sum()).item()) * cfg.kv_heads * cfg.head_dim * 2 * 2
    q_bytes = B * cfg.q_width * 2 * 2
    out = {}
    t = timed(lambda: ops.decode_attention(step.q, engine.arena.keys[0], engine.arena.values[0], pos,
                                           context=step.context, out=step.attn, workspace=step.ws_attn))
    out["decode_attention"] = {"seconds": t, "bytes": kv_bytes + q_bytes, "per_step": cfg.layers,
                               "seconds_in_graph": attention_in_graph(cfg, engine, step, pos)}
    eps = cfg.eps if layer.folded else None   # QKV and gate/up carry the folded RMSNorm
    for name, w, x, o, epi, res, norm in (
            ("linear_gate_up", layer.gate_up, step.h, step.act, _lib.EPI_SWIGLU_PAIRED, None, eps),
            ("linear_qkv", layer.qkv, step.h, step.qkv, _lib.EPI_STORE, None, eps),
            ("linear_down", layer.down, step.act, step.h, _lib.EPI_RESIDUAL, step.h, None),
            ("linear_o", layer.o, step.attn.view(B, -1), step.h, _lib.EPI_RESIDUAL, step.h, None)):
        t = timed(lambda: ops.linear(x, w, out=o, epilogue=epi, residual=res, row_norm_eps=norm))
        nbytes = w.numel() * 2 + x.numel() * 2 + o.numel() * 2 * (2 if res is not None else 1)
        out[name] = {"seconds": t, "bytes": nbytes, "per_step": cfg.layers}
    del flush
    return out


# ---------------------------------------------------------------------- reference (CPU) arm
def run_reference(args, dist: Dist):
    from qwen3_tts_b200.config import TALKER
    work = Workload(args.seed)
    layers = 2
    [(per_step, threads)] = cpu_decode_sample(TALKER, work.positions, args.warmup + args.steps, layers, args.seed)
    value = SLOTS / per_step
    return {
        "metric": f"codec frames/s (talker decode step, C={SLOTS})", "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"BASELINE config 2: talker decode step, {SLOTS} slots, ctx U[64,2048]",
                   "model": "qwen3-tts talker 28L h2048 (random init)", "global_batch": SLOTS,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"oracle fp32 talker, {layers} of 28 layers at full width, 32 slots, "
                                   f"ragged ctx; median step time scaled by 28/{layers}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def op_costs(args) -> None:
    """In-graph cost of each op of a talker layer: one CUDA graph of 28 back-to-back launches
    of the same op cycling through the 28 layers' weights and KV (nothing stays in L2), timed
    with CUDA events; one JSON line per op (us per launch, achieved GB/s)."""
    from qwen3_tts_b200 import _lib, ops
    from qwen3_tts_b200.config import TALKER
    from qwen3_tts_b200.talker import TalkerDecoder
    from qwen3_tts_b200.weights import decoder_weights

    dev = torch.device("cuda:0")
    cfg, L = TALKER, TALKER.layers
    work = Workload(args.seed)
    positions = work.positions.to(dev)
    engine = TalkerDecoder(cfg, decoder_weights(cfg, args.seed, dev), SLOTS, CAPACITY, dev, use_graphs=False)
    step = engine.step_for(SLOTS, CAPACITY)
    for plane in engine.arena.keys + engine.arena.values:
        plane.normal_()
    W = engine.weights["layers"]
    eps = cfg.eps if W[0].folded else None
    # the step's split-KV plan, as TalkerStep.compute makes it once per step
    ops.attention_plan(positions, step.ws_attn, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                       context=CAPACITY)

    def graph_us(fn, replays=10):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(L):
                fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for i in range(L):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(replays):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3 / (L * replays)

    kv = int(((work.positions + 1).sum()).item()) * cfg.kv_heads * cfg.head_dim * 2 * 2
    B = SLOTS
    costs = {
        "linear_qkv": (lambda i: ops.linear(step.h, W[i].qkv, out=step.qkv, row_norm_eps=eps), W[0].qkv.numel() * 2),
        "qk_norm_rope_kv": (lambda i: ops.qk_norm_rope_kv(
            step.qkv, W[i].q_norm, W[i].k_norm, cfg.eps, engine.cos, engine.sin, positions, positions,
            engine.arena.keys[i], engine.arena.values[i], q_heads=cfg.q_heads, kv_heads=cfg.kv_heads,
            head_dim=cfg.head_dim, query_out=step.q), B * cfg.qkv_width * 2 * 2),
        "decode_attention": (lambda i: ops.decode_attention(
            step.q, engine.arena.keys[i], engine.arena.values[i], positions, context=CAPACITY, out=step.attn,
            workspace=step.ws_attn), kv),
        "decode_attention_qkv (fused q/k norm, RoPE, KV write)": (lambda i: ops.decode_attention_qkv(
            step.qkv, W[i].q_norm, W[i].k_norm, cfg.eps, engine.cos, engine.sin, positions, engine.arena.keys[i],
            engine.arena.values[i], positions, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
            context=CAPACITY, out=step.attn, workspace=step.ws_attn), kv),
        "linear_o": (lambda i: ops.linear(step.attn.view(B, -1), W[i].o, out=step.h, epilogue=_lib.EPI_RESIDUAL,
                                          residual=step.h), W[0].o.numel() * 2),
        "linear_gate_up": (lambda i: ops.linear(step.h, W[i].gate_up, out=step.act, epilogue=_lib.EPI_SWIGLU_PAIRED,
                                                row_norm_eps=eps), W[0].gate_up.numel() * 2),
        "linear_down": (lambda i: ops.linear(step.act, W[i].down, out=step.h, epilogue=_lib.EPI_RESIDUAL,
                                             residual=step.h), W[0].down.numel() * 2),
    }
    total = 0.0
    step_ops = {"linear_qkv", "decode_attention_qkv (fused q/k norm, RoPE, KV write)", "linear_o", "linear_gate_up",
                "linear_down"}
    for name, (fn, nbytes) in costs.items():
        us = graph_us(fn)
        total += us if name in step_ops else 0.0
        print(json.dumps({"op": name, "us_per_launch": round(us, 2), "GBps": round(nbytes / us / 1e3, 1)}))
    print(json.dumps({"layer_us (ops of the decode step)": round(total, 1), "step_ms_28_layers": round(total * L / 1e3, 3),
                      "status": ops.read_status(dev)}))


def serving_requests(seed: int, count: int):
    """BASELINE config 5 synthetic requests: text ids U[0, 151936) of length U[20, 200], one of two
    speakers, target audio frames U[50, 400] (max_new_tokens = target + 1, so each ends at its target)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(count):
        length = int(torch.randint(20, 201, (1,), generator=g))
        ids = torch.randint(0, 151936, (length,), generator=g).tolist()
        target = int(torch.randint(50, 401, (1,), generator=g))
        out.append({"input": "", "input_ids": ids, "voice": ("voice_a", "voice_b")[i % 2], "language": "english",
                    "instructions": "", "max_new_tokens": target + 1, "seed": seed * 1000 + i})
    return out


def run_serving(args) -> dict:
    """Closed-loop serving through ContinuousModel.tick at `concurrency` requests in flight.

    A first pass over the same request set captures every graph shape (untimed); the
    second pass is timed on the host clock (the engine synchronises once per tick).
    Metrics follow the reference's service benchmark (``metrics.summarize``): frames/s =
    delivered audio x 12.5 / wall time; TTFA = submission -> first PCM chunk (p50/p95,
    interpolated); RTF = mean over requests of latency / audio duration. A request ends at
    its synthetic target length (the max_new_tokens cap stands in for EOS at the target)."""
    from qwen3_tts_b200.continuous import ContinuousModel
    from qwen3_tts_b200.metrics import summarize
    slots = 1 << max(0, (args.concurrency - 1).bit_length())
    engine = dict(max_slots=slots, initial_capacity=1024, seed=args.seed, codec_batch_size=4,
                  codec_streams=args.codec_streams)
    gpus = max(1, args.gpus)
    if gpus > 1:
        # request-level data parallelism: one engine process per GPU behind the host dispatcher,
        # `concurrency` requests in flight per GPU
        from qwen3_tts_b200.dispatcher import Dispatcher
        model = Dispatcher.start(gpus, engine, per_engine=args.concurrency)
    else:
        model = ContinuousModel(None, torch.device("cuda:0"), **engine)
    concurrency = args.concurrency * gpus
    requests = serving_requests(args.seed, args.requests * gpus)

    def one_pass():
        pending = list(enumerate(requests))
        submitted, first_audio, done, frames = {}, {}, {}, 0
        in_flight = 0

        def emit(identifier, pcm, rate):
            if len(pcm):
                first_audio.setdefault(identifier, time.perf_counter())

        start = time.perf_counter()
        while pending or in_flight:
            subs = []
            while pending and in_flight + len(subs) < concurrency:
                subs.append(pending.pop(0))
            now = time.perf_counter()
            for identifier, _ in subs:
                submitted[identifier] = now
            in_flight += len(subs)
            for identifier, result in model.tick(subs, emit=emit):
                done[identifier] = (time.perf_counter(), result)
                frames += result["codec_frames"]
                in_flight -= 1
        wall = time.perf_counter() - start
        records = []
        for i in submitted:
            finished, result = done[i]
            records.append({"success": result["finish_reason"] in ("stop", "length") and result["codec_frames"] > 0
                            and i in first_audio, "audio_seconds": result["codec_frames"] / 12.5,
                            "elapsed_seconds": finished - submitted[i],
                            "ttfa_seconds": first_audio.get(i, finished) - submitted[i]})
        return dict(summarize(records, wall, 12.5), frames=frames)

    one_pass()                       # graph capture for every (batch, context) and codec shape met
    res = one_pass()
    model.close()
    return {"frames_per_s": res["throughput_frames_s"], "frames": res["frames"], "wall_s": res["wall_seconds"],
            "ttfa_p50_ms": res["ttfa_p50_ms"], "ttfa_p95_ms": res["ttfa_p95_ms"], "rtf": res["rtf_mean"],
            "status": res["status"], "failed_requests": res["failed_requests"], "slots": slots, "gpus": gpus}


# BASELINE config 3 per predictor step: 5 layers (QKV, O, gate/up, down) + input projection +
# one head, bf16 = 165.7 MB; one frame runs 15 steps.
PREDICTOR_STEP_BYTES = (5 * (1024 * 4096 + 2048 * 1024 + 3 * 1024 * 3072) + 2048 * 1024 + 1024 * 2048) * 2


def timed_region(fn, count: int) -> float:
    """CUDA-event milliseconds of `count` calls of fn on the current stream; the region is also
    bracketed by cudaProfilerStart/Stop (no-ops without a profiler) for ncu --profile-from-start off."""
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(count):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    return a.elapsed_time(b)


def run_predictor(args) -> dict:
    """the 15-codebook code predictor for `batch` rows (64), Philox sampling
    with T 0.9, top-k 50, top-p 0.95, over `frames` frames (200). One frame = PredictorStep.run:
    the talker hidden state and first code of every row copied in, then one replay of the
    captured chain (15 steps x 5 layers, heads, sampling, frame embedding). Inputs are
    device-resident seeded N(0,1) hidden states and uniform first codes."""
    from qwen3_tts_b200 import ops
    from qwen3_tts_b200.config import PREDICTOR
    from qwen3_tts_b200.predictor import PredictorStep
    from qwen3_tts_b200.weights import decoder_weights, pack_decoder
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    B, F = args.batch, args.frames
    g = torch.Generator(device=dev).manual_seed(args.seed)
    weights = pack_decoder(decoder_weights(PREDICTOR, args.seed, dev), dev)
    talker_emb = (torch.randn(3072, PREDICTOR.talker_hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    step = PredictorStep(PREDICTOR, weights, talker_emb, B, dev, temperature=0.9, top_k=50, top_p=0.95,
                         philox_seed=args.seed)
    step.capture()
    total = F + args.warmup
    hidden = torch.randn(total, B, PREDICTOR.talker_hidden, generator=g, device=dev).to(torch.bfloat16)
    first = torch.randint(0, 2048, (total, B), generator=g, device=dev)
    offsets = torch.zeros(B, dtype=torch.long, device=dev)

    def frame(i):
        offsets.add_(16)  # each frame draws 15 Philox uniforms per row
        step.run(hidden[i], first[i], offsets=offsets, clone=False)

    for i in range(args.warmup):
        frame(i)
    ms = timed_region(lambda i: frame(args.warmup + i), F)
    status = ops.read_status(dev)
    step.close()
    per_frame_bytes = 15 * PREDICTOR_STEP_BYTES
    fps = B * F / (ms / 1e3)
    peak, peak_kind = measured_peaks()
    return {"frames_per_s": fps, "ms_per_frame": ms / F, "status": status,
            "hbm_fraction": per_frame_bytes * (F / (ms / 1e3)) / (peak * 1e9), "peak_kind": peak_kind}


def run_codec(args) -> dict:
    """incremental codec decode of `batch` streams (64) in 4-frame chunks.
    One step = CodecSlots.decode of every stream's next 4 frames (codes uniform over 2048,
    seeded, device-resident): RVQ, pre-conv, 8-layer sliding-window transformer, upsampling,
    decoder convolutions, PCM16, as one captured graph per (batch, frames)."""
    from qwen3_tts_b200 import ops
    from qwen3_tts_b200.codec import CodecSlots, pack_codec
    from qwen3_tts_b200.codec_weights import random_codec
    from qwen3_tts_b200.config import CODEC
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    B, T = args.batch, 4
    codec = CodecSlots(CODEC, pack_codec(random_codec(CODEC, args.seed), dev), B, dev, max_chunk_frames=8)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    total = args.steps + args.warmup
    codes = torch.randint(0, CODEC.codebook_size, (total, B, CODEC.codebooks, T), generator=g, device=dev)
    indices = list(range(B))
    for i in range(args.warmup):
        codec.decode(indices, codes[i])
    ms = timed_region(lambda i: codec.decode(indices, codes[args.warmup + i]), args.steps)
    status = ops.read_status(dev)
    codec.close()
    return {"frames_per_s": B * T * args.steps / (ms / 1e3), "ms_per_step": ms / args.steps, "status": status}


def main():
    global SLOTS
    args = parse_args()
    if args.slots < 1 or args.slots > 64:
        raise SystemExit("--slots must be within 1..64")
    SLOTS = args.slots
    if args.op_costs:
        op_costs(args)
        return
    if args.workload == "predictor":
        res = run_predictor(args)
        print(json.dumps({
            "metric": f"codec frames/s (code predictor, batch {args.batch})", "value": res["frames_per_s"],
            "unit": UNIT, "n_gpus": 1, "frames": args.frames, "warmup": args.warmup, "ms_per_frame": res["ms_per_frame"],
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded random-init weights, N(0,1) hidden)",
            "config": {"workload": "BASELINE config 3: 15-codebook predictor, T 0.9, top-k 50, top-p 0.95, Philox",
                       "batch": args.batch},
            "hbm_fraction": res["hbm_fraction"], "peak_kind": res["peak_kind"], "status_word": res["status"]}))
        return
    if args.workload == "codec":
        res = run_codec(args)
        print(json.dumps({
            "metric": f"codec frames/s (incremental codec decode, {args.batch} streams x 4-frame chunks)",
            "value": res["frames_per_s"], "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"], "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (seeded random-init codec, uniform codes)",
            "config": {"workload": "BASELINE config 4: incremental codec decode", "streams": args.batch,
                       "chunk_frames": 4}, "status_word": res["status"]}))
        return
    if args.workload == "serving":
        if int(os.environ.get("RANK", 0)) != 0:
            return  # one host process drives every GPU through the dispatcher
        res = run_serving(args)
        print(json.dumps({
            "metric": f"codec frames/s (end-to-end serving, C={args.concurrency} per GPU)", "value": res["frames_per_s"],
            "unit": UNIT, "n_gpus": res["gpus"], "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (BASELINE config 5 request recipe, seeded random-init weights)",
            "config": {"workload": "BASELINE config 5: talker -> code predictor -> incremental codec, closed loop",
                       "concurrency": args.concurrency, "requests": args.requests * res["gpus"], "slots": res["slots"],
                       "codec_streams": args.codec_streams},
            "ttfa_p50_ms": res["ttfa_p50_ms"], "ttfa_p95_ms": res["ttfa_p95_ms"], "rtf": res["rtf"],
            "frames": res["frames"], "wall_s": res["wall_s"], "status": res["status"],
            "failed_requests": res["failed_requests"]}))
        return
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", 0))
        if rank != 0:
            return
        print(json.dumps(run_reference(args, Dist.__new__(Dist))))
        return
    dist = Dist("nccl")
    res = run_b200(args, dist)
    cfg = res["cfg"]
    frames = SLOTS * args.steps * dist.world
    seconds = res["elapsed_ms"] / 1e3
    value = frames / seconds
    kernels = res["kernels"]
    # dominant kernel = largest share of the step (seconds x launches per step)
    dom_name = max(kernels, key=lambda k: kernels[k]["seconds"] * kernels[k]["per_step"])
    dom = kernels[dom_name]
    peak, peak_kind = measured_peaks()
    in_graph = dom.get("seconds_in_graph")
    achieved = dom["bytes"] / (in_graph or dom["seconds"]) / 1e9
    positions = res["positions"]
    kv_step = int(((positions + 1).sum()).item()) * cfg.kv_heads * cfg.head_dim * 2 * 2 * cfg.layers
    step_bytes = cfg.weight_bytes() + kv_step
    e2e_value = SLOTS * res["e2e_steps"] * dist.world / (res["e2e_ms"] / 1e3)
    line = {
        "metric": f"codec frames/s (talker decode step, C={SLOTS})", "value": value, "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res["elapsed_ms"] / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights)",
        "config": {"workload": f"BASELINE config 2: talker decode step, {SLOTS} slots, ctx U[64,2048], "
                               "greedy, evict/admit 4 slots every 16 steps",
                   "layers": cfg.layers, "global_batch": SLOTS * dist.world, "slots_per_gpu": SLOTS,
                   "parallelism": f"replicas x{dist.world} (request-level data parallel)",
                   "l2": f"inputs > L2 ({step_bytes / 1e9:.1f} GB streamed per step)",
                   "hbm_fraction_step": step_bytes / (res["elapsed_ms"] / args.steps / 1e3) / (peak * 1e9),
                   "bytes_per_step": step_bytes},
        "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": profile_traffic(dom_name),
                     "method": ("in graph: the step's back-to-back launches over every layer's K/V, CUDA events"
                                if in_graph else "alone, L2 flushed between launches, CUDA events"),
                     "achieved_alone": dom["bytes"] / dom["seconds"] / 1e9},
        "kernels": {k: {"us": v["seconds"] * 1e6, "GBps": v["bytes"] / v["seconds"] / 1e9,
                        "frac": v["bytes"] / v["seconds"] / 1e9 / peak} for k, v in kernels.items()},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
        "gpu_launches": res["launches_per_step"] * args.steps,
        "status_word": res["status"],
        "clocks": res["clocks"],
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        (per_step, threads), (per_step4, _) = cpu_decode_sample(cfg, positions, 3, 2, args.seed, (None, 4))
        line["cpu_baseline"] = {"value": SLOTS / per_step, "unit": UNIT, "cores": threads, "kind": "port",
                                "value_4_threads": SLOTS / per_step4,
                                "sample": f"oracle fp32 talker, 2 of 28 layers at full width, {SLOTS} slots, "
                                          "same contexts, median of 3 steps scaled by 14; value_4_threads = the "
                                          "same at 4 threads (the reference's default torch thread count)"}
    if dist.rank == 0:
        print(json.dumps(line))
    dist.close()


if __name__ == "__main__":
    main()
