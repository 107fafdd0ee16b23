#!/usr/bin/env python
"""Benchmark of the B200 Qwen3-TTS decode path.

Default (the contract line): BASELINE config 5, end-to-end serving of the full
talker -> code predictor -> incremental codec pipeline at concurrency 64 per
GPU, random-init weights of the 1.7B geometry, synthetic requests from a seed
(text ids U[0, 151936) of length U[20, 200], one of two speakers, U[50, 400]
target frames). BASELINE's corpus (Seed-TTS transcripts) is not used.

* ``value``: device pipeline throughput in codec frames/s. One step = one
  steady-state engine tick for 64 active slots, all device-resident: the tick
  graph (frame embedding -> 15-codebook predictor -> 28-layer talker -> semantic
  sampling -> commit) plus the incremental codec decode of 64 frames of audio
  (8 streams x 8-frame chunks, rotating over the slots) and PCM16. W untimed
  steps, then exactly K steps between CUDA events.
* ``e2e``: the same metric through the public API, ``ContinuousModel.tick``, in
  a closed loop over the request set (admission and prefill, host token reads,
  PCM16 copied to the host every tick), timed with CUDA events; TTFA p50/p95
  and RTF follow the reference's service benchmark (benchmark.py:17-34).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 (torchrun, one rank per GPU) runs one engine per GPU over its own shard of
requests (request-level data parallelism: no collective on the data path); the
timed regions are bracketed by barriers and the max over ranks is reported.
Other workloads: ``--workload step`` (config 2, the talker decode step),
``predictor`` (config 3), ``codec`` (config 4), ``dispatch`` (closed-loop
serving through the host dispatcher over several GPUs from one process).
"""
from __future__ import annotations

import argparse
import collections
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

UNIT = "frames/s"
SERVING_SLOTS = 64          # BASELINE config 5 at C=64 per GPU
SERVING_CODEC_BATCH = 8     # streams per codec call (the reference's largest --codec-batch-size)
SERVING_CHUNK = 8           # frames per steady-state codec chunk
SLOTS = 32
CAPACITY = 4096
ADMIT_EVERY = 16
ADMIT_SLOTS = 4


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", choices=["serving", "step", "predictor", "codec", "dispatch", "chain", "prefill"],
                   default="serving",
                   help="serving: BASELINE config 5 (default); step: config 2; predictor: config 3; codec: config 4; "
                        "dispatch: closed-loop serving through the host dispatcher; chain: one layer's "
                        "projections as q3t_linear_chain against four linear launches")
    p.add_argument("--layers", type=int, default=28, help="step: talker depth (28 = the benchmarked model)")
    p.add_argument("--slots", type=int, default=SLOTS,
                   help="step: concurrent slots (32 = BASELINE config 2; 64 = the C=64 roofline target)")
    p.add_argument("--concurrency", type=int, default=SERVING_SLOTS, help="serving/dispatch: requests in flight")
    p.add_argument("--requests", type=int, default=128, help="serving/dispatch: synthetic requests per GPU")
    p.add_argument("--batch", type=int, default=64, help="predictor / codec: rows or streams (BASELINE configs 3, 4)")
    p.add_argument("--codec-streams", type=int, default=2, choices=[1, 2],
                   help="serving/dispatch: codec decode lanes (ContinuousModel codec_streams)")
    p.add_argument("--frames", type=int, default=200, help="predictor: timed frames (BASELINE config 3)")
    p.add_argument("--no-pipeline", action="store_true",
                   help="serving: decode each tick's audio before the next tick (pipeline_audio off)")
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

    def sum(self, value: float) -> float:
        if not self.enabled:
            return value
        import torch.distributed as dist
        t = torch.tensor([value], dtype=torch.float64,
                         device="cuda" if dist.get_backend() == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
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


# DRAM bytes per launch of a kernel, from one ncu capture each (dram__bytes_read.sum +
# dram__bytes_write.sum), with the capture it came from; None where no capture exists.
TRAFFIC = {
    "decode_attention": (146493952, "ncu, 2 launches of the 32-slot decode attention, ctx U[64,2048] "
                                    "(bench.py --workload step --layers 2)"),
}


def traffic(kernel: str):
    entry = TRAFFIC.get(kernel)
    return (entry[0], entry[1]) if entry else (None, None)


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
def step_config(cfg, slots: int, world: int) -> dict:
    """The `config` of the step workload, shared by both arms."""
    return {"workload": f"BASELINE config 2: talker decode step, {slots} slots, ctx U[64,2048], "
                        "greedy, evict/admit 4 slots every 16 steps",
            "model": f"qwen3-tts talker {cfg.layers}L h{cfg.hidden} (random init)", "layers": cfg.layers,
            "global_batch": slots * world, "slots_per_gpu": slots,
            "parallelism": f"replicas x{world} (request-level data parallel)"}


def run_reference(args, dist: Dist):
    """The reference arm of the step workload: the CPU port of the talker step."""
    from qwen3_tts_b200.config import TALKER
    work = Workload(args.seed, SLOTS)
    layers = 2
    [(per_step, threads)] = cpu_decode_sample(TALKER, work.positions, args.warmup + args.steps, layers, args.seed)
    value = SLOTS / per_step
    return {
        "metric": f"codec frames/s (talker decode step, C={SLOTS})", "value": value, "unit": UNIT,
        "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded random-init weights)",
        "config": step_config(TALKER, SLOTS, args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"oracle fp32 talker, {layers} of 28 layers at full width, {SLOTS} slots, "
                                   f"ragged ctx; median step time scaled by 28/{layers}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


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


def closed_loop(model, requests, concurrency: int, timed: bool = False) -> dict:
    """Serve `requests` through model.tick with at most `concurrency` in flight (closed loop:
    a finished request is replaced by the next one). Metrics follow the reference's service
    benchmark (``metrics.summarize``, benchmark.py:17-34): frames/s = delivered audio x 12.5 /
    wall time; TTFA = submission -> first PCM chunk (p50/p95, interpolated); RTF = mean over
    requests of latency / audio duration. A request ends at its synthetic target length (the
    max_new_tokens cap stands in for EOS at the target). With `timed`, the pass is also timed
    with CUDA events on the engine's stream, and the host<->device bytes are counted: per
    request the prompt ids and the uniform table going in, per tick the token ids and status
    word coming out, and every PCM16 chunk delivered."""
    from qwen3_tts_b200.metrics import summarize
    pending = list(enumerate(requests))
    submitted, first_audio, done = {}, {}, {}
    counts = {"frames": 0, "ticks": 0, "pcm_bytes": 0, "token_bytes": 0, "h2d": 0}
    in_flight = 0

    def emit(identifier, pcm, rate):
        counts["pcm_bytes"] += len(pcm)
        if len(pcm):
            first_audio.setdefault(identifier, time.perf_counter())

    table_rows = getattr(getattr(model, "state", None), "table_rows", 0)
    events = None
    if timed:
        torch.cuda.synchronize()
        events = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        events[0].record()
    start = time.perf_counter()
    while pending or in_flight:
        subs = []
        while pending and in_flight + len(subs) < concurrency:
            subs.append(pending.pop(0))
        now = time.perf_counter()
        for identifier, payload in subs:
            submitted[identifier] = now
            counts["h2d"] += len(payload["input_ids"]) * 8 + table_rows * 16 * 4 + 64
        in_flight += len(subs)
        counts["token_bytes"] += in_flight * 8 + 4
        counts["ticks"] += 1
        for identifier, result in model.tick(subs, emit=emit):
            done[identifier] = (time.perf_counter(), result)
            counts["frames"] += result["codec_frames"]
            in_flight -= 1
    wall = time.perf_counter() - start
    device_ms = None
    if timed:
        events[1].record()
        torch.cuda.synchronize()
        device_ms = events[0].elapsed_time(events[1])
    records = []
    for i in submitted:
        finished, result = done[i]
        records.append({"success": result["finish_reason"] in ("stop", "length") and result["codec_frames"] > 0
                        and i in first_audio, "audio_seconds": result["codec_frames"] / 12.5,
                        "elapsed_seconds": finished - submitted[i],
                        "ttfa_seconds": first_audio.get(i, finished) - submitted[i]})
    return dict(summarize(records, wall, 12.5), device_ms=device_ms, **counts)


def serving_engine(args, device):
    from qwen3_tts_b200.continuous import ContinuousModel
    slots = 1 << max(0, (args.concurrency - 1).bit_length())
    return ContinuousModel(None, device, max_slots=slots, initial_capacity=1024, seed=args.seed,
                           codec_batch_size=SERVING_CODEC_BATCH, codec_streams=args.codec_streams,
                           pipeline_audio=not args.no_pipeline)


def steady_state(model, requests, steps: int, warmup: int, seed: int, dist) -> dict:
    """Device pipeline throughput at full concurrency: the engine holds `max_slots` active
    requests in mid-stream (positions = prompt length + U[0, target) frames already decoded);
    one step = one replay of the (batch, context) tick graph plus the codec decode of
    SERVING_CHUNK-frame chunks for max_slots / SERVING_CHUNK streams (rotating over the slots:
    every slot's audio is decoded once per SERVING_CHUNK steps, as in steady-state serving),
    PCM16 on the device. Nothing is copied to the host and the host never waits inside the
    timed region. Returns frames/s (max_slots frames per step) and the timing."""
    from qwen3_tts_b200.batching import context_bucket
    slots = model.max_slots
    subs = [(("steady", i), dict(req, max_new_tokens=4000)) for i, req in enumerate(requests[:slots])]
    model.tick(subs)                                   # admission: batched prefill + first frame
    states, S = model.states, model.state
    advance = torch.tensor(steady_advance(requests[:slots], seed), dtype=torch.long)
    S.positions[:slots] += advance.to(S.positions.device)
    S.rotary[:slots] += advance.to(S.rotary.device)
    for state, extra in zip(states, advance.tolist()):
        state.position += extra
    priming = SERVING_CHUNK
    top = max(state.position for state in states) + priming + warmup + steps + 1
    model.ensure_capacity(top)
    graph = model._tick_graph(slots, context_bucket(top + 1, model.arena.capacity))
    model._set_active(slots)
    groups = slots // SERVING_CHUNK

    def tick_only():
        graph.run()
        for state in states:
            state.frames += 1

    # pipelined audio in flight: the last few steps' buffers stay referenced (a server releases a
    # tick's audio once delivered); older ones return to the pinned-memory cache once their copies
    # complete, so steps reuse host buffers instead of allocating new pinned memory each step
    flights = collections.deque(maxlen=4)

    def step(i):
        tick_only()
        due = states[(i % groups) * SERVING_CHUNK:(i % groups + 1) * SERVING_CHUNK] if groups else states
        for state in due:
            state.emitted = state.frames - SERVING_CHUNK
        if model.pipeline_audio:
            # as a pipelined tick: this step's chunks decode on the codec lanes, overlapping the next
            # step's graph; nothing waits on the host
            flights.append(model._launch_audio(due, []))
        else:
            model.decode_chunks(due)

    def join_lanes():
        main = torch.cuda.current_stream()
        for lane in getattr(model, "_audio_lanes", []):
            main.wait_stream(lane)

    engine_stream = getattr(model, "_engine_stream", None) if model.pipeline_audio else None
    if engine_stream is not None:   # the engine's high-priority stream, as its ticks use it
        engine_stream.wait_stream(torch.cuda.current_stream())
        torch.cuda.set_stream(engine_stream)
    for _ in range(priming):                            # fill every slot's code ring
        tick_only()
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    from qwen3_tts_b200 import _lib
    codec_graphs = list(model.codec.graphs.values())
    replays = [c.replays for c in codec_graphs]
    ticks, host = graph.replays, _lib.launch_count()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    join_lanes()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()   # cudaProfilerStart/Stop: no-ops unless a profiler is attached
    a.record()
    for i in range(steps):
        step(warmup + i)
    join_lanes()
    b.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    flights.clear()
    if engine_stream is not None:
        torch.cuda.set_stream(torch.cuda.default_stream())
    dist.barrier()
    elapsed_ms = dist.max(a.elapsed_time(b))
    # this library's kernels in the timed region: graph replays x kernels captured per replay,
    # plus the kernels launched directly (code ring reads)
    launches = (graph.replays - ticks) * graph.launches + (_lib.launch_count() - host)
    launches += sum((c.replays - r) * c.launches for c, r in zip(codec_graphs, replays))
    context = graph.context
    mean_position = sum(state.position for state in states) / len(states)
    model.states.clear()
    model._set_active(0)
    return {"elapsed_ms": elapsed_ms, "frames": slots * steps, "context": context, "mean_position": mean_position,
            "launches": launches, "tick_launches": graph.launches}


def gemm_roofline(model, peak: float) -> dict:
    """The dominant kernel of a serving step: the projection GEMM (tcgen05 linear kernel), which
    carries the code predictor's and the talker's weight streams. Timed as the predictor runs it
    at 64 rows: one CUDA graph with one codebook step's projections (5 layers x QKV, O, gate/up,
    down, then the head) launched back to back, replayed, CUDA events on the replay stream.
    achieved = weight + activation bytes per launch / mean launch time."""
    from qwen3_tts_b200 import _lib, ops
    cfg, w = model.predictor_config, model.predictor_weights
    dev = model.device
    rows = model.max_slots
    x = torch.zeros(rows, cfg.hidden, dtype=torch.bfloat16, device=dev)
    qkv = torch.zeros(rows, cfg.qkv_width, dtype=torch.bfloat16, device=dev)
    attn = torch.zeros(rows, cfg.q_width, dtype=torch.bfloat16, device=dev)
    act = torch.zeros(rows, cfg.ffn, dtype=torch.bfloat16, device=dev)
    logits = torch.zeros(rows, cfg.vocab, dtype=torch.float32, device=dev)
    calls, nbytes = [], 0

    def add(fn, weight, x_bytes, out_bytes):
        nonlocal nbytes
        calls.append(fn)
        nbytes += weight.numel() * 2 + x_bytes + out_bytes

    for layer in w["layers"]:
        add(lambda l=layer: ops.linear(x, l.qkv, out=qkv, row_norm_eps=cfg.eps), layer.qkv, x.numel() * 2,
            qkv.numel() * 2)
        add(lambda l=layer: ops.linear(attn, l.o, out=x, epilogue=_lib.EPI_RESIDUAL, residual=x), layer.o,
            attn.numel() * 2, 2 * x.numel() * 2)
        add(lambda l=layer: ops.linear(x, l.gate_up, out=act, epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=cfg.eps),
            layer.gate_up, x.numel() * 2, act.numel() * 2)
        add(lambda l=layer: ops.linear(act, l.down, out=x, epilogue=_lib.EPI_RESIDUAL, residual=x), layer.down,
            act.numel() * 2, 2 * x.numel() * 2)
    head = w["heads"][0]
    add(lambda: ops.linear(x, head, out=logits, out_dtype=torch.float32, row_norm_eps=cfg.eps), head, x.numel() * 2,
        logits.numel() * 4)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for fn in calls:
            fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for fn in calls:
            fn()
    replays = 20
    with torch.cuda.stream(side):
        graph.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(side)
        for _ in range(replays):
            graph.replay()
        b.record(side)
    torch.cuda.synchronize()
    graph.reset()
    seconds = a.elapsed_time(b) / 1e3 / (replays * len(calls))
    per_launch = nbytes / len(calls)
    achieved = per_launch / seconds / 1e9
    return {"bound": "hbm", "kernel": "linear_kernel (tcgen05 projection GEMM, 64 rows)", "achieved": achieved,
            "peak": peak, "unit": "GB/s", "frac": achieved / peak, "launch_us": seconds * 1e6,
            "bytes_per_launch": per_launch,
            "method": "in graph: one predictor codebook step's 21 projections back to back, CUDA events"}


def serving_contract(args, dist) -> dict:
    """BASELINE config 5 at C=64 per GPU on this rank's GPU (see the module docstring)."""
    from qwen3_tts_b200 import ops
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    model = serving_engine(args, dev)
    requests = serving_requests(args.seed + 7919 * dist.rank, args.requests)
    closed_loop(model, requests, args.concurrency)     # captures every graph shape the pass meets
    dist.barrier()
    e2e = closed_loop(model, requests, args.concurrency, timed=True)
    dist.barrier()
    e2e_ms = dist.max(e2e["device_ms"])
    frames_all = dist.sum(e2e["frames"])
    clocks = ClockSampler(dev.index)
    clocks.start()
    steady = steady_state(model, serving_requests(args.seed + 104729 + dist.rank, SERVING_SLOTS), args.steps,
                          args.warmup, args.seed + dist.rank, dist)
    clock_info = clocks.stop()
    status = ops.read_status(dev)
    peak, peak_kind = measured_peaks()
    roofline = gemm_roofline(model, peak)
    roofline["peak_kind"] = peak_kind
    roofline["traffic"], roofline["traffic_source"] = traffic("linear_kernel")
    model.close()
    return {"steady": steady, "e2e": e2e, "e2e_ms": e2e_ms, "e2e_frames_all": frames_all, "clocks": clock_info,
            "status": status, "roofline": roofline}


def run_dispatch(args) -> dict:
    """Closed-loop serving through the host dispatcher: one engine process per GPU (--gpus N),
    `concurrency` requests in flight per GPU, from this single process. A first pass over the
    same requests captures the graph shapes; the second is timed on the host clock."""
    from qwen3_tts_b200.continuous import ContinuousModel
    slots = 1 << max(0, (args.concurrency - 1).bit_length())
    engine = dict(max_slots=slots, initial_capacity=1024, seed=args.seed, codec_batch_size=SERVING_CODEC_BATCH,
                  codec_streams=args.codec_streams)
    gpus = max(1, args.gpus)
    if gpus > 1:
        from qwen3_tts_b200.dispatcher import Dispatcher
        model = Dispatcher.start(gpus, engine, per_engine=args.concurrency)
    else:
        model = ContinuousModel(None, torch.device("cuda:0"), **engine)
    requests = serving_requests(args.seed, args.requests * gpus)
    closed_loop(model, requests, args.concurrency * gpus)
    res = closed_loop(model, requests, args.concurrency * gpus)
    model.close()
    return {"frames_per_s": res["throughput_frames_s"], "frames": res["frames"], "wall_s": res["wall_seconds"],
            "ttfa_p50_ms": res["ttfa_p50_ms"], "ttfa_p95_ms": res["ttfa_p95_ms"], "rtf": res["rtf_mean"],
            "status": res["status"], "failed_requests": res["failed_requests"], "gpus": gpus}


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


def run_prefill(args) -> list:
    """Admission prefill of the talker (PrefillGraph, prefill_graph.py:31-50): the 28-layer causal
    stack over a group of prompts, K/V written into arena slots, last-token hidden state and
    logits. Two groups: 16 prompts of 256 tokens (no padding either way: the GEMM and attention
    rate at 4,096 rows) and the first 16 prompts of the serving recipe (
    lengths 29-209 with the CustomVoice prefix), each as the padded graph (power-of-two length,
    the reference's shape) and the packed graph (prompts end to end, 512-row buckets). Each
    line: mean CUDA-event ms over `steps` graph replays after `warmup`, and the projection
    GEMMs' FLOP/s over the real prompt rows (2 x rows x projection weights x 28 layers)."""
    from qwen3_tts_b200.batching import packed_rows, packed_tables, packed_units
    from qwen3_tts_b200.config import TALKER
    from qwen3_tts_b200.talker import PackedPrefill, SlotArena, TalkerPrefill, rope_tables
    from qwen3_tts_b200.weights import decoder_weights, pack_decoder
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = TALKER
    weights = pack_decoder(decoder_weights(cfg, args.seed, dev), dev)
    arena = SlotArena(cfg, 16, 256, dev)
    cos, sin = rope_tables(4096, cfg.head_dim, cfg.theta, dev)
    per_row = 2 * cfg.layers * (cfg.hidden * cfg.qkv_width + cfg.q_width * cfg.hidden + cfg.hidden * 2 * cfg.ffn
                                + cfg.ffn * cfg.hidden)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    recipe = [len(r["input_ids"]) + PROMPT_PREFIX for r in serving_requests(args.seed, 16)]
    out = []
    for name, lengths in (("16x256", [256] * 16), ("serving recipe, 16 prompts", recipe)):
        total = sum(lengths)
        x = (torch.randn(total, cfg.hidden, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        padded_len = 1 << (max(lengths) - 1).bit_length()
        graphs = {}
        padded = TalkerPrefill(cfg, weights, arena, 16, padded_len, cos, sin)
        padded.capture()
        embeds = torch.zeros(16, padded_len, cfg.hidden, dtype=torch.bfloat16, device=dev)
        offset = 0
        for b, n in enumerate(lengths):
            embeds[b, :n] = x[offset:offset + n]
            offset += n
        lens = torch.tensor(lengths, device=dev)
        slots = torch.arange(16, device=dev)
        graphs["padded"] = (padded, lambda i: padded.run(embeds, lens, slots), 16 * padded_len)
        rows = packed_rows(total)
        packed = PackedPrefill(cfg, weights, arena, rows, 16, cos, sin)
        packed.capture()
        px = torch.cat([x, x[-1:].expand(rows - total, -1)])
        tables = [t.to(dev) for t in packed_tables(lengths, 0, rows, 16)] + [packed_units(lengths, 0, rows, 16).to(dev)]
        graphs["packed"] = (packed, lambda i: packed.run(px, *tables), rows)
        for form, (graph, call, graph_rows) in graphs.items():
            for i in range(args.warmup):
                call(i)
            ms = timed_region(call, args.steps) / args.steps
            out.append({"workload": "prefill", "group": name, "form": form, "prompts": 16, "real_rows": total,
                        "graph_rows": graph_rows, "ms": ms, "ttfa_share_ms_per_prompt": ms / 16,
                        "projection_tflops_real_rows": per_row * total / (ms / 1e3) / 1e12})
            graph.close()
    return out


def run_chain(args) -> list:
    """One decode layer's projections after its attention (O + residual, gate/up with the folded
    RMSNorm and SwiGLU, down + residual, the next layer's QKV with the folded RMSNorm) at the
    predictor's and the talker's widths, as one q3t_linear_chain launch and as four q3t_linear
    launches, each form captured in a CUDA graph and replayed (CUDA events, mean of 20)."""
    from qwen3_tts_b200 import _lib, ops
    from qwen3_tts_b200.talker import mlp_stages, qkv_stage
    from qwen3_tts_b200.weights import PackedLayer
    dev = torch.device("cuda:0")
    bf = torch.bfloat16

    def tiles(o, i, g):
        return ops.pack_tiles((torch.randn(o, i, generator=g) * i ** -0.5).to(bf).to(dev))

    def graph_us(fn, n=20):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            fn()
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        graph.reset()
        return a.elapsed_time(b) * 1e3 / n

    out = []
    for name, hidden, ffn, rows in (("predictor", 1024, 3072, 64), ("talker", 2048, 6144, 32),
                                    ("talker", 2048, 6144, 64)):
        g = torch.Generator().manual_seed(args.seed + 1)
        layer = PackedLayer(input_norm=None, qkv=tiles(4096, hidden, g), q_norm=None, k_norm=None,
                            o=tiles(hidden, 2048, g), post_norm=None, gate_up=tiles(2 * ffn, hidden, g),
                            down=tiles(hidden, ffn, g), folded=True)
        attn = torch.randn(rows, 2048, generator=g).to(bf).to(dev)
        x = torch.randn(rows, hidden, generator=g).to(bf).to(dev)
        h, act = torch.empty_like(x), torch.empty(rows, ffn, dtype=bf, device=dev)
        qkv = torch.empty(rows, 4096, dtype=bf, device=dev)
        ws = ops.linear_chain_workspace(rows, dev)
        stages = mlp_stages(attn, x, layer, h, act, 1e-6) + [qkv_stage(h, layer, qkv, 1e-6, depends=2)]

        def separate():
            ops.linear(attn, layer.o, out=h, epilogue=_lib.EPI_RESIDUAL, residual=x)
            ops.linear(h, layer.gate_up, out=act, epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=1e-6)
            ops.linear(act, layer.down, out=h, epilogue=_lib.EPI_RESIDUAL, residual=h)
            ops.linear(h, layer.qkv, out=qkv, row_norm_eps=1e-6)
        weights = sum(t.tiles.numel() for t in (layer.qkv, layer.o, layer.gate_up, layer.down))
        out.append({"layer": name, "rows": rows, "weight_bytes": weights,
                    "chain_us": graph_us(lambda: ops.linear_chain(stages, ws)), "linear_x4_us": graph_us(separate),
                    "status_word": ops.read_status(dev)})
    return out


# ---------------------------------------------------------------------- CPU tick (serving arms)
PROMPT_PREFIX = 9   # CustomVoice prompt rows around the text ids (role, speaker, language, codec tags)


def steady_advance(requests, seed: int) -> list:
    """Frames already decoded per slot in the steady state (U[0, target)), shared by both arms."""
    g = torch.Generator().manual_seed(seed + 17)
    return [int(torch.randint(0, max(1, r["max_new_tokens"] - 1), (1,), generator=g)) for r in requests]


class CpuTick:
    """One steady-state serving tick of the CPU port (the oracle, fp32) for `slots` active
    requests, in bounded samples: the talker step as one of its 28 layers at full width over
    the slots' contexts (scaled by 28) plus the LM head; the whole code-predictor frame (5
    layers, 15 codebooks, heads and top-k sampling) for every slot; the incremental codec
    decode of one stream's 8-frame chunk, scaled by the slots / 8 streams a tick decodes."""

    def __init__(self, slots: int, positions, seed: int, steps: int):
        from dataclasses import replace

        from oracle import codec as OC
        from oracle import decoder as OD
        from qwen3_tts_b200.config import CODEC, PREDICTOR, TALKER
        from qwen3_tts_b200.weights import decoder_weights

        def fp32(weights):
            for layer in weights["layers"]:
                for key in list(layer):
                    layer[key] = layer[key].float()
            for key in list(weights):
                if isinstance(weights[key], torch.Tensor):
                    weights[key] = weights[key].float()
            return weights

        self.OD, self.slots = OD, slots
        self.talker_cfg = replace(TALKER, layers=1)
        self.talker = fp32(decoder_weights(self.talker_cfg, seed, dtype=torch.bfloat16))
        self.positions = torch.tensor(positions, dtype=torch.long).view(-1, 1)
        cap = int(self.positions.max()) + steps + 2
        self.tables = OD.Tables(cap + 1, TALKER.head_dim, TALKER.theta)
        self.cache = OD.new_cache(self.talker_cfg, slots, cap)
        self.predictor_cfg = PREDICTOR
        self.predictor = fp32(decoder_weights(PREDICTOR, seed + 1, dtype=torch.bfloat16))
        self.ptables = OD.Tables(PREDICTOR.groups + 1, PREDICTOR.head_dim, PREDICTOR.theta)
        g = torch.Generator().manual_seed(seed + 2)
        self.h = torch.randn(slots, 1, TALKER.hidden, generator=g) * 0.1
        self.first = torch.randn(slots, PREDICTOR.talker_hidden, generator=g) * 0.02
        self.draws = torch.rand(slots, 16, generator=g)
        self.codec = OC.IncrementalOracle(OC.randomize(OC.CodecDecoder(CODEC), seed + 3))
        self.codec_state = self.codec.new_state()
        self.codes = torch.randint(0, CODEC.codebook_size, (1, CODEC.codebooks, SERVING_CHUNK), generator=g)
        self.streams = max(1, slots // SERVING_CHUNK)

    def step(self) -> float:
        """Seconds of one tick (sampled parts scaled)."""
        OD = self.OD
        t0 = time.perf_counter()
        x = OD.layer_forward(self.talker_cfg, self.talker["layers"][0], self.h, self.positions, *self.cache[0],
                             self.positions, self.tables, "fp32")
        t1 = time.perf_counter()
        hidden = OD._rms(x, self.talker["norm"], self.talker_cfg.eps, "fp32")
        torch.argmax(hidden[:, 0] @ self.talker["head"].T, dim=-1)
        t2 = time.perf_counter()
        OD.predictor_frame(self.predictor_cfg, self.predictor, self.h[:, 0].float(), self.first, self.draws,
                           self.ptables, "fp32")
        t3 = time.perf_counter()
        self.codec.decode(self.codes, self.codec_state)
        t4 = time.perf_counter()
        self.positions += 1
        return (t1 - t0) * 28 + (t2 - t1) + (t3 - t2) + (t4 - t3) * self.streams


def cpu_serving_sample(args, steps: int, threads=None):
    """Seconds per CPU tick (median of `steps`) and the thread count used (`threads`, default every
    host core), on the serving workload's steady state (same requests and contexts as the GPU
    arm's)."""
    requests = serving_requests(args.seed + 104729, SERVING_SLOTS)
    advance = steady_advance(requests, args.seed)
    positions = [len(r["input_ids"]) + PROMPT_PREFIX + a for r, a in zip(requests, advance)]
    torch.set_num_threads(threads or os.cpu_count() or 1)
    tick = CpuTick(SERVING_SLOTS, positions, args.seed, steps)
    times = [tick.step() for _ in range(steps)]
    used = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    return float(np.median(times)), used


CPU_SERVING_SAMPLE = ("oracle fp32 serving tick at 64 slots (steady state, same requests and contexts): talker 1 of "
                      "28 layers at full width x 28 + LM head, the full 15-codebook predictor frame, one of 8 "
                      "streams' 8-frame codec chunks x 8; median tick time")


def serving_config(args, world: int) -> dict:
    """The `config` of the serving workload, shared by both arms."""
    return {"workload": "BASELINE config 5: talker -> code predictor -> incremental codec, C=64 per GPU; value: "
                        "steady-state tick (64 slots, 8 streams x 8-frame codec chunks per step); e2e: closed loop "
                        "through ContinuousModel.tick",
            "model": "qwen3-tts 1.7B CustomVoice geometry (talker 28L h2048, predictor 5L h1024, codec 8L h512 / "
                     "1536-ch decoder), random init",
            "concurrency": args.concurrency, "requests_per_gpu": args.requests, "global_batch": SERVING_SLOTS * world,
            "codec_batch": SERVING_CODEC_BATCH, "codec_streams": args.codec_streams,
            "pipeline_audio": not args.no_pipeline,
            "parallelism": f"replicas x{world} (request-level data parallel, one engine per GPU)",
            "l2": "inputs > L2 (talker 2.8 GB + predictor 2.5 GB of weights streamed per step)"}


SERVING_METRIC = "codec frames/s (end-to-end serving, C=64 per GPU)"


def run_reference_serving(args) -> dict:
    per_tick, threads = cpu_serving_sample(args, args.warmup + args.steps)
    value = SERVING_SLOTS / per_tick
    return {
        "metric": SERVING_METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_tick * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (BASELINE config 5 request recipe, seeded random-init weights)",
        "config": serving_config(args, args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": CPU_SERVING_SAMPLE},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    global SLOTS
    args = parse_args()
    if args.slots < 1 or args.slots > 64:
        raise SystemExit("--slots must be within 1..64")
    if args.concurrency != SERVING_SLOTS and args.workload == "serving":
        raise SystemExit("the serving contract runs at C=64 per GPU (use --workload dispatch for other C)")
    SLOTS = args.slots
    rank = int(os.environ.get("RANK", 0))
    if args.impl == "reference":
        if rank != 0:
            return            # the CPU arm runs on rank 0 alone
        if args.workload == "serving":
            print(json.dumps(run_reference_serving(args)))
        elif args.workload == "step":
            print(json.dumps(run_reference(args, Dist.__new__(Dist))))
        else:
            print(json.dumps({"impl": "reference", "unavailable": f"no CPU arm for --workload {args.workload}"}))
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
    if args.workload == "prefill":
        for row in run_prefill(args):
            print(json.dumps(row))
        return
    if args.workload == "chain":
        for row in run_chain(args):
            print(json.dumps(row))
        return
    if args.workload == "dispatch":
        if rank != 0:
            return  # one host process drives every GPU through the dispatcher
        res = run_dispatch(args)
        print(json.dumps({
            "metric": f"codec frames/s (end-to-end serving through the dispatcher, C={args.concurrency} per GPU)",
            "value": res["frames_per_s"], "unit": UNIT, "n_gpus": res["gpus"], "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic (BASELINE config 5 request recipe, seeded random-init weights)",
            "config": {"workload": "BASELINE config 5: talker -> code predictor -> incremental codec, closed loop",
                       "concurrency": args.concurrency, "requests": args.requests * res["gpus"],
                       "codec_streams": args.codec_streams},
            "ttfa_p50_ms": res["ttfa_p50_ms"], "ttfa_p95_ms": res["ttfa_p95_ms"], "rtf": res["rtf"],
            "frames": res["frames"], "wall_s": res["wall_s"], "status": res["status"],
            "failed_requests": res["failed_requests"]}))
        return
    dist = Dist("nccl")
    if args.workload == "serving":
        line = serving_line(args, dist)
    else:
        line = step_line(args, dist)
    if dist.rank == 0:
        print(json.dumps(line))
    dist.close()


def serving_line(args, dist) -> dict:
    res = serving_contract(args, dist)
    steady, e2e = res["steady"], res["e2e"]
    seconds = steady["elapsed_ms"] / 1e3
    value = steady["frames"] * dist.world / seconds
    e2e_value = res["e2e_frames_all"] / (res["e2e_ms"] / 1e3)
    ticks = max(1, e2e["ticks"])
    line = {
        "metric": SERVING_METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": steady["elapsed_ms"] / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": value / REFERENCE_C64_FRAMES, "dtype": "bf16",
        "data": "synthetic (BASELINE config 5 request recipe, seeded random-init weights)",
        "config": dict(serving_config(args, dist.world), steady_context=steady["context"],
                       steady_mean_position=steady["mean_position"]),
        "roofline": res["roofline"],
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": e2e["h2d"] / ticks,
                "d2h_bytes_per_step": (e2e["pcm_bytes"] + e2e["token_bytes"]) / ticks, "ticks": e2e["ticks"],
                "frames": e2e["frames"], "ms": res["e2e_ms"], "method": "CUDA events around the closed-loop pass"},
        "ttfa_p50_ms": e2e["ttfa_p50_ms"], "ttfa_p95_ms": e2e["ttfa_p95_ms"], "rtf": e2e["rtf_mean"],
        "failed_requests": e2e["failed_requests"],
        "gpu_launches": steady["launches"], "tick_graph_kernels": steady["tick_launches"],
        "status_word": res["status"],
        "clocks": res["clocks"],
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        per_tick, threads = cpu_serving_sample(args, 3)
        per_tick4, _ = cpu_serving_sample(args, 1, threads=4)
        line["cpu_baseline"] = {"value": SERVING_SLOTS / per_tick, "unit": UNIT, "cores": threads, "kind": "port",
                                "value_4_threads": SERVING_SLOTS / per_tick4,
                                "sample": CPU_SERVING_SAMPLE + " of 3 ticks; value_4_threads = one tick of the same "
                                          "at 4 threads (the reference's default torch thread count)"}
    return line


# the reference's published throughput at C=64 (1x Ascend 910B1, bf16, mean of 3 runs)
REFERENCE_C64_FRAMES = 549.39


def step_line(args, dist) -> dict:
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
    dom_traffic, dom_source = traffic(dom_name) if SLOTS == 32 else (None, None)
    line = {
        "metric": f"codec frames/s (talker decode step, C={SLOTS})", "value": value, "unit": UNIT,
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["elapsed_ms"] / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights)",
        "config": dict(step_config(cfg, SLOTS, dist.world),
                       l2=f"inputs > L2 ({step_bytes / 1e9:.1f} GB streamed per step)",
                       hbm_fraction_step=step_bytes / (res["elapsed_ms"] / args.steps / 1e3) / (peak * 1e9),
                       bytes_per_step=step_bytes),
        "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind, "traffic": dom_traffic,
                     "traffic_source": dom_source,
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
    return line


if __name__ == "__main__":
    main()
