"""Continuous-batching talker -> code-predictor -> codec engine (ContinuousModel,
continuous.py:251-672 of the reference engine) on device-resident slot state.

Slot i holds the i-th active request, as in the reference (states are dense;
a finished or cancelled request is replaced by the last one). What the
reference keeps per request in Python (token, hidden, seen mask, uniform
table, position, frame counter, trailing text, pad embedding, recent codes) is
here a set of [slots, ...] device arrays (``SlotState``), so one tick is one
CUDA graph per (batch bucket, context bucket):

    tick_gather -> predictor chain (15 codebooks) -> talker step (28 layers,
    LM head) -> semantic sampling (penalty, mask, EOS gate, top-k, CDF) ->
    tick_commit (code ring, hidden, counters)

followed by one device->host copy of the new tokens (the reference's
``.tolist()`` sync, continuous.py:623) for the host's stop/emit decisions.
Admission is a batched prefill graph over the prompts packed end to end (no
padding to the longest) that writes K/V straight into the arena slots (no intermediate cache copy) and samples each first token on the
device. Audio chunks are decoded by the slot-indexed incremental codec from
the device code ring, converted to PCM16 on the device and copied to the host
in one transfer per tick.

The tick's outputs follow the reference contract:
``tick(submissions, emit=None, cancelled=()) -> [(identifier, {"pcm", "sample_rate",
"codec_frames", "finish_reason"})]`` with ``emit(identifier, pcm_bytes, 24000)``
called for every delivered chunk.
"""
from __future__ import annotations

import logging
import time
from pathlib import Path
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, checkpoint, ops
from .batching import (MAX_PACKED_ROWS, context_bucket, decode_batch_size, emission_target, packed_groups,
                       packed_rows, packed_tables, packed_units)
from .code_buffer import CodecCodeBuffer
from .codec import CodecGraph, CodecSlots, pack_codec
from .codec_weights import random_codec
from .config import CODEC, PREDICTOR, PROMPT, TALKER, CodecConfig, PredictorConfig, PromptConfig, TalkerConfig
from .predictor import PredictorStep
from .prompt import SUPPORTED_SAMPLING, CustomVoicePrompt, prompt_weights
from .sampling import random_table
from .talker import PackedPrefill, SlotArena, TalkerPrefill, TalkerStep, rope_tables
from .weights import decoder_weights, pack_decoder

BF16 = torch.bfloat16
SAMPLE_RATE = 24000


@dataclass
class EngineStats:
    """Per-engine counters, updated on the owner thread once per tick (served by /health)."""
    ticks: int = 0
    frames: int = 0           # codec frames decoded (one per active slot per tick)
    admitted: int = 0
    finished: int = 0
    cancelled: int = 0
    active: int = 0           # slots decoded by the last tick
    batch: int = 0            # the last tick's decode batch bucket
    last_tick_ms: float = 0.0
    tick_seconds: float = 0.0

    def as_dict(self) -> dict:
        return dict(vars(self))


@dataclass
class RequestState:
    """Host-side mirror of one request (continuous.py:232-247); tensors live in SlotState."""
    identifier: object
    payload: dict
    position: int
    rope_delta: int
    max_new_tokens: int
    frames: int = 0
    emitted: int = 0
    audio: list = field(default_factory=list)
    codec_slot: int = -1      # the request's row of the incremental codec's state (fixed for its life)
    cancelled: bool = False


@dataclass
class AudioInFlight:
    """One tick's audio on the codec lanes (pipeline_audio): per group the (state, frames decoded
    up to) pairs and the pinned PCM16 block, the requests that ended with this tick, and the
    event after the last copy."""
    finished: list
    blocks: list = field(default_factory=list)
    status: object = None
    done: object = None


class SlotState:
    """Per-slot decode state as dense device arrays ([slots, ...])."""

    def __init__(self, slots: int, hidden: int, vocab: int, codebooks: int, table_rows: int, trailing_rows: int,
                 ring_depth: int, device):
        dev = torch.device(device)
        self.slots, self.table_rows, self.trailing_rows = slots, table_rows, trailing_rows
        self.active = torch.zeros(1, dtype=torch.long, device=dev)
        self.tokens = torch.zeros(slots, dtype=torch.long, device=dev)
        self.hidden = torch.zeros(slots, hidden, dtype=BF16, device=dev)
        self.seen = torch.zeros(slots, vocab, dtype=torch.bool, device=dev)
        self.positions = torch.zeros(slots, dtype=torch.long, device=dev)
        self.rotary = torch.zeros(slots, dtype=torch.long, device=dev)
        self.frames = torch.zeros(slots, dtype=torch.long, device=dev)
        self.tables = torch.full((slots, table_rows, 16), 0.5, dtype=torch.float32, device=dev)
        self.trailing = torch.zeros(slots, trailing_rows, hidden, dtype=BF16, device=dev)
        self.trailing_len = torch.zeros(slots, dtype=torch.long, device=dev)
        self.pad = torch.zeros(slots, hidden, dtype=BF16, device=dev)
        self.codes = CodecCodeBuffer(slots, codebooks, dev, depth=ring_depth)
        self.arrays = [self.tokens, self.hidden, self.seen, self.positions, self.rotary, self.frames, self.tables,
                       self.trailing, self.trailing_len, self.pad, self.codes.data]

    def move(self, source: int, destination: int) -> None:
        if source != destination:
            for array in self.arrays:
                ops.slot_move(array, source, destination)


class TickGraph:
    """One tick for `batch` rows attending over `context` keys, captured as one CUDA graph."""

    def __init__(self, engine: "ContinuousModel", batch: int, context: int):
        self.engine, self.batch, self.context = engine, batch, context
        e = engine
        self.pred = e.predictor_step(batch)
        self.talk = TalkerStep(e.talker_config, e.talker_weights, e.arena, batch, context, e.cos, e.sin)
        shared = e.batch_buffers(batch)
        self.talk.inputs = self.pred.embeds          # frame embedding + text feeds the talker directly
        self.talk.positions, self.talk.rotary = shared["positions"], shared["rotary"]
        self.uniform, self.steps = shared["uniform"], shared["steps"]
        self.graph = None
        self.launches = 0          # this library's kernels per replay (counted at capture)
        self.replays = 0

    def compute(self) -> None:
        e, S, B, p, t = self.engine, self.engine.state, self.batch, self.pred, self.talk
        ops.tick_gather(S.active, S.tokens, S.hidden, e.codec_embedding, S.tables, S.frames, S.trailing,
                        S.trailing_len, S.pad, S.positions, S.rotary, pred_inputs=p.inputs, codes=p.codes,
                        draws=p.draws, talker_uniform=self.uniform, steps=self.steps, text=p.text,
                        step_positions=t.positions, step_rotary=t.rotary, rows=B)
        p.compute()
        t.compute()
        ops.sample(t.logits, uniforms=self.uniform, seen=S.seen[:B], allowed=e.allowed, steps=self.steps, eos=e.eos,
                   min_steps=2, penalty=e.penalty, temperature=e.temperature, top_k=e.top_k, top_p=e.top_p,
                   seen_out=S.seen[:B], tokens=S.tokens[:B].view(B, 1))
        ops.tick_commit(S.active, p.codes, t.hidden, S.hidden, S.codes.data, S.frames, S.positions, S.rotary, rows=B)

    @torch.inference_mode()
    def capture(self, warmup: int = 2) -> None:
        """Warm up with every row as padding (commit skips them), then capture. Padding rows
        still write K/V at position 0 and the sampled token/seen row of slots 0..batch-1,
        so those are saved and restored around the capture."""
        e, S, B = self.engine, self.engine.state, self.batch
        saved_kv = e.arena.packed[:, :B, :, 0].clone()
        saved = (S.tokens[:B].clone(), S.seen[:B].clone(), S.active.clone())
        S.active.zero_()
        stream = torch.cuda.Stream(device=e.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.compute()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize(e.device)
        self.graph = torch.cuda.CUDAGraph()
        before = _lib.launch_count()
        with torch.cuda.graph(self.graph, stream=stream):
            self.compute()
        self.launches = _lib.launch_count() - before     # this library's kernels per replay
        torch.cuda.synchronize(e.device)
        e.arena.packed[:, :B, :, 0].copy_(saved_kv)
        S.tokens[:B].copy_(saved[0])
        S.seen[:B].copy_(saved[1])
        S.active.copy_(saved[2])

    def run(self) -> None:
        if self.graph is None:
            self.compute()
        else:
            self.graph.replay()
            self.replays += 1

    def close(self) -> None:
        if self.graph is not None:
            torch.cuda.synchronize(self.engine.device)
            self.graph.reset()
            self.graph = None


class ContinuousModel:
    """Drop-in for the reference ContinuousModel on one CUDA device.

    ``model_path`` is a checkpoint directory (``model.safetensors`` or a sharded
    index, ``config.json``, and ``speech_tokenizer/model.safetensors`` for the
    codec; ``checkpoint.load_model`` / ``checkpoint.load_codec``): the
    geometry and prompt ids come from the checkpoint and override the config
    arguments. With ``model_path=None`` the engine serves seeded random-init
    weights of the 1.7B CustomVoice geometry (``seed``), or caller-provided
    weight dicts (``weights={"talker", "predictor", "prompt"}``) and a codec
    decoder module tree (``codec_decoder``); a checkpoint without a codec
    directory gets the seeded codec. Reference flags that select between NPU
    kernel variants are accepted and ignored (there is one CUDA path).

    Admission packs the prompts end to end (``packed_prefill``, groups of at most
    ``max_prefill_rows`` rows: wide-tile projection GEMMs and the causal tcgen05
    prefill attention); ``packed_prefill=False`` keeps the reference's padded
    power-of-two prefill graphs in groups of ``max_prefill_batch``.
    """

    def __init__(self, model_path=None, device="cuda:0", max_slots=64, initial_capacity=512, *, seed: int = 0,
                 talker_config: TalkerConfig = TALKER, predictor_config: PredictorConfig = PREDICTOR,
                 codec_config: CodecConfig = CODEC, prompt_config: PromptConfig = PROMPT, weights=None,
                 codec_decoder=None, codec_left_context=72, codec_batch_size=4, incremental_codec=True,
                 codec_chunk_frames=8, codec_streams=1, decode_bucket_step=0, prewarm_codec=False,
                 prewarm_prefill=False, bucket_prefill=True, max_frames=4096, max_prefill_batch=16, use_graphs=True,
                 temperature=0.9, top_k=50, top_p=1.0, subtalker_temperature=0.9, subtalker_top_k=50,
                 subtalker_top_p=1.0, penalty=1.05, pipeline_audio=False, packed_prefill=True,
                 max_prefill_rows=MAX_PACKED_ROWS, **flags):
        if codec_chunk_frames not in (8, 16) or (codec_chunk_frames != 8 and not incremental_codec):
            raise ValueError("16-frame chunks require the incremental codec")
        if codec_streams not in (1, 2) or (codec_streams == 2 and not incremental_codec):
            raise ValueError("Two Codec streams require incremental codec")
        if max_slots < 1 or max_slots & (max_slots - 1):
            raise ValueError("Continuous slot count must be a positive power of two")
        decode_batch_size(1, max_slots, decode_bucket_step)
        self.flags = flags
        self.device = torch.device(device)
        torch.cuda.set_device(self.device)
        if model_path is not None:
            loaded = checkpoint.load_model(model_path, self.device, prompt_base=prompt_config)
            talker_config, predictor_config = loaded["talker_config"], loaded["predictor_config"]
            prompt_config, weights = loaded["prompt_config"], loaded["weights"]
            codec_dir = Path(model_path) / "speech_tokenizer"
            if codec_decoder is None and codec_dir.is_dir():
                codec_decoder = checkpoint.load_codec(codec_dir, codec_config)
        self.max_slots, self.decode_bucket_step = max_slots, decode_bucket_step
        self.talker_config, self.predictor_config = talker_config, predictor_config
        self.codec_config, self.prompt_config = codec_config, prompt_config
        self.incremental_codec, self.codec_chunk_frames = incremental_codec, codec_chunk_frames
        self.codec_streams, self.codec_batch_size = codec_streams, codec_batch_size
        self.context = codec_left_context
        self.bucket_prefill, self.max_prefill_batch = bucket_prefill, max_prefill_batch
        if not 1 <= max_prefill_rows <= MAX_PACKED_ROWS:
            raise ValueError(f"max_prefill_rows must be within 1..{MAX_PACKED_ROWS}")
        self.packed_prefill, self.max_prefill_rows = packed_prefill, max_prefill_rows
        self.use_graphs = use_graphs
        self.temperature, self.top_k, self.top_p, self.penalty = temperature, top_k, top_p, penalty
        self.max_frames = max_frames
        self.speakers = [name for name, _ in prompt_config.speakers]
        self.languages = ["auto"] + [name for name, _ in prompt_config.languages]

        weights = weights or {}
        talker = weights.get("talker") or decoder_weights(talker_config, seed, self.device)
        predictor = weights.get("predictor") or decoder_weights(predictor_config, seed + 1, self.device)
        prompt = weights.get("prompt") or prompt_weights(prompt_config, seed + 2, self.device)
        self.talker_weights = pack_decoder(talker, self.device)
        self.predictor_weights = pack_decoder(predictor, self.device)
        self.codec_embedding = self.talker_weights["embedding"]
        self.prompt_builder = CustomVoicePrompt(prompt_config, prompt, self.codec_embedding, self.device)
        self.arena = SlotArena(talker_config, max_slots, initial_capacity, self.device)
        self.cos, self.sin = rope_tables(1 << 15, talker_config.head_dim, talker_config.theta, self.device)
        self.eos = talker_config.eos
        self.allowed = torch.ones(talker_config.vocab, dtype=torch.bool, device=self.device)
        self.allowed[-1024:] = False
        self.allowed[self.eos] = True
        ring = codec_chunk_frames if incremental_codec else 1 << (codec_left_context + 16).bit_length()
        self.state = SlotState(max_slots, talker_config.hidden, talker_config.vocab, talker_config.codebooks,
                               max_frames + 1, 1, max(8, ring), self.device)
        self.codec_codes = self.state.codes
        packed_codec = pack_codec(codec_decoder if codec_decoder is not None else random_codec(codec_config, seed + 3),
                                  self.device)
        if incremental_codec:
            self.codec = CodecSlots(codec_config, packed_codec, max_slots, self.device,
                                    max_chunk_frames=codec_chunk_frames, use_graphs=use_graphs,
                                    streams=codec_streams)
            if prewarm_codec:
                self.codec.prewarm(min(codec_batch_size, max_slots))
        else:
            self.codec = CodecGraph(codec_config, packed_codec, self.device, max_batch=codec_batch_size,
                                    use_graphs=use_graphs)
        self.subtalker = dict(temperature=subtalker_temperature, top_k=subtalker_top_k, top_p=subtalker_top_p)
        # Every request owns one row of the incremental codec's state from admission to its end
        # (compaction moves only the talker-side slot rows). With pipeline_audio the chunks a tick
        # makes due are decoded on the codec lanes while the next tick's graph runs, and are
        # delivered (emit, finished results) by that next tick; a finished request's codec row is
        # reused only after its last chunk has been delivered.
        self.pipeline_audio = bool(pipeline_audio) and incremental_codec
        self._codec_free = list(range(max_slots)) if incremental_codec else []
        self._codec_held: list = []          # rows whose last chunk is still being decoded
        self._inflight = None                # the previous tick's audio in flight (pipeline_audio)
        if self.pipeline_audio:
            self._audio_lanes = (self.codec.lanes if self.codec.lanes
                                 else [torch.cuda.Stream(device=self.device)])
            self._engine_stream = torch.cuda.Stream(device=self.device, priority=-16)
        self.states: list[RequestState] = []
        self.stats = EngineStats()
        # Optional observer of every decoded frame: on_codes(identifier, frame, codes, next_token)
        # (one extra device->host copy per tick when set; used for auditing and parity checks).
        self.on_codes = None
        self.graphs: dict[tuple[int, int], TickGraph] = {}
        self.prefills: dict[tuple[int, int], TalkerPrefill] = {}
        self.packed: dict[int, PackedPrefill] = {}
        self._predictors: dict[int, PredictorStep] = {}
        self._buffers: dict[int, dict] = {}
        self._active = 0
        self._zeros = torch.zeros(max_slots, dtype=torch.long, device=self.device)
        self._host_tokens = torch.zeros(max_slots, dtype=torch.long).pin_memory()
        self._host_status = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.status = ops.status_word(self.device)
        if prewarm_prefill:
            for batch in (1, 2, 4):
                for length in (32, 64, 128):
                    if batch <= max_slots and length <= self.arena.capacity:
                        self._prefill(batch, length)

    # ------------------------------------------------------------------ shared buffers and graphs
    def predictor_step(self, batch: int) -> PredictorStep:
        step = self._predictors.get(batch)
        if step is None:
            step = PredictorStep(self.predictor_config, self.predictor_weights, self.codec_embedding, batch,
                                 self.device, **self.subtalker)
            self._predictors[batch] = step
        return step

    def batch_buffers(self, batch: int) -> dict:
        buffers = self._buffers.get(batch)
        if buffers is None:
            dev = self.device
            buffers = {"positions": torch.zeros(batch, dtype=torch.long, device=dev),
                       "rotary": torch.zeros(batch, dtype=torch.long, device=dev),
                       "uniform": torch.full((batch,), 0.5, dtype=torch.float32, device=dev),
                       "steps": torch.zeros(batch, dtype=torch.long, device=dev)}
            self._buffers[batch] = buffers
        return buffers

    def _tick_graph(self, batch: int, context: int) -> TickGraph:
        key = (batch, context)
        graph = self.graphs.get(key)
        if graph is None:
            graph = TickGraph(self, batch, context)
            if self.use_graphs:
                graph.capture()
            self.graphs[key] = graph
        return graph

    def _prefill(self, batch: int, length: int) -> TalkerPrefill:
        key = (batch, length)
        graph = self.prefills.get(key)
        if graph is None:
            graph = TalkerPrefill(self.talker_config, self.talker_weights, self.arena, batch, length, self.cos,
                                  self.sin)
            if self.use_graphs:
                graph.capture()
            self.prefills[key] = graph
        return graph

    def _packed_prefill(self, rows: int) -> PackedPrefill:
        graph = self.packed.get(rows)
        if graph is None:
            graph = PackedPrefill(self.talker_config, self.talker_weights, self.arena, rows, self.max_slots, self.cos,
                                  self.sin)
            if self.use_graphs:
                graph.capture()
            self.packed[rows] = graph
        return graph

    def _drop_graphs(self) -> None:
        for graph in list(self.graphs.values()) + list(self.prefills.values()) + list(self.packed.values()):
            graph.close()
        self.graphs.clear()
        self.prefills.clear()
        self.packed.clear()

    def ensure_capacity(self, required: int) -> None:
        """Double the KV arena when `required` does not fit (continuous.py:353-363); every
        graph that points into the old arena is dropped and recaptured lazily."""
        if required < self.arena.capacity:
            return
        self._drop_graphs()
        new = max(self.arena.capacity * 2, 1 << int(required).bit_length())
        self.arena = self.arena.grown(new)

    def _set_active(self, count: int) -> None:
        if count != self._active:
            self.state.active.fill_(count)
            self._active = count

    # ------------------------------------------------------------------ admission
    def prepare_prompt(self, payload: dict) -> dict:
        prompt = self.prompt_builder.build(payload)
        for key, value in SUPPORTED_SAMPLING.items():
            if prompt.get(key) != value:
                raise ValueError(f"Unsupported native sampling setting: {key}={prompt.get(key)}")
        if not 1 <= prompt["max_new_tokens"] <= self.max_frames:
            raise ValueError(f"max_new_tokens must be within 1..{self.max_frames}")
        return prompt

    def prepare_prompts(self, payloads) -> tuple:
        """prepare_prompt for several payloads with one text projection (CustomVoicePrompt
        .build_many): the prompts' rows packed end to end and the per-request prompt dicts."""
        packed, prompts = self.prompt_builder.build_many(payloads)
        for prompt in prompts:
            for key, value in SUPPORTED_SAMPLING.items():
                if prompt.get(key) != value:
                    raise ValueError(f"Unsupported native sampling setting: {key}={prompt.get(key)}")
            if not 1 <= prompt["max_new_tokens"] <= self.max_frames:
                raise ValueError(f"max_new_tokens must be within 1..{self.max_frames}")
        return packed, prompts

    @torch.inference_mode()
    def admit_batch(self, submissions) -> None:
        """Batched prefill into slots len(states).. (continuous.py:424-473): prompts packed end to
        end in groups of at most `max_prefill_rows` rows, or (packed_prefill=False) padded to a
        power-of-two length in groups of `max_prefill_batch` as the reference pads them."""
        submissions = list(submissions)
        if len(self.states) + len(submissions) > self.max_slots:
            raise ValueError("Insufficient continuous request slots")
        if not self.packed_prefill:
            for offset in range(0, len(submissions), self.max_prefill_batch):
                self._admit_group(submissions[offset:offset + self.max_prefill_batch])
            return
        packed, prompts = self.prepare_prompts([payload for _, payload in submissions])
        lengths = [p["inputs_embeds"].shape[1] for p in prompts]
        offsets = np.cumsum([0] + lengths).tolist()
        for start, end in packed_groups(lengths, self.max_prefill_rows):
            self._admit_group(submissions[start:end], prompts[start:end], packed[offsets[start]:offsets[end]])

    def _prefill_padded(self, prompts, lengths, count):
        n = len(prompts)
        padded = 1 << (max(lengths) - 1).bit_length()
        batch = 1 << (n - 1).bit_length() if self.bucket_prefill else n
        self.ensure_capacity(padded - 1)
        H = self.talker_config.hidden
        embeds = torch.zeros(batch, padded, H, dtype=BF16, device=self.device)
        for row, (prompt, length) in enumerate(zip(prompts, lengths)):
            embeds[row, :length] = prompt["inputs_embeds"][0]
        # graph padding rows repeat the last request (same slot, same values: benign duplicate writes)
        embeds[n:] = embeds[n - 1]
        host = torch.tensor([count + min(r, n - 1) for r in range(batch)] + [lengths[min(r, n - 1)]
                                                                             for r in range(batch)],
                            dtype=torch.long).pin_memory()
        table = host.to(self.device, non_blocking=True)
        slots, lens = table[:batch], table[batch:]
        return self._prefill(batch, padded).run(embeds, lens, slots)

    def _prefill_packed(self, prompts, lengths, count, embeds=None):
        n, total = len(prompts), sum(lengths)
        rows = packed_rows(total)
        self.ensure_capacity(max(lengths) - 1)
        graph = self._packed_prefill(rows)
        if embeds is None:
            embeds = torch.cat([p["inputs_embeds"][0] for p in prompts])
        packed = torch.empty(rows, self.talker_config.hidden, dtype=BF16, device=self.device)
        packed[:total] = embeds
        packed[total:] = embeds[-1]
        row_slots, row_pos, last = packed_tables(lengths, count, rows, self.max_slots)
        units = packed_units(lengths, count, rows, self.max_slots)
        host = torch.cat([row_slots, row_pos, last, units.view(torch.int64).view(-1)]).pin_memory()
        table = host.to(self.device, non_blocking=True)
        end = 2 * rows + self.max_slots
        return graph.run(packed, table[:rows], table[rows:2 * rows], table[2 * rows:end],
                         table[end:].view(torch.int32).view(-1, 4))

    def _admit_group(self, submissions, prompts=None, embeds=None) -> None:
        if prompts is None:
            prompts = [self.prepare_prompt(payload) for _, payload in submissions]
        lengths = [p["inputs_embeds"].shape[1] for p in prompts]
        count, n = len(self.states), len(submissions)
        S = self.state
        if self.packed_prefill:
            hidden, logits = self._prefill_packed(prompts, lengths, count, embeds)
        else:
            hidden, logits = self._prefill_padded(prompts, lengths, count)
        # per-slot state of the new requests
        # uniform tables: only the rows the requests can reach cross the bus; the rest of each
        # slot's table is reset on the device
        used = max(p["max_new_tokens"] for p in prompts) + 1
        tables = torch.full((n, used, 16), 0.5, dtype=torch.float32)
        for row, ((_, payload), prompt) in enumerate(zip(submissions, prompts)):
            table = random_table(int(payload.get("seed", 0)), prompt["max_new_tokens"])
            tables[row, :table.shape[0]] = table
        S.tables[count:count + n, :used].copy_(tables.pin_memory(), non_blocking=True)
        if used < S.table_rows:
            S.tables[count:count + n, used:].fill_(0.5)
        ints = torch.tensor([lengths, lengths, [0] * n, [1] * n], dtype=torch.long).pin_memory()
        ints = ints.to(self.device, non_blocking=True)
        S.positions[count:count + n].copy_(ints[0])
        S.rotary[count:count + n].copy_(ints[1])
        S.frames[count:count + n].copy_(ints[2])
        S.trailing_len[count:count + n].copy_(ints[3])
        S.hidden[count:count + n].copy_(hidden[:n])
        S.trailing[count:count + n, 0].copy_(torch.cat([p["trailing_text_hidden"][0, :1] for p in prompts]))
        S.pad[count:count + n].copy_(torch.cat([p["tts_pad_embed"][0, :1] for p in prompts]))
        # first semantic token: table[0, 0], no seen tokens, EOS blocked (continuous.py:409-422)
        ops.sample(logits[:n], uniforms=S.tables[count:count + n, 0, 0], seen=None, allowed=self.allowed,
                   steps=self._zeros[:n], eos=self.eos, min_steps=2, penalty=self.penalty,
                   temperature=self.temperature, top_k=self.top_k, top_p=self.top_p, seen_out=S.seen[count:count + n],
                   tokens=S.tokens[count:count + n].view(n, 1))
        rows = self._take_codec_rows(n) if self.incremental_codec else [-1] * n
        for ((identifier, payload), prompt, length), row in zip(zip(submissions, prompts, lengths), rows):
            self.states.append(RequestState(identifier, payload, length, 0, prompt["max_new_tokens"], codec_slot=row))

    def _take_codec_rows(self, n: int) -> list:
        """The n lowest free codec rows, cleared for a fresh stream (contiguous runs in one call each)."""
        self._codec_free.sort()
        rows, self._codec_free = self._codec_free[:n], self._codec_free[n:]
        start = 0
        for i in range(1, n + 1):
            if i == n or rows[i] != rows[i - 1] + 1:
                self.codec.reset_range(rows[start], i - start)
                start = i
        return rows

    def _release_codec_row(self, state) -> None:
        if state.codec_slot < 0:
            return
        (self._codec_held if self._inflight is not None else self._codec_free).append(state.codec_slot)
        state.codec_slot = -1

    # ------------------------------------------------------------------ compaction
    def _move_slot(self, source: int, destination: int) -> None:
        self.arena.move(source, destination)
        self.state.move(source, destination)

    def _remove(self, index: int) -> None:
        last = len(self.states) - 1
        if self.incremental_codec:
            self._release_codec_row(self.states[index])
        self._move_slot(last, index)
        if index != last:
            self.states[index] = self.states[last]
        self.states.pop()

    # ------------------------------------------------------------------ audio
    def emit_audio(self, selected, emit) -> None:
        """Decode due chunks grouped by length (<= codec_batch_size streams per call), convert
        to PCM16 on the device and deliver after one host copy (continuous.py:475-539)."""
        pending = self.decode_chunks(selected)
        if not pending:
            return
        for (group, _), block in zip(pending, self._to_host([pcm for _, pcm in pending])):
            for row, (state, _, skip) in enumerate(group):
                data = block[row, skip:].astype("<i2").tobytes()
                state.audio.append(data)
                state.emitted = state.frames
                if emit is not None:
                    emit(state.identifier, data, SAMPLE_RATE)

    def decode_chunks(self, selected) -> list:
        """The device half of emit_audio: decode every pending chunk of `selected` (frames
        state.emitted .. state.frames, or the windowed span with its left context) and return
        [(group, pcm16 device block)], group = [(state, start frame, samples to skip)]. Nothing
        is copied to the host and no request state changes."""
        slots = {id(state): index for index, state in enumerate(self.states)}
        groups: dict[int, list] = {}
        for state in selected:
            if state.frames == state.emitted:
                continue
            start = state.emitted if self.incremental_codec else max(0, state.emitted - self.context)
            groups.setdefault(state.frames - start, []).append((state, start, (state.emitted - start) * 1920))
        pending = []
        lanes = []   # with two codec streams: every group's (indices, codes), decoded on alternating lanes
        for length, entries in groups.items():
            for offset in range(0, len(entries), self.codec_batch_size):
                group = entries[offset:offset + self.codec_batch_size]
                indices = [slots[id(entry[0])] for entry in group]          # code ring rows (talker slots)
                if self.incremental_codec and getattr(self, "codec_streams", 1) == 2:
                    lanes.append((group, [entry[0].codec_slot for entry in group],
                                  self.codec_codes.read(indices, [entry[1] for entry in group], length)))
                else:
                    pending.append((group, self._decode_group(indices, [entry[1] for entry in group], length,
                                                              [entry[0].codec_slot for entry in group])))
        if lanes:
            outputs = self.codec.decode_groups([(indices, codes) for _, indices, codes in lanes])
            pending += [(group, out[1]) for (group, _, _), out in zip(lanes, outputs)]
        return pending

    # ------------------------------------------------------------------ pipelined audio
    def _launch_audio(self, due, finished) -> "AudioInFlight":
        """Decode the chunks of `due` on the codec lanes without waiting: the code rows are read on
        the engine stream (ordered after this tick's graph and before any later compaction), each
        lane waits for that, decodes its groups and copies their PCM16 into pinned host buffers.
        The next tick's graph runs on the engine stream meanwhile."""
        slots = {id(state): index for index, state in enumerate(self.states)}
        groups: dict[int, list] = {}
        for state in due:
            if state.frames > state.emitted:
                groups.setdefault(state.frames - state.emitted, []).append(state)
        reads = []
        for length, states in groups.items():
            for offset in range(0, len(states), self.codec_batch_size):
                group = states[offset:offset + self.codec_batch_size]
                codes = self.codec_codes.read([slots[id(st)] for st in group], [st.emitted for st in group], length)
                reads.append(([(st, st.frames) for st in group], [st.codec_slot for st in group], codes))
        flight = AudioInFlight(finished=list(finished))
        if not reads:
            return flight
        producer = torch.cuda.current_stream(self.device)
        lanes = self._audio_lanes
        for lane in lanes:
            lane.wait_stream(producer)
        for index, (group, rows, codes) in enumerate(reads):
            k = index % len(lanes)
            with torch.cuda.stream(lanes[k]):
                codes.record_stream(lanes[k])
                _, pcm = self.codec.decode(rows, codes, lane=k if self.codec.stream_count == 2 else 0)
                host = torch.empty(pcm.shape, dtype=torch.int16, pin_memory=True)
                host.copy_(pcm, non_blocking=True)
            flight.blocks.append((group, host))
        with torch.cuda.stream(lanes[-1]):
            for lane in lanes[:-1]:
                lanes[-1].wait_stream(lane)
            flight.status = torch.empty(1, dtype=torch.int32, pin_memory=True)
            flight.status.copy_(self.status[:1], non_blocking=True)
            flight.done = torch.cuda.Event()
            flight.done.record(lanes[-1])
        return flight

    def _deliver(self, flight, emit) -> list:
        """Wait for a launched tick's audio, hand its chunks to `emit` and return the results of
        the requests that ended with it; their codec rows become free again."""
        if flight is None:
            return []
        if flight.done is not None:
            flight.done.synchronize()
            if int(flight.status[0]) & ops.STATUS_NONFINITE:
                self.status.zero_()
                raise ValueError("Native codec emitted nonfinite audio")
        for group, host in flight.blocks:
            block = host.numpy()
            for row, (state, upto) in enumerate(group):
                data = block[row].astype("<i2").tobytes()
                state.audio.append(data)
                state.emitted = upto
                if emit is not None and not state.cancelled:
                    emit(state.identifier, data, SAMPLE_RATE)
        results = [(state.identifier, {"pcm": b"".join(state.audio), "sample_rate": SAMPLE_RATE,
                                       "codec_frames": state.frames, "finish_reason": reason})
                   for state, reason in flight.finished if not state.cancelled]
        self._codec_free.extend(self._codec_held)
        self._codec_held = []
        return results

    def _decode_group(self, indices, starts, length, rows=None):
        """PCM16 [len(indices), length * 1920] (device) of frames starts[i] .. + length of talker
        slots `indices`, decoded in codec rows `rows` (incremental codec)."""
        codes = self.codec_codes.read(indices, starts, length)
        if self.incremental_codec:
            return self.codec.decode(rows, codes)[1]
        return self.codec.decode(codes)[1]

    def _to_host(self, blocks):
        """One device->host copy of every PCM block; raises on nonfinite codec output."""
        flat = torch.cat([block.reshape(-1) for block in blocks])
        if flat.device.type == "cuda":
            host = torch.empty(flat.shape, dtype=torch.int16, pin_memory=True)
            host.copy_(flat, non_blocking=True)
            self._host_status.copy_(self.status[:1], non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            if int(self._host_status[0]) & ops.STATUS_NONFINITE:
                self.status.zero_()
                raise ValueError("Native codec emitted nonfinite audio")
            flat = host
        audio = flat.numpy()
        out, offset = [], 0
        for block in blocks:
            out.append(audio[offset:offset + block.numel()].reshape(block.shape))
            offset += block.numel()
        return out

    def _report_codes(self, tokens) -> None:
        """on_codes(identifier, frame, codes[16], next_token) for the frame each slot just decoded."""
        depth = self.codec_codes.depth
        rows = torch.tensor([i * depth + s.frames % depth for i, s in enumerate(self.states)], device=self.device)
        codes = self.codec_codes.data.view(-1, self.codec_codes.codebooks).index_select(0, rows).cpu().tolist()
        for state, frame_codes, token in zip(self.states, codes, tokens):
            self.on_codes(state.identifier, state.frames, frame_codes, token)

    def _run_tick(self, count: int) -> list:
        """Replay the (batch, context) tick graph for `count` active slots; return their new tokens."""
        batch = decode_batch_size(count, self.max_slots, self.decode_bucket_step)
        required = max(state.position for state in self.states)
        self.ensure_capacity(required)
        context = context_bucket(required + 1, self.arena.capacity)
        graph = self._tick_graph(batch, context)
        self._set_active(count)
        graph.run()
        self._host_tokens[:count].copy_(self.state.tokens[:count], non_blocking=True)
        self._host_status.copy_(self.status[:1], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        if int(self._host_status[0]):
            bits = int(self._host_status[0])
            self.status.zero_()
            raise RuntimeError(f"Device status 0x{bits:x} raised during the tick")
        return self._host_tokens[:count].tolist()

    # ------------------------------------------------------------------ one scheduler iteration
    @torch.inference_mode()
    def tick(self, submissions=(), emit=None, cancelled=()):
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        if self.pipeline_audio:
            # the tick's own work runs on a high-priority stream, so that the codec lanes decoding the
            # previous tick's audio take only the SMs its dependent kernels leave free
            self._engine_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self._engine_stream):
                return self._tick(submissions, emit, cancelled)
        return self._tick(submissions, emit, cancelled)

    def _tick(self, submissions, emit, cancelled):
        started = time.perf_counter()
        stats = self.stats
        cancelled = set(cancelled)
        for index in reversed(range(len(self.states))):
            if self.states[index].identifier in cancelled:
                self.states[index].cancelled = True
                self._remove(index)
                stats.cancelled += 1
        if self._inflight is not None:   # requests that ended last tick, awaiting their last chunk
            for state, _ in self._inflight.finished:
                if state.identifier in cancelled:
                    state.cancelled = True
        if submissions:
            before = len(self.states)
            self.admit_batch(submissions)
            stats.admitted += len(self.states) - before
        if not self.states:
            flight, self._inflight = self._inflight, None
            return self._deliver(flight, emit)
        stats.active = len(self.states)
        stats.batch = decode_batch_size(stats.active, self.max_slots, self.decode_bucket_step)
        tokens = self._run_tick(len(self.states))
        if self.on_codes is not None:
            self._report_codes(tokens)
        results = []
        if self.pipeline_audio:
            # the previous tick's chunks decoded while this tick's graph ran: deliver them before
            # this tick's emission schedule is evaluated
            flight, self._inflight = self._inflight, None
            results += self._deliver(flight, emit)
        due, finished = [], []
        for index, state in enumerate(self.states):
            state.frames += 1
            state.position += 1
            stopped = tokens[index] == self.eos
            limited = state.frames >= state.max_new_tokens - 1
            if state.frames >= emission_target(state.emitted, self.codec_chunk_frames) or stopped or limited:
                due.append(state)
            if stopped or limited:
                finished.append((index, state, "stop" if stopped else "length"))
        if self.pipeline_audio:
            # this tick's chunks decode on the codec lanes while the next tick's graph runs
            self._inflight = self._launch_audio(due, [(state, reason) for _, state, reason in finished])
            for index, _, _ in reversed(finished):
                self._remove(index)
        else:
            self.emit_audio(due, emit)
            for index, state, reason in reversed(finished):
                results.append((state.identifier, {"pcm": b"".join(state.audio), "sample_rate": SAMPLE_RATE,
                                                   "codec_frames": state.frames, "finish_reason": reason}))
                self._remove(index)
        elapsed = time.perf_counter() - started
        stats.ticks += 1
        stats.frames += stats.active
        stats.finished += len(results)
        stats.last_tick_ms = elapsed * 1e3
        stats.tick_seconds += elapsed
        return results

    def generate(self, payloads, emit=None):
        """The batch API of the reference's CustomVoiceModel.generate (model.py:58-129): run
        `payloads` to completion and return one result record per payload, in order;
        `emit(index, pcm, sample_rate)` streams audio chunks under the payload's index. Served by
        the continuous tick: at most `max_slots` requests in flight, the rest admitted as slots
        free up. Raises ValueError while continuous requests are active (one mode at a time)."""
        if self.states:
            raise ValueError("generate() needs an idle engine; continuous requests are active")
        pending = [(("batch", index), payload) for index, payload in enumerate(payloads)]
        relay = None if emit is None else (lambda ident, pcm, rate: emit(ident[1], pcm, rate))
        results = {}
        while pending or self.states or self._inflight is not None:
            free = self.max_slots - len(self.states)
            submissions, pending = pending[:free], pending[free:]
            for ident, record in self.tick(submissions, emit=relay):
                results[ident[1]] = record
        return [results[index] for index in range(len(payloads))]

    def close(self) -> None:
        if self._inflight is not None and self._inflight.done is not None:
            self._inflight.done.synchronize()
        self._inflight = None
        logging.getLogger(__name__).info("Captured graph shapes: prefill=%s tick=%s codec=%s", sorted(self.prefills),
                                         sorted(self.graphs), sorted(self.codec.slots.graphs
                                                                     if isinstance(self.codec, CodecGraph)
                                                                     else self.codec.graphs))
        self._drop_graphs()
        for step in self._predictors.values():
            step.close()
        self._predictors.clear()
        self.codec.close()
