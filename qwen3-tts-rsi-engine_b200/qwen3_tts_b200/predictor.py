"""Code predictor: the 15-codebook autoregressive chain per frame, one CUDA graph per batch.

Mirrors ``UniformPredictor`` (continuous.py:20-94): step 0 runs the talker
hidden state and the semantic code's embedding as two tokens at positions
[0, 1] with a causal mask; step i runs the embedding of code i (codebook i-1
table) at position i+1; head i samples code i+1 from ``draws[:, i+1]``
(the request's uniform table) or from Philox (seed, per-row stream offset).
With ``graph_embeddings`` the frame embedding (talker codec embedding of the
semantic code plus the 15 predictor embeddings, summed once, plus the text
embedding) is produced in the same graph (continuous.py:63-67, 590-601).

All 15 steps x 5 layers and the sampling run as ~425 kernels from
``libq3t_b200.so`` replayed as one graph; the RoPE coefficients of the 16
fixed positions are precomputed (fixed_predictor_rotary.py). With the packed
weights of ``pack_decoder`` a step i >= 1 gathers its input row from the
pre-projected codebook table (proj and bias applied once at load), runs q/k
norm, RoPE and the K/V write inside the attention kernel, and the final
RMSNorm is folded into the codebook heads.
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .config import PredictorConfig
from . import talker
from .talker import mlp_stages, qkv_stage, rope_tables
from .weights import pack_decoder

BF16 = torch.bfloat16


class PredictorStep:
    def __init__(self, cfg: PredictorConfig, weights: dict, talker_embedding: torch.Tensor, batch: int, device, *,
                 temperature: float = 0.9, top_k: int = 50, top_p: float = 1.0, philox_seed=None,
                 record_logits: bool = False):
        self.cfg, self.w, self.batch = cfg, weights, batch
        self.device = torch.device(device)
        self.talker_embedding = talker_embedding
        self.temperature, self.top_k, self.top_p = temperature, top_k, top_p
        self.philox_seed = philox_seed
        dev, B, Hp, Ht = self.device, batch, cfg.hidden, cfg.talker_hidden
        positions = cfg.groups + 1
        self.cos, self.sin = rope_tables(positions, cfg.head_dim, cfg.theta, dev)
        self.inputs = torch.zeros(B, 2, Ht, dtype=BF16, device=dev)          # (hidden, first)
        self.draws = torch.full((B, 16), 0.5, dtype=torch.float32, device=dev)
        self.offsets = torch.zeros(B, dtype=torch.long, device=dev)         # Philox stream per row
        self.codes = torch.zeros(B, cfg.groups + 1, dtype=torch.long, device=dev)
        self.text = torch.zeros(B, Ht, dtype=BF16, device=dev)
        self.embeds = torch.zeros(B, Ht, dtype=BF16, device=dev)            # next talker input
        self.x = torch.zeros(2 * B, Hp, dtype=BF16, device=dev)
        self.xn = torch.zeros(2 * B, Hp, dtype=BF16, device=dev)
        self.qkv = torch.zeros(2 * B, cfg.qkv_width, dtype=BF16, device=dev)
        self.q = torch.zeros(2 * B, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.attn = torch.zeros(2 * B, cfg.q_heads, cfg.head_dim, dtype=BF16, device=dev)
        self.act = torch.zeros(2 * B, cfg.ffn, dtype=BF16, device=dev)
        self.e = torch.zeros(B, Ht, dtype=BF16, device=dev)
        self.logits = torch.zeros(B, cfg.vocab, dtype=torch.float32, device=dev)
        # optional per-step logits (parity checks); the head GEMMs write there directly
        self.step_logits = (torch.zeros(cfg.groups, B, cfg.vocab, dtype=torch.float32, device=dev)
                            if record_logits else None)
        self.cache = torch.zeros(2 * cfg.layers, B, cfg.kv_heads, positions, cfg.head_dim, dtype=BF16, device=dev)
        self.pos0 = torch.tensor([0, 1] * B, dtype=torch.long, device=dev)
        self.pos = torch.arange(2, positions, dtype=torch.long, device=dev).view(-1, 1).repeat(1, B).contiguous()
        gemms = [(Ht, Hp), (Hp, cfg.qkv_width), (cfg.q_width, Hp), (Hp, 2 * cfg.ffn), (cfg.ffn, Hp), (Hp, cfg.vocab)]
        need = max(ops.linear_workspace_bytes(2 * B, k, n) for k, n in gemms)
        self.ws_linear = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
        need = ops.decode_attention_workspace_bytes(2 * B, cfg.q_heads, cfg.head_dim, positions)
        self.ws_attn = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
        self.status = ops.status_word(dev)
        self.prefetch_weights = True  # GEMMs pull the next GEMM's weights into L2
        # steps >= 1 (one row per slot, <= 64 rows): each layer's O, gate/up, down and the next
        # layer's QKV (or the codebook head after the last layer) run as one q3t_linear_chain launch
        self.use_chain = (talker.CHAIN_PROJECTIONS and B <= 64 and weights["layers"][0].folded and weights.get("heads_folded", False)
                          and isinstance(weights["layers"][0].qkv, ops.TiledWeight))
        self.ws_chain = ops.linear_chain_workspace(B, dev) if self.use_chain else None
        # Layers [0, keep_layers) load their weights evict-last (Q3T_LINEAR_KEEP_WEIGHTS) to keep them
        # in L2 across the 15 codebook steps; measured no faster (the GEMMs are latency-bound), so off.
        self.keep_layers = 0
        self.graph = None

    def _layers(self, rows: int, length: int, positions: torch.Tensor, tail=None) -> None:
        """The decoder layers on x[:rows]; `tail` is the weight used after them (L2 prefetch target)."""
        cfg, lw = self.cfg, ops.linear
        x = self.x[:rows]
        L = cfg.layers
        layers = self.w["layers"]
        # each GEMM pulls the next GEMM's weights into L2 while it runs
        pf = (lambda t: t) if self.prefetch_weights else (lambda t: None)
        for i, layer in enumerate(layers):
            keys, values = self.cache[i], self.cache[L + i]
            following = layers[i + 1].qkv if i + 1 < L else tail
            keep = i < self.keep_layers
            if layer.folded:
                lw(x, layer.qkv, out=self.qkv[:rows], row_norm_eps=cfg.eps, prefetch=pf(layer.o), keep_weights=keep)
            else:
                ops.rms_norm(x, layer.input_norm, cfg.eps, out=self.xn[:rows])
                lw(self.xn[:rows], layer.qkv, out=self.qkv[:rows], workspace=self.ws_linear, prefetch=pf(layer.o),
                   keep_weights=keep)
            if length == 1:
                # one query row per slot: q/k norm, RoPE and the K/V write run inside attention
                ops.decode_attention_qkv(self.qkv[:rows], layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin,
                                         positions, keys, values, positions, q_heads=cfg.q_heads,
                                         kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, context=keys.shape[2],
                                         out=self.attn[:rows], workspace=self.ws_attn)
            else:
                ops.qk_norm_rope_kv(self.qkv[:rows], layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin,
                                    positions, positions, keys, values, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads,
                                    head_dim=cfg.head_dim, length=length, query_out=self.q[:rows])
                ops.decode_attention(self.q[:rows], keys, values, positions, context=keys.shape[2],
                                     rows_per_slot=length, out=self.attn[:rows], workspace=self.ws_attn)
            lw(self.attn[:rows].view(rows, cfg.q_width), layer.o, out=x, epilogue=_lib.EPI_RESIDUAL, residual=x,
               workspace=self.ws_linear, prefetch=pf(layer.gate_up), keep_weights=keep)
            if layer.folded:
                lw(x, layer.gate_up, out=self.act[:rows], epilogue=_lib.EPI_SWIGLU_PAIRED, row_norm_eps=cfg.eps,
                   prefetch=pf(layer.down), keep_weights=keep)
            else:
                ops.rms_norm(x, layer.post_norm, cfg.eps, out=self.xn[:rows])
                lw(self.xn[:rows], layer.gate_up, out=self.act[:rows], epilogue=_lib.EPI_SWIGLU_PAIRED,
                   workspace=self.ws_linear, prefetch=pf(layer.down), keep_weights=keep)
            lw(self.act[:rows], layer.down, out=x, epilogue=_lib.EPI_RESIDUAL, residual=x, workspace=self.ws_linear,
               prefetch=pf(following) if following is not None else None, keep_weights=keep)
        if not self.w.get("heads_folded", False):
            ops.rms_norm(x, self.w["norm"], self.cfg.eps, out=self.xn[:rows])

    def _chained_step(self, step: int) -> None:
        """Steps >= 1 with the projections as chains: QKV of layer 0, then per layer the fused
        attention and one chain (O, gate/up, down, next QKV; the last layer's chain ends with
        codebook head `step`, final norm folded in, fp32 logits)."""
        cfg, B = self.cfg, self.batch
        x = self.x[:B]
        layers = self.w["layers"]
        positions = self.pos[step - 1]
        ops.linear_chain([qkv_stage(x, layers[0], self.qkv[:B], cfg.eps, depends=-1)], self.ws_chain)
        for i, layer in enumerate(layers):
            keys, values = self.cache[i], self.cache[cfg.layers + i]
            ops.decode_attention_qkv(self.qkv[:B], layer.q_norm, layer.k_norm, cfg.eps, self.cos, self.sin,
                                     positions, keys, values, positions, q_heads=cfg.q_heads,
                                     kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, context=keys.shape[2],
                                     out=self.attn[:B], workspace=self.ws_attn)
            stages = mlp_stages(self.attn[:B].view(B, cfg.q_width), x, layer, x, self.act[:B], cfg.eps)
            if i + 1 < len(layers):
                stages.append(qkv_stage(x, layers[i + 1], self.qkv[:B], cfg.eps, depends=2))
            else:
                stages.append({"x": x, "weight": self.w["heads"][step], "out": self._logits(step),
                               "row_norm_eps": cfg.eps, "depends": 2})
            ops.linear_chain(stages, self.ws_chain)

    def _head(self, step: int, last: slice) -> None:
        """Codebook head `step` on the last decoder row of every slot (`last` picks those rows of
        x / xn). With folded heads the final RMSNorm weight is inside the head matrix and the GEMM
        applies the row RMS to the raw residual rows itself."""
        w = self.w
        following = w["layers"][0].qkv if self.prefetch_weights and step + 1 < self.cfg.groups else None
        if w.get("heads_folded", False):
            ops.linear(self.x[last], w["heads"][step], out=self._logits(step), out_dtype=torch.float32,
                       row_norm_eps=self.cfg.eps, prefetch=following)
        else:
            ops.linear(self.xn[last], w["heads"][step], out=self._logits(step), out_dtype=torch.float32,
                       workspace=self.ws_linear, prefetch=following)

    def _logits(self, step: int) -> torch.Tensor:
        return self.logits if self.step_logits is None else self.step_logits[step]

    def _sample(self, step: int) -> None:
        tokens = self.codes[:, step + 1]
        logits = self._logits(step)
        if self.philox_seed is None:
            ops.sample(logits, uniforms=self.draws[:, step + 1], temperature=self.temperature, top_k=self.top_k,
                       top_p=self.top_p, tokens=tokens)
        else:
            ops.sample(logits, seed=self.philox_seed, philox_offsets=self.offsets, philox_add=step,
                       temperature=self.temperature, top_k=self.top_k, top_p=self.top_p, tokens=tokens)

    def compute(self) -> None:
        cfg, w, B, lw = self.cfg, self.w, self.batch, ops.linear
        lw(self.inputs.view(2 * B, cfg.talker_hidden), w["proj"], w["proj_bias"], out=self.x, workspace=self.ws_linear)
        self._layers(2 * B, 2, self.pos0, tail=w["heads"][0])
        self._head(0, slice(1, 2 * B, 2))  # second row of every slot
        self._sample(0)
        tables = w.get("proj_tables")
        for step in range(1, cfg.groups):
            if tables is not None:  # projected row of codebook table step-1 (proj and bias applied at load)
                ops.embedding(self.codes[:, step], tables[step - 1], out=self.x[:B])
            else:
                ops.embedding(self.codes[:, step], w["embeddings"][step - 1], out=self.e)
                lw(self.e, w["proj"], w["proj_bias"], out=self.x[:B], workspace=self.ws_linear)
            if self.use_chain:
                self._chained_step(step)
            else:
                self._layers(B, 1, self.pos[step - 1], tail=w["heads"][step])
                self._head(step, slice(0, B))
            self._sample(step)
        ops.frame_embed(self.codes, self.talker_embedding, w["embeddings"], self.text, out=self.embeds)

    @torch.inference_mode()
    def capture(self, warmup: int = 2) -> None:
        stream = torch.cuda.Stream(device=self.device)
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

    @torch.inference_mode()
    def run(self, hidden, first_codes, draws=None, text=None, offsets=None, clone: bool = True):
        """hidden [B, Ht]; first_codes [B] semantic codes -> (codes [B, 16], talker input embeddings [B, Ht])."""
        B = self.batch
        self.inputs[:, 0].copy_(hidden)
        ops.embedding(first_codes.view(-1), self.talker_embedding, out=self.inputs[:, 1])
        self.codes[:, 0].copy_(first_codes.view(-1))
        if draws is not None:
            self.draws.copy_(draws)
        if offsets is not None:
            self.offsets.copy_(offsets)
        if text is not None:
            self.text.copy_(text)
        if self.graph is None:
            self.compute()
        else:
            self.graph.replay()
        if clone:
            return self.codes.clone(), self.embeds.clone()
        return self.codes, self.embeds

    def close(self) -> None:
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None


class CodePredictor:
    """Predictor weights plus one captured chain per batch size (UniformPredictor.captures)."""

    def __init__(self, cfg: PredictorConfig, weights: dict, talker_embedding: torch.Tensor, device, packed=False,
                 use_graphs=True, **sampling):
        self.cfg = cfg
        self.device = torch.device(device)
        self.weights = weights if packed else pack_decoder(weights, self.device)
        self.talker_embedding = talker_embedding
        self.use_graphs = use_graphs
        self.sampling = sampling
        self.captures: dict[int, PredictorStep] = {}

    def step_for(self, batch: int) -> PredictorStep:
        step = self.captures.get(batch)
        if step is None:
            step = PredictorStep(self.cfg, self.weights, self.talker_embedding, batch, self.device, **self.sampling)
            if self.use_graphs:
                step.capture()
            self.captures[batch] = step
        return step

    def run(self, hidden, first_codes, draws=None, text=None, offsets=None):
        return self.step_for(hidden.shape[0]).run(hidden, first_codes, draws=draws, text=text, offsets=offsets)

    def close(self) -> None:
        for step in self.captures.values():
            step.close()
        self.captures.clear()
