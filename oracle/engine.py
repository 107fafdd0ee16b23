"""One request of the continuous-batching engine restated on the CPU, teacher-forced.

TEST INFRASTRUCTURE ONLY (see the package docstring).

Follows ContinuousModel (continuous.py): admission prefill and first token
(continuous.py:424-473, 409-422), then per tick the predictor chain on
(hidden, codec embedding of the semantic code) with draws = table[frames]
(continuous.py:575-589), the frame embedding plus text (continuous.py:590-601),
the talker step at position/rotary (continuous.py:602-613) and semantic
sampling with steps = frames + 1 and u = table[frames + 1, 0]
(continuous.py:614-619). Sampling here is greedy (top-k 1), so each draw has
one answer up to ties: the oracle consumes the ENGINE's codes as its history
(teacher forcing) and records, for every draw, the gap between the best score
and the score of the engine's choice. A gap of zero is an exact match; a
small positive gap is a near tie that bf16 rounding may legitimately flip.
"""
from __future__ import annotations

import torch

from . import decoder as OD
from .elementwise import bf
from .sampling import allowed_mask


def semantic_scores(logits, seen, steps, allowed, eos, penalty=1.05, min_steps=2):
    """Scores the semantic sampler ranks (continuous.py:365-370) before temperature/top-k."""
    scores = logits.float().clone()
    scores = torch.where(seen, torch.where(scores < 0, scores * penalty, scores / penalty), scores)
    scores = scores.masked_fill(~allowed, -float("inf"))
    if steps < min_steps:
        scores[eos] = -float("inf")
    return scores


def gap(scores, token: int) -> float:
    best = float(scores.max())
    value = float(scores[token])
    return best - value if value != -float("inf") else float("inf")


class RequestOracle:
    def __init__(self, talker_cfg, predictor_cfg, talker_w, predictor_w, inputs_embeds, pad, table, capacity,
                 mode="bf16f"):
        self.tc, self.pc, self.tw, self.pw = talker_cfg, predictor_cfg, talker_w, predictor_w
        self.mode, self.pad, self.table = mode, pad.float(), table
        self.allowed = allowed_mask(talker_cfg.vocab, talker_cfg.eos)
        self.ttables = OD.Tables(capacity, talker_cfg.head_dim, talker_cfg.theta)
        self.ptables = OD.Tables(predictor_cfg.groups + 1, predictor_cfg.head_dim, predictor_cfg.theta)
        self.cache = OD.new_cache(talker_cfg, 1, capacity)
        L = inputs_embeds.shape[0]
        pos = torch.arange(L)[None]
        h = OD.decoder_forward(talker_cfg, talker_w, inputs_embeds.float()[None], pos, self.cache, pos, self.ttables,
                               mode)
        self.hidden = h[0, -1]
        self.logits = self._head(self.hidden)
        self.position, self.frames = L, 0
        self.seen = torch.zeros(talker_cfg.vocab, dtype=torch.bool)
        self.token = None
        self.gaps: list[float] = []
        self.labels: list[tuple] = []   # (frame, draw kind, step, engine token, best token) per gap

    def _head(self, hidden):
        logits = hidden @ self.tw["head"].float().T
        return bf(logits) if self.mode in ("bf16", "bf16f") else logits

    def _record(self, scores, token, kind, step):
        self.gaps.append(gap(scores, token))
        self.labels.append((self.frames, kind, step, int(token), int(scores.argmax())))

    def first(self, engine_token: int) -> None:
        scores = semantic_scores(self.logits, self.seen, 0, self.allowed, self.tc.eos)
        self._record(scores, engine_token, "first", 0)
        self.seen[engine_token] = True
        self.token = engine_token

    def frame(self, engine_codes, engine_next: int) -> None:
        """Consume one engine frame (16 codes) and the engine's next semantic token."""
        codes = [int(c) for c in engine_codes]
        if codes[0] != self.token:
            raise AssertionError(f"frame {self.frames}: semantic code {codes[0]} != carried token {self.token}")
        first = self.tw["embedding"][codes[0]].float()
        draws = self.table[self.frames][None]
        subcodes, acc, logits = OD.predictor_frame(self.pc, self.pw, self.hidden[None], first[None], draws,
                                                   self.ptables, self.mode, top_k=1,
                                                   forced_codes=torch.tensor([codes[1:]]))
        for step in range(self.pc.groups):
            self._record(logits[step, 0].float(), codes[1 + step], "predictor", step)
        embeds = bf(bf(acc) + self.pad) if self.mode in ("bf16", "bf16f") else acc + self.pad
        hidden, logits = OD.talker_decode_step(self.tc, self.tw, embeds, torch.tensor([self.position]),
                                               torch.tensor([0]), self.cache, self.ttables, self.mode)
        self.hidden = hidden[0]
        scores = semantic_scores(logits[0], self.seen, self.frames + 1, self.allowed, self.tc.eos)
        self._record(scores, engine_next, "talker", 0)
        self.seen[engine_next] = True
        self.token = engine_next
        self.frames += 1
        self.position += 1
