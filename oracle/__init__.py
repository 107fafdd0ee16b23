"""CPU oracle for the Qwen3-TTS talker -> code-predictor -> codec decode path.

TEST INFRASTRUCTURE ONLY. This package restates, on the CPU, the reference
engine's algorithms (InferMatrixLab/qwen3-tts-rsi-engine, package
``qwen3_tts_engine``) and the parts of the third-party ``qwen-tts==0.1.1``
model that the reference calls (absent from this environment; restated from
the reference's call sites and the model shapes). Every function cites the
reference ``file:line`` it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and ``--impl reference`` legs may import it, and only as the checker or the
timed CPU baseline. The product package never imports it and has no CPU path.

Pinning: the reference-owned pieces (batching, sampling, KV scatter/copy,
code buffer, request views, incremental-codec state logic, RVQ decode) are
checked against golden fixtures produced by importing the reference itself
(``tests/golden/make_golden.py``). The ``qwen-tts`` model internals (decoder
layer, code-predictor projection, codec module stack) have no reference
implementation available here: at that boundary parity is unpinned and the
restatement follows the reference call sites and BASELINE shapes.
"""
