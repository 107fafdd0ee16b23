"""B200-native (sm_100a) engine for the Qwen3-TTS talker -> code-predictor -> codec decode path.

The compute path is ``libq3t_b200.so`` (hand-written CUDA kernels behind the C ABI
in ``include/q3t.h``), loaded through ctypes by ``_lib``; host scheduling mirrors
the reference engine's Python surface. Modules, by the reference module they stand in for:

* ``continuous`` (ContinuousModel, tick / generate), ``talker`` (SlotArena, the decode and
  prefill graphs), ``predictor`` (the 15-codebook predictor), ``codec`` (CodecSlots,
  CodecGraph), ``code_buffer``, ``request_views``, ``batching``, ``sampling``;
* ``kernels`` (the reference's kernel wrappers: write, rotary, snake, select,
  scatter_rows, copy_packed_prefix) over ``ops`` (tensor-level wrappers of the C ABI);
* ``operators``, ``packed_attention``, ``packed_mlp``, ``fused_decoder`` (module-replacement
  plugins with the reference's install functions);
* ``server`` (SpeechService and the command line), ``dispatcher`` (one engine process per
  GPU), ``prompt`` (CustomVoice prompt preparation), ``checkpoint`` (safetensors loading),
  ``metrics`` (service metrics), ``tracing`` (phase tracing);
* ``config``, ``weights``, ``codec_weights`` (geometry, seeded weights and device layouts).
"""
__version__ = "0.1.0"
