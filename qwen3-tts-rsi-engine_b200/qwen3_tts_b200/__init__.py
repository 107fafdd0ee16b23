"""B200-native (sm_100a) engine for the Qwen3-TTS talker -> code-predictor -> codec decode path.

The compute path is ``libq3t_b200.so`` (hand-written CUDA kernels behind the C ABI
in ``include/q3t.h``), loaded through ctypes by ``_lib``; host scheduling mirrors
the reference engine's Python surface.
"""
__version__ = "0.1.0"
