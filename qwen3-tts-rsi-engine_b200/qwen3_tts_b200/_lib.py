"""ctypes binding of the C ABI in ``include/q3t.h`` (``libq3t_b200.so``).

Loading is lazy and loud: if the shared library is missing or fails to load,
every operation raises - there is no CPU or library fallback behind these ops.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIBRARY_PATH = _HERE / "libq3t_b200.so"

Q3T_OK, Q3T_EINVAL, Q3T_EUNSUPPORTED, Q3T_ECUDA, Q3T_ESPACE = 0, -1, -2, -3, -4
Q3T_BF16, Q3T_F32 = 0, 1
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU_PAIRED, EPI_RESIDUAL_SCALED, EPI_GELU, EPI_SILU, EPI_SNAKE = 0, 1, 2, 3, 4, 5, 6
LINEAR_KEEP_WEIGHTS = 1
LINEAR_NARROW = 2
NORM_REFERENCE, NORM_NATIVE = 0, 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t

CHAIN_MAX_STAGES = 8


class ChainStage(ctypes.Structure):
    """q3t_chain_stage (include/q3t.h): one projection of a q3t_linear_chain."""
    _fields_ = [("x", ctypes.c_void_p), ("x_stride", ctypes.c_int64), ("weight_tiles", ctypes.c_void_p),
                ("in_features", ctypes.c_int64), ("out_features", ctypes.c_int64), ("out", ctypes.c_void_p),
                ("out_stride", ctypes.c_int64), ("out_dtype", ctypes.c_int), ("epilogue", ctypes.c_int),
                ("residual", ctypes.c_void_p), ("residual_stride", ctypes.c_int64), ("bias", ctypes.c_void_p),
                ("row_norm_eps", ctypes.c_float), ("depends", ctypes.c_int)]


# name -> (restype, argtypes); mirrors include/q3t.h exactly.
SIGNATURES: dict[str, tuple[object, list]] = {
    "q3t_abi_version": (_i32, []),
    "q3t_last_error": (ctypes.c_char_p, []),
    "q3t_launch_count": (_u64, []),
    "q3t_kv_write": (_i32, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _p, _p]),
    "q3t_copy_packed_prefix": (_i32, [_p, _p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _p]),
    "q3t_slot_move": (_i32, [_p, _i64, _i64, _i64, _i64, _i32, _i64, _i64, _p]),
    "q3t_copy_rows": (_i32, [_p, _i64, _p, _i64, _i64, _i64, _p]),
    "q3t_slot_zero": (_i32, [_p, _i64, _i64, _i64, _i64, _i32, _i64, _i64, _p]),
    "q3t_advance": (_i32, [_p, _i64, _i64, _p]),
    "q3t_rms_norm": (_i32, [_p, _i64, _p, _p, _i64, _i64, _f32, _i32, _p]),
    "q3t_add_rms_norm": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _f32, _i32, _p]),
    "q3t_rotary": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "q3t_swiglu": (_i32, [_p, _p, _i64, _i64, _p]),
    "q3t_snake": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _p]),
    "q3t_linear_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "q3t_attention_plan": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _p, _sz, _p]),
    "q3t_decode_attention_qkv": (_i32, [_p, _i64, _p, _p, _f32, _p, _p, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                        _i64, _i64, _i64, _i64, _f32, _p, _sz, _p, _p]),
    "q3t_decode_attention_qkv_ex": (_i32, [_p, _i64, _p, _p, _f32, _p, _p, _i64, _p, _p, _p, _p, _p, _i64, _i64,
                                           _i64, _i64, _i64, _i64, _i64, _f32, _p, _sz, _p, _sz, _p, _sz, _p, _p]),
    "q3t_linear_rownorm": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _p, _p, _i64, _i32, _i32, _p, _i64, _p, _f32, _p,
                                  _p, _p]),
    "q3t_linear": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _p, _p, _i64, _i32, _i32, _p, _i64, _p, _p, _p, _sz,
                          _p, _p]),
    "q3t_linear_ex": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _p, _p, _i64, _i32, _i32, _p, _i64, _p, _f32, _p, _p,
                             _sz, _i32, _p, _p]),
    "q3t_weight_tiles_bytes": (_sz, [_i64, _i64]),
    "q3t_pack_weight_tiles": (_i32, [_p, _i64, _i64, _p, _p]),
    "q3t_qk_norm_rope_kv": (_i32, [_p, _i64, _p, _p, _f32, _p, _p, _i64, _p, _p, _p, _p, _p, _i64, _i64, _p, _i64,
                                   _i64, _i64, _i64, _p, _p]),
    "q3t_decode_attention_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "q3t_decode_attention": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _f32, _p, _sz, _p, _p]),
    "q3t_decode_attention_noalloc": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                            _i64, _f32, _p, _p]),
    "q3t_prefill_attention": (_i32, [_p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p,
                                     _p]),
    "q3t_cdf_select": (_i32, [_p, _p, _p, _i64, _i64, _p]),
    "q3t_sample": (_i32, [_p, _i32, _i64, _p, _i64, _p, _p, _i64, _i64, _f32, _f32, _i64, _f32, _p, _i64, _u64,
                          _p, _i64, _p, _i64, _p, _i64, _i64, _i64, _p]),
    "q3t_philox_uniforms": (_i32, [_u64, _u64, _p, _i64, _p]),
    "q3t_frame_embed": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _p, _p]),
    "q3t_embedding": (_i32, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _p, _p]),
    "q3t_scatter_rows": (_i32, [_p, _i64, _p, _p, _i32, _p, _p, _i32, _p, _p]),
    "q3t_rvq_gather": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "q3t_conv_gather": (_i32, [_p, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _i64, _i32, _p, _p, _p, _p]),
    "q3t_conv_pad": (_i32, [_p, _i64, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _p, _p]),
    "q3t_conv_linear": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _p, _i64, _p, _p, _i64, _i32, _p, _i64,
                               _p, _p, _p, _p, _p]),
    "q3t_conv_history": (_i32, [_p, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "q3t_dwconv_layernorm": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _p, _p, _f32, _p, _p]),
    "q3t_codec_positions": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p, _i32, _p]),
    "q3t_pcm16": (_i32, [_p, _i64, _p, _p, _p, _p]),
    "q3t_tick_gather": (_i32, [_p, _p, _p, _p, _i64, _p, _i64, _p, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _p, _p,
                               _p, _p, _p, _p, _i64, _i64, _p, _p]),
    "q3t_tick_commit": (_i32, [_p, _p, _i64, _i64, _p, _p, _p, _i64, _p, _p, _p, _i64, _i64, _p]),
    "q3t_code_ring_write": (_i32, [_p, _i64, _p, _p, _i64, _i64, _i64, _p]),
    "q3t_code_ring_read": (_i32, [_p, _i64, _i64, _i64, _p, _p, _i64, _i64, _p, _p, _p]),
    "q3t_linear_chain_workspace_bytes": (_sz, [_i64]),
    "q3t_linear_chain": (_i32, [_p, _i32, _i64, _p, _sz, _p, _p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class KernelError(RuntimeError):
    """A CUDA-side failure reported by the library."""


def load() -> ctypes.CDLL:
    """Load the kernel library once; raise if it is missing (no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY_PATH.exists():
                raise ImportError(
                    f"{LIBRARY_PATH.name} is not built; run __graft_entry__.build() "
                    "(nvcc, sm_100a) before using the CUDA path")
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().q3t_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Translate a C status into the reference's error behaviour."""
    if rc == Q3T_OK:
        return
    message = last_error() or what
    if rc in (Q3T_EINVAL, Q3T_EUNSUPPORTED, Q3T_ESPACE):
        raise ValueError(message)
    raise KernelError(f"{what}: {message}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def launch_count() -> int:
    return int(load().q3t_launch_count())


def i64_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (ctypes.c_int64 * len(values))(*values)
