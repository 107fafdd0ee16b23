"""Tensor-level wrappers over the C ABI: validate, allocate outputs, launch.

Every function enqueues on the current CUDA stream and never synchronises, so
all of them can be recorded into CUDA graphs (after one warm-up call has sized
any scratch). Invalid arguments raise ``ValueError`` before anything is
written, as the reference wrappers do.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib
from ._lib import call, i64_array

BF16 = torch.bfloat16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and (not isinstance(t, torch.Tensor) or t.device.type != "cuda"):
            raise ValueError("Expected CUDA tensors")


def _capturing() -> bool:
    return torch.cuda.is_current_stream_capturing()


# ------------------------------------------------------------------ scratch and status
class Scratch:
    """Per-device, per-tag zero-filled workspaces and status words.

    Kernels leave their scratch ready for the next call (tickets reset to
    zero), so a workspace is zeroed only when it is (re)allocated. Growth is
    refused while a CUDA graph is being captured: warm up first.
    """

    def __init__(self) -> None:
        self._buffers: dict[tuple, torch.Tensor] = {}
        self._status: dict[int, torch.Tensor] = {}

    def workspace(self, nbytes: int, device: torch.device, tag: str = "default") -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), tag)
        buf = self._buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            if _capturing():
                raise RuntimeError(f"workspace '{tag}' must be sized by a warm-up call before graph capture")
            size = max(nbytes, 1 << 20)
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            self._buffers[key] = buf
        return buf

    def status(self, device: torch.device) -> torch.Tensor:
        index = device.index if device.index is not None else torch.cuda.current_device()
        word = self._status.get(index)
        if word is None:
            if _capturing():
                raise RuntimeError("status word must exist before graph capture")
            word = torch.zeros(4, dtype=torch.int32, device=device)
            self._status[index] = word
        return word


SCRATCH = Scratch()


def status_word(device: torch.device) -> torch.Tensor:
    return SCRATCH.status(device)


def read_status(device: torch.device, clear: bool = True) -> int:
    """Synchronise and return the error bits kernels raised on `device`."""
    word = SCRATCH.status(device)
    value = int(word[0].item())
    if clear and value:
        word.zero_()
    return value


# ------------------------------------------------------------------ KV arena
def kv_write(keys, values, target_keys, target_values, positions) -> None:
    """target[b, h, positions[b]] = source[b, h, 0] for K and V (kv_triton_ascend.py:39)."""
    _need_cuda(keys, values, target_keys, target_values, positions)
    if keys.ndim != 4 or keys.shape[2] != 1 or values.shape != keys.shape:
        raise ValueError("Expected matching single-token BNSD K/V")
    batch, heads, _, width = keys.shape
    if (target_keys.shape != target_values.shape or tuple(target_keys.shape[:2]) != (batch, heads)
            or target_keys.shape[-1] != width or not target_keys.is_contiguous()
            or not target_values.is_contiguous() or tuple(positions.shape) != (batch,)
            or not positions.is_contiguous() or positions.dtype != torch.int64):
        raise ValueError("Invalid contiguous KV arena or position vector")
    if any(t.dtype != keys.dtype for t in (values, target_keys, target_values)):
        raise ValueError("KV tensors must share dtype and device")
    if keys.dtype not in (BF16, torch.float32):
        raise ValueError("KV write supports BF16 and FP32 tensors")
    dtype = _lib.Q3T_BF16 if keys.dtype == BF16 else _lib.Q3T_F32
    ks = i64_array((keys.stride(0), keys.stride(1), keys.stride(3)))
    vs = i64_array((values.stride(0), values.stride(1), values.stride(3)))
    call("q3t_kv_write", keys.data_ptr(), ks, values.data_ptr(), vs, target_keys.data_ptr(),
         target_values.data_ptr(), positions.data_ptr(), batch, heads, width, target_keys.shape[2], dtype,
         status_word(keys.device).data_ptr(), _stream())


def copy_packed_prefix(target, source, slot, row=0, length=None) -> None:
    """target[:, slot, :, :length] = source[:, row, :, :length] (packed_kv.py:6)."""
    if (not isinstance(target, torch.Tensor) or not isinstance(source, torch.Tensor) or target.ndim != 5
            or source.ndim != 5 or any(s <= 0 for s in tuple(target.shape) + tuple(source.shape))
            or (target.shape[0], target.shape[2], target.shape[4]) != (source.shape[0], source.shape[2], source.shape[4])
            or target.device != source.device or target.dtype != source.dtype
            or target.untyped_storage().data_ptr() == source.untyped_storage().data_ptr()):
        raise ValueError("Expected independent compatible packed KV tensors")
    length = source.shape[3] if length is None else length
    if (type(slot) is not int or not 0 <= slot < target.shape[1] or type(row) is not int
            or not 0 <= row < source.shape[1] or type(length) is not int
            or not 0 < length <= min(target.shape[3], source.shape[3])):
        raise ValueError("Expected a valid packed KV row and prefix length")
    _need_cuda(target, source)
    call("q3t_copy_packed_prefix", target.data_ptr(), i64_array(target.shape), i64_array(target.stride()),
         source.data_ptr(), i64_array(source.shape), i64_array(source.stride()), target.element_size(), slot, row,
         length, _stream())


def _slot_geometry(tensor: torch.Tensor, dim: int):
    if not tensor.is_contiguous():
        raise ValueError("Slot buffers must be contiguous")
    planes = math.prod(tensor.shape[:dim]) if dim > 0 else 1
    plane_stride = tensor.stride(dim - 1) if dim > 0 else 0
    return planes, plane_stride, tensor.stride(dim), math.prod(tensor.shape[dim + 1:])


def slot_move(tensor: torch.Tensor, source: int, destination: int, dim: int = 0) -> None:
    """tensor[..., destination, ...] = tensor[..., source, ...] along `dim` (SlotArena.move)."""
    _need_cuda(tensor)
    if not (0 <= source < tensor.shape[dim] and 0 <= destination < tensor.shape[dim]):
        raise ValueError("Slot index out of range")
    planes, pstride, sstride, elems = _slot_geometry(tensor, dim)
    call("q3t_slot_move", tensor.data_ptr(), planes, pstride, sstride, elems, tensor.element_size(), source,
         destination, _stream())


def slot_zero(tensor: torch.Tensor, start: int, count: int = 1, dim: int = 0) -> None:
    """Zero `count` slots from `start` along `dim` (CodecSlots.reset_range)."""
    _need_cuda(tensor)
    if type(start) is not int or type(count) is not int or start < 0 or count < 0 or start + count > tensor.shape[dim]:
        raise ValueError("Expected a valid contiguous slot range")
    planes, pstride, sstride, elems = _slot_geometry(tensor, dim)
    call("q3t_slot_zero", tensor.data_ptr(), planes, pstride, sstride, elems, tensor.element_size(), start, count,
         _stream())


def advance(values: torch.Tensor, delta: int = 1) -> None:
    """values += delta for device-resident int64 counters (positions, frames)."""
    _need_cuda(values)
    if values.dtype != torch.int64 or not values.is_contiguous():
        raise ValueError("advance expects a contiguous int64 tensor")
    call("q3t_advance", values.data_ptr(), values.numel(), int(delta), _stream())


def copy_prefix_along(target: torch.Tensor, source: torch.Tensor, dim: int) -> None:
    """target[..., :n, ...] = source along `dim` (capacity doubling, continuous.py:362-363)."""
    _need_cuda(target, source)
    if not target.is_contiguous() or not source.is_contiguous() or target.dtype != source.dtype:
        raise ValueError("Expected contiguous tensors of one dtype")
    rows = math.prod(source.shape[:dim]) if dim > 0 else 1
    row_bytes = source.stride(dim - 1) * source.element_size() if dim > 0 else source.numel() * source.element_size()
    dst_pitch = target.stride(dim - 1) * target.element_size() if dim > 0 else row_bytes
    call("q3t_copy_rows", target.data_ptr(), dst_pitch, source.data_ptr(), row_bytes, row_bytes, rows, _stream())


# ------------------------------------------------------------------ norms, rotary, activations
def rms_norm(x, weight, eps: float, mode: int = _lib.NORM_REFERENCE, out=None):
    _need_cuda(x, weight)
    if x.dtype != BF16 or weight.dtype != BF16 or x.stride(-1) != 1:
        raise ValueError("RMSNorm expects BF16 rows with unit inner stride")
    width = x.shape[-1]
    rows = x.numel() // width
    x2 = x.reshape(rows, width) if x.is_contiguous() else x
    out = torch.empty(x.shape, dtype=BF16, device=x.device) if out is None else out
    call("q3t_rms_norm", x2.data_ptr(), x2.stride(0) if x2.ndim == 2 else width, weight.data_ptr(), out.data_ptr(),
         rows, width, float(eps), mode, _stream())
    return out


def add_rms_norm(a, h, weight, eps: float, mode: int = _lib.NORM_REFERENCE):
    """(normalized, residual) with residual = a + h (npu_add_rms_norm contract)."""
    _need_cuda(a, h, weight)
    if a.shape != h.shape or a.dtype != BF16 or h.dtype != BF16 or not a.is_contiguous() or not h.is_contiguous():
        raise ValueError("add_rms_norm expects matching contiguous BF16 tensors")
    width = a.shape[-1]
    rows = a.numel() // width
    normalized = torch.empty_like(a)
    residual = torch.empty_like(a)
    call("q3t_add_rms_norm", a.data_ptr(), h.data_ptr(), weight.data_ptr(), normalized.data_ptr(),
         residual.data_ptr(), rows, width, float(eps), mode, _stream())
    return normalized, residual


def rotary(hidden, cos, sin):
    """BSND rotary with bf16 rounding after each multiply and add (rotary_triton_ascend.py:29)."""
    if not isinstance(hidden, torch.Tensor) or hidden.ndim != 4 or hidden.device.type != "cuda" or hidden.dtype != BF16:
        raise ValueError("Expected BF16 BSND CUDA input")
    batch, length, heads, width = hidden.shape
    if heads not in (8, 16) or width not in (64, 128) or batch * length < 1:
        raise ValueError("Unsupported rotary shape")
    if tuple(cos.shape) != (batch, length, width) or sin.shape != cos.shape:
        raise ValueError("Rotary coefficients must match batch, length and width")
    if any(t.device != hidden.device or t.dtype != hidden.dtype or not t.is_contiguous() for t in (hidden, cos, sin)):
        raise ValueError("Rotary tensors must be contiguous with matching dtype/device")
    out = torch.empty_like(hidden)
    call("q3t_rotary", hidden.data_ptr(), cos.data_ptr(), sin.data_ptr(), out.data_ptr(), batch, length, heads, width,
         _stream())
    return out


def swiglu(packed):
    """silu(gate) * up over packed [.., 2*w] (npu_swiglu at packed_mlp.py:23)."""
    _need_cuda(packed)
    if packed.dtype != BF16 or not packed.is_contiguous() or packed.shape[-1] % 2:
        raise ValueError("swiglu expects contiguous BF16 [..., 2*width]")
    width = packed.shape[-1] // 2
    out = torch.empty(*packed.shape[:-1], width, dtype=BF16, device=packed.device)
    call("q3t_swiglu", packed.data_ptr(), out.data_ptr(), packed.numel() // packed.shape[-1], width, _stream())
    return out


def snake(hidden, alpha, inverse_beta):
    """SnakeBeta x + inv_beta * sin(x * alpha)^2 on NCT (snake_triton_ascend.py:28)."""
    if (not isinstance(hidden, torch.Tensor) or hidden.device.type != "cuda" or hidden.ndim != 3
            or not hidden.is_contiguous() or hidden.dtype not in (BF16, torch.float32)):
        raise ValueError("Snake kernel requires contiguous NCT BF16/FP32 CUDA input")
    if alpha.numel() != hidden.shape[1] or inverse_beta.numel() != hidden.shape[1]:
        raise ValueError("Snake coefficients must match the channel count")
    if hidden.numel() == 0:
        raise ValueError("Snake input must be nonempty")
    alpha = alpha.reshape(-1).contiguous()
    inverse_beta = inverse_beta.reshape(-1).contiguous()
    if alpha.dtype != inverse_beta.dtype:
        inverse_beta = inverse_beta.to(alpha.dtype)
    dtype = _lib.Q3T_BF16 if hidden.dtype == BF16 else _lib.Q3T_F32
    cdt = _lib.Q3T_BF16 if alpha.dtype == BF16 else _lib.Q3T_F32
    if cdt == _lib.Q3T_F32 and alpha.dtype != torch.float32:
        raise ValueError("Snake coefficients must be BF16 or FP32")
    out = torch.empty_like(hidden)
    call("q3t_snake", hidden.data_ptr(), alpha.data_ptr(), inverse_beta.data_ptr(), out.data_ptr(), hidden.shape[0],
         hidden.shape[1], hidden.shape[2], dtype, cdt, _stream())
    return out


# ------------------------------------------------------------------ dense projections
def linear_workspace_bytes(rows: int, in_features: int, out_features: int) -> int:
    return int(_lib.load().q3t_linear_workspace_bytes(rows, in_features, out_features))


class TiledWeight:
    """A [out, in] weight in the pre-swizzled tile layout of q3t_pack_weight_tiles."""

    def __init__(self, tiles: torch.Tensor, out_features: int, in_features: int):
        self.tiles, self.out_features, self.in_features = tiles, out_features, in_features
        self.shape = (out_features, in_features)
        self.dtype = BF16
        self.device = tiles.device

    def numel(self) -> int:
        return self.out_features * self.in_features


def pack_tiles(weight: torch.Tensor) -> TiledWeight:
    """Re-layout a contiguous bf16 [out, in] weight as contiguous swizzled 16 KB tiles."""
    _need_cuda(weight)
    if weight.dtype != BF16 or weight.ndim != 2 or not weight.is_contiguous():
        raise ValueError("pack_tiles expects a contiguous BF16 [out, in] weight")
    n, k = weight.shape
    nbytes = int(_lib.load().q3t_weight_tiles_bytes(n, k))
    tiles = torch.empty(nbytes, dtype=torch.uint8, device=weight.device)
    call("q3t_pack_weight_tiles", weight.data_ptr(), n, k, tiles.data_ptr(), _stream())
    return TiledWeight(tiles, n, k)


def linear(x, weight, bias=None, *, out=None, out_dtype=BF16, epilogue: int = _lib.EPI_STORE, residual=None,
           scale=None, row_norm_eps: Optional[float] = None, workspace: Optional[torch.Tensor] = None,
           prefetch=None, keep_weights: bool = False, narrow: bool = False, tag: str = "linear"):
    """out = x @ weight.T (+ bias) with a fused epilogue, on tcgen05 tensor cores.

    `weight` is a contiguous bf16 [out, in] tensor or a TiledWeight. With
    `row_norm_eps`, row r of the product is scaled by rsqrt(mean(x[r]^2) + eps):
    an RMSNorm of x folded into the GEMM (the norm weight must already be
    multiplied into `weight`, see weights.fold_norm). `prefetch` (a weight
    tensor or TiledWeight, normally the next GEMM's) is pulled into L2 while
    this GEMM runs; `keep_weights` loads the weight tiles evict-last so that a
    chain that re-reads them finds them in L2 (q3t_linear_ex). Row counts in the thousands run
    the persistent wide-tile kernel unless `narrow` keeps the split-K kernel."""
    tiled = isinstance(weight, TiledWeight)
    _need_cuda(x, weight.tiles if tiled else weight)
    if x.dtype != BF16 or (not tiled and (weight.dtype != BF16 or weight.ndim != 2 or not weight.is_contiguous())):
        raise ValueError("linear expects BF16 activations and a contiguous BF16 [out, in] weight")
    n_rows_w, in_features = weight.shape
    if x.shape[-1] != in_features or x.stride(-1) != 1:
        raise ValueError("linear: activation width must match the weight")
    rows = x.numel() // in_features if x.is_contiguous() else x.shape[0]
    x2 = x.reshape(rows, in_features) if x.is_contiguous() else x
    if x2.ndim != 2:
        raise ValueError("linear: non-contiguous activations must be 2-D")
    n_out = n_rows_w // 2 if epilogue == _lib.EPI_SWIGLU_PAIRED else n_rows_w
    if out is None:
        out = torch.empty(*x.shape[:-1], n_out, dtype=out_dtype, device=x.device)
    out2 = out.reshape(rows, n_out) if out.is_contiguous() else out
    res2 = None
    if residual is not None:
        res2 = residual.reshape(rows, n_out) if residual.is_contiguous() else residual
    odt = _lib.Q3T_BF16 if out.dtype == BF16 else _lib.Q3T_F32
    if prefetch is not None or keep_weights or narrow:
        pre = prefetch.tiles if isinstance(prefetch, TiledWeight) else prefetch
        if pre is not None:
            _need_cuda(pre)
        call("q3t_linear_ex", x2.data_ptr(), x2.stride(0), rows, in_features,
             None if tiled else weight.data_ptr(), n_rows_w, _ptr(bias), out2.data_ptr(), out2.stride(0), odt,
             epilogue, _ptr(res2), res2.stride(0) if res2 is not None else 0, _ptr(scale),
             float(row_norm_eps) if row_norm_eps is not None else 0.0, weight.tiles.data_ptr() if tiled else None,
             _ptr(pre), (pre.numel() * pre.element_size()) // 16 * 16 if pre is not None else 0,
             (_lib.LINEAR_KEEP_WEIGHTS if keep_weights else 0) | (_lib.LINEAR_NARROW if narrow else 0),
             status_word(x.device).data_ptr(), _stream())
        return out
    if row_norm_eps is not None:
        call("q3t_linear_rownorm", x2.data_ptr(), x2.stride(0), rows, in_features,
             None if tiled else weight.data_ptr(), n_rows_w, _ptr(bias), out2.data_ptr(), out2.stride(0), odt,
             epilogue, _ptr(res2), res2.stride(0) if res2 is not None else 0, _ptr(scale), float(row_norm_eps),
             weight.tiles.data_ptr() if tiled else None, status_word(x.device).data_ptr(), _stream())
        return out
    call("q3t_linear", x2.data_ptr(), x2.stride(0), rows, in_features, None if tiled else weight.data_ptr(), n_rows_w,
         _ptr(bias), out2.data_ptr(), out2.stride(0), odt, epilogue, _ptr(res2),
         res2.stride(0) if res2 is not None else 0, _ptr(scale), weight.tiles.data_ptr() if tiled else None,
         _ptr(workspace), workspace.numel() if workspace is not None else 0, status_word(x.device).data_ptr(),
         _stream())
    return out


def linear_chain_workspace(rows: int, device) -> torch.Tensor:
    """Zeroed workspace of q3t_linear_chain for `rows` activation rows (one per stream of chains)."""
    nbytes = int(_lib.load().q3t_linear_chain_workspace_bytes(rows))
    if nbytes == 0:
        raise ValueError("linear_chain: rows must be within 1..64")
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def linear_chain(stages, workspace: torch.Tensor) -> None:
    """A chain of dependent projections in one persistent launch (q3t_linear_chain).

    Each stage is a dict: x (bf16 [rows, in], unit inner stride), weight (TiledWeight), out
    (bf16 or fp32 [rows, out or out/2 for SwiGLU]), and optionally epilogue (EPI_STORE,
    EPI_RESIDUAL, EPI_SWIGLU_PAIRED), residual, bias, row_norm_eps (folded RMSNorm), depends
    (the earlier stage whose output this stage reads; default: the previous stage, -1 for
    the first). Stage s computes what ops.linear(x, weight, ...) would, with every SM
    streaming weights across the whole chain."""
    if not 1 <= len(stages) <= _lib.CHAIN_MAX_STAGES:
        raise ValueError(f"linear_chain: 1..{_lib.CHAIN_MAX_STAGES} stages")
    rows = None
    table = (_lib.ChainStage * len(stages))()
    for i, st in enumerate(stages):
        x, w, out = st["x"], st["weight"], st["out"]
        if not isinstance(w, TiledWeight):
            raise ValueError("linear_chain: weights must be TiledWeight (ops.pack_tiles)")
        _need_cuda(x, w.tiles, out)
        if x.dtype != BF16 or x.ndim != 2 or x.stride(1) != 1 or x.shape[1] != w.in_features:
            raise ValueError("linear_chain: x must be BF16 [rows, in_features] with unit inner stride")
        if rows is None:
            rows = x.shape[0]
        epi = st.get("epilogue", _lib.EPI_STORE)
        n_out = w.out_features // 2 if epi == _lib.EPI_SWIGLU_PAIRED else w.out_features
        if x.shape[0] != rows or out.ndim != 2 or out.shape != (rows, n_out) or out.stride(1) != 1:
            raise ValueError("linear_chain: every stage has the same rows; out must be [rows, out_features]")
        res, bias = st.get("residual"), st.get("bias")
        if res is not None and (res.shape != out.shape or res.stride(1) != 1 or res.dtype != BF16):
            raise ValueError("linear_chain: residual must be BF16 shaped like out")
        eps = st.get("row_norm_eps")
        e = table[i]
        e.x, e.x_stride, e.weight_tiles = x.data_ptr(), x.stride(0), w.tiles.data_ptr()
        e.in_features, e.out_features = w.in_features, w.out_features
        e.out, e.out_stride = out.data_ptr(), out.stride(0)
        e.out_dtype = _lib.Q3T_BF16 if out.dtype == BF16 else _lib.Q3T_F32
        e.epilogue = epi
        e.residual, e.residual_stride = _ptr(res), res.stride(0) if res is not None else 0
        e.bias = _ptr(bias)
        e.row_norm_eps = float(eps) if eps is not None else 0.0
        e.depends = int(st.get("depends", i - 1))
    call("q3t_linear_chain", ctypes.cast(table, ctypes.c_void_p), len(stages), rows, workspace.data_ptr(),
         workspace.numel(), status_word(workspace.device).data_ptr(), _stream())


# ------------------------------------------------------------------ attention
def qk_norm_rope_kv(qkv, q_norm_weight, k_norm_weight, eps, cos_table, sin_table, rotary_positions, cache_positions,
                    target_keys, target_values, *, q_heads, kv_heads, head_dim, length=1, query_out=None, slots=None):
    """Per-head q/k RMSNorm, rotary and KV write for packed QKV rows (packed_attention.py:42-74)."""
    _need_cuda(qkv, cos_table, sin_table, rotary_positions, cache_positions, target_keys, target_values)
    rows = qkv.shape[0]
    if qkv.ndim != 2 or qkv.stride(1) != 1 or qkv.dtype != BF16:
        raise ValueError("qkv must be BF16 [rows, (q+2kv)*head_dim] with unit inner stride")
    if query_out is None:
        query_out = torch.empty(rows, q_heads, head_dim, dtype=BF16, device=qkv.device)
    call("q3t_qk_norm_rope_kv", qkv.data_ptr(), qkv.stride(0), _ptr(q_norm_weight), _ptr(k_norm_weight), float(eps),
         cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], rotary_positions.data_ptr(),
         cache_positions.data_ptr(), query_out.data_ptr(), target_keys.data_ptr(), target_values.data_ptr(), rows,
         length, _ptr(slots), q_heads, kv_heads, head_dim, target_keys.shape[2], status_word(qkv.device).data_ptr(),
         _stream())
    return query_out


def decode_attention_workspace_bytes(batch, q_heads, head_dim, context) -> int:
    return int(_lib.load().q3t_decode_attention_workspace_bytes(batch, q_heads, head_dim, context))


def decode_attention(query, keys, values, positions, *, context=None, scale=None, out=None, rows_per_slot=1,
                     window=0, slots=None, ring=0, workspace: Optional[torch.Tensor] = None, tag: str = "attention"):
    """GQA attention of query row r over keys [max(0, p-window+1), p] of slot r // rows_per_slot
    (or slots[r // rows_per_slot]), p = positions[r]; ring > 0 stores position p in row p % ring."""
    _need_cuda(query, keys, values, positions)
    rows, q_heads, head_dim = query.shape
    n_slots, kv_heads, capacity, width = keys.shape
    if (width != head_dim or values.shape != keys.shape or (slots is None and n_slots * rows_per_slot < rows)
            or not keys.is_contiguous()
            or not values.is_contiguous() or not query.is_contiguous() or query.dtype != BF16
            or keys.dtype != BF16 or values.dtype != BF16 or positions.dtype != torch.int64):
        raise ValueError("Expected BF16 query [rows,Hq,D] and contiguous BF16 KV arena [slots,Hkv,cap,D]")
    context = capacity if context is None else context
    scale = head_dim ** -0.5 if scale is None else scale
    out = torch.empty_like(query) if out is None else out
    need = decode_attention_workspace_bytes(rows, q_heads, head_dim, context)
    ws = workspace if workspace is not None else SCRATCH.workspace(need, query.device, tag)
    call("q3t_decode_attention", query.data_ptr(), keys.data_ptr(), values.data_ptr(), positions.data_ptr(),
         out.data_ptr(), rows, rows_per_slot, _ptr(slots), int(ring), q_heads, kv_heads, head_dim, n_slots, capacity,
         context, window, float(scale), ws.data_ptr(), ws.numel(), status_word(query.device).data_ptr(), _stream())
    return out


def prefill_attention(query, keys, values, positions, units, *, out, scale=None):
    """Causal attention of packed prompt rows over their own slot's keys (q3t_prefill_attention):
    `units` int32 [n, 4] = {first_row, count, keys, slot} from batching.packed_units; rows no
    unit covers are left as they are in `out`."""
    _need_cuda(query, keys, values, positions, units, out)
    rows, q_heads, head_dim = query.shape
    n_slots, kv_heads, capacity, width = keys.shape
    if (width != head_dim or values.shape != keys.shape or not keys.is_contiguous() or not values.is_contiguous()
            or not query.is_contiguous() or not out.is_contiguous() or out.shape != query.shape
            or query.dtype != BF16 or keys.dtype != BF16 or values.dtype != BF16 or out.dtype != BF16
            or positions.dtype != torch.int64 or units.dtype != torch.int32 or units.ndim != 2
            or units.shape[1] != 4 or not units.is_contiguous()):
        raise ValueError("Expected BF16 query/out [rows,Hq,D], a contiguous BF16 KV arena and int32 units [n, 4]")
    scale = head_dim ** -0.5 if scale is None else scale
    call("q3t_prefill_attention", query.data_ptr(), keys.data_ptr(), values.data_ptr(), positions.data_ptr(),
         units.data_ptr(), units.shape[0], out.data_ptr(), rows, q_heads, kv_heads, head_dim, n_slots, capacity,
         float(scale), status_word(query.device).data_ptr(), _stream())
    return out


def attention_plan(positions, workspace, *, q_heads, kv_heads, head_dim, context):
    """Per-step split-KV chunk plan (q3t_attention_plan) for the decode attention calls that use
    `workspace`: one wave of resident CTAs over this batch's contexts."""
    _need_cuda(positions, workspace)
    if positions.dtype != torch.int64 or positions.ndim != 1:
        raise ValueError("positions must be int64 [rows]")
    call("q3t_attention_plan", positions.data_ptr(), positions.shape[0], q_heads, kv_heads, head_dim, context,
         workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream())


def _prefetch_range(weight):
    """(pointer, bytes) of a weight tensor or TiledWeight for an L2 prefetch hint, or (None, 0)."""
    if weight is None:
        return None, 0
    t = weight.tiles if isinstance(weight, TiledWeight) else weight
    _need_cuda(t)
    return t.data_ptr(), (t.numel() * t.element_size()) // 16 * 16


def decode_attention_qkv(qkv, q_norm_weight, k_norm_weight, eps, cos_table, sin_table, rotary_positions, keys,
                         values, positions, *, q_heads, kv_heads, head_dim, context=None, scale=None, out=None,
                         workspace: Optional[torch.Tensor] = None, prefetch=(), tag: str = "attention"):
    """Decode attention straight from the QKV projection rows: per-head q/k RMSNorm, RoPE and the
    K/V write of each row's position fused into the attention kernel (one query row per slot).
    `prefetch`: up to two weights (tensors or TiledWeights, normally the projections that follow)
    that the kernel pulls into L2 while the keys stream (q3t_decode_attention_qkv_ex)."""
    _need_cuda(qkv, cos_table, sin_table, rotary_positions, keys, values, positions)
    prefetch = [w for w in prefetch if w is not None]
    if len(prefetch) > 2:
        raise ValueError("decode_attention_qkv: at most two prefetch ranges")
    rows = qkv.shape[0]
    n_slots, kvh, capacity, width = keys.shape
    if (qkv.ndim != 2 or qkv.stride(1) != 1 or qkv.dtype != BF16 or width != head_dim or kvh != kv_heads
            or values.shape != keys.shape or not keys.is_contiguous() or not values.is_contiguous()
            or keys.dtype != BF16 or positions.dtype != torch.int64 or rotary_positions.dtype != torch.int64):
        raise ValueError("Expected BF16 QKV rows and a contiguous BF16 KV arena [slots, Hkv, cap, D]")
    context = capacity if context is None else context
    scale = head_dim ** -0.5 if scale is None else scale
    out = torch.empty(rows, q_heads, head_dim, dtype=BF16, device=qkv.device) if out is None else out
    need = decode_attention_workspace_bytes(rows, q_heads, head_dim, context)
    ws = workspace if workspace is not None else SCRATCH.workspace(need, qkv.device, tag)
    if prefetch:
        (p0, n0), (p1, n1) = (list(map(_prefetch_range, prefetch)) + [(None, 0)])[:2]
        call("q3t_decode_attention_qkv_ex", qkv.data_ptr(), qkv.stride(0), _ptr(q_norm_weight), _ptr(k_norm_weight),
             float(eps), cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], rotary_positions.data_ptr(),
             keys.data_ptr(), values.data_ptr(), positions.data_ptr(), out.data_ptr(), rows, q_heads, kv_heads,
             head_dim, n_slots, capacity, context, float(scale), ws.data_ptr(), ws.numel(), p0, n0, p1, n1,
             status_word(qkv.device).data_ptr(), _stream())
        return out
    call("q3t_decode_attention_qkv", qkv.data_ptr(), qkv.stride(0), _ptr(q_norm_weight), _ptr(k_norm_weight),
         float(eps), cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], rotary_positions.data_ptr(),
         keys.data_ptr(), values.data_ptr(), positions.data_ptr(), out.data_ptr(), rows, q_heads, kv_heads, head_dim,
         n_slots, capacity, context, float(scale), ws.data_ptr(), ws.numel(), status_word(qkv.device).data_ptr(),
         _stream())
    return out


# ------------------------------------------------------------------ sampling
def cdf_select(cdf, uniforms):
    """token = #{cdf / cdf[-1] <= u} per row (cdf_triton_ascend.py:20)."""
    if (not isinstance(cdf, torch.Tensor) or cdf.device.type != "cuda" or cdf.dtype != torch.float32
            or cdf.ndim != 2 or not cdf.is_contiguous() or not 1 <= cdf.shape[1] <= 4096):
        raise ValueError("CDF must be contiguous FP32 CUDA rows of width 1..4096")
    if (uniforms.device != cdf.device or uniforms.dtype != torch.float32
            or tuple(uniforms.shape) != (cdf.shape[0],) or not uniforms.is_contiguous()):
        raise ValueError("Uniforms must be one contiguous FP32 value per CDF row")
    if cdf.shape[0] < 1:
        raise ValueError("Empty CDF batch")
    out = torch.empty((cdf.shape[0], 1), device=cdf.device, dtype=torch.long)
    call("q3t_cdf_select", cdf.data_ptr(), uniforms.data_ptr(), out.data_ptr(), cdf.shape[0], cdf.shape[1], _stream())
    return out


def sample(logits, *, uniforms=None, seed: int = 0, philox_offsets=None, philox_add: int = 0, temperature=0.9,
           top_k=50, top_p=1.0, seen=None, allowed=None, steps=None, eos=0, min_steps=2, penalty=1.05,
           seen_out=None, tokens=None):
    """Fused categorical sampling (sampling.py:5 + continuous.py:365-370 + sampling_graph.py:14-16)."""
    _need_cuda(logits)
    if logits.ndim != 2 or logits.stride(1) != 1 or logits.dtype not in (BF16, torch.float32):
        raise ValueError("logits must be [rows, vocab] BF16/FP32 with unit inner stride")
    rows, width = logits.shape
    if uniforms is None and philox_offsets is None:
        raise ValueError("Provide uniforms or Philox offsets")
    if uniforms is not None:
        if uniforms.dtype != torch.float32 or uniforms.shape[0] != rows or uniforms.device != logits.device \
                or uniforms.ndim != 1:
            raise ValueError("Uniforms must be one FP32 value per row")
    if philox_offsets is not None and (philox_offsets.dtype != torch.int64 or philox_offsets.shape[0] != rows):
        raise ValueError("Philox offsets must be one int64 per row")
    for t in (seen, allowed, seen_out):
        if t is not None and t.dtype != torch.bool:
            raise ValueError("seen/allowed masks must be bool")
    if tokens is None:
        tokens = torch.empty((rows, 1), dtype=torch.long, device=logits.device)
    call("q3t_sample", logits.data_ptr(), _lib.Q3T_BF16 if logits.dtype == BF16 else _lib.Q3T_F32, logits.stride(0),
         _ptr(seen), seen.stride(0) if seen is not None else 0, _ptr(allowed), _ptr(steps), int(eos), int(min_steps),
         float(penalty), float(temperature), int(top_k), float(top_p), _ptr(uniforms),
         uniforms.stride(0) if uniforms is not None else 0, int(seed) & ((1 << 64) - 1), _ptr(philox_offsets),
         int(philox_add), tokens.data_ptr(), tokens.stride(0), _ptr(seen_out), seen_out.stride(0) if seen_out is not None else 0, rows,
         width, _stream())
    return tokens


def philox_uniforms(seed: int, offset: int, count: int, device) -> torch.Tensor:
    out = torch.empty(count, dtype=torch.float32, device=device)
    call("q3t_philox_uniforms", int(seed) & ((1 << 64) - 1), int(offset), out.data_ptr(), count, _stream())
    return out


# ------------------------------------------------------------------ embeddings and codec state
def frame_embed(codes, first_table, group_tables, text=None, out=None):
    """E_first[codes[:,0]] + sum_g E_g[codes[:,g+1]] (one rounding) + text (continuous.py:584-601)."""
    _need_cuda(codes, first_table, group_tables)
    batch, hidden = codes.shape[0], first_table.shape[1]
    out = torch.empty(batch, hidden, dtype=BF16, device=codes.device) if out is None else out
    call("q3t_frame_embed", codes.data_ptr(), codes.stride(0), first_table.data_ptr(), first_table.shape[0],
         group_tables.data_ptr(), group_tables.shape[0], group_tables.shape[1], _ptr(text),
         text.stride(0) if text is not None else 0, out.data_ptr(), batch, hidden,
         status_word(codes.device).data_ptr(), _stream())
    return out


def embedding(ids, table, out=None):
    _need_cuda(ids, table)
    rows = ids.shape[0]
    out = torch.empty(rows, table.shape[1], dtype=table.dtype, device=ids.device) if out is None else out
    call("q3t_embedding", ids.data_ptr(), ids.stride(0) if ids.ndim else 1, table.data_ptr(), table.shape[0],
         out.data_ptr(), out.stride(0), rows, table.shape[1], status_word(ids.device).data_ptr(), _stream())
    return out


def scatter_rows(target, indices, source) -> None:
    """target[indices[i]] = source[i] (codec_row_scatter.py:48); caller guarantees unique indices."""
    if (not isinstance(target, torch.Tensor) or target.device.type != "cuda" or source.device != target.device
            or indices.device != target.device or indices.dtype != torch.long or indices.ndim != 1
            or not indices.is_contiguous() or not target.is_contiguous() or not 1 <= target.ndim <= 4
            or source.ndim != target.ndim or source.dtype != target.dtype
            or tuple(source.shape[1:]) != tuple(target.shape[1:]) or source.shape[0] != indices.numel()
            or source.numel() == 0
            or source.untyped_storage().data_ptr() == target.untyped_storage().data_ptr()):
        raise ValueError("Expected independent source and contiguous selected-row target")
    call("q3t_scatter_rows", target.data_ptr(), target.shape[0], indices.data_ptr(), source.data_ptr(), source.ndim,
         i64_array(source.shape), i64_array(source.stride()), source.element_size(),
         status_word(target.device).data_ptr(), _stream())


# ------------------------------------------------------------------ incremental codec
def rvq_gather(codes, tables, semantic: int, out=None):
    """[sum of semantic codebook rows | sum of the rest] per (stream, frame) (cached_quantizer.py:17-30).

    codes int64 [B, n_q, T]; tables bf16 [n_q, bins, dim] (normalised codebooks) -> [B*T, 2*dim]."""
    _need_cuda(codes, tables)
    B, n_q, T = codes.shape
    dim = tables.shape[2]
    out = torch.empty(B * T, 2 * dim, dtype=BF16, device=codes.device) if out is None else out
    call("q3t_rvq_gather", codes.data_ptr(), codes.stride(0), codes.stride(1), codes.stride(2), tables.data_ptr(),
         n_q, semantic, tables.shape[1], dim, B, T, out.data_ptr(), status_word(codes.device).data_ptr(), _stream())
    return out


def conv_gather(x, batch: int, frames: int, *, taps: int, dilation: int = 1, reverse: bool = False, history=None,
                slots=None, alpha=None, inverse_beta=None, out=None):
    """im2col rows of a causal conv over time-major x [batch*frames, C] with per-slot history."""
    _need_cuda(x)
    C = x.shape[-1]
    H = history.shape[1] if history is not None else 0
    out = torch.empty(batch * frames, taps * C, dtype=BF16, device=x.device) if out is None else out
    call("q3t_conv_gather", x.data_ptr(), x.stride(0), batch, frames, C, _ptr(history), H, _ptr(slots), taps,
         dilation, int(reverse), _ptr(alpha), _ptr(inverse_beta), out.data_ptr(), _stream())
    return out


def conv_pad(x, batch: int, frames: int, *, history=None, slots=None, alpha=None, inverse_beta=None, out=None):
    """Padded input of an implicit causal conv: snake([history[slot] | x[b]]) as [batch*(H+frames), C]."""
    _need_cuda(x)
    C = x.shape[-1]
    H = history.shape[1] if history is not None else 0
    out = torch.empty(batch * (H + frames), C, dtype=BF16, device=x.device) if out is None else out
    if out.shape != (batch * (H + frames), C) or not out.is_contiguous():
        raise ValueError("conv_pad: out must be a contiguous [batch*(history+frames), channels] buffer")
    call("q3t_conv_pad", x.data_ptr(), x.stride(0), batch, frames, C, _ptr(history), H, _ptr(slots), _ptr(alpha),
         _ptr(inverse_beta), out.data_ptr(), _stream())
    return out


def conv_weight_tiles(weight: torch.Tensor, taps: int) -> TiledWeight:
    """Conv weight [C_out, taps*C_in] (K ordered (tap, channel)) -> tiles of q3t_conv_linear, with the
    channels of every tap zero-padded to a multiple of 64."""
    c_out, k = weight.shape
    c_in = k // taps
    cp = -(-c_in // 64) * 64
    if cp != c_in:
        padded = torch.zeros(c_out, taps, cp, dtype=weight.dtype, device=weight.device)
        padded[:, :, :c_in] = weight.view(c_out, taps, c_in)
        weight = padded.view(c_out, taps * cp)
    return pack_tiles(weight.contiguous())


def conv_linear(xs, batch: int, frames: int, pad: int, weight: TiledWeight, *, taps: int, dilation: int = 1,
                reverse: bool = False, bias=None, out=None, epilogue: int = _lib.EPI_STORE, residual=None, scale=None,
                snake=None):
    """Causal conv over conv_pad's buffer as an implicit GEMM (q3t_conv_linear) -> [batch*frames, C_out]."""
    _need_cuda(xs, weight.tiles)
    C = xs.shape[-1]
    if not isinstance(weight, TiledWeight) or weight.in_features != taps * (-(-C // 64) * 64):
        raise ValueError("conv_linear: weight must be conv_weight_tiles of [C_out, taps*C_in]")
    if xs.shape != (batch * (pad + frames), C) or not xs.is_contiguous():
        raise ValueError("conv_linear: xs must be conv_pad's [batch*(pad+frames), channels] buffer")
    n = weight.out_features
    out = torch.empty(batch * frames, n, dtype=BF16, device=xs.device) if out is None else out
    alpha, inv = snake if snake is not None else (None, None)
    call("q3t_conv_linear", xs.data_ptr(), batch, frames, pad, C, taps, dilation, int(reverse), weight.tiles.data_ptr(),
         n, _ptr(bias), out.data_ptr(), out.stride(0), epilogue, _ptr(residual),
         residual.stride(0) if residual is not None else 0, _ptr(scale), _ptr(alpha), _ptr(inv),
         status_word(xs.device).data_ptr(), _stream())
    return out


def conv_history(x, batch: int, frames: int, history, slots=None) -> None:
    """history[slot] = last H frames of [history[slot] | x[b]]."""
    _need_cuda(x, history)
    call("q3t_conv_history", x.data_ptr(), x.stride(0), batch, frames, x.shape[-1], history.data_ptr(),
         history.shape[1], _ptr(slots), _stream())


def dwconv_layernorm(x, batch: int, frames: int, history, slots, weight, bias, ln_weight, ln_bias, eps, out=None):
    _need_cuda(x)
    C = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    call("q3t_dwconv_layernorm", x.data_ptr(), batch, frames, C, _ptr(history),
         history.shape[1] if history is not None else 0, _ptr(slots), weight.data_ptr(), bias.data_ptr(),
         ln_weight.data_ptr(), ln_bias.data_ptr(), float(eps), out.data_ptr(), _stream())
    return out


def codec_positions(frames_by_slot, slots, batch: int, frames: int, ring: int, rotary, cache, advance: bool) -> None:
    call("q3t_codec_positions", frames_by_slot.data_ptr(), _ptr(slots), batch, frames, ring, rotary.data_ptr(),
         cache.data_ptr(), int(advance), _stream())


STATUS_BAD_INDEX = 1 << 3
STATUS_NONFINITE = 1 << 4


def pcm16(x, wave=None, pcm=None) -> None:
    """wave = clip(x, -1, 1) (fp32) and/or pcm = int16(wave * 32767) on the device;
    a nonfinite sample raises STATUS_NONFINITE in the device status word."""
    _need_cuda(x)
    call("q3t_pcm16", x.data_ptr(), x.numel(), _ptr(wave), _ptr(pcm), status_word(x.device).data_ptr(), _stream())


# ------------------------------------------------------------------ engine slot state
def tick_gather(active, tokens, hidden_state, codec_embedding, tables, frames, trailing, trailing_len, pad, positions,
                rotary, *, pred_inputs, codes, draws, talker_uniform, steps, text, step_positions, step_rotary,
                rows: int) -> None:
    """State arrays -> one tick's predictor/talker inputs (continuous.py:575-606)."""
    hidden = hidden_state.shape[-1]
    call("q3t_tick_gather", active.data_ptr(), tokens.data_ptr(), hidden_state.data_ptr(), codec_embedding.data_ptr(),
         codec_embedding.shape[0], tables.data_ptr(), tables.shape[1], frames.data_ptr(), trailing.data_ptr(),
         trailing.shape[1], trailing_len.data_ptr(), pad.data_ptr(), positions.data_ptr(), rotary.data_ptr(),
         pred_inputs.data_ptr(), codes.data_ptr(), codes.stride(0), draws.data_ptr(), talker_uniform.data_ptr(),
         steps.data_ptr(), text.data_ptr(), step_positions.data_ptr(), step_rotary.data_ptr(), rows, hidden,
         status_word(tokens.device).data_ptr(), _stream())


def tick_commit(active, codes, step_hidden, hidden_state, ring, frames, positions, rotary, *, rows: int) -> None:
    """Step outputs -> state arrays and the code ring (continuous.py:618-635)."""
    call("q3t_tick_commit", active.data_ptr(), codes.data_ptr(), codes.stride(0), ring.shape[2], step_hidden.data_ptr(),
         hidden_state.data_ptr(), ring.data_ptr(), ring.shape[1], frames.data_ptr(), positions.data_ptr(),
         rotary.data_ptr(), rows, hidden_state.shape[-1], _stream())


def code_ring_write(ring, codes, frame_indices) -> None:
    """ring[i, frame_indices[i] % depth] = codes[i] (codec_code_buffer.py:12-17)."""
    _need_cuda(ring, codes, frame_indices)
    call("q3t_code_ring_write", codes.data_ptr(), codes.stride(0), frame_indices.data_ptr(), ring.data_ptr(),
         ring.shape[1], ring.shape[2], codes.shape[0], _stream())


def code_ring_read(ring, indices, starts, length: int, out=None):
    """[batch, codebooks, length] codes of retained frames (codec_code_buffer.py:19-27)."""
    _need_cuda(ring, indices, starts)
    batch = indices.numel()
    out = torch.empty(batch, ring.shape[2], length, dtype=torch.long, device=ring.device) if out is None else out
    call("q3t_code_ring_read", ring.data_ptr(), ring.shape[0], ring.shape[1], ring.shape[2], indices.data_ptr(),
         starts.data_ptr(), batch, length, out.data_ptr(), status_word(ring.device).data_ptr(), _stream())
    return out
