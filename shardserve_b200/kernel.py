"""Drop-in replacement for shardserve/kernel.py on B200.

`ragged_attention_direct` keeps the reference's exact signature, argument meaning and
error behaviour (shardserve/kernel.py:11-82): the same `KernelUnsupported(ValueError)` is
raised, with the same messages, for the same unsupported inputs.  The work is done by the
hand-written sm_100a kernels in `libshardserve_b200.so` (TMA page gather + tensor-core
split-K decode); there is no Triton and no CPU fallback.

`kv_append` is the device half of `Cache.write` (shardserve/cache.py:47-49).

Both calls launch on torch's current CUDA stream, allocate only through the torch caching
allocator (the output; the split-K workspace is allocated once per device and reused), and
never synchronise, so they can be captured in a CUDA graph exactly like the reference's
decode buckets (shardserve/runtime.py:51-80).  Warm up once with the largest token count
before capturing, as the reference does, so the workspace exists before capture.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Any

from . import _native

SUPPORTED_RAGGED_HEAD_DIMS = (64, 128)
SUPPORTED_BLOCK_SIZE = 16


class KernelUnsupported(ValueError):
    pass


_ws_lock = threading.Lock()
_workspaces: dict[int, Any] = {}


def _workspace(device, tokens: int, heads: int, kv_heads: int, head_dim: int):
    """Per-device workspace (error word, split-K partial states, split descriptors).

    Every call rewrites the scratch it reads, so the buffer is reused without clearing.
    One buffer per device: calls on one device must not overlap in time on different
    streams (the reference issues them from one thread on one stream).
    """
    import torch

    need = ctypes.c_size_t(0)
    rc = _native.lib().ss_attention_workspace_bytes(device.index, tokens, heads, kv_heads,
                                                    head_dim, ctypes.byref(need))
    if rc != _native.SS_OK:
        raise RuntimeError(f"ss_attention_workspace_bytes: {_native.last_error()}")
    with _ws_lock:
        ws = _workspaces.get(device.index)
        if ws is None or ws.numel() < need.value:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "ragged_attention_direct: workspace must grow during CUDA graph capture; "
                    "run the same shapes once before capturing")
            size = max(need.value, 2 * (ws.numel() if ws is not None else 0), 1 << 20)
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _workspaces[device.index] = ws
        return ws


def workspace_for(device):
    """The workspace tensor of `device` (None before the first attention call on it)."""
    return _workspaces.get(device.index)


def device_errors(device, clear: bool = True) -> int:
    """Reads the SS_DEVERR_* bits accumulated on `device` (synchronises; debug only)."""
    import torch

    ws = _workspaces.get(device.index)
    if ws is None:
        return 0
    flags = ctypes.c_uint32(0)
    stream = torch.cuda.current_stream(device).cuda_stream
    rc = _native.lib().ss_fetch_device_errors(ctypes.c_void_p(ws.data_ptr()), int(clear),
                                              ctypes.byref(flags), ctypes.c_void_p(stream))
    if rc != _native.SS_OK:
        raise RuntimeError(_native.last_error())
    return flags.value


def last_attention_path() -> int:
    """1 = TMA tensor-core split-K kernel, 2 = generic strided kernel, 3 = split-K kernel
    plus tcgen05 chunked-prefill tiles, 0 = none yet."""
    return _native.lib().ss_last_attention_path()


def _index_flag(t, name: str) -> int:
    import torch

    if t.dtype == torch.int64:
        return 1
    if t.dtype == torch.int32:
        return 0
    raise KernelUnsupported(f"{name} must be int32 or int64, got {t.dtype}")


def ragged_attention_direct(
    q: Any,
    k_pool_layer: Any,
    v_pool_layer: Any,
    block_tables: Any,
    query_seq_ids: Any,
    positions: Any,
    sm_scale: float,
) -> Any:
    """Attention for a flat mixed-query batch over physical KV blocks.

    Each query token carries its sequence row (`query_seq_ids`) and absolute position
    (`positions`); it attends to keys 0..position of its row, which makes decode rows and
    causal chunked-prefill rows one launch (reference kernel.py:20-25).
    """
    import torch

    # Checks and messages of the reference wrapper, kernel.py:28-49.
    if q.device.type != "cuda" or q.dtype != torch.bfloat16:
        raise KernelUnsupported("ragged kernel requires BF16 CUDA queries")
    if q.dim() != 3 or q.shape[-1] not in SUPPORTED_RAGGED_HEAD_DIMS:
        raise KernelUnsupported(
            f"ragged q must be [tokens, heads, 64|128], got {tuple(q.shape)}"
        )
    if k_pool_layer.shape != v_pool_layer.shape or k_pool_layer.dim() != 4:
        raise KernelUnsupported("ragged K/V pools must have identical rank-4 shapes")
    if k_pool_layer.dtype != torch.bfloat16 or k_pool_layer.shape[1] != SUPPORTED_BLOCK_SIZE:
        raise KernelUnsupported("ragged KV pools must be BF16 with block_size=16")
    if k_pool_layer.shape[-1] != q.shape[-1]:
        raise KernelUnsupported("query and KV head dimensions differ")
    if block_tables.device != q.device or block_tables.dim() != 2:
        raise KernelUnsupported("block_tables must be a device-resident rank-2 tensor")
    if query_seq_ids.numel() != q.shape[0] or positions.numel() != q.shape[0]:
        raise KernelUnsupported("one sequence id and absolute position are required per query")
    if q.shape[0] < 1:
        raise KernelUnsupported("ragged batch cannot be empty")
    tokens, num_heads, head_dim = q.shape
    kv_heads = k_pool_layer.shape[2]
    if num_heads % kv_heads:
        raise KernelUnsupported("query heads must be divisible by KV heads")
    # The Triton kernel would read these from the same device; say so explicitly here.
    for name, t in (("k_pool_layer", k_pool_layer), ("v_pool_layer", v_pool_layer),
                    ("query_seq_ids", query_seq_ids), ("positions", positions)):
        if t.device != q.device:
            raise KernelUnsupported(f"{name} must be on {q.device}")
    if v_pool_layer.dtype != torch.bfloat16:
        raise KernelUnsupported("ragged KV pools must be BF16 with block_size=16")
    bt64 = _index_flag(block_tables, "block_tables")
    seq64 = _index_flag(query_seq_ids, "query_seq_ids")
    pos64 = _index_flag(positions, "positions")
    seqs = query_seq_ids.reshape(-1)
    pos = positions.reshape(-1)
    if not seqs.is_contiguous():
        seqs = seqs.contiguous()
    if not pos.is_contiguous():
        pos = pos.contiguous()

    out = torch.empty_like(q)
    ws = _workspace(q.device, tokens, num_heads, kv_heads, head_dim)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    L = _native.lib()
    rc = L.ss_ragged_paged_attention(
        q.data_ptr(), _native.strides(q.stride()),
        k_pool_layer.data_ptr(), _native.strides(k_pool_layer.stride()),
        v_pool_layer.data_ptr(), _native.strides(v_pool_layer.stride()),
        block_tables.data_ptr(), _native.strides(block_tables.stride()),
        block_tables.shape[0], block_tables.shape[1], bt64,
        seqs.data_ptr(), seq64, pos.data_ptr(), pos64,
        out.data_ptr(), _native.strides(out.stride()),
        tokens, num_heads, kv_heads, head_dim, k_pool_layer.shape[0], float(sm_scale),
        ws.data_ptr(), ws.numel(), stream)
    if rc == _native.SS_ERR_INVALID:
        raise KernelUnsupported(_native.last_error())
    if rc != _native.SS_OK:
        raise RuntimeError(f"ss_ragged_paged_attention: {_native.last_error()}")
    return out


def kv_append(k_pool_layer: Any, v_pool_layer: Any, k: Any, v: Any, slots: Any) -> None:
    """Writes k[i], v[i] into row slots[i] % 16 of page slots[i] // 16 (cache.py:47-49)."""
    import torch

    if k_pool_layer.device.type != "cuda":
        raise KernelUnsupported("KV append requires CUDA pools")
    if k_pool_layer.dtype != torch.bfloat16 or v_pool_layer.dtype != torch.bfloat16:
        raise KernelUnsupported("KV pools must be BF16")
    if k_pool_layer.shape != v_pool_layer.shape or k_pool_layer.dim() != 4 \
            or k_pool_layer.shape[1] != SUPPORTED_BLOCK_SIZE:
        raise KernelUnsupported("ragged K/V pools must have identical rank-4 shapes")
    kv_heads, head_dim = k_pool_layer.shape[2], k_pool_layer.shape[3]
    if k.dim() != 3 or tuple(k.shape[1:]) != (kv_heads, head_dim) or k.shape != v.shape:
        raise KernelUnsupported(
            f"k/v must be [tokens, {kv_heads}, {head_dim}], got {tuple(k.shape)}/{tuple(v.shape)}")
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise KernelUnsupported("k/v must be BF16")
    for name, t in (("v_pool_layer", v_pool_layer), ("k", k), ("v", v), ("slots", slots)):
        if t.device != k_pool_layer.device:
            raise KernelUnsupported(f"{name} must be on {k_pool_layer.device}")
    if slots.numel() != k.shape[0]:
        raise KernelUnsupported("one slot is required per appended token")
    s64 = _index_flag(slots, "slots")
    sl = slots.reshape(-1)
    if not sl.is_contiguous():
        sl = sl.contiguous()
    ws = _workspaces.get(k_pool_layer.device.index)
    stream = torch.cuda.current_stream(k_pool_layer.device).cuda_stream
    rc = _native.lib().ss_kv_append(
        k.data_ptr(), _native.strides(k.stride()), v.data_ptr(), _native.strides(v.stride()),
        k_pool_layer.data_ptr(), _native.strides(k_pool_layer.stride()),
        v_pool_layer.data_ptr(), _native.strides(v_pool_layer.stride()),
        sl.data_ptr(), s64, k.shape[0], k_pool_layer.shape[0], kv_heads, head_dim,
        ws.data_ptr() if ws is not None else None, stream)
    if rc == _native.SS_ERR_INVALID:
        raise KernelUnsupported(_native.last_error())
    if rc != _native.SS_OK:
        raise RuntimeError(f"ss_kv_append: {_native.last_error()}")


def rope_kv_append(q: Any, k: Any, v: Any, cos: Any, sin: Any, positions: Any,
                   k_pool_layer: Any, v_pool_layer: Any, slots: Any, out: Any = None) -> Any:
    """One launch for `q, k = apply_rope(q, k, cos, sin, positions)` (shardserve/math.py:28-38,
    model.py:25) followed by `Cache.write(layer, k, v, slots)` (cache.py:47-49, model.py:32).

    q [tokens, heads, D], k / v [tokens, kv_heads, D] bf16; cos / sin fp32 [rows, D] (the
    tables of math.build_rope_cache); positions / slots int32 or int64 [tokens].  Returns the
    rotated q (in `out` if given; `out` may be q itself).  Bit-exact with the reference's
    bf16 arithmetic."""
    import torch

    if k_pool_layer.device.type != "cuda":
        raise KernelUnsupported("RoPE + KV append requires CUDA pools")
    if k_pool_layer.dtype != torch.bfloat16 or v_pool_layer.dtype != torch.bfloat16:
        raise KernelUnsupported("KV pools must be BF16")
    if k_pool_layer.shape != v_pool_layer.shape or k_pool_layer.dim() != 4 \
            or k_pool_layer.shape[1] != SUPPORTED_BLOCK_SIZE:
        raise KernelUnsupported("ragged K/V pools must have identical rank-4 shapes")
    kv_heads, head_dim = k_pool_layer.shape[2], k_pool_layer.shape[3]
    if q.dim() != 3 or q.shape[2] != head_dim or q.dtype != torch.bfloat16:
        raise KernelUnsupported(f"q must be BF16 [tokens, heads, {head_dim}]")
    if k.dim() != 3 or tuple(k.shape[1:]) != (kv_heads, head_dim) or k.shape != v.shape:
        raise KernelUnsupported(
            f"k/v must be [tokens, {kv_heads}, {head_dim}], got {tuple(k.shape)}/{tuple(v.shape)}")
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise KernelUnsupported("k/v must be BF16")
    if q.shape[0] != k.shape[0] or q.shape[1] % kv_heads:
        raise KernelUnsupported("q and k/v must have the same tokens and a whole GQA group")
    if head_dim % 2:
        raise KernelUnsupported("RoPE needs an even head_dim")
    for name, t in (("cos", cos), ("sin", sin)):
        if t.dtype != torch.float32 or t.dim() != 2 or t.shape[1] != head_dim:
            raise KernelUnsupported(f"{name} must be float32 [rows, {head_dim}]")
    if cos.shape != sin.shape:
        raise KernelUnsupported("cos and sin tables must have the same shape")
    for name, t in (("v_pool_layer", v_pool_layer), ("q", q), ("k", k), ("v", v), ("cos", cos),
                    ("sin", sin), ("positions", positions), ("slots", slots)):
        if t.device != k_pool_layer.device:
            raise KernelUnsupported(f"{name} must be on {k_pool_layer.device}")
    tokens = q.shape[0]
    if slots.numel() != tokens or positions.numel() != tokens:
        raise KernelUnsupported("one position and one slot are required per token")
    p64 = _index_flag(positions, "positions")
    s64 = _index_flag(slots, "slots")
    pos = positions.reshape(-1)
    sl = slots.reshape(-1)
    pos = pos if pos.is_contiguous() else pos.contiguous()
    sl = sl if sl.is_contiguous() else sl.contiguous()
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != torch.bfloat16 or out.device != q.device:
        raise KernelUnsupported("out must be a BF16 tensor shaped like q on q's device")
    ws = _workspaces.get(k_pool_layer.device.index)
    stream = torch.cuda.current_stream(k_pool_layer.device).cuda_stream
    rc = _native.lib().ss_rope_kv_append(
        q.data_ptr(), _native.strides(q.stride()), out.data_ptr(), _native.strides(out.stride()),
        k.data_ptr(), _native.strides(k.stride()), v.data_ptr(), _native.strides(v.stride()),
        cos.data_ptr(), _native.strides(cos.stride()), sin.data_ptr(),
        _native.strides(sin.stride()), cos.shape[0], pos.data_ptr(), p64,
        k_pool_layer.data_ptr(), _native.strides(k_pool_layer.stride()),
        v_pool_layer.data_ptr(), _native.strides(v_pool_layer.stride()),
        sl.data_ptr(), s64, tokens, q.shape[1], kv_heads, head_dim, k_pool_layer.shape[0],
        ws.data_ptr() if ws is not None else None, stream)
    if rc == _native.SS_ERR_INVALID:
        raise KernelUnsupported(_native.last_error())
    if rc != _native.SS_OK:
        raise RuntimeError(f"ss_rope_kv_append: {_native.last_error()}")
    return out
