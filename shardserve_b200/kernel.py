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
from typing import Any

from . import _native

SUPPORTED_RAGGED_HEAD_DIMS = (64, 128)
SUPPORTED_BLOCK_SIZE = 16


class KernelUnsupported(ValueError):
    pass


def _workspace(device, tokens: int, heads: int, kv_heads: int, head_dim: int):
    """Per-device workspace (error word, split-K partial states, split descriptors), kept
    by the torch binding: one zero-filled buffer per device, grown to what
    ss_attention_workspace_bytes asks for (never during CUDA graph capture).

    Every call rewrites the scratch it reads, so the buffer is reused without clearing.
    One buffer per device: calls on one device must not overlap in time on different
    streams (the reference issues them from one thread on one stream).
    """
    return _native.ops().ensure_workspace(device.index, tokens, heads, kv_heads, head_dim)


def workspace_for(device):
    """The workspace tensor of `device` (None before the first attention call on it)."""
    return _native.ops().workspace_for(device.index)


def device_errors(device, clear: bool = True) -> int:
    """Reads the SS_DEVERR_* bits accumulated on `device` (synchronises; debug only)."""
    import torch

    ws = workspace_for(device)
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
    plus tcgen05 chunked-prefill tiles, 4 = split-K kernel with the KV append folded in
    (kv_append_attention), 0 = none yet."""
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
    # Checks (the reference wrapper's, kernel.py:28-49, same order and messages) and the
    # launch run in the torch binding (csrc/torch_binding.cpp).
    return _native.ops().ragged_attention_direct(q, k_pool_layer, v_pool_layer, block_tables,
                                                 query_seq_ids, positions, sm_scale)


def kv_append_attention(k_pool_layer: Any, v_pool_layer: Any, k: Any, v: Any, slots: Any,
                        q: Any, block_tables: Any, query_seq_ids: Any, positions: Any,
                        sm_scale: float) -> Any:
    """`kv_append(k_pool_layer, v_pool_layer, k, v, slots)` then
    `ragged_attention_direct(q, k_pool_layer, v_pool_layer, block_tables, query_seq_ids,
    positions, sm_scale)` in one call, as the reference model makes them per layer
    (cache.write then ragged_attention_direct, model.py:32-37).  For a decode step (one query
    token per row) the append runs inside the attention kernel; slots must then be each
    token's own position in its row, as the reference builds them (runtime.py:38).  Other
    batches run the append kernel first."""
    return _native.ops().kv_append_attention(k_pool_layer, v_pool_layer, k, v, slots, q,
                                             block_tables, query_seq_ids, positions, sm_scale)


def kv_append(k_pool_layer: Any, v_pool_layer: Any, k: Any, v: Any, slots: Any) -> None:
    """Writes k[i], v[i] into row slots[i] % 16 of page slots[i] // 16 (cache.py:47-49)."""
    _native.ops().kv_append(k_pool_layer, v_pool_layer, k, v, slots)


def rope_kv_append(q: Any, k: Any, v: Any, cos: Any, sin: Any, positions: Any,
                   k_pool_layer: Any, v_pool_layer: Any, slots: Any, out: Any = None) -> Any:
    """One launch for `q, k = apply_rope(q, k, cos, sin, positions)` (shardserve/math.py:28-38,
    model.py:25) followed by `Cache.write(layer, k, v, slots)` (cache.py:47-49, model.py:32).

    q [tokens, heads, D], k / v [tokens, kv_heads, D] bf16; cos / sin fp32 [rows, D] (the
    tables of math.build_rope_cache); positions / slots int32 or int64 [tokens].  Returns the
    rotated q (in `out` if given; `out` may be q itself).  Bit-exact with the reference's
    bf16 arithmetic."""
    return _native.ops().rope_kv_append(q, k, v, cos, sin, positions, k_pool_layer,
                                        v_pool_layer, slots, out)
