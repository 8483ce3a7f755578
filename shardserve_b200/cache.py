"""Paged KV pool for B200, a drop-in for shardserve/cache.py's `Cache`.

`Cache` owns the device pools `k`, `v` of shape
[layers, blocks + 8, 16, kv_heads / world, head_dim] (cache.py:37-45; the last eight pages
are graph-padding scratch, runtime.py:41-44) and appends through the sm_100a kernel
(`Cache.write`, cache.py:47-49).  The logical page allocator `Cache.blocks` (free list and
per-request block tables, cache.py:6-35) is host-side engine code, not part of the device
path: it is the engine's own class, by default the reference's `shardserve.cache.Blocks`,
or any class passed as `allocator`.

Layout in HBM: one contiguous bf16 tensor per K and per V; page p of layer l for KV head h
is the 16 x head_dim block at [l, p, :, h, :], so one page of all KV heads of a layer is a
contiguous 16 * kv_heads * head_dim * 2 byte run (8 KiB at Qwen2.5-3B TP1), which the
attention kernel moves with a single TMA box.
"""
from __future__ import annotations

from .kernel import KernelUnsupported, kv_append, rope_kv_append


def default_allocator():
    """The engine's logical page allocator class: shardserve.cache.Blocks (cache.py:6-35)."""
    try:
        from shardserve.cache import Blocks
    except ImportError as e:
        raise ImportError(
            "Cache needs the engine's logical page allocator: pass allocator=<class taking the "
            "block count> or make the shardserve package importable") from e
    return Blocks


class Cache:
    """Device KV pool with the reference constructor signature (cache.py:37-45).  `allocator`
    builds `self.blocks` from the block count (default: the reference's Blocks).
    `scratch_pages` trailing pages serve graph-padding rows, one page per padding row (the
    reference keeps 8 for its buckets of up to 8 rows; DecodeGraphs buckets of up to n rows
    need n)."""

    def __init__(self, c, world, blocks, device, dtype, allocator=None, scratch_pages=8):
        import torch

        if torch.device(device).type != "cuda" or dtype != torch.bfloat16:
            raise KernelUnsupported("the B200 KV pool is a BF16 CUDA tensor")
        if scratch_pages < 0:
            raise KernelUnsupported("scratch_pages must be >= 0")
        self.blocks = (allocator or default_allocator())(blocks)
        self.scratch_pages = int(scratch_pages)
        self.shape = (c["num_hidden_layers"], blocks + self.scratch_pages, 16,
                      c["num_key_value_heads"] // world, c["hidden_size"] // c["num_attention_heads"])
        self.k = torch.zeros(self.shape, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.bytes = 2 * self.k.numel() * self.k.element_size()

    def write(self, layer, k, v, slots):
        """Appends k, v [tokens, kv_heads, head_dim] at `slots` of `layer` (cache.py:47-49)."""
        kv_append(self.k[layer], self.v[layer], k, v, slots)

    def write_rope(self, layer, q, k, v, cos, sin, positions, slots, out=None):
        """Rotates q and k with RoPE at `positions` (math.py:28-38) and appends the rotated
        k and v at `slots` of `layer` in one launch; returns the rotated q."""
        return rope_kv_append(q, k, v, cos, sin, positions, self.k[layer], self.v[layer], slots,
                              out=out)
