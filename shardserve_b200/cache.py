"""Paged KV pool for B200, a drop-in for shardserve/cache.py's `Blocks` and `Cache`.

`Blocks` is the host-side logical page allocator (all-or-nothing reservations, reference
cache.py:6-35); `Cache` owns the device pools `k`, `v` of shape
[layers, blocks + 8, 16, kv_heads / world, head_dim] (cache.py:37-45; the last eight pages
are graph-padding scratch, runtime.py:41-44) and appends through the sm_100a kernel
(`Cache.write`, cache.py:47-49).

Layout in HBM: one contiguous bf16 tensor per K and per V; page p of layer l for KV head h
is the 16 x head_dim block at [l, p, :, h, :], so one page of all KV heads of a layer is a
contiguous 16 * kv_heads * head_dim * 2 byte run (8 KiB at Qwen2.5-3B TP1), which the
attention kernel moves with a single TMA box.
"""
from __future__ import annotations

import math

from .kernel import KernelUnsupported, kv_append, rope_kv_append


class Blocks:
    """Free-list page allocator with all-or-nothing reservations (reference cache.py:6-35)."""

    def __init__(self, count):
        if type(count) is not int or count < 1:
            raise ValueError("positive block count required")
        self.count = count
        self.free = list(range(count))
        self.tables = {}

    def reserve(self, requests):
        """Reserves ceil(n / 16) pages for every request of {key: tokens}, or none at all."""
        if any(key in self.tables for key in requests):
            raise ValueError("duplicate reservation")
        if any(type(n) is not int or n < 1 for n in requests.values()):
            raise ValueError("invalid reservation")
        sizes = {key: math.ceil(n / 16) for key, n in requests.items()}
        if sum(sizes.values()) > len(self.free):
            raise MemoryError("KV capacity exhausted")
        for key, n in sizes.items():
            # Pages come off the end of the free list, as in the reference (cache.py:23).
            self.tables[key] = [self.free.pop() for _ in range(n)]
        self.check()

    def release(self, key):
        if key not in self.tables:
            raise ValueError("double/foreign release")
        self.free.extend(self.tables.pop(key))
        self.check()

    def check(self):
        owned = [b for table in self.tables.values() for b in table]
        assert sorted(owned + self.free) == list(range(self.count)), "leak/duplicate ownership"


class Cache:
    """Device KV pool with the reference constructor signature (cache.py:37-45)."""

    def __init__(self, c, world, blocks, device, dtype):
        import torch

        if torch.device(device).type != "cuda" or dtype != torch.bfloat16:
            raise KernelUnsupported("the B200 KV pool is a BF16 CUDA tensor")
        self.blocks = Blocks(blocks)
        self.shape = (c["num_hidden_layers"], blocks + 8, 16, c["num_key_value_heads"] // world,
                      c["hidden_size"] // c["num_attention_heads"])
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
