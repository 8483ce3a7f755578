"""Generates tests/golden/rope_<case>.npz by running the REFERENCE RoPE + append itself.

For every case below this script imports ShardServe unchanged from the reference checkout
(the directory named by the SHARDSERVE_REFERENCE environment variable), builds the fp32 cos / sin
tables with the reference's `build_rope_cache` (shardserve/math.py:12-20), rotates seeded
bf16 q / k with the reference's `apply_rope` (math.py:28-38, torch CPU, bf16 tensors), and
appends the rotated k and the raw v with the reference's `Cache.write` (cache.py:47-49).
Stored (bf16 as uint16 bit patterns):

* inputs: q, k, v, positions, slots, and the cos / sin table rows at the used positions
  (`table_pos`, `cos_rows`, `sin_rows`; the full table has `max_len` rows);
* outputs: q_rot, k_rot (bit-exact targets) and the sha256 of both pools after the append.

Run once in a container that has the reference (it is not needed afterwards):
    python tests/golden/make_golden_rope.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("SHARDSERVE_REFERENCE")
if not REF:
    sys.exit("set SHARDSERVE_REFERENCE to the reference checkout (its shardserve package)")
sys.path.insert(0, REF)
from shardserve.cache import Cache as RefCache  # noqa: E402
from shardserve.math import apply_rope, build_rope_cache  # noqa: E402

# name: (tokens, heads, kv_heads, head_dim, theta, max_len, pool_pages, kind, seed)
CASES = {
    "rope_decode": (16, 16, 2, 128, 1.0e6, 4096, 64, "decode", 11),
    "rope_chunk_mha_d64": (40, 8, 8, 64, 1.0e4, 512, 16, "chunk", 12),
    "rope_tp2_long": (8, 8, 1, 128, 1.0e6, 32768, 16, "long", 13),
    "rope_wide_range": (12, 4, 2, 128, 1.0e6, 8192, 8, "wide", 14),
}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def build_inputs(name: str):
    T, H, KVH, D, theta, max_len, pages, kind, seed = CASES[name]
    g = torch.Generator().manual_seed(seed)
    if kind == "decode":
        pos = torch.randint(0, max_len, (T,), generator=g)
    elif kind == "chunk":
        pos = torch.arange(100, 100 + T)
    elif kind == "long":
        pos = torch.randint(16000, max_len, (T,), generator=g)
    else:
        pos = torch.randint(0, max_len, (T,), generator=g)
    q = torch.randn(T, H, D, generator=g)
    k = torch.randn(T, KVH, D, generator=g)
    v = torch.randn(T, KVH, D, generator=g)
    if kind == "wide":  # magnitudes from 2^-60 to 2^40: exercises the fp32 sum's own rounding
        q = q * torch.pow(2.0, torch.randint(-60, 41, (T, H, D), generator=g).float())
        k = k * torch.pow(2.0, torch.randint(-60, 41, (T, KVH, D), generator=g).float())
    slots = torch.randperm(pages * 16, generator=g)[:T].to(torch.int64)
    return (q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16),
            pos.to(torch.int64), slots, (T, H, KVH, D, theta, max_len, pages))


def run_case(name: str) -> dict:
    q, k, v, pos, slots, (T, H, KVH, D, theta, max_len, pages) = build_inputs(name)
    cos, sin = build_rope_cache(D, max_len, theta, "cpu")
    q_rot, k_rot = apply_rope(q, k, cos, sin, pos)
    c = RefCache.__new__(RefCache)
    c.k = torch.zeros(1, pages, 16, KVH, D, dtype=torch.bfloat16)
    c.v = torch.zeros_like(c.k)
    c.shape = tuple(c.k.shape)
    c.write(0, k_rot, v, slots)
    table_pos = torch.unique(pos)
    return {
        "q": _bits(q), "k": _bits(k), "v": _bits(v),
        "positions": pos.numpy(), "slots": slots.numpy(),
        "table_pos": table_pos.numpy(),
        "cos_rows": cos[table_pos].numpy().astype(np.float32),
        "sin_rows": sin[table_pos].numpy().astype(np.float32),
        "dims": np.array([T, H, KVH, D, max_len, pages], dtype=np.int64),
        "theta": np.array([theta], dtype=np.float64),
        "q_rot": _bits(q_rot), "k_rot": _bits(k_rot),
        "kpool_sha256": np.array(_digest(_bits(c.k[0]))),
        "vpool_sha256": np.array(_digest(_bits(c.v[0]))),
    }


def main() -> None:
    for name in CASES:
        rec = run_case(name)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
        print(name, "q_rot", rec["q_rot"].shape, "rows", rec["table_pos"].size)


if __name__ == "__main__":
    main()
