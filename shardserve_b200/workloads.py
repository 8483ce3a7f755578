"""Seeded synthetic decode workloads with the shapes of the benchmark configurations.

No dataset is involved: contexts are drawn uniformly in [lo, hi], K/V/Q are N(0, 1) rounded
to bf16, and every sequence's pages are a slice of a seeded random permutation of the pool
(pool = total pages x slack + 8 graph-padding scratch pages, as the reference pool keeps 8,
shardserve/cache.py:42).  Each decode token sits at position L - 1 of its sequence, and the
new token's K/V row is appended at that position's slot first (runtime.py:38, model.py:32).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

BLOCK = 16


@dataclass
class DecodeBatch:
    q: object          # bf16 [T, H, D]
    k_pool: object     # bf16 [N, 16, KVH, D]
    v_pool: object
    block_tables: object  # int32 [T, W]
    seq_ids: object    # int32 [T]
    positions: object  # int64 [T]
    slots: object      # int64 [T]
    k_new: object      # bf16 [T, KVH, D]
    v_new: object
    lengths: list      # context lengths (keys attended) per sequence
    heads: int
    kv_heads: int
    head_dim: int

    @property
    def tokens(self) -> int:
        return len(self.lengths)


def decode_batch(lengths, heads=16, kv_heads=2, head_dim=128, slack=1.1, seed=0,
                 device="cuda") -> DecodeBatch:
    """One query token per sequence at position L - 1, pages scattered over the pool."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    lengths = [int(x) for x in lengths]
    pages = [math.ceil(L / BLOCK) for L in lengths]
    data_pages = int(math.ceil(sum(pages) * slack))
    N = data_pages + 8
    perm = torch.randperm(data_pages, generator=g).to(torch.int32)
    W = max(pages)
    T = len(lengths)
    bt = torch.zeros(T, W, dtype=torch.int32)
    off = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[off:off + n]
        off += n
    pos = torch.tensor([L - 1 for L in lengths], dtype=torch.int64)
    seq = torch.arange(T, dtype=torch.int32)
    slots = bt[seq.long(), pos // BLOCK].long() * BLOCK + pos % BLOCK
    dg = torch.Generator(device=device).manual_seed(seed + 1)
    shape = (N, BLOCK, kv_heads, head_dim)
    kp = torch.randn(shape, generator=dg, device=device, dtype=torch.float32).to(torch.bfloat16)
    vp = torch.randn(shape, generator=dg, device=device, dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((T, heads, head_dim), generator=dg, device=device).to(torch.bfloat16)
    kn = torch.randn((T, kv_heads, head_dim), generator=dg, device=device).to(torch.bfloat16)
    vn = torch.randn((T, kv_heads, head_dim), generator=dg, device=device).to(torch.bfloat16)
    return DecodeBatch(q=q, k_pool=kp, v_pool=vp, block_tables=bt.to(device),
                       seq_ids=seq.to(device), positions=pos.to(device), slots=slots.to(device),
                       k_new=kn, v_new=vn, lengths=lengths, heads=heads, kv_heads=kv_heads,
                       head_dim=head_dim)


def uniform_lengths(n, lo, hi, seed):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def attention_bytes(lengths, heads, kv_heads, head_dim) -> int:
    """Algorithmic HBM bytes of one decode attention launch, each byte counted once:
    K and V of every attended key (GQA re-reads not credited), q in, out, the block-table
    entries used, and per-token seq id (4 B) + position (8 B)."""
    T = len(lengths)
    kv = sum(lengths) * kv_heads * head_dim * 2 * 2
    qo = 2 * T * heads * head_dim * 2
    tables = sum(math.ceil(L / BLOCK) for L in lengths) * 4
    return kv + qo + tables + T * (4 + 8)


def append_bytes(tokens, kv_heads, head_dim) -> int:
    """K and V rows read plus written, and the int64 slot per token."""
    return tokens * kv_heads * head_dim * 2 * 2 * 2 + tokens * 8
