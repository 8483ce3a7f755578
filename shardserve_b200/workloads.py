"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No dataset is involved: contexts are drawn uniformly, K/V/Q are N(0, 1) rounded to bf16,
and every sequence's pages are a slice of a seeded random permutation of the pool
(pool = total pages x slack + 8 graph-padding scratch pages, as the reference pool keeps 8,
shardserve/cache.py:42).  A sequence with `n` query tokens after `ctx` cached tokens gets
positions ctx .. ctx+n-1 (decode: n = 1; chunked prefill: n > 1), and every query token's
own K/V row is appended at its slot `table[p // 16] * 16 + p % 16` first (runtime.py:38,
model.py:32).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

BLOCK = 16


@dataclass
class RaggedBatch:
    q: object          # bf16 [T, H, D]
    k_pool: object     # bf16 [N, 16, KVH, D]  (or [layers, N, 16, KVH, D])
    v_pool: object
    block_tables: object  # int32 [B, W]
    seq_ids: object    # int32 [T]
    positions: object  # int64 [T]
    slots: object      # int64 [T]
    k_new: object      # bf16 [T, KVH, D]
    v_new: object
    rows: list         # (cached context, query tokens) per sequence
    heads: int
    kv_heads: int
    head_dim: int

    @property
    def tokens(self) -> int:
        return sum(n for _, n in self.rows)

    @property
    def lengths(self) -> list:
        """Keys attended by the last query token of every sequence."""
        return [c + n for c, n in self.rows]


def _tables(rows, slack, gen):
    import torch

    pages = [math.ceil((c + n) / BLOCK) for c, n in rows]
    data_pages = int(math.ceil(sum(pages) * slack))
    perm = torch.randperm(data_pages, generator=gen).to(torch.int32)
    bt = torch.zeros(len(rows), max(pages), dtype=torch.int32)
    off = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[off:off + n]
        off += n
    return bt, data_pages + 8


def _tokens(rows, bt):
    import torch

    seq, pos = [], []
    for i, (c, n) in enumerate(rows):
        seq += [i] * n
        pos += list(range(c, c + n))
    seq = torch.tensor(seq, dtype=torch.int32)
    pos = torch.tensor(pos, dtype=torch.int64)
    slots = bt[seq.long(), pos // BLOCK].long() * BLOCK + pos % BLOCK
    return seq, pos, slots


def ragged_batch(rows, heads=16, kv_heads=2, head_dim=128, slack=1.1, seed=0, device="cuda",
                 layers=None, pool_pages=None) -> RaggedBatch:
    """A flat ragged batch.  `layers` gives a [layers, N, ...] pool; `pool_pages` forces the
    pool size (pages are then scattered over the whole pool)."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    if pool_pages is None:
        bt, N = _tables(rows, slack, g)
    else:
        pages = [math.ceil((c + n) / BLOCK) for c, n in rows]
        N = int(pool_pages)
        if sum(pages) > N - 8:
            raise ValueError("pool too small for the batch")
        # Scattered over the whole pool without materialising a permutation of N pages.
        pick = torch.randint(0, N - 8, (int(sum(pages) * 1.3) + 64,), generator=g).unique()
        pick = pick[torch.randperm(pick.numel(), generator=g)][:sum(pages)].to(torch.int32)
        if pick.numel() < sum(pages):
            raise ValueError("could not draw distinct pages")
        bt = torch.zeros(len(rows), max(pages), dtype=torch.int32)
        off = 0
        for i, n in enumerate(pages):
            bt[i, :n] = pick[off:off + n]
            off += n
    seq, pos, slots = _tokens(rows, bt)
    T = int(seq.numel())
    dg = torch.Generator(device=device).manual_seed(seed + 1)
    shape = (N, BLOCK, kv_heads, head_dim) if layers is None else (layers, N, BLOCK, kv_heads, head_dim)
    kp = torch.empty(shape, device=device, dtype=torch.bfloat16)
    vp = torch.empty_like(kp)
    for pool in (kp, vp):  # bf16 directly, in slices, so no fp32 copy of a large pool exists
        flat = pool.view(-1)
        step = 1 << 28
        for i in range(0, flat.numel(), step):
            flat[i:i + step].normal_(generator=dg)
    q = torch.randn((T, heads, head_dim), generator=dg, device=device).to(torch.bfloat16)
    kn = torch.randn((T, kv_heads, head_dim), generator=dg, device=device).to(torch.bfloat16)
    vn = torch.randn((T, kv_heads, head_dim), generator=dg, device=device).to(torch.bfloat16)
    return RaggedBatch(q=q, k_pool=kp, v_pool=vp, block_tables=bt.to(device),
                       seq_ids=seq.to(device), positions=pos.to(device), slots=slots.to(device),
                       k_new=kn, v_new=vn, rows=list(rows), heads=heads, kv_heads=kv_heads,
                       head_dim=head_dim)


def decode_batch(lengths, heads=16, kv_heads=2, head_dim=128, slack=1.1, seed=0,
                 device="cuda") -> RaggedBatch:
    """One query token per sequence at position L - 1, pages scattered over the pool."""
    return ragged_batch([(int(L) - 1, 1) for L in lengths], heads, kv_heads, head_dim, slack,
                        seed, device)


def uniform_lengths(n, lo, hi, seed):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def mixed_rows(seed, chunks=8, decode_rows=56, chunk=512):
    """The mixed chunked-prefill batch: `decode_rows` decode rows with context U[256, 4096]
    first (as the reference scheduler packs decode rows first, scheduler.py:119-131), then
    `chunks` prefill chunks of `chunk` query tokens on cached context U[0, 2048]."""
    import torch

    g = torch.Generator().manual_seed(seed)
    decode = [(int(c) - 1, 1) for c in torch.randint(256, 4097, (decode_rows,), generator=g)]
    prefill = [(int(c), chunk) for c in torch.randint(0, 2049, (chunks,), generator=g)]
    return decode, prefill


def attention_bytes(lengths, heads, kv_heads, head_dim, tokens=None) -> int:
    """Algorithmic HBM bytes of one decode attention launch, each byte counted once:
    K and V of every attended key (GQA re-reads not credited), q in, out, the block-table
    entries used, and per-token seq id (4 B) + position (8 B)."""
    T = len(lengths) if tokens is None else tokens
    kv = sum(lengths) * kv_heads * head_dim * 2 * 2
    qo = 2 * T * heads * head_dim * 2
    tables = sum(math.ceil(L / BLOCK) for L in lengths) * 4
    return kv + qo + tables + T * (4 + 8)


def prefill_flops(rows, heads, head_dim) -> int:
    """QK^T + PV FLOPs of the causal keys every query token attends: 4 H D sum(pos + 1)."""
    keys = sum(sum(range(c + 1, c + n + 1)) for c, n in rows)
    return 4 * heads * head_dim * keys


def append_bytes(tokens, kv_heads, head_dim) -> int:
    """K and V rows read plus written, and the int64 slot per token."""
    return tokens * kv_heads * head_dim * 2 * 2 * 2 + tokens * 8
