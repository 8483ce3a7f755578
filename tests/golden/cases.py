"""Seeded ragged-attention cases shared by the golden-fixture script and the tests.

Each case is a flat batch in the reference's per-token contract (shardserve/kernel.py:11-19,
shardserve/runtime.py:28-49): every query token has a sequence row and an absolute
position; a sequence with `n` query tokens after `ctx` cached tokens contributes positions
ctx .. ctx+n-1 (causal chunked prefill when n > 1, decode when n == 1).  Page tables are
slices of a seeded random permutation of the pool's pages; the last `scratch` pages are the
graph-padding scratch pages of the reference (cache.py:42, runtime.py:41-44), used by
`padding` rows exactly as runtime.metadata builds them.

Inputs are generated with numpy only (no torch), so the same bytes can be rebuilt on any
host; `input_digest` fingerprints them so a fixture can never silently pair with different
inputs.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np

BLOCK = 16


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) >> 16).astype(np.uint16)


def _bf16_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


# name -> spec.  seqs: (cached context before this step, query tokens this step).
CASES = {
    # The reference's CPU-runnable decode case: contexts {17, 64, 200, 511}, one query token each, Qwen2.5-3B
    # geometry, 64-page pool, tables from a seeded permutation of page ids.
    "config1_decode": dict(H=16, KVH=2, D=128, seqs=[(16, 1), (63, 1), (199, 1), (510, 1)],
                           pages=64, scratch=0, padding=0, seed=1101),
    # Chunks crossing page edges (15|16, 16|17, 31|32, 47|48), decode rows, padding rows.
    "chunked_mixed": dict(H=16, KVH=2, D=128,
                          seqs=[(30, 20), (70, 1), (0, 5), (15, 18), (0, 1)],
                          pages=24, scratch=8, padding=2, seed=1103),
    # TP2 per-rank head layout: 8 query heads, 1 KV head (docs/implementation.md:15).
    "tp2_decode": dict(H=8, KVH=1, D=128, seqs=[(0, 1), (15, 1), (16, 1), (299, 1), (999, 1)],
                       pages=100, scratch=0, padding=0, seed=1104),
    # head_dim 64, 4 query heads per KV head, a 40-token chunk and a 9-token chunk.
    "d64_group4": dict(H=8, KVH=2, D=64, seqs=[(100, 40), (33, 1), (250, 1), (7, 9)],
                       pages=56, scratch=8, padding=0, seed=1105),
    # Multi-head attention (one query head per KV head), four KV heads.
    "mha_d64": dict(H=4, KVH=4, D=64, seqs=[(64, 1), (500, 1), (31, 3)],
                    pages=48, scratch=0, padding=0, seed=1106),
    # A CUDA-graph decode bucket of 8 with 3 live rows and 5 padding rows.
    "graph_padding": dict(H=16, KVH=2, D=128, seqs=[(47, 1), (128, 1), (5, 1)],
                          pages=16, scratch=8, padding=5, seed=1107),
    # Long decode contexts up to the reference's 4096 limit (256-page tables).
    "long_decode": dict(H=16, KVH=2, D=128, seqs=[(4095, 1), (2499, 1), (1, 1)],
                        pages=420, scratch=0, padding=0, seed=1108),
    # 16 query heads per KV head (fills the 16-row tensor-core tile).
    "gqa16": dict(H=32, KVH=2, D=128, seqs=[(300, 1), (40, 12)],
                  pages=32, scratch=0, padding=0, seed=1109),
    # 32 query heads per KV head: served by the generic strided kernel.
    "group32_generic": dict(H=32, KVH=1, D=64, seqs=[(90, 1), (17, 4)],
                            pages=16, scratch=0, padding=0, seed=1110),
    # TP2 geometry with a 64-token prefill chunk on 600 cached tokens plus a long decode row.
    "tp2_chunk_long": dict(H=8, KVH=1, D=128, seqs=[(600, 64), (3000, 1)],
                           pages=260, scratch=0, padding=0, seed=1111),
}


def build(name: str) -> dict:
    """Deterministic inputs of case `name` (numpy arrays; bf16 tensors as uint16 bits)."""
    if name == "preflight_kat":
        return preflight_kat()
    c = CASES[name]
    H, KVH, D = c["H"], c["KVH"], c["D"]
    rng = np.random.default_rng(c["seed"])
    N = c["pages"] + c["scratch"]
    lengths = [ctx + n for ctx, n in c["seqs"]]
    need = [math.ceil(L / BLOCK) for L in lengths]
    assert sum(need) <= c["pages"], name
    W = max(need)
    B = len(c["seqs"]) + c["padding"]
    perm = rng.permutation(c["pages"]).astype(np.int32)
    bt = np.zeros((B, W), dtype=np.int32)
    off = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[off:off + n]
        off += n
    seqs, pos = [], []
    for i, (ctx, n) in enumerate(c["seqs"]):
        seqs += [i] * n
        pos += list(range(ctx, ctx + n))
    for j in range(c["padding"]):  # runtime.py:41-44
        row = len(c["seqs"]) + j
        block = c["pages"] + j
        bt[row, 0] = block
        seqs.append(row)
        pos.append(0)
    seqs = np.asarray(seqs, dtype=np.int32)
    pos = np.asarray(pos, dtype=np.int64)
    T = len(seqs)
    slots = (bt[seqs, pos // BLOCK].astype(np.int64) * BLOCK + pos % BLOCK).astype(np.int64)
    kp = _bf16_bits(rng.standard_normal((N, BLOCK, KVH, D), dtype=np.float32))
    vp = _bf16_bits(rng.standard_normal((N, BLOCK, KVH, D), dtype=np.float32))
    q = _bf16_bits(rng.standard_normal((T, H, D), dtype=np.float32))
    k_new = _bf16_bits(rng.standard_normal((T, KVH, D), dtype=np.float32))
    v_new = _bf16_bits(rng.standard_normal((T, KVH, D), dtype=np.float32))
    return dict(name=name, H=H, KVH=KVH, D=D, N=N, scale=float(D) ** -0.5, q=q, k_pool=kp,
                v_pool=vp, k_new=k_new, v_new=v_new, block_tables=bt, seq_ids=seqs,
                positions=pos, slots=slots, append=True)


def preflight_kat() -> dict:
    """The reference's kernel known-answer test (shardserve/preflight.py:20-26): q = 1,
    K = 1, V = 2 on one page, position 0 (int32 ids and positions) -> every output is 2."""
    one = _bf16_bits(np.ones(1, np.float32))[0]
    two = _bf16_bits(np.full(1, 2.0, np.float32))[0]
    return dict(name="preflight_kat", H=8, KVH=1, D=128, N=1, scale=128 ** -0.5,
                q=np.full((1, 8, 128), one, np.uint16),
                k_pool=np.full((1, 16, 1, 128), one, np.uint16),
                v_pool=np.full((1, 16, 1, 128), two, np.uint16),
                k_new=None, v_new=None, block_tables=np.zeros((1, 1), np.int32),
                seq_ids=np.zeros(1, np.int32), positions=np.zeros(1, np.int32),
                slots=None, append=False)


def names() -> list[str]:
    return ["preflight_kat", *CASES]


def as_f32(bits: np.ndarray) -> np.ndarray:
    return _bf16_f32(bits)


def input_digest(inp: dict) -> str:
    h = hashlib.sha256()
    for key in ("q", "k_pool", "v_pool", "k_new", "v_new", "block_tables", "seq_ids",
                "positions", "slots"):
        a = inp[key]
        if a is not None:
            h.update(key.encode())
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
