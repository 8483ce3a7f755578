"""CPU oracle for the ShardServe attention hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this module, and only as the checker (or, in bench.py, as the timed CPU baseline).  The
product path (shardserve_b200) never calls it.

It restates, in numpy, the reference's own algorithm:

* `kv_append`        — Cache.write, shardserve/cache.py:47-49: `pool.flatten(0, 1)` indexed
                       by int64 slots receives k / v rows (index_copy_).  Bit-exact.
* `ragged_attention` — the Triton kernel shardserve/kernel.py:115-166 and the diagnostic
                       path shardserve/cache.py:51-61.  For each query token t:
                         seq = query_seq_ids[t], L = positions[t] + 1       (kernel.py:117-119)
                         key i in [0, L) lives at slot table[seq, i // 16] * 16 + i % 16
                                                                       (cache.py:55-56,
                                                                        kernel.py:130-141)
                         query head h reads KV head h // (H / KVH)         (kernel.py:120;
                                                                        repeat_interleave,
                                                                        cache.py:57-58)
                         s = q . k * sm_scale in fp32                      (kernel.py:143)
                         out = softmax(s) . v, fp32 probabilities         (kernel.py:146-162)
                       The online softmax of the kernel equals the plain softmax used here
                       up to rounding; probabilities stay fp32 as in the Triton kernel (the
                       diagnostic path rounds them to the pool dtype, cache.py:60, which only
                       matters for bf16 pools).

Parity of this restatement is pinned against vectors produced by the reference itself
(the Triton kernel under TRITON_INTERPRET=1 and Cache.write + Cache.diagnostic), stored in
tests/golden/*.npz by tests/golden/make_golden.py and checked in tests/test_oracle_golden.py.
"""
from __future__ import annotations

import concurrent.futures as _cf
import os

import numpy as np

BLOCK = 16


# ---- bf16 helpers (round-to-nearest-even, as torch's float->bfloat16 conversion) ------
def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(bf16_bits(x))


# ---- append ---------------------------------------------------------------------------
def kv_append(k_pool: np.ndarray, v_pool: np.ndarray, k: np.ndarray, v: np.ndarray,
              slots: np.ndarray) -> None:
    """In-place slot-mapped append (cache.py:47-49).  Works on any dtype (bit copies)."""
    n, blk, kvh, d = k_pool.shape
    assert blk == BLOCK
    flat_k = k_pool.reshape(n * blk, kvh, d)
    flat_v = v_pool.reshape(n * blk, kvh, d)
    s = np.asarray(slots, dtype=np.int64)
    flat_k[s] = k
    flat_v[s] = v


def token_slots(block_tables: np.ndarray, seq: int, length: int) -> np.ndarray:
    """Slots of keys 0..length-1 of row `seq` (cache.py:55-56)."""
    i = np.arange(length, dtype=np.int64)
    return block_tables[seq, i // BLOCK].astype(np.int64) * BLOCK + i % BLOCK


def _attend_tokens(q, k_flat, v_flat, block_tables, seqs, positions, sm_scale, tokens, out,
                   acc_dtype):
    H = q.shape[1]
    KVH = k_flat.shape[1]
    G = H // KVH
    for t in tokens:
        L = int(positions[t]) + 1
        if L <= 0:
            out[t] = 0.0
            continue
        sl = token_slots(block_tables, int(seqs[t]), L)
        kk = k_flat[sl].astype(acc_dtype)  # [L, KVH, D]
        vv = v_flat[sl].astype(acc_dtype)
        qg = q[t].astype(acc_dtype).reshape(KVH, G, -1)  # [KVH, G, D]
        s = np.matmul(qg, kk.transpose(1, 2, 0)) * acc_dtype(sm_scale)  # [KVH, G, L]
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        o = np.matmul(p, vv.transpose(1, 0, 2))  # [KVH, G, D]
        out[t] = o.reshape(H, -1)


def ragged_attention(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray,
                     block_tables: np.ndarray, query_seq_ids: np.ndarray,
                     positions: np.ndarray, sm_scale: float, acc_dtype=np.float32,
                     threads: int = 1) -> np.ndarray:
    """Reference attention for a flat ragged batch; inputs are float arrays holding the
    bf16-rounded values.  Returns [T, H, D] in `acc_dtype`."""
    T, H, D = q.shape
    n, blk, kvh, d = k_pool.shape
    assert blk == BLOCK and d == D and H % kvh == 0
    k_flat = k_pool.reshape(n * blk, kvh, d)
    v_flat = v_pool.reshape(n * blk, kvh, d)
    out = np.zeros((T, H, D), dtype=acc_dtype)
    if threads <= 1:
        _attend_tokens(q, k_flat, v_flat, block_tables, query_seq_ids, positions, sm_scale,
                       range(T), out, acc_dtype)
        return out
    chunks = [range(i, T, threads) for i in range(threads)]
    with _cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda c: _attend_tokens(q, k_flat, v_flat, block_tables, query_seq_ids,
                                             positions, sm_scale, c, out, acc_dtype), chunks))
    return out


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
