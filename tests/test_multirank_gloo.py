"""Multi-rank host logic on CPU: two gloo ranks (spawned processes, 127.0.0.1 rendezvous).

* Request sharding: each rank takes its `shard_requests` share of a ragged decode batch,
  builds its own pool/tables for those requests and computes attention (CPU oracle); the
  gathered per-rank outputs equal the single-rank result, and the shards' total contexts are
  balanced.
* TP2 head split (the reference's layout, docs/implementation.md:15): rank r computes query
  heads [8r, 8r+8) against KV head r; concatenating the ranks' heads equals full attention.
* The timing reduction the benchmark uses (max over ranks) is the MAX all-reduce.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from shardserve_b200.sharding import shard_requests, tp_head_slice


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(lengths, H, KVH, D, seed):
    rng = np.random.default_rng(seed)
    pages = [-(-L // 16) for L in lengths]
    N = sum(pages) + 8
    perm = rng.permutation(N - 8).astype(np.int32)
    bt = np.zeros((len(lengths), max(pages)), np.int32)
    off = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[off:off + n]
        off += n
    f = lambda *s: oracle.bf16_round(rng.standard_normal(s, dtype=np.float32))
    return dict(kp=f(N, 16, KVH, D), vp=f(N, 16, KVH, D), bt=bt,
                pos=np.asarray(lengths, np.int64) - 1, seq=np.arange(len(lengths), dtype=np.int32))


def _worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths = [int(x) for x in np.random.default_rng(5).integers(16, 700, 24)]
        shards = shard_requests(lengths, world)
        mine = shards[rank]
        # Request-sharded: this rank's requests only, in its own pool.
        my_len = [lengths[i] for i in mine]
        b = _batch(my_len, 16, 2, 64, seed=100 + rank)
        q = oracle.bf16_round(np.random.default_rng([7, rank]).standard_normal(
            (len(mine), 16, 64), dtype=np.float32))
        out = oracle.ragged_attention(q, b["kp"], b["vp"], b["bt"], b["seq"], b["pos"], 0.125)
        # Local check against the same requests computed one at a time (independence).
        for j in range(len(mine)):
            one = oracle.ragged_attention(q[j:j + 1], b["kp"], b["vp"], b["bt"][j:j + 1],
                                          np.zeros(1, np.int32), b["pos"][j:j + 1], 0.125)
            assert np.array_equal(one[0], out[j])
        loads = [None] * world
        dist.all_gather_object(loads, sum(my_len))
        # TP2 head split of one shared batch (same seed on both ranks).
        full = _batch(lengths[:6], 16, 2, 64, seed=42)
        qf = oracle.bf16_round(np.random.default_rng(43).standard_normal((6, 16, 64), dtype=np.float32))
        hs, ks = tp_head_slice(rank, world, 16, 2)
        part = oracle.ragged_attention(qf[:, hs], full["kp"][:, :, ks], full["vp"][:, :, ks],
                                       full["bt"], full["seq"], full["pos"], 0.125)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        t = torch.tensor([float(rank + 1) * 1.5], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            ref = oracle.ragged_attention(qf, full["kp"], full["vp"], full["bt"], full["seq"],
                                          full["pos"], 0.125)
            np.save(result_path, dict(loads=loads, tp_equal=bool(
                np.allclose(np.concatenate(parts, axis=1), ref, atol=1e-6, rtol=0)),
                tmax=float(t.item()), shards=shards), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks(tmp_path):
    if not dist.is_gloo_available():
        pytest.skip("gloo backend missing")
    path = str(tmp_path / "result.npy")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, start_method="spawn",
                       join=True)
    r = np.load(path, allow_pickle=True).item()
    assert sorted(i for s in r["shards"] for i in s) == list(range(24))
    assert max(r["loads"]) <= 1.1 * min(r["loads"])
    assert r["tp_equal"]
    assert r["tmax"] == 3.0


def test_shard_requests_partitions_and_balances():
    lengths = list(np.random.default_rng(3).integers(128, 4097, 512))
    for world in (1, 2, 4, 8):
        shards = shard_requests(lengths, world)
        assert sorted(i for s in shards for i in s) == list(range(512))
        loads = [sum(lengths[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(lengths)
    with pytest.raises(ValueError):
        shard_requests(lengths, 0)
    assert tp_head_slice(1, 2, 16, 2) == (slice(8, 16), slice(1, 2))
    with pytest.raises(ValueError):
        tp_head_slice(0, 2, 16, 1)
