"""CUDA-graph decode buckets above the reference's 8 rows (DecodeGraphs, shardserve/runtime.py:
51-80, extended to 64 and 256): replaying a bucket after its static metadata is rebuilt in
place gives the same bits as running the same step eagerly with the same padded metadata,
and within the attention tolerance of the unpadded eager step; the KV appends land in the
same slots; padding rows touch only scratch pages."""
import random

import pytest
import torch

import shardserve_b200 as sb
from helpers import MAX_ABS_TOL, MEAN_ABS_TOL, page_allocator
from shardserve_b200.graphs import DecodeGraphs

pytestmark = pytest.mark.gpu
LAYERS, H, KVH, D, VOCAB, CONTEXT = 2, 16, 2, 128, 1000, 4096


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


def _setup(dev, blocks=16000, scratch=256):
    c = dict(num_hidden_layers=LAYERS, num_key_value_heads=KVH, hidden_size=H * D,
             num_attention_heads=H)
    cache = sb.Cache(c, 1, blocks, dev, torch.bfloat16, allocator=page_allocator(),
                     scratch_pages=scratch)
    g = torch.Generator(device=dev).manual_seed(5)
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    emb = [(torch.randn(VOCAB, n * D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
           for n in (H, KVH, KVH)]

    def forward(ids, positions, tables, seqs, slots):
        outs = []
        for layer in range(LAYERS):
            T = ids.numel()
            q = emb[0][ids].view(T, H, D) + layer
            k = emb[1][ids].view(T, KVH, D) - layer
            v = emb[2][ids].view(T, KVH, D)
            cache.write(layer, k, v, slots)
            outs.append(sb.ragged_attention_direct(q, cache.k[layer], cache.v[layer], tables,
                                                   seqs, positions, D ** -0.5))
        return torch.stack(outs)

    return cache, forward


def _plan(rnd, cache, n, step):
    rows = []
    for i in range(n):
        key = f"r{i}"
        if key not in cache.blocks.tables:
            cache.blocks.reserve({key: rnd.randint(64, 1800) + 64})
        ctx = len(cache.blocks.tables[key]) * 16 - 64 + step  # a decode position inside
        rows.append(dict(request_id=key, tokens=[rnd.randint(1, VOCAB - 1)], context=ctx,
                         positions=[ctx], offset=i, query_length=1, sample=True))
    return {"rows": rows}


@pytest.mark.parametrize("rows,size", [(40, 64), (200, 256)])
def test_bucket_replay_equals_eager(dev, rows, size):
    cache, forward = _setup(dev)
    meta = sb.DeviceMetadata(cache.blocks, dev, CONTEXT)
    graphs = DecodeGraphs(forward, meta, dev, cache.shape[1], sizes=(16, 64, 256))
    assert graphs.bucket(rows) == size and graphs.captures == 3
    rnd = random.Random(rows)
    for step in range(2):  # two replays with different metadata in the same static tensors
        plan = _plan(rnd, cache, rows, step)
        k_before = cache.k.clone()
        out = graphs.run(plan)
        torch.cuda.synchronize()
        got = out[:, :rows].clone()
        k_graph = cache.k.clone()
        # The same step eagerly with the same padded metadata: the same launches, same bits.
        cache.k.copy_(k_before)
        data = meta.build(plan, size)
        data.pop("selected")
        eager_padded = forward(**data)
        assert torch.equal(eager_padded[:, :rows], got)
        assert torch.equal(cache.k, k_graph)
        # Unpadded eager step: within the attention tolerance (another split-K partition).
        data = meta.build(plan)
        data.pop("selected")
        eager = forward(**data)
        err = (eager.float() - got.float()).abs()
        assert err.max().item() <= MAX_ABS_TOL and err.mean().item() <= MEAN_ABS_TOL
        # Padding rows wrote only into scratch pages (after the allocator's pages).
        changed = (cache.k != k_before).flatten(2).any(-1).any(0).nonzero().flatten()
        real = {p for r in plan["rows"] for p in cache.blocks.tables[r["request_id"]]}
        assert all(int(p) in real or int(p) >= cache.blocks.count for p in changed)
    graphs.close()


def test_bucket_needs_scratch_pages(dev):
    cache, forward = _setup(dev, blocks=512, scratch=8)
    meta = sb.DeviceMetadata(cache.blocks, dev, CONTEXT)
    with pytest.raises(sb.KernelUnsupported):
        DecodeGraphs(forward, meta, dev, cache.shape[1], sizes=(64,))
