"""kv_append_attention (ss_append_ragged_paged_attention): Cache.write + ragged_attention_direct
in one call, the append folded into the decode kernel for decode-only launches.

It must give the bits of the two separate calls — the outputs and the appended pools — on
decode steps (batch-64 and TP2 shapes, head_dim 64, a sequence with two query tokens in a
decode-only launch), fall back to the append kernel on batches with chunked-prefill runs, flag
a slot that is not the token's own position, and replay from a CUDA graph.  Reference:
shardserve/model.py:32-37, cache.py:47-49, runtime.py:38.
"""
import numpy as np
import pytest
import torch

import cases
import oracle
import shardserve_b200 as sb
from helpers import MAX_ABS_TOL, MEAN_ABS_TOL, bf16_tensor, load_golden, oracle_inputs
from shardserve_b200 import kernel as K
from shardserve_b200.workloads import ragged_batch, uniform_lengths

pytestmark = pytest.mark.gpu
SCALE = 128 ** -0.5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


def both(b, scale=SCALE):
    """(fused output, fused pools, separate output, separate pools, fused path)."""
    kp, vp = b.k_pool.clone(), b.v_pool.clone()
    fused = sb.kv_append_attention(kp, vp, b.k_new, b.v_new, b.slots, b.q, b.block_tables,
                                   b.seq_ids, b.positions, scale)
    path = K.last_attention_path()
    kp2, vp2 = b.k_pool.clone(), b.v_pool.clone()
    sb.kv_append(kp2, vp2, b.k_new, b.v_new, b.slots)
    sep = sb.ragged_attention_direct(b.q, kp2, vp2, b.block_tables, b.seq_ids, b.positions, scale)
    torch.cuda.synchronize()
    return fused, (kp, vp), sep, (kp2, vp2), path


@pytest.mark.parametrize("n,lo,hi,H,KVH,D", [
    (64, 128, 4096, 16, 2, 128),   # batch-64 decode step
    (8, 16384, 32768, 8, 1, 128),  # TP2 per-rank heads, long contexts
    (33, 1, 700, 16, 4, 64),       # head_dim 64, two KV-head blocks, pages ending anywhere
])
def test_fused_append_matches_separate_calls(dev, n, lo, hi, H, KVH, D):
    lengths = uniform_lengths(n, lo, hi, n + lo)
    b = ragged_batch([(L - 1, 1) for L in lengths], H, KVH, D, seed=n, device=dev)
    K.device_errors(dev, clear=True)
    fused, pf, sep, ps, path = both(b, D ** -0.5)
    assert path == 4, "the append was not folded into the decode kernel"
    assert torch.equal(fused, sep)
    assert torch.equal(pf[0], ps[0]) and torch.equal(pf[1], ps[1])
    assert K.device_errors(dev) == 0


def test_fused_append_with_two_tokens_of_one_sequence(dev):
    """A decode-only launch (tokens <= table rows) holding two consecutive positions of one
    sequence: the second token attends to the first one's new row."""
    rows = [(40, 2), (100, 1), (15, 1), (300, 0 + 1)]
    b = ragged_batch(rows, 16, 2, 128, seed=9, device=dev)
    pad = torch.zeros(2, b.block_tables.shape[1], dtype=b.block_tables.dtype, device=dev)
    b.block_tables = torch.cat([b.block_tables, pad])  # more table rows than query tokens
    assert b.tokens <= b.block_tables.shape[0]
    fused, pf, sep, ps, path = both(b)
    assert path == 4
    assert torch.equal(fused, sep)
    assert torch.equal(pf[0], ps[0]) and torch.equal(pf[1], ps[1])
    f = lambda x: x.float().cpu().numpy()
    ref = oracle.ragged_attention(f(b.q), f(ps[0]), f(ps[1]), b.block_tables.cpu().numpy(),
                                  b.seq_ids.cpu().numpy(), b.positions.cpu().numpy(), SCALE)
    err = np.abs(f(fused) - ref)
    assert err.max() <= MAX_ABS_TOL and err.mean() <= MEAN_ABS_TOL


def test_fused_append_falls_back_on_prefill_runs(dev):
    b = ragged_batch([(500, 1), (20, 100), (1000, 1)], 16, 2, 128, seed=10, device=dev)
    fused, pf, sep, ps, path = both(b)
    assert path == 3
    assert torch.equal(fused, sep)
    assert torch.equal(pf[0], ps[0])


@pytest.mark.parametrize("name", ["config1_decode", "tp2_decode", "d64_group4"])
def test_fused_append_against_reference_vectors(dev, name):
    inp = cases.build(name)
    want, _ = load_golden(name)
    q, kp, vp = (bf16_tensor(inp[x], dev) for x in ("q", "k_pool", "v_pool"))
    out = sb.kv_append_attention(kp, vp, bf16_tensor(inp["k_new"], dev),
                                 bf16_tensor(inp["v_new"], dev),
                                 torch.from_numpy(inp["slots"]).to(dev), q,
                                 torch.from_numpy(inp["block_tables"]).to(dev),
                                 torch.from_numpy(inp["seq_ids"]).to(dev),
                                 torch.from_numpy(np.asarray(inp["positions"])).to(dev),
                                 inp["scale"])
    err = np.abs(out.float().cpu().numpy() - want)
    assert err.max() <= MAX_ABS_TOL and err.mean() <= MEAN_ABS_TOL
    q32, k32, v32 = oracle_inputs(inp)
    ref = oracle.ragged_attention(q32, k32, v32, inp["block_tables"], inp["seq_ids"],
                                  inp["positions"], inp["scale"])
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= MAX_ABS_TOL and err.mean() <= MEAN_ABS_TOL


def test_fused_append_flags_a_slot_off_the_tokens_position(dev):
    lengths = uniform_lengths(16, 100, 900, 3)
    b = ragged_batch([(L - 1, 1) for L in lengths], 16, 2, 128, seed=11, device=dev)
    slots = b.slots.clone()
    slots[3] = slots[3] + 1 if int(b.positions[3]) % 16 != 15 else slots[3] - 1
    K.device_errors(dev, clear=True)
    sb.kv_append_attention(b.k_pool, b.v_pool, b.k_new, b.v_new, slots, b.q, b.block_tables,
                           b.seq_ids, b.positions, SCALE)
    assert K.device_errors(dev) & 0x8


def test_fused_append_replays_from_a_cuda_graph(dev):
    lengths = uniform_lengths(64, 128, 4096, 12)
    b = ragged_batch([(L - 1, 1) for L in lengths], 16, 2, 128, seed=12, device=dev)
    kp0, vp0 = b.k_pool.clone(), b.v_pool.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            sb.kv_append_attention(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots, b.q,
                                   b.block_tables, b.seq_ids, b.positions, SCALE)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = sb.kv_append_attention(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots, b.q,
                                     b.block_tables, b.seq_ids, b.positions, SCALE)
    b.k_pool.copy_(kp0)
    b.v_pool.copy_(vp0)
    b.q.copy_(torch.randn_like(b.q.float()).to(torch.bfloat16))
    g.replay()
    torch.cuda.synchronize()
    kp2, vp2 = kp0.clone(), vp0.clone()
    sb.kv_append(kp2, vp2, b.k_new, b.v_new, b.slots)
    want = sb.ragged_attention_direct(b.q, kp2, vp2, b.block_tables, b.seq_ids, b.positions,
                                      SCALE)
    assert torch.equal(out, want)
    assert torch.equal(b.k_pool, kp2)
