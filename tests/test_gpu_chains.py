"""Long chains of calls on one stream, the way a model's layers issue them: RoPE + append
then attention, append then attention, and the fused append + attention, 200 times each on
a batch-256 decode step (context U[512, 8192], 16 q / 2 kv heads).

The decode kernel's split-K merge runs after a grid barrier.  An append kernel that
released the attention kernel early, or a decode grid of another shape, left SMs that could
hold only two attention CTAs, so some CTAs of the next grid were not resident while the
others waited for them.  The barrier now gives up after ~0.5 ms and the call's last arrival
merges for the CTAs that gave up.  These chains check that no call sets a device error and
that the last call's output equals the same call made alone.
Reference composition: shardserve/model.py:25-37 (apply_rope, Cache.write, attention).
"""
import pytest
import torch

import shardserve_b200 as sb
from shardserve_b200 import kernel as K
from shardserve_b200.workloads import ragged_batch, uniform_lengths

pytestmark = pytest.mark.gpu
CALLS = 200
SCALE = 128 ** -0.5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def batch(dev):
    lengths = uniform_lengths(256, 512, 8192, 2024)
    return ragged_batch([(L - 1, 1) for L in lengths], 16, 2, 128, seed=2024, device=dev)


def _attention(b, q):
    return sb.ragged_attention_direct(q, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                      b.positions, SCALE)


@pytest.mark.parametrize("chain", ["rope_append", "kv_append", "fused"])
def test_long_call_chain_never_times_out(dev, batch, chain):
    b = batch
    cos = torch.ones(8192, 128, device=dev)
    sin = torch.zeros(8192, 128, device=dev)  # identity rotation: q, k unchanged
    q = b.q.clone()
    torch.cuda.synchronize()
    K.device_errors(dev, clear=True)
    for _ in range(CALLS):
        if chain == "rope_append":
            sb.rope_kv_append(q, b.k_new, b.v_new, cos, sin, b.positions, b.k_pool, b.v_pool,
                              b.slots, out=q)
            out = _attention(b, q)
        elif chain == "kv_append":
            sb.kv_append(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots)
            out = _attention(b, q)
        else:
            out = sb.kv_append_attention(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots, q,
                                         b.block_tables, b.seq_ids, b.positions, SCALE)
    torch.cuda.synchronize()
    assert K.device_errors(dev, clear=True) == 0
    alone = _attention(b, q)
    torch.cuda.synchronize()
    assert torch.equal(out, alone)


def test_alternating_decode_kernel_shapes_never_time_out(dev, batch):
    """Back-to-back attention calls whose decode grids are different kernel instances (16 q /
    2 kv heads at head_dim 128, the TP2 8 q / 1 kv layout, head_dim 64), each released early
    by the one before it: the chain in which some grids are not fully resident and their
    barrier waiters give up, so the call's last arrival merges every item."""
    tp2 = ragged_batch([(L - 1, 1) for L in uniform_lengths(16, 4096, 16384, 7)], 8, 1, 128,
                       seed=7, device=dev)
    d64 = ragged_batch([(L - 1, 1) for L in uniform_lengths(64, 128, 4096, 8)], 16, 4, 64,
                       seed=8, device=dev)
    calls = [(batch, SCALE), (tp2, SCALE), (d64, 64 ** -0.5)]

    def call(i):
        b, scale = calls[i]
        return sb.ragged_attention_direct(b.q, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                          b.positions, scale)

    alone = []
    for i in range(len(calls)):  # each call made alone (the stream drained around it)
        torch.cuda.synchronize()
        alone.append(call(i))
        torch.cuda.synchronize()
    K.device_errors(dev, clear=True)
    # Every call of the chain, including any whose barrier waiters gave up and whose last
    # arrival merged every item, must give the lone call's bits (compared on the device).
    differs = torch.zeros((), dtype=torch.bool, device=dev)
    for _ in range(CALLS):
        for i in range(len(calls)):
            differs |= (call(i) != alone[i]).any()
    torch.cuda.synchronize()
    assert K.device_errors(dev, clear=True) == 0
    assert not differs.item()
