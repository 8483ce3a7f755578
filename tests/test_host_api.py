"""The Python boundary mirrors the reference wrapper's validation (shardserve/kernel.py:28-49)
and fails loudly without CUDA instead of falling back to a CPU path."""
import pytest
import torch

import shardserve_b200 as sb
from shardserve_b200 import kernel as K
from helpers import FreeListPages, reference_blocks
from shardserve_b200.cache import Cache, default_allocator


def _args(**over):
    a = dict(q=torch.zeros(2, 8, 128, dtype=torch.bfloat16),
             k=torch.zeros(4, 16, 1, 128, dtype=torch.bfloat16),
             v=torch.zeros(4, 16, 1, 128, dtype=torch.bfloat16),
             bt=torch.zeros(2, 1, dtype=torch.int32), seq=torch.zeros(2, dtype=torch.int32),
             pos=torch.zeros(2, dtype=torch.int64))
    a.update(over)
    return a


def _call(a):
    return sb.ragged_attention_direct(a["q"], a["k"], a["v"], a["bt"], a["seq"], a["pos"], 0.1)


def test_same_names_as_reference():
    assert issubclass(sb.KernelUnsupported, ValueError)
    assert sb.SUPPORTED_RAGGED_HEAD_DIMS == (64, 128)
    assert sb.SUPPORTED_BLOCK_SIZE == 16


@pytest.mark.parametrize("over,msg", [
    ({}, "ragged kernel requires BF16 CUDA queries"),
    (dict(q=torch.zeros(2, 8, 128)), "ragged kernel requires BF16 CUDA queries"),
])
def test_cpu_or_fp32_query_is_rejected_like_the_reference(over, msg):
    with pytest.raises(sb.KernelUnsupported, match=msg):
        _call(_args(**over))


def test_no_cpu_fallback_for_append():
    a = _args()
    with pytest.raises(sb.KernelUnsupported):
        sb.kv_append(a["k"][:, :, :, :], a["v"], torch.zeros(2, 1, 128, dtype=torch.bfloat16),
                     torch.zeros(2, 1, 128, dtype=torch.bfloat16), torch.zeros(2, dtype=torch.int64))


def test_cache_refuses_cpu_pools():
    c = dict(num_hidden_layers=2, num_key_value_heads=2, hidden_size=32, num_attention_heads=4)
    with pytest.raises(sb.KernelUnsupported):
        Cache(c, 1, 8, "cpu", torch.float32)


def test_cache_uses_the_engines_own_page_allocator():
    """The drop-in Cache keeps no allocator of its own: Cache.blocks is the reference's
    Blocks (cache.py:6-35) or the class the engine passes."""
    Blocks = reference_blocks()
    if Blocks is None:
        pytest.skip("the reference package is not installed here")
    assert default_allocator() is Blocks
    # The reference allocator's free-list order, which the block tables (and so the
    # slot/table parity fixtures) follow: pages come off the end of the free list.
    b = Blocks(4)
    b.reserve({"a": 17})
    assert b.tables["a"] == [3, 2]
    with pytest.raises(MemoryError):
        b.reserve({"b": 33, "c": 1})
    b.release("a")
    b.check()


def test_free_list_stand_in_matches_the_reference_order():
    Blocks = reference_blocks()
    if Blocks is None:
        pytest.skip("the reference package is not installed here")
    a, b = Blocks(64), FreeListPages(64)
    for step, req in enumerate([{"x": 17}, {"y": 100, "z": 1}, {"w": 33}]):
        a.reserve(req)
        b.reserve(req)
        if step == 1:
            a.release("x")
            b.release("x")
    assert a.tables == b.tables and a.free == b.free


def test_index_dtype_checked():
    with pytest.raises(sb.KernelUnsupported):
        K._index_flag(torch.zeros(2, dtype=torch.float32), "positions")
    assert K._index_flag(torch.zeros(2, dtype=torch.int64), "positions") == 1
    assert K._index_flag(torch.zeros(2, dtype=torch.int32), "positions") == 0
