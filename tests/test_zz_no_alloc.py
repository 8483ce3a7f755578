"""GPU test of ss_ragged_paged_attention_noalloc, the allocation-free entry point.

Callers that cannot allocate device memory around an attention call (code recorded into a
CUDA graph, serving loops with a fixed memory plan, FFI hosts without a caching allocator)
use this entry point; it keeps its split-K scratch in the library's own fixed device array.
The test drives it through the C ABI directly and checks, on two different calls in a row,
that its output matches the ordinary entry point (which takes a caller workspace) within
the attention tolerance used throughout the tests.  The file name makes pytest collect it
last.
"""
import ctypes

import numpy as np
import pytest
import torch

import cases
import shardserve_b200 as sb
from helpers import MAX_ABS_TOL, MEAN_ABS_TOL, bf16_tensor
from shardserve_b200 import _native

pytestmark = pytest.mark.gpu


def _device_inputs(name, dev):
    inp = cases.build(name)
    t = dict(q=bf16_tensor(inp["q"], dev), kp=bf16_tensor(inp["k_pool"], dev),
             vp=bf16_tensor(inp["v_pool"], dev),
             bt=torch.from_numpy(inp["block_tables"]).to(dev),
             seq=torch.from_numpy(inp["seq_ids"]).to(dev),
             pos=torch.from_numpy(np.asarray(inp["positions"])).to(dev, torch.int64))
    if inp["append"]:
        sb.kv_append(t["kp"], t["vp"], bf16_tensor(inp["k_new"], dev),
                     bf16_tensor(inp["v_new"], dev), torch.from_numpy(inp["slots"]).to(dev))
    return inp, t


def _noalloc(t, scale):
    q, kp, vp, bt = t["q"], t["kp"], t["vp"], t["bt"]
    out = torch.empty_like(q)
    s = _native.strides
    rc = _native.lib().ss_ragged_paged_attention_noalloc(
        q.data_ptr(), s(q.stride()), kp.data_ptr(), s(kp.stride()), vp.data_ptr(),
        s(vp.stride()), bt.data_ptr(), s(bt.stride()), bt.shape[0], bt.shape[1], 0,
        t["seq"].data_ptr(), 0, t["pos"].data_ptr(), 1, out.data_ptr(), s(out.stride()),
        q.shape[0], q.shape[1], kp.shape[2], q.shape[2], kp.shape[0], ctypes.c_float(scale),
        torch.cuda.current_stream().cuda_stream)
    assert rc == _native.SS_OK, _native.last_error()
    return out


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    assert torch.cuda.is_available()
    dev = torch.device("cuda", 0)
    for name in ("long_decode", "chunked_mixed"):  # two calls in a row, different shapes
        inp, t = _device_inputs(name, dev)
        want = sb.ragged_attention_direct(t["q"], t["kp"], t["vp"], t["bt"], t["seq"],
                                          t["pos"], inp["scale"])
        got = _noalloc(t, inp["scale"])
        torch.cuda.synchronize()
        err = (got.float() - want.float()).abs()
        assert err.max().item() <= MAX_ABS_TOL
        assert err.mean().item() <= MEAN_ABS_TOL


def test_noalloc_rejects_calls_beyond_its_fixed_scratch():
    assert torch.cuda.is_available()
    dev = torch.device("cuda", 0)
    inp, t = _device_inputs("config1_decode", dev)
    huge = 10 ** 7  # split descriptors alone would need 160 MB
    s = _native.strides
    q = t["q"]
    rc = _native.lib().ss_ragged_paged_attention_noalloc(
        q.data_ptr(), s(q.stride()), t["kp"].data_ptr(), s(t["kp"].stride()),
        t["vp"].data_ptr(), s(t["vp"].stride()), t["bt"].data_ptr(), s(t["bt"].stride()),
        t["bt"].shape[0], t["bt"].shape[1], 0, t["seq"].data_ptr(), 0, t["pos"].data_ptr(), 1,
        q.data_ptr(), s(q.stride()), huge, 16, 2, 128, t["kp"].shape[0], ctypes.c_float(0.1),
        torch.cuda.current_stream().cuda_stream)
    assert rc == _native.SS_ERR_WORKSPACE
    assert "no-allocation" in _native.last_error()
