"""GPU test of ss_ragged_paged_attention_noalloc, the allocation-free entry point.

Callers that cannot allocate device memory around an attention call (code recorded into a
CUDA graph, where cudaMalloc is not allowed; serving loops with a fixed memory plan, where
an allocation can stall the device; FFI hosts without a caching allocator to keep a
workspace alive) use this entry point: it keeps its split-K scratch in the library's own
fixed device array.  The test drives it through the C ABI directly, on two different calls
in a row, and checks that its output is bit-identical to the ordinary entry point (which
takes a caller workspace and runs the same kernels on the same inputs) and within the
attention tolerance of the CPU oracle; that the fast kernels ran; that the error word of
the fixed scratch reports an out-of-range page through ss_noalloc_fetch_device_errors; and
that calls beyond the fixed scratch are rejected.  The file name makes pytest collect it
last.
"""
import ctypes

import numpy as np
import pytest
import torch

import cases
import oracle
import shardserve_b200 as sb
from helpers import MAX_ABS_TOL, MEAN_ABS_TOL, bf16_tensor, oracle_inputs
from shardserve_b200 import _native
from shardserve_b200 import kernel as K

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


def _noalloc(t, scale, bt=None):
    q, kp, vp = t["q"], t["kp"], t["vp"]
    bt = t["bt"] if bt is None else bt
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


def _noalloc_errors(dev, clear=True):
    flags = ctypes.c_uint32(0)
    rc = _native.lib().ss_noalloc_fetch_device_errors(
        dev.index, int(clear), ctypes.byref(flags), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _native.SS_OK, _native.last_error()
    return flags.value


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    assert torch.cuda.is_available()
    dev = torch.device("cuda", 0)
    # The first call on a device resolves the scratch address; it must come before any
    # stream capture, which this test does not do.
    for name in ("long_decode", "chunked_mixed"):  # two calls in a row, different shapes
        inp, t = _device_inputs(name, dev)
        want = sb.ragged_attention_direct(t["q"], t["kp"], t["vp"], t["bt"], t["seq"],
                                          t["pos"], inp["scale"])
        path = K.last_attention_path()
        got = _noalloc(t, inp["scale"])
        torch.cuda.synchronize()
        assert _native.lib().ss_last_attention_path() == path
        assert path in (1, 3), "the TMA / tensor-core kernels did not run"
        # Same kernels, same inputs, same launch shapes: the same bits.
        assert torch.equal(got, want)
        q, kp, vp = oracle_inputs(inp)
        ref = oracle.ragged_attention(q, kp, vp, inp["block_tables"], inp["seq_ids"],
                                      inp["positions"], inp["scale"])
        err = np.abs(got.float().cpu().numpy() - ref)
        assert err.max() <= MAX_ABS_TOL, err.max()
        assert err.mean() <= MEAN_ABS_TOL, err.mean()
    assert _noalloc_errors(dev) == 0


def test_noalloc_error_word_reports_a_page_outside_the_pool():
    assert torch.cuda.is_available()
    dev = torch.device("cuda", 0)
    inp, t = _device_inputs("config1_decode", dev)
    _noalloc(t, inp["scale"])
    _noalloc_errors(dev, clear=True)
    bt = t["bt"].clone()
    bt[0, 0] = t["kp"].shape[0] + 1000  # outside the pool: the page reads as zeros
    _noalloc(t, inp["scale"], bt=bt)
    _noalloc(t, inp["scale"])  # a clean call after it keeps the bit
    assert _noalloc_errors(dev, clear=True) & _native.SS_DEVERR_PAGE
    assert _noalloc_errors(dev) == 0


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
