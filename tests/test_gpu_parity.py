"""GPU parity: the sm_100a kernels (called through the C ABI) against the reference.

* append: bit-exact against the reference's Cache.write (fixture SHA-256 of the pools);
* attention: max-abs <= 2e-2 and mean-abs <= 2e-3 (bf16 output vs fp32 reference) against
  the reference Triton kernel's own output (fixtures) and the CPU oracle.
"""
import numpy as np
import pytest
import torch

import cases
import oracle
import shardserve_b200 as sb
from helpers import (MAX_ABS_TOL, MEAN_ABS_TOL, bf16_tensor, bits_of, load_golden,
                     oracle_inputs, page_allocator)
from shardserve_b200 import kernel as K

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


def to_device(inp, dev, pos_dtype=torch.int64, seq_dtype=torch.int32, bt_dtype=torch.int32):
    t = dict(
        q=bf16_tensor(inp["q"], dev),
        kp=bf16_tensor(inp["k_pool"], dev),
        vp=bf16_tensor(inp["v_pool"], dev),
        bt=torch.from_numpy(inp["block_tables"]).to(dev, bt_dtype),
        seq=torch.from_numpy(inp["seq_ids"]).to(dev, seq_dtype),
        pos=torch.from_numpy(np.asarray(inp["positions"])).to(dev, pos_dtype),
    )
    if inp["append"]:
        t["k_new"] = bf16_tensor(inp["k_new"], dev)
        t["v_new"] = bf16_tensor(inp["v_new"], dev)
        t["slots"] = torch.from_numpy(inp["slots"]).to(dev)
    return t


def expected_path(inp):
    """2: generic kernel; 3: split-K + tcgen05 prefill tiles (more tokens than rows, 8 query
    heads per KV head, head_dim 128); 1: split-K only."""
    group = inp["H"] // inp["KVH"]
    if group > 16:
        return 2
    T, B = len(inp["seq_ids"]), inp["block_tables"].shape[0]
    return 3 if (T > B and group == 8 and inp["D"] == 128) else 1


def run(inp, t, q=None, kp=None, vp=None):
    kp = t["kp"] if kp is None else kp
    vp = t["vp"] if vp is None else vp
    if inp["append"]:
        sb.kv_append(kp, vp, t["k_new"], t["v_new"], t["slots"])
    return sb.ragged_attention_direct(t["q"] if q is None else q, kp, vp, t["bt"], t["seq"],
                                      t["pos"], inp["scale"])


def check_close(got, want):
    err = (got.float().cpu().numpy() - want).__abs__()
    assert err.max() <= MAX_ABS_TOL, f"max-abs {err.max():.3e}"
    assert err.mean() <= MEAN_ABS_TOL, f"mean-abs {err.mean():.3e}"
    return err


@pytest.mark.parametrize("name", cases.names())
def test_golden_case(name, dev):
    inp = cases.build(name)
    want, meta = load_golden(name)
    t = to_device(inp, dev, pos_dtype=torch.int32 if name == "preflight_kat" else torch.int64)
    K.device_errors(dev, clear=True)
    out = run(inp, t)
    torch.cuda.synchronize()
    # Append: bit-exact against the reference's Cache.write.
    assert cases.digest(bits_of(t["kp"])) == meta["kpool_sha256"]
    assert cases.digest(bits_of(t["vp"])) == meta["vpool_sha256"]
    # Attention: against the reference kernel's output and against the oracle.
    check_close(out, want)
    q, kp, vp = oracle_inputs(inp)
    ref = oracle.ragged_attention(q, kp, vp, inp["block_tables"], inp["seq_ids"],
                                  inp["positions"], inp["scale"])
    check_close(out, ref)
    assert K.last_attention_path() == expected_path(inp)
    assert K.device_errors(dev) == 0


def test_preflight_known_answer_exact(dev):
    inp = cases.build("preflight_kat")
    t = to_device(inp, dev, pos_dtype=torch.int32)
    out = run(inp, t)
    assert torch.equal(out, torch.full_like(out, 2))


@pytest.mark.parametrize("pos_dtype,seq_dtype,bt_dtype", [
    (torch.int32, torch.int32, torch.int32),
    (torch.int64, torch.int64, torch.int64),
    (torch.int32, torch.int64, torch.int32),
])
def test_index_dtypes_give_identical_results(dev, pos_dtype, seq_dtype, bt_dtype):
    inp = cases.build("chunked_mixed")
    base = run(inp, to_device(inp, dev))
    other = run(inp, to_device(inp, dev, pos_dtype, seq_dtype, bt_dtype))
    assert torch.equal(base, other)


def test_strided_query_output_and_pool_views(dev):
    """Non-contiguous q (a head slice), a pool that is a layer view of a larger cache, and a
    pool with padded KV-head rows: all stay on the TMA path and give the same bits."""
    inp = cases.build("config1_decode")
    t = to_device(inp, dev)
    base = run(inp, t)
    T, H, D = t["q"].shape
    wide = torch.zeros(T, 2 * H, D, dtype=torch.bfloat16, device=dev)
    wide[:, 1::2] = t["q"]
    qv = wide[:, 1::2]
    assert not qv.is_contiguous()
    t2 = to_device(inp, dev)
    layers = torch.zeros((3, *t2["kp"].shape), dtype=torch.bfloat16, device=dev)
    layers[1].copy_(t2["kp"])
    vlayers = torch.zeros_like(layers)
    vlayers[1].copy_(t2["vp"])
    out = run(inp, t2, q=qv, kp=layers[1], vp=vlayers[1])
    assert K.last_attention_path() == expected_path(inp)
    assert torch.equal(out, base)
    t3 = to_device(inp, dev)
    N, P, KVH, _ = t3["kp"].shape
    padk = torch.zeros(N, P, KVH, D + 64, dtype=torch.bfloat16, device=dev)
    padv = torch.zeros_like(padk)
    padk[..., :D] = t3["kp"]
    padv[..., :D] = t3["vp"]
    out3 = run(inp, t3, kp=padk[..., :D], vp=padv[..., :D])
    assert K.last_attention_path() == expected_path(inp)
    assert torch.equal(out3, base)


def test_generic_path_for_non_unit_head_dim_stride(dev):
    inp = cases.build("tp2_decode")
    want, _ = load_golden("tp2_decode")
    t = to_device(inp, dev)
    wide_k = torch.zeros((*t["kp"].shape[:-1], 2 * t["kp"].shape[-1]), dtype=torch.bfloat16,
                         device=dev)
    wide_v = torch.zeros_like(wide_k)
    wide_k[..., ::2] = t["kp"]
    wide_v[..., ::2] = t["vp"]
    kp_t, vp_t = wide_k[..., ::2], wide_v[..., ::2]  # head_dim stride 2
    assert kp_t.stride(-1) == 2
    out = run(inp, t, kp=kp_t, vp=vp_t)
    assert K.last_attention_path() == 2
    check_close(out, want)


@pytest.mark.parametrize("name", ["config1_decode", "tp2_decode"])
def test_generic_path_for_queries_not_16_byte_addressable(dev, name):
    """The split-K kernel reads q rows as 16-byte vectors; a q view that starts one element
    into its buffer (or has odd strides) runs on the generic kernel, same results."""
    inp = cases.build(name)
    want, _ = load_golden(name)
    t = to_device(inp, dev)
    T, H, D = t["q"].shape
    buf = torch.zeros(T * H * D + 1, dtype=torch.bfloat16, device=dev)
    q_off = buf[1:].view(T, H, D)
    q_off.copy_(t["q"])
    assert q_off.data_ptr() % 16 != 0
    out = run(inp, t, q=q_off)
    assert K.last_attention_path() == 2
    check_close(out, want)
    odd = torch.zeros(T, H, D + 1, dtype=torch.bfloat16, device=dev)[..., :D]
    odd.copy_(t["q"])
    assert odd.stride(1) % 8 != 0
    t2 = to_device(inp, dev)
    out2 = run(inp, t2, q=odd)
    assert K.last_attention_path() == 2
    check_close(out2, want)


def test_repeated_calls_are_bitwise_deterministic(dev):
    """The split-K tickets are reset by each call: a second call reuses the workspace."""
    inp = cases.build("long_decode")
    t = to_device(inp, dev)
    a = run(inp, t)
    outs = [sb.ragged_attention_direct(t["q"], t["kp"], t["vp"], t["bt"], t["seq"], t["pos"],
                                       inp["scale"]) for _ in range(3)]
    for o in outs:
        assert torch.equal(o, a)


def test_cuda_graph_capture_and_replay(dev):
    """Capture append + attention like DecodeGraphs (runtime.py:51-80) and replay with new
    metadata copied into the captured buffers."""
    inp = cases.build("graph_padding")
    t = to_device(inp, dev)
    eager = run(inp, to_device(inp, dev))
    static = {k: v.clone() for k, v in t.items()}
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            run(inp, static)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    # Reset the pools, then capture.
    static["kp"].copy_(t["kp"])
    static["vp"].copy_(t["vp"])
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = run(inp, static)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # New step: other queries, same shapes, replayed through the graph.
    q2 = torch.randn_like(t["q"].float()).to(torch.bfloat16)
    static["q"].copy_(q2)
    g.replay()
    torch.cuda.synchronize()
    want = sb.ragged_attention_direct(q2, static["kp"], static["vp"], static["bt"],
                                      static["seq"], static["pos"], inp["scale"])
    assert torch.equal(out, want)


def test_workspace_growth_keeps_a_captured_graphs_buffer_alive(dev):
    """A decode graph is captured, then a larger call grows the per-device workspace (as an
    eager chunked-prefill step after start-up bucket capture does).  The graph still
    replays into the old buffer, so that buffer must stay allocated: a tensor allocated
    after the growth must not receive the graph's writes, and the replay stays correct."""
    from shardserve_b200 import _native

    inp = cases.build("graph_padding")
    eager = run(inp, to_device(inp, dev))
    static = to_device(inp, dev)
    kp0, vp0 = static["kp"].clone(), static["vp"].clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            run(inp, static)
    torch.cuda.current_stream().wait_stream(s)
    static["kp"].copy_(kp0)
    static["vp"].copy_(vp0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = run(inp, static)
    torch.cuda.synchronize()
    old = K.workspace_for(dev)
    old_ptr, old_n = old.data_ptr(), old.numel()
    del old
    # A token count whose workspace need (asked of the library) outgrows the current buffer.
    import ctypes

    tokens, need = 1024, ctypes.c_size_t(0)
    while True:
        assert _native.lib().ss_attention_workspace_bytes(dev.index, tokens, 16, 2, 128,
                                                          ctypes.byref(need)) == _native.SS_OK
        if need.value > old_n:
            break
        tokens *= 2
    _native.ops().ensure_workspace(dev.index, tokens, 16, 2, 128)
    assert K.workspace_for(dev).data_ptr() != old_ptr
    canary = torch.full((old_n,), 0x5A, dtype=torch.uint8, device=dev)
    static["kp"].copy_(kp0)
    static["vp"].copy_(vp0)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert bool((canary == 0x5A).all()), "a graph replay wrote into memory it no longer owns"


def test_out_of_range_metadata_is_flagged_not_faulted(dev):
    inp = cases.build("config1_decode")
    t = to_device(inp, dev)
    run(inp, t)
    torch.cuda.synchronize()
    K.device_errors(dev, clear=True)
    bt = t["bt"].clone()
    bt[0, 0] = 10 ** 6  # page outside the pool: reads as zeros
    sb.ragged_attention_direct(t["q"], t["kp"], t["vp"], bt, t["seq"], t["pos"], inp["scale"])
    assert K.device_errors(dev) & 0x1
    seq = t["seq"].clone()
    seq[1] = 99  # row outside the block table: zero output
    out = sb.ragged_attention_direct(t["q"], t["kp"], t["vp"], t["bt"], seq, t["pos"],
                                     inp["scale"])
    assert K.device_errors(dev) & 0x2
    assert torch.count_nonzero(out[1]) == 0
    pos = t["pos"].clone()
    pos[2] = 16 * t["bt"].shape[1] + 5  # past the table width: clamped
    sb.ragged_attention_direct(t["q"], t["kp"], t["vp"], t["bt"], t["seq"], pos, inp["scale"])
    assert K.device_errors(dev) & 0x4
    slots = torch.tensor([10 ** 9], device=dev)
    before = t["kp"].clone()
    sb.kv_append(t["kp"], t["vp"], t["k_new"][:1], t["v_new"][:1], slots)
    assert K.device_errors(dev) & 0x8
    assert torch.equal(before, t["kp"])


def _big_decode(dev, n_seq, lo, hi, H, KVH, seed):
    """Config-2-style batch: contexts U[lo, hi], scattered pages, N(0,1) bf16."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    L = torch.randint(lo, hi + 1, (n_seq,), generator=g)
    pages = (L + 15) // 16
    N = int(pages.sum().item() * 1.1) + 8
    perm = torch.randperm(N - 8, generator=g).to(torch.int32)
    W = int(pages.max())
    bt = torch.zeros(n_seq, W, dtype=torch.int32)
    off = 0
    for i in range(n_seq):
        bt[i, :pages[i]] = perm[off:off + pages[i]]
        off += int(pages[i])
    kp = torch.randn(N, 16, KVH, 128, generator=g).to(torch.bfloat16)
    vp = torch.randn(N, 16, KVH, 128, generator=g).to(torch.bfloat16)
    q = torch.randn(n_seq, H, 128, generator=g).to(torch.bfloat16)
    pos = (L - 1).to(torch.int64)
    seq = torch.arange(n_seq, dtype=torch.int32)
    return dict(q=q, kp=kp, vp=vp, bt=bt, seq=seq, pos=pos)


@pytest.mark.parametrize("n_seq,lo,hi,H,KVH", [
    (64, 128, 4096, 16, 2),      # batch-64 decode, contexts U[128, 4096]
    (8, 16384, 32768, 8, 1),     # TP2 long-context layout (per rank: 8 q heads, 1 kv head)
    (256, 1, 300, 16, 2),        # many short rows
    (40000, 1, 16, 16, 2),       # one-page rows: ~90 rows per CTA, more than its row table
])
def test_full_size_decode_against_oracle(dev, n_seq, lo, hi, H, KVH):
    c = _big_decode(dev, n_seq, lo, hi, H, KVH, seed=n_seq + lo)
    d = {k: v.to(dev) for k, v in c.items()}
    out = sb.ragged_attention_direct(d["q"], d["kp"], d["vp"], d["bt"], d["seq"], d["pos"],
                                     128 ** -0.5)
    assert K.last_attention_path() == 1
    f = lambda x: x.float().numpy()
    ref = oracle.ragged_attention(f(c["q"]), f(c["kp"]), f(c["vp"]), c["bt"].numpy(),
                                  c["seq"].numpy(), c["pos"].numpy(), 128 ** -0.5,
                                  threads=oracle.host_threads())
    check_close(out, ref)
    assert K.device_errors(dev) == 0


def test_full_size_properties(dev):
    """Size-independent checks at batch 64 x U[128, 4096]: relocating every page (same
    contents, new block table) changes no bit, and doubling V doubles the output exactly."""
    c = _big_decode(dev, 64, 128, 4096, 16, 2, seed=7)
    d = {k: v.to(dev) for k, v in c.items()}
    base = sb.ragged_attention_direct(d["q"], d["kp"], d["vp"], d["bt"], d["seq"], d["pos"],
                                      128 ** -0.5)
    N = d["kp"].shape[0]
    perm = torch.randperm(N, device=dev)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(N, device=dev)
    kp2, vp2 = d["kp"][perm], d["vp"][perm]  # page p moves to index inv[p]
    bt2 = inv[d["bt"].long()].to(torch.int32)
    moved = sb.ragged_attention_direct(d["q"], kp2, vp2, bt2, d["seq"], d["pos"], 128 ** -0.5)
    assert torch.equal(moved, base)
    doubled = sb.ragged_attention_direct(d["q"], d["kp"], d["vp"] * 2, d["bt"], d["seq"],
                                         d["pos"], 128 ** -0.5)
    assert torch.equal(doubled, base * 2)


def test_cache_object_matches_reference_layout(dev):
    c = dict(num_hidden_layers=3, num_key_value_heads=2, hidden_size=2048, num_attention_heads=16)
    cache = sb.Cache(c, 1, 64, dev, torch.bfloat16, allocator=page_allocator())
    assert cache.shape == (3, 72, 16, 2, 128)
    inp = cases.build("config1_decode")
    t = to_device(inp, dev)
    cache.write(1, t["k_new"], t["v_new"], t["slots"])
    flat = cache.k[1].flatten(0, 1)
    assert torch.equal(flat[t["slots"]], t["k_new"])
    assert torch.count_nonzero(cache.k[0]) == 0 and torch.count_nonzero(cache.k[2]) == 0


def test_mixed_geometries_share_one_workspace(dev):
    """Calls with different token counts, head layouts and head dims reuse the per-device
    workspace in any order: the ticket region never aliases another call's partial states."""
    order = ["chunked_mixed", "tp2_chunk_long", "config1_decode", "d64_group4",
             "tp2_chunk_long", "mha_d64", "chunked_mixed", "long_decode", "tp2_chunk_long"]
    for name in order:
        inp = cases.build(name)
        want, _ = load_golden(name)
        check_close(run(inp, to_device(inp, dev)), want)


def _ragged_rows_case(dev, rows, H, KVH, seed):
    """Device + oracle inputs for (cached context, query tokens) rows, appended first."""
    from shardserve_b200.workloads import ragged_batch

    b = ragged_batch(rows, H, KVH, 128, seed=seed, device=dev)
    sb.kv_append(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots)
    out = sb.ragged_attention_direct(b.q, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                     b.positions, 128 ** -0.5)
    path = K.last_attention_path()
    f = lambda x: x.float().cpu().numpy()
    ref = oracle.ragged_attention(f(b.q), f(b.k_pool), f(b.v_pool), b.block_tables.cpu().numpy(),
                                  b.seq_ids.cpu().numpy(), b.positions.cpu().numpy(), 128 ** -0.5,
                                  threads=oracle.host_threads())
    return out, ref, path


def test_prefill_tiles_with_short_runs_and_window_straddles(dev):
    """Runs of 2..20 tokens packed so one 16-token tile window holds several runs (and a
    decode row), runs cross tile boundaries, and contexts cross 128-key blocks."""
    rows = [(10, 3), (50, 5), (0, 7), (200, 1), (100, 2), (33, 20), (127, 2), (128, 16), (0, 1)]
    out, ref, path = _ragged_rows_case(dev, rows, 16, 2, seed=31)
    assert path == 3
    check_close(out, ref)
    assert K.device_errors(dev) == 0


def test_prefill_tiles_config3_shape_against_oracle(dev):
    """Mixed chunked-prefill batch of the benchmark's shape (reduced: 4 chunks of 512 on
    cached context up to 2048 and 16 decode rows) against the CPU oracle."""
    g = torch.Generator().manual_seed(3)
    decode = [(int(c) - 1, 1) for c in torch.randint(256, 4097, (16,), generator=g)]
    prefill = [(int(c), 512) for c in torch.randint(0, 2049, (4,), generator=g)]
    out, ref, path = _ragged_rows_case(dev, decode + prefill, 16, 2, seed=32)
    assert path == 3
    check_close(out, ref)
    assert K.device_errors(dev) == 0


def test_prefill_tiles_tp2_layout_against_oracle(dev):
    """TP2 per-rank heads (8 query heads, 1 KV head) with a 300-token chunk on 1000 cached."""
    out, ref, path = _ragged_rows_case(dev, [(1000, 300), (4000, 1), (5, 40)], 8, 1, seed=33)
    assert path == 3
    check_close(out, ref)


def test_prefill_work_queue_spans_more_items_than_sms(dev):
    """More (window, KV head) work items than SMs, so CTAs take several items each from the
    workspace work counter; repeated and interleaved calls check that every launch leaves
    the counter at zero (a stale counter would skip items and leave rows unwritten)."""
    g = torch.Generator().manual_seed(5)
    prefill = [(int(c), 512) for c in torch.randint(0, 1025, (12,), generator=g)]
    decode = [(int(c) - 1, 1) for c in torch.randint(64, 2049, (8,), generator=g)]
    rows = decode[:4] + prefill + decode[4:]
    out, ref, path = _ragged_rows_case(dev, rows, 16, 2, seed=34)
    assert path == 3
    check_close(out, ref)
    small, small_ref, _ = _ragged_rows_case(dev, [(300, 40), (10, 1), (0, 33)], 16, 2, seed=35)
    check_close(small, small_ref)
    again, _, _ = _ragged_rows_case(dev, rows, 16, 2, seed=34)
    assert torch.equal(again, out)
    assert K.device_errors(dev) == 0


@pytest.mark.parametrize("seq_dtype,pos_dtype,H,KVH", [
    (torch.int32, torch.int64, 16, 2),
    (torch.int64, torch.int32, 16, 2),
    (torch.int32, torch.int64, 8, 1),   # TP2 per-rank heads: the one-KV-head wide shape
])
def test_mixed_batch_index_arrays_staged_or_not_give_identical_results(dev, seq_dtype, pos_dtype,
                                                                       H, KVH):
    """The wide decode shape next to the prefill tiles copies 16-byte aligned sequence-id and
    position arrays into shared memory for its scan, and scans them from global memory
    otherwise.  The same batch with the arrays as offset views (not 16-byte aligned) must give
    bit-identical outputs."""
    from shardserve_b200.workloads import ragged_batch

    g = torch.Generator().manual_seed(41)
    decode = [(int(c) - 1, 1) for c in torch.randint(256, 4097, (24,), generator=g)]
    prefill = [(int(c), 512) for c in torch.randint(0, 2049, (3,), generator=g)]
    b = ragged_batch(decode + prefill, H, KVH, 128, seed=41, device=dev)
    seq = b.seq_ids.to(seq_dtype)
    pos = b.positions.to(pos_dtype)
    args = (b.q, b.k_pool, b.v_pool, b.block_tables)
    aligned = sb.ragged_attention_direct(*args, seq, pos, 128 ** -0.5)
    assert K.last_attention_path() == 3
    T = seq.numel()
    seq_off = torch.empty(T + 1, dtype=seq_dtype, device=dev)[1:]
    pos_off = torch.empty(T + 1, dtype=pos_dtype, device=dev)[1:]
    seq_off.copy_(seq)
    pos_off.copy_(pos)
    assert seq_off.data_ptr() % 16 and pos_off.data_ptr() % 16
    offset = sb.ragged_attention_direct(*args, seq_off, pos_off, 128 ** -0.5)
    assert torch.equal(aligned, offset)
    assert K.device_errors(dev) == 0


@pytest.mark.parametrize("rows,H,KVH", [
    ([(5, 2)], 16, 2),                       # one run of two query tokens, nothing else
    ([(100, 40), (0, 7), (300, 33)], 16, 2),  # prefill runs only: no decode row at all
    ([(1000, 64)], 8, 1),                    # TP2 heads, one chunk
])
def test_prefill_only_launches_against_oracle(dev, rows, H, KVH):
    """Launches whose every token belongs to a prefill run: the decode kernel beside the tiles
    finds no units, and every one of its CTAs leaves right after its prologue."""
    out, ref, path = _ragged_rows_case(dev, rows, H, KVH, seed=51)
    assert path == 3
    check_close(out, ref)
    assert K.device_errors(dev) == 0


@pytest.mark.parametrize("chunks", [
    40,   # 20,508 tokens, 641 windows: ranked longest first, straddling windows not split
    70,   # 35,868 tokens, 1,121 windows: more windows than the ranking holds, taken in order
])
def test_prefill_tiles_beyond_the_ranked_window_limits(dev, chunks):
    """Batches with more 32-token windows than the tile kernel's longest-first ranking splits
    (512) or ranks at all (1024).  The decode rows come first, so every chunk starts inside a
    window and windows straddle two chunks."""
    g = torch.Generator().manual_seed(61 + chunks)
    decode = [(int(c) - 1, 1) for c in torch.randint(64, 1025, (28,), generator=g)]
    prefill = [(int(c), 512) for c in torch.randint(0, 301, (chunks,), generator=g)]
    out, ref, path = _ragged_rows_case(dev, decode + prefill, 16, 2, seed=61 + chunks)
    assert path == 3
    check_close(out, ref)
    assert K.device_errors(dev) == 0
