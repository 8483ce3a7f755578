"""GPU parity at the benchmark configurations' own scale, against the CPU oracle.

* Long-context TP2 layout on a pool filling ~60 % of HBM: every K/V tensor holds more than
  2^31 elements and every sequence's pages sit, scattered, in the far end of the pool, so
  page offsets, append slots and TMA page coordinates all run past 32-bit element offsets.
  Both attention kernels (the TMA split-K kernel and the generic strided kernel) and both
  append kernels (16-byte vectors and single elements) run on it.  The oracle sees only the
  pages the block tables touch, gathered to the host.
* The exact mixed chunked-prefill batch of the benchmark (8 chunks of 512 query tokens on
  cached context U[0, 2048] plus 56 decode rows with context U[256, 4096]).
* One layer of the 36-layer decode step: 256 sequences with context U[512, 8192], 16 query
  and 2 KV heads, q / k / v from random-init projections, RoPE (theta 1e6) fused with the
  append, then attention.

Reference: shardserve/kernel.py:115-166 (int64 page offsets, kernel.py:130-142),
shardserve/cache.py:47-61, shardserve/math.py:28-38.
"""
import numpy as np
import pytest
import torch

import oracle
import shardserve_b200 as sb
from helpers import MAX_ABS_TOL, MEAN_ABS_TOL
from shardserve_b200 import kernel as K
from shardserve_b200.workloads import mixed_rows, ragged_batch, uniform_lengths

pytestmark = pytest.mark.gpu
SCALE = 128 ** -0.5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


def check_close(got, want):
    err = np.abs(got.float().cpu().numpy() - want)
    assert err.max() <= MAX_ABS_TOL, f"max-abs {err.max():.3e}"
    assert err.mean() <= MEAN_ABS_TOL, f"mean-abs {err.mean():.3e}"


def f32(t):
    return t.float().cpu().numpy()


def test_long_context_tp2_layout_on_a_pool_past_2_31_elements(dev):
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info(dev)
    page_bytes = 16 * 1 * 128 * 2  # one page of one KV head, d 128, bf16: 4 KiB
    N = int(free * 0.6 / (2 * page_bytes))  # K and V pools together: ~60 % of free HBM
    assert N * 16 * 128 > 2 ** 31, "the pool must hold more than 2^31 elements"
    kp = torch.empty((N, 16, 1, 128), dtype=torch.bfloat16, device=dev)
    vp = torch.empty_like(kp)
    try:
        g = torch.Generator().manual_seed(55)
        n_seq = 16
        lengths = torch.randint(16384, 32769, (n_seq,), generator=g)
        pages = ((lengths + 15) // 16).tolist()
        W = max(pages)
        # Pages scattered over the last ~8 % of the pool (the scratch pages excluded).
        hi, lo = N - 8, N - 8 - int(0.08 * N)
        pick = torch.randperm(hi - lo, generator=g)[:sum(pages)].to(torch.int64) + lo
        assert pick.numel() == sum(pages) and int(pick.min()) * 16 * 128 > 2 ** 31
        bt = torch.zeros(n_seq, W, dtype=torch.int32)
        off = 0
        for i, n in enumerate(pages):
            bt[i, :n] = pick[off:off + n].to(torch.int32)
            off += n
        touched = pick.to(dev)
        gd = torch.Generator(device=dev).manual_seed(56)
        kp[touched] = torch.randn((touched.numel(), 16, 1, 128), generator=gd,
                                  device=dev).to(torch.bfloat16)
        vp[touched] = torch.randn((touched.numel(), 16, 1, 128), generator=gd,
                                  device=dev).to(torch.bfloat16)
        pos = (lengths - 1).to(torch.int64)
        seq = torch.arange(n_seq, dtype=torch.int32)
        slots = bt[seq.long(), pos // 16].to(torch.int64) * 16 + pos % 16
        assert int(slots.min()) * 128 > 2 ** 31
        kn = torch.randn((n_seq, 1, 128), generator=gd, device=dev).to(torch.bfloat16)
        vn = torch.randn((n_seq, 1, 128), generator=gd, device=dev).to(torch.bfloat16)
        d_bt, d_seq, d_pos, d_slots = bt.to(dev), seq.to(dev), pos.to(dev), slots.to(dev)
        K.device_errors(dev, clear=True)
        # Append: the first half of the tokens by 16-byte vectors, the second half through
        # element-wise copies (a source whose head_dim stride is 2 is not 16-byte addressable).
        h = n_seq // 2
        sb.kv_append(kp, vp, kn[:h], vn[:h], d_slots[:h])
        kn2 = torch.zeros((n_seq - h, 1, 256), dtype=torch.bfloat16, device=dev)
        vn2 = torch.zeros_like(kn2)
        kn2[..., ::2] = kn[h:]
        vn2[..., ::2] = vn[h:]
        sb.kv_append(kp, vp, kn2[..., ::2], vn2[..., ::2], d_slots[h:])
        # The oracle's view: the touched pages only, renumbered.
        order = torch.sort(pick).values
        remap = {int(p): i for i, p in enumerate(order.tolist())}
        cbt = np.vectorize(lambda p: remap.get(int(p), 0))(bt.numpy()).astype(np.int32)
        cpos = pos.numpy()
        cseq = seq.numpy()
        ck, cv = f32(kp[order.to(dev)]), f32(vp[order.to(dev)])
        # Append bit-exact: every appended row holds the new k / v.
        cslots = cbt[cseq, cpos // 16].astype(np.int64) * 16 + cpos % 16
        np.testing.assert_array_equal(ck.reshape(-1, 1, 128)[cslots], f32(kn))
        np.testing.assert_array_equal(cv.reshape(-1, 1, 128)[cslots], f32(vn))
        for H, path in ((8, 1), (32, 2)):  # TP2 per-rank heads (TMA kernel); group 32 (generic)
            q = torch.randn((n_seq, H, 128), generator=gd, device=dev).to(torch.bfloat16)
            out = sb.ragged_attention_direct(q, kp, vp, d_bt, d_seq, d_pos, SCALE)
            assert K.last_attention_path() == path
            ref = oracle.ragged_attention(f32(q), ck, cv, cbt, cseq, cpos, SCALE,
                                          threads=oracle.host_threads())
            check_close(out, ref)
        assert K.device_errors(dev) == 0
    finally:
        del kp, vp
        torch.cuda.empty_cache()


def _oracle_of_batch(b):
    return oracle.ragged_attention(f32(b.q), f32(b.k_pool), f32(b.v_pool),
                                   b.block_tables.cpu().numpy(), b.seq_ids.cpu().numpy(),
                                   b.positions.cpu().numpy(), SCALE, threads=oracle.host_threads())


def test_exact_mixed_chunked_prefill_batch(dev):
    """The benchmark's mixed batch exactly (its row generator and seed)."""
    decode, prefill = mixed_rows(2024)
    assert len(decode) == 56 and len(prefill) == 8
    b = ragged_batch(decode + prefill, 16, 2, 128, seed=2024, device=dev)
    assert b.tokens == 56 + 8 * 512
    K.device_errors(dev, clear=True)
    sb.kv_append(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots)
    out = sb.ragged_attention_direct(b.q, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                     b.positions, SCALE)
    assert K.last_attention_path() == 3
    check_close(out, _oracle_of_batch(b))
    assert K.device_errors(dev) == 0


def test_one_layer_of_the_36_layer_decode_step(dev):
    """256 sequences, context U[512, 8192], 16 q / 2 kv heads: q / k / v projected from
    N(0,1) hidden states by random-init weights with bias, RoPE (theta 1e6) + append in one
    launch, then attention; against the oracle's RoPE + append + attention."""
    lengths = uniform_lengths(256, 512, 8192, 2024)
    b = ragged_batch([(L - 1, 1) for L in lengths], 16, 2, 128, seed=77, device=dev)
    T, hidden = b.tokens, 2048
    gen = torch.Generator(device=dev).manual_seed(78)
    x = torch.randn(T, hidden, generator=gen, device=dev).to(torch.bfloat16)

    def proj(o):
        w = (torch.randn(o, hidden, generator=gen, device=dev) * hidden ** -0.5).to(torch.bfloat16)
        bias = (torch.randn(o, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        return torch.nn.functional.linear(x, w, bias)

    q = proj(16 * 128).view(T, 16, 128).contiguous()
    k = proj(2 * 128).view(T, 2, 128).contiguous()
    v = proj(2 * 128).view(T, 2, 128).contiguous()
    cos, sin = oracle.rope_tables(128, 8192, 1e6)
    kp_before, vp_before = f32(b.k_pool), f32(b.v_pool)
    K.device_errors(dev, clear=True)
    qr = sb.rope_kv_append(q, k, v, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev),
                           b.positions, b.k_pool, b.v_pool, b.slots)
    out = sb.ragged_attention_direct(qr, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                     b.positions, SCALE)
    assert K.last_attention_path() == 1

    def bits(t):
        return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)

    pos = b.positions.cpu().numpy()
    q_rot = oracle.apply_rope_bits(bits(q), cos, sin, pos)
    k_rot = oracle.apply_rope_bits(bits(k), cos, sin, pos)
    np.testing.assert_array_equal(bits(qr), q_rot)
    oracle.kv_append(kp_before, vp_before, oracle.bf16_to_f32(k_rot), f32(v),
                     b.slots.cpu().numpy())
    np.testing.assert_array_equal(f32(b.k_pool), kp_before)
    np.testing.assert_array_equal(f32(b.v_pool), vp_before)
    ref = oracle.ragged_attention(oracle.bf16_to_f32(q_rot), kp_before, vp_before,
                                  b.block_tables.cpu().numpy(), b.seq_ids.cpu().numpy(), pos,
                                  SCALE, threads=oracle.host_threads())
    check_close(out, ref)
    assert K.device_errors(dev) == 0
