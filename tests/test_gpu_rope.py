"""GPU parity of the fused RoPE + KV append (ss_rope_kv_append) — bit-exact.

Against the reference's own vectors (tests/golden/rope_*.npz, from shardserve/math.py and
Cache.write), against the CPU oracle on seeded inputs, and against torch's bf16 arithmetic
on the GPU (the reference's apply_rope expression evaluated by torch on the same device).
"""
import os

import numpy as np
import pytest
import torch

import oracle
import shardserve_b200 as sb
from shardserve_b200 import kernel as K

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
ROPE_CASES = ["rope_decode", "rope_chunk_mha_d64", "rope_tp2_long", "rope_wide_range"]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda:0")


def bits_tensor(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def load_rope(name, dev):
    z = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    T, H, KVH, D, max_len, pages = (int(x) for x in z["dims"])
    cos = np.zeros((max_len, D), np.float32)
    sin = np.zeros((max_len, D), np.float32)
    cos[z["table_pos"]] = z["cos_rows"]
    sin[z["table_pos"]] = z["sin_rows"]
    return z, (T, H, KVH, D, pages), torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)


def torch_apply_rope(q, cos, sin, positions):
    """The reference expression (math.py:36-38) evaluated by torch on bf16 GPU tensors."""
    c = cos[positions][:, None, :].to(q.dtype)
    s = sin[positions][:, None, :].to(q.dtype)
    half = q.shape[-1] // 2
    rot = torch.cat((-q[..., half:], q[..., :half]), dim=-1)
    return (q * c) + (rot * s)


@pytest.mark.parametrize("name", ROPE_CASES)
@pytest.mark.parametrize("layout", ["contiguous", "strided", "in_place"])
def test_rope_append_matches_reference_vectors(dev, name, layout):
    z, (T, H, KVH, D, pages), cos, sin = load_rope(name, dev)
    q = bits_tensor(z["q"], dev)
    k = bits_tensor(z["k"], dev)
    v = bits_tensor(z["v"], dev)
    pos = torch.from_numpy(z["positions"]).to(dev)
    slots = torch.from_numpy(z["slots"]).to(dev)
    kp = torch.zeros(pages, 16, KVH, D, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    out = None
    if layout == "strided":  # non-unit inner strides: the scalar path
        q = torch.empty(T, H, D, 2, dtype=torch.bfloat16, device=dev)[..., 0].copy_(q)
        k = torch.empty(T, KVH, D, 2, dtype=torch.bfloat16, device=dev)[..., 0].copy_(k)
        cos = torch.empty(cos.shape[0], D, 2, device=dev)[..., 0].copy_(cos)
        sin = torch.empty(sin.shape[0], D, 2, device=dev)[..., 0].copy_(sin)
    elif layout == "in_place":
        out = q
    got = sb.rope_kv_append(q, k, v, cos, sin, pos, kp, vp, slots, out=out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits_of(got), z["q_rot"])
    flat_k = kp.reshape(-1, KVH, D)[slots]
    flat_v = vp.reshape(-1, KVH, D)[slots]
    np.testing.assert_array_equal(bits_of(flat_k), z["k_rot"])
    np.testing.assert_array_equal(bits_of(flat_v), z["v"])


@pytest.mark.parametrize("H,KVH,D,theta", [(16, 2, 128, 1e6), (32, 8, 64, 1e4), (8, 1, 128, 1e6)])
def test_rope_append_matches_oracle_and_torch(dev, H, KVH, D, theta):
    T, pages, max_len = 200, 40, 8192
    g = torch.Generator().manual_seed(H * 1000 + D)
    cos_np, sin_np = oracle.rope_tables(D, max_len, theta)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    q = torch.randn(T, H, D, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(T, KVH, D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(T, KVH, D, generator=g).to(torch.bfloat16).to(dev)
    pos = torch.randint(0, max_len, (T,), generator=g).to(dev)
    slots = torch.randperm(pages * 16, generator=g)[:T].to(dev)
    kp = torch.zeros(pages, 16, KVH, D, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    got = sb.rope_kv_append(q, k, v, cos, sin, pos.to(torch.int32), kp, vp, slots)
    want_q = oracle.apply_rope_bits(bits_of(q), cos_np, sin_np, pos.cpu().numpy())
    want_k = oracle.apply_rope_bits(bits_of(k), cos_np, sin_np, pos.cpu().numpy())
    np.testing.assert_array_equal(bits_of(got), want_q)
    np.testing.assert_array_equal(bits_of(kp.reshape(-1, KVH, D)[slots]), want_k)
    assert torch.equal(got, torch_apply_rope(q, cos, sin, pos))
    assert torch.equal(kp.reshape(-1, KVH, D)[slots], torch_apply_rope(k, cos, sin, pos))


def test_rope_append_then_attention_equals_separate_ops(dev):
    """The fused op feeds attention exactly like apply_rope + Cache.write (model.py:25-37)."""
    from shardserve_b200.workloads import ragged_batch

    b = ragged_batch([(100, 1), (37, 20), (500, 1)], 16, 2, 128, seed=41, device=dev)
    cos_np, sin_np = oracle.rope_tables(128, 2048, 1e6)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    kp2, vp2 = b.k_pool.clone(), b.v_pool.clone()
    q_f = sb.rope_kv_append(b.q, b.k_new, b.v_new, cos, sin, b.positions, b.k_pool, b.v_pool,
                            b.slots)
    out_f = sb.ragged_attention_direct(q_f, b.k_pool, b.v_pool, b.block_tables, b.seq_ids,
                                       b.positions, 128 ** -0.5)
    q_s = torch_apply_rope(b.q, cos, sin, b.positions)
    k_s = torch_apply_rope(b.k_new, cos, sin, b.positions)
    sb.kv_append(kp2, vp2, k_s, b.v_new, b.slots)
    out_s = sb.ragged_attention_direct(q_s, kp2, vp2, b.block_tables, b.seq_ids, b.positions,
                                       128 ** -0.5)
    assert torch.equal(kp2, b.k_pool) and torch.equal(vp2, b.v_pool)
    assert torch.equal(out_f, out_s)


def test_out_of_table_position_is_flagged_and_skipped(dev):
    T, H, KVH, D = 4, 8, 2, 128
    cos = torch.ones(16, D, device=dev)
    sin = torch.zeros(16, D, device=dev)
    q = torch.randn(T, H, D, device=dev).to(torch.bfloat16)
    k = torch.randn(T, KVH, D, device=dev).to(torch.bfloat16)
    kp = torch.zeros(4, 16, KVH, D, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    K._workspace(dev, T, H, KVH, D)
    K.device_errors(dev, clear=True)
    pos = torch.tensor([0, 16, 3, -1], device=dev)
    slots = torch.tensor([1, 2, 3, 4], device=dev)
    out = torch.full_like(q, 7.0)
    sb.rope_kv_append(q, k, k.clone(), cos, sin, pos, kp, vp, slots, out=out)
    torch.cuda.synchronize()
    assert K.device_errors(dev) & 0x4  # SS_DEVERR_POS
    assert torch.equal(out[0], q[0]) and torch.equal(out[2], q[2])  # cos 1, sin 0: identity
    assert torch.all(out[1] == 7.0) and torch.all(out[3] == 7.0)    # skipped rows untouched
    flat = kp.reshape(-1, KVH, D)
    assert torch.equal(flat[1], k[0]) and torch.equal(flat[3], k[2])
    assert torch.all(flat[2] == 0) and torch.all(flat[4] == 0)
    K.device_errors(dev, clear=True)
