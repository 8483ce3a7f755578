"""The torch binding (csrc/torch_binding.cpp) raises the reference wrapper's errors with its
messages (shardserve/kernel.py:28-49) for inputs that only a CUDA tensor reaches, and the
calls run through it."""
import os

import pytest
import torch

import shardserve_b200 as sb
from shardserve_b200 import _native
from shardserve_b200 import kernel as K

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


def _inputs(dev, **over):
    a = dict(q=torch.zeros(2, 8, 128, dtype=BF, device=dev),
             k=torch.zeros(4, 16, 1, 128, dtype=BF, device=dev),
             v=torch.zeros(4, 16, 1, 128, dtype=BF, device=dev),
             bt=torch.zeros(2, 1, dtype=torch.int32, device=dev),
             seq=torch.zeros(2, dtype=torch.int32, device=dev),
             pos=torch.zeros(2, dtype=torch.int64, device=dev))
    a.update(over)
    return a


def _attn(a):
    return sb.ragged_attention_direct(a["q"], a["k"], a["v"], a["bt"], a["seq"], a["pos"], 0.1)


def test_binding_is_the_in_tree_module():
    assert os.path.dirname(_native.ops().__file__) == os.path.dirname(_native.LIB_PATH)


def _z(*shape, dtype=BF, dev="cuda"):
    return torch.zeros(*shape, dtype=dtype, device=dev)


@pytest.mark.parametrize("make,msg", [
    (lambda: dict(q=_z(2, 8, 100)), r"ragged q must be \[tokens, heads, 64\|128\], got \(2, 8, 100\)"),
    (lambda: dict(k=_z(4, 16, 1, 128), v=_z(4, 16, 1, 64)),
     "ragged K/V pools must have identical rank-4 shapes"),
    (lambda: dict(k=_z(4, 8, 1, 128), v=_z(4, 8, 1, 128)), "ragged KV pools must be BF16 with block_size=16"),
    (lambda: dict(k=_z(4, 16, 1, 64), v=_z(4, 16, 1, 64)), "query and KV head dimensions differ"),
    (lambda: dict(bt=_z(2, dtype=torch.int32)), "block_tables must be a device-resident rank-2 tensor"),
    (lambda: dict(seq=_z(3, dtype=torch.int32)), "one sequence id and absolute position are required per query"),
    (lambda: dict(q=_z(0, 8, 128), seq=_z(0, dtype=torch.int32), pos=_z(0, dtype=torch.int64)),
     "ragged batch cannot be empty"),
    (lambda: dict(q=_z(2, 3, 128), k=_z(4, 16, 2, 128), v=_z(4, 16, 2, 128)),
     "query heads must be divisible by KV heads"),
    (lambda: dict(pos=_z(2, dtype=torch.int64, dev="cpu")), "positions must be on cuda:0"),
    (lambda: dict(v=_z(4, 16, 1, 128, dtype=torch.float16)), "ragged KV pools must be BF16 with block_size=16"),
    (lambda: dict(pos=_z(2, dtype=torch.float32)), "positions must be int32 or int64, got torch.float32"),
    (lambda: dict(bt=_z(2, 1, dtype=torch.int16)), "block_tables must be int32 or int64, got torch.int16"),
])
def test_attention_rejections_match_reference(dev, make, msg):
    with pytest.raises(sb.KernelUnsupported, match=msg):
        _attn(_inputs(dev, **make()))


def test_append_rejections_match_reference(dev):
    kp = torch.zeros(4, 16, 1, 128, dtype=BF, device=dev)
    vp = torch.zeros_like(kp)
    k = torch.zeros(2, 1, 128, dtype=BF, device=dev)
    slots = torch.zeros(2, dtype=torch.int64, device=dev)
    with pytest.raises(sb.KernelUnsupported,
                       match=r"k/v must be \[tokens, 1, 128\], got \(2, 1, 128\)/\(2, 1, 64\)"):
        sb.kv_append(kp, vp, k, k[:, :, :64], slots)
    with pytest.raises(sb.KernelUnsupported, match="one slot is required per appended token"):
        sb.kv_append(kp, vp, k, k, slots[:1])
    with pytest.raises(sb.KernelUnsupported, match="slots must be on cuda:0"):
        sb.kv_append(kp, vp, k, k, slots.cpu())
    with pytest.raises(sb.KernelUnsupported, match="slots must be int32 or int64, got torch.float64"):
        sb.kv_append(kp, vp, k, k, slots.double())


def test_rope_rejections_match_reference(dev):
    kp = torch.zeros(4, 16, 1, 128, dtype=BF, device=dev)
    q = torch.zeros(2, 8, 128, dtype=BF, device=dev)
    k = torch.zeros(2, 1, 128, dtype=BF, device=dev)
    tab = torch.zeros(8, 128, device=dev)
    pos = torch.zeros(2, dtype=torch.int64, device=dev)
    with pytest.raises(sb.KernelUnsupported, match=r"cos must be float32 \[rows, 128\]"):
        sb.rope_kv_append(q, k, k, tab.double(), tab, pos, kp, kp.clone(), pos)
    with pytest.raises(sb.KernelUnsupported, match="cos and sin tables must have the same shape"):
        sb.rope_kv_append(q, k, k, tab, tab[:4], pos, kp, kp.clone(), pos)
    with pytest.raises(sb.KernelUnsupported, match="out must be a BF16 tensor shaped like q"):
        sb.rope_kv_append(q, k, k, tab, tab, pos, kp, kp.clone(), pos, out=q[:1])


def test_workspace_is_shared_with_the_c_abi_error_reader(dev):
    inp = _inputs(dev)
    _attn(inp)
    ws = K.workspace_for(dev)
    assert ws is not None and ws.dtype == torch.uint8 and ws.device == dev
    assert K.device_errors(dev) == 0


def test_plain_ctypes_binding_matches_the_torch_binding(dev):
    """The minimal ctypes binding a maintainer would add beside the reference's kernel.py
    (C ABI only, no torch extension) gives bit-identical output to the torch binding."""
    import ctypes

    from shardserve_b200.workloads import decode_batch

    lib = ctypes.CDLL(_native.LIB_PATH)
    lib.ss_last_error_message.restype = ctypes.c_char_p
    I64 = ctypes.c_int64

    def strides(t):
        return (I64 * t.dim())(*t.stride())

    def attention(q, kp, vp, tables, seqs, pos, scale, ws):
        out = torch.empty_like(q)
        rc = lib.ss_ragged_paged_attention(
            ctypes.c_void_p(q.data_ptr()), strides(q), ctypes.c_void_p(kp.data_ptr()), strides(kp),
            ctypes.c_void_p(vp.data_ptr()), strides(vp), ctypes.c_void_p(tables.data_ptr()),
            strides(tables), I64(tables.shape[0]), I64(tables.shape[1]), 0,
            ctypes.c_void_p(seqs.data_ptr()), 0, ctypes.c_void_p(pos.data_ptr()), 1,
            ctypes.c_void_p(out.data_ptr()), strides(out), I64(q.shape[0]), q.shape[1],
            kp.shape[2], q.shape[2], I64(kp.shape[0]), ctypes.c_float(scale),
            ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if rc:
            raise RuntimeError(lib.ss_last_error_message().decode())
        return out

    b = decode_batch([300, 17, 2049, 64], 16, 2, 128, seed=71, device=dev)
    sb.kv_append(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots)
    need = ctypes.c_size_t()
    assert lib.ss_attention_workspace_bytes(0, I64(4), 16, 2, 128, ctypes.byref(need)) == 0
    ws = torch.zeros(need.value, dtype=torch.uint8, device=dev)
    seqs = b.seq_ids.to(torch.int32)
    pos = b.positions.to(torch.int64)
    tables = b.block_tables.to(torch.int32)
    via_ctypes = attention(b.q, b.k_pool, b.v_pool, tables, seqs, pos, 128 ** -0.5, ws)
    via_torch = sb.ragged_attention_direct(b.q, b.k_pool, b.v_pool, tables, seqs, pos, 128 ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(via_ctypes, via_torch)


def test_output_rows_not_16_byte_addressable_run_on_the_generic_kernel(dev):
    """The split-K and tile kernels write output rows as vectors; an output view that starts
    one element into its buffer, or has an odd head stride, goes to the generic kernel
    through the C ABI, with results within the attention tolerance of the fast path."""
    import ctypes

    from helpers import MAX_ABS_TOL, MEAN_ABS_TOL
    from shardserve_b200.workloads import decode_batch

    lib = ctypes.CDLL(_native.LIB_PATH)
    lib.ss_last_error_message.restype = ctypes.c_char_p
    I64 = ctypes.c_int64

    def strides(t):
        return (I64 * t.dim())(*t.stride())

    b = decode_batch([300, 17, 2049, 64, 900], 16, 2, 128, seed=72, device=dev)
    sb.kv_append(b.k_pool, b.v_pool, b.k_new, b.v_new, b.slots)
    need = ctypes.c_size_t()
    assert lib.ss_attention_workspace_bytes(0, I64(5), 16, 2, 128, ctypes.byref(need)) == 0
    ws = torch.zeros(need.value, dtype=torch.uint8, device=dev)
    seqs = b.seq_ids.to(torch.int32)
    pos = b.positions.to(torch.int64)
    tables = b.block_tables.to(torch.int32)
    T, H, D = b.q.shape

    def attention(out):
        rc = lib.ss_ragged_paged_attention(
            ctypes.c_void_p(b.q.data_ptr()), strides(b.q), ctypes.c_void_p(b.k_pool.data_ptr()),
            strides(b.k_pool), ctypes.c_void_p(b.v_pool.data_ptr()), strides(b.v_pool),
            ctypes.c_void_p(tables.data_ptr()), strides(tables), I64(tables.shape[0]),
            I64(tables.shape[1]), 0, ctypes.c_void_p(seqs.data_ptr()), 0,
            ctypes.c_void_p(pos.data_ptr()), 1, ctypes.c_void_p(out.data_ptr()), strides(out),
            I64(T), H, 2, D, I64(b.k_pool.shape[0]), ctypes.c_float(D ** -0.5),
            ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.ss_last_error_message().decode()
        return lib.ss_last_attention_path()

    fast = torch.empty_like(b.q)
    assert attention(fast) == 1
    shifted = torch.zeros(T * H * D + 1, dtype=torch.bfloat16, device=dev)[1:].view(T, H, D)
    odd = torch.zeros(T, H, D + 1, dtype=torch.bfloat16, device=dev)[..., :D]
    for out in (shifted, odd):
        assert attention(out) == 2
        torch.cuda.synchronize()
        err = (out.float() - fast.float()).abs()
        assert err.max().item() <= MAX_ABS_TOL and err.mean().item() <= MEAN_ABS_TOL
