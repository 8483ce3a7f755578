"""TP2 attention output projection fused with its all-reduce (two ranks, NVLink peer memory).

In the reference's TP2 layout (docs/implementation.md:15) each rank holds 8 query heads / 1
KV head and the matching column shard of o_proj, and each layer does
`hidden = hidden + reduce(F.linear(attention, w_o))` with `reduce` = a two-rank NCCL
all-reduce (shardserve/model.py:40, runtime.py:17-24).  `TP2OprojAllReduce` computes
`reduce(F.linear(attention, w_o))` in one kernel launch per rank: the GEMM tiles run on the
tensor cores, each rank stores its bf16 partial of every tile, six values per 16-byte vector
tagged with the call number, straight into the other rank's inbox over NVLink and adds the
other rank's partial from its own inbox once its tags match, so both ranks return the same
bf16 sum.  The inboxes are
plain device allocations shared with CUDA IPC once, at construction (a collective over
`group`).
"""
from __future__ import annotations

import ctypes
from typing import Any

from . import _native
from .kernel import KernelUnsupported


class TP2OprojAllReduce:

    def __init__(self, group: Any, device: Any, max_tokens: int, out_features: int,
                 in_features: int):
        import torch
        import torch.distributed as dist

        if dist.get_world_size(group) != 2:
            raise KernelUnsupported("TP2OprojAllReduce needs a group of exactly two ranks")
        if out_features % 128 or in_features % 256:
            raise KernelUnsupported("out_features must be a multiple of 128 and in_features of 256")
        self.device = torch.device(device)
        self.rank = dist.get_rank(group)
        self.max_tokens, self.n, self.k = int(max_tokens), int(out_features), int(in_features)
        lib = _native.lib()
        with torch.cuda.device(self.device):
            self._local = {}
            # Two halves (call parity) of [32-row blocks][feature groups][6][32] 16-byte
            # vectors: 6 * rows rounded up to 32 * out_features bytes.
            inbox = 6 * ((self.max_tokens + 31) // 32) * 32 * self.n
            for name, nbytes in (("inbox", inbox), ("err", 256),
                                 ("epoch", 256)):
                p = ctypes.c_void_p()
                if lib.ss_device_alloc_zeroed(nbytes, ctypes.byref(p)) != _native.SS_OK:
                    raise RuntimeError(f"ss_device_alloc_zeroed: {_native.last_error()}")
                self._local[name] = p.value
            handles = {}
            for name in ("inbox",):
                h = ctypes.create_string_buffer(64)
                if lib.ss_ipc_handle(self._local[name], h) != _native.SS_OK:
                    raise RuntimeError(f"ss_ipc_handle: {_native.last_error()}")
                handles[name] = h.raw
            gathered = [None, None]
            dist.all_gather_object(gathered, handles, group=group)
            self._peer = {}
            for name, raw in gathered[1 - self.rank].items():
                p = ctypes.c_void_p()
                if lib.ss_ipc_open(ctypes.create_string_buffer(raw, 64), ctypes.byref(p)) \
                        != _native.SS_OK:
                    raise RuntimeError(f"ss_ipc_open: {_native.last_error()}")
                self._peer[name] = p.value
            dist.barrier(group=group)

    def __call__(self, attn: Any, w_o: Any, out: Any = None) -> Any:
        """reduce(F.linear(attn, w_o)) over the two ranks: attn bf16 [T, in_features] (this
        rank's heads), w_o bf16 [out_features, in_features] (this rank's shard)."""
        import torch

        if attn.dtype != torch.bfloat16 or w_o.dtype != torch.bfloat16:
            raise KernelUnsupported("attn and w_o must be BF16")
        if attn.dim() != 2 or attn.shape[1] != self.k or tuple(w_o.shape) != (self.n, self.k):
            raise KernelUnsupported(
                f"attn must be [T, {self.k}] and w_o [{self.n}, {self.k}]")
        if attn.shape[0] > self.max_tokens:
            raise KernelUnsupported("more tokens than the inbox holds")
        if out is None:
            out = torch.empty((attn.shape[0], self.n), dtype=torch.bfloat16, device=attn.device)
        rc = _native.lib().ss_tp2_oproj_allreduce(
            attn.data_ptr(), _native.strides(attn.stride()), w_o.data_ptr(),
            _native.strides(w_o.stride()), out.data_ptr(), _native.strides(out.stride()),
            attn.shape[0], self.n, self.k, self._local["inbox"], self._peer["inbox"],
            self.max_tokens, self._local["epoch"], self._local["err"],
            torch.cuda.current_stream(attn.device).cuda_stream)
        if rc == _native.SS_ERR_INVALID:
            raise KernelUnsupported(_native.last_error())
        if rc != _native.SS_OK:
            raise RuntimeError(f"ss_tp2_oproj_allreduce: {_native.last_error()}")
        return out

    def device_errors(self) -> int:
        """SS_DEVERR_* bits of this rank's calls (synchronises)."""
        import torch

        torch.cuda.synchronize(self.device)
        flags = ctypes.c_uint32()
        rc = _native.lib().ss_fetch_device_errors(self._local["err"], 1, ctypes.byref(flags), None)
        if rc != _native.SS_OK:
            raise RuntimeError(f"ss_fetch_device_errors: {_native.last_error()}")
        return flags.value

    def close(self) -> None:
        lib = _native.lib()
        for p in self._peer.values():
            lib.ss_ipc_close(p)
        for p in self._local.values():
            lib.ss_device_free(p)
        self._peer, self._local = {}, {}
