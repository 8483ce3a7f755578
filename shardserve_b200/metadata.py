"""Device-side per-step attention metadata, a drop-in for shardserve/runtime.py:28-49.

The reference's `metadata(plan, cache, device, context, bucket)` walks every query token
in Python, then makes six device tensors with separate host-to-device copies, one more per
row for its block table.  `DeviceMetadata` keeps the block list of every live request on
the device (copied once, when the request first appears in a plan) and per step sends one
packed int64 buffer (row descriptors, sampled indices, token ids) through a pinned staging
buffer; `ss_build_metadata` then writes tables, ids, positions, seqs, slots and selected on
the device, bit-exact with the reference, optionally straight into a captured graph's
static input tensors (the copies of DecodeGraphs.run, runtime.py:75-78, disappear).

Block lists come from the allocator's `tables` ({request_id: [blocks]}, cache.py:14-24);
a request whose list object changed (released and reserved again) is copied again, and
rows of released requests are reused when the store fills up.
"""
from __future__ import annotations

from typing import Any

import numpy as np

from . import _native
from .kernel import KernelUnsupported, workspace_for

_OUT_KEYS = ("ids", "positions", "tables", "seqs", "slots", "selected")


class DeviceMetadata:
    def __init__(self, blocks, device, context: int, capacity: int = 1024):
        import torch

        self.blocks = blocks
        self.device = torch.device(device)
        self.context = int(context)
        self.width = (self.context + 15) // 16
        self.capacity = int(capacity)
        self.store = torch.zeros((self.capacity, self.width), dtype=torch.int32,
                                 device=self.device)
        self.lens = torch.zeros(self.capacity, dtype=torch.int32, device=self.device)
        self._row_of: dict = {}     # request_id -> (store row, block list object)
        self._free = list(range(self.capacity - 1, -1, -1))
        self._pinned = [torch.empty(0, dtype=torch.int64).pin_memory() for _ in range(2)]
        self._staged = [torch.empty(0, dtype=torch.int64, device=self.device) for _ in range(2)]
        self._events = [None, None]
        self._flip = 0

    # ---- request block lists --------------------------------------------------------------
    def _sweep(self):
        live = self.blocks.tables
        for key in [k for k, (_, tab) in self._row_of.items() if live.get(k) is not tab]:
            self._free.append(self._row_of.pop(key)[0])

    def _row(self, key) -> int:
        import torch

        table = self.blocks.tables[key]
        hit = self._row_of.get(key)
        if hit is not None and hit[1] is table:
            return hit[0]
        if hit is not None:
            self._free.append(self._row_of.pop(key)[0])
        if not self._free:
            self._sweep()
        if not self._free:
            raise MemoryError("device metadata store is full; raise capacity")
        if len(table) > self.width:
            raise KernelUnsupported(f"request {key!r} holds more blocks than the context allows")
        row = self._free.pop()
        host = torch.zeros(self.width, dtype=torch.int32)
        host[:len(table)] = torch.tensor(table, dtype=torch.int32)
        self.store[row].copy_(host.to(self.device, non_blocking=False))
        self.lens[row] = len(table)
        self._row_of[key] = (row, table)
        return row

    # ---- per-step build -------------------------------------------------------------------
    def build(self, plan: dict, bucket: int | None = None, out: dict | None = None) -> dict:
        """Same outputs as runtime.metadata(plan, cache, device, context, bucket); writes
        into `out` (a dict of correctly shaped device tensors, e.g. a graph's static inputs)
        when given."""
        import torch

        rows = plan["rows"]
        n = bucket or len(rows)
        if n < len(rows):
            raise KernelUnsupported("bucket smaller than the plan")
        nreal = sum(r["query_length"] for r in rows)
        tokens = nreal + (n - len(rows))
        desc = np.empty((n, 4), dtype=np.int64)
        sel, ids = [], []
        off = 0
        for i, r in enumerate(rows):
            ql = r["query_length"]
            pos = r["positions"]
            if len(pos) != ql or len(r["tokens"]) != ql or \
                    (ql and pos[-1] - pos[0] != ql - 1):
                raise KernelUnsupported("row positions must be one consecutive run per row")
            desc[i] = (self._row(r["request_id"]), ql, pos[0] if ql else 0, off)
            ids.extend(r["tokens"])
            if r["sample"]:
                sel.append(r["offset"] + ql - 1)
            off += ql
        for i in range(len(rows), n):
            desc[i] = (-1, 1, 0, off)
            ids.append(0)
            off += 1
        packed = np.concatenate([desc.reshape(-1), np.asarray(sel, dtype=np.int64),
                                 np.asarray(ids, dtype=np.int64)])
        # Alternate two pinned staging buffers; wait until the copy that last used one ended.
        k = self._flip = self._flip ^ 1
        if self._events[k] is not None:
            self._events[k].synchronize()
        if self._pinned[k].numel() < packed.size:
            self._pinned[k] = torch.empty(max(packed.size, 2 * self._pinned[k].numel()),
                                          dtype=torch.int64).pin_memory()
            self._staged[k] = torch.empty(self._pinned[k].numel(), dtype=torch.int64,
                                          device=self.device)
        self._pinned[k][:packed.size].numpy()[:] = packed
        self._staged[k][:packed.size].copy_(self._pinned[k][:packed.size], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._events[k] = ev
        if out is None:
            dev = self.device
            out = dict(ids=torch.empty(tokens, dtype=torch.long, device=dev),
                       positions=torch.empty(tokens, dtype=torch.long, device=dev),
                       tables=torch.empty((n, self.width), dtype=torch.int32, device=dev),
                       seqs=torch.empty(tokens, dtype=torch.int32, device=dev),
                       slots=torch.empty(tokens, dtype=torch.long, device=dev),
                       selected=torch.empty(len(sel), dtype=torch.long, device=self.device))
        else:
            if "selected" not in out:  # a graph's static inputs carry no sampled indices
                out = dict(out, selected=torch.empty(len(sel), dtype=torch.long,
                                                     device=self.device))
            self._check_out(out, n, tokens, len(sel))
        ws = workspace_for(self.device)
        rc = _native.lib().ss_build_metadata(
            self._staged[k].data_ptr(), n, len(sel), tokens, self.store.data_ptr(),
            self.lens.data_ptr(), self.capacity, self.store.stride(0), self.blocks.count,
            out["tables"].data_ptr(), self.width, out["tables"].stride(0), out["ids"].data_ptr(),
            out["positions"].data_ptr(), out["seqs"].data_ptr(), out["slots"].data_ptr(),
            out["selected"].data_ptr() if len(sel) else None,
            ws.data_ptr() if ws is not None else None,
            torch.cuda.current_stream(self.device).cuda_stream)
        if rc != _native.SS_OK:
            raise RuntimeError(f"ss_build_metadata: {_native.last_error()}")
        return out

    def _check_out(self, out: dict, n: int, tokens: int, nsel: int) -> None:
        import torch

        want = dict(ids=((tokens,), torch.long), positions=((tokens,), torch.long),
                    tables=((n, self.width), torch.int32), seqs=((tokens,), torch.int32),
                    slots=((tokens,), torch.long), selected=((nsel,), torch.long))
        for key, (shape, dtype) in want.items():
            t = out[key]
            if tuple(t.shape) != shape or t.dtype != dtype or t.device != self.device or \
                    (t.dim() == 1 and t.numel() > 0 and t.stride(0) != 1) or \
                    (t.dim() == 2 and t.stride(1) != 1):
                raise KernelUnsupported(f"out[{key!r}] must be {dtype} {shape} on {self.device}")


_builders: dict = {}


def metadata(plan: dict, cache: Any, device, context: int, bucket: int | None = None) -> dict:
    """Drop-in for shardserve.runtime.metadata (runtime.py:28-49): same arguments, same
    outputs, built on the device.  One DeviceMetadata is kept per (cache, device, context)."""
    key = (id(cache), str(device), int(context))
    b = _builders.get(key)
    if b is None or b.blocks is not cache.blocks:
        b = _builders[key] = DeviceMetadata(cache.blocks, device, context)
    return b.build(plan, bucket)
