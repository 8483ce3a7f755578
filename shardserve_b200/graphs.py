"""CUDA-graph decode buckets for batches larger than the reference engine's, a drop-in for
shardserve/runtime.py's DecodeGraphs (runtime.py:51-80).

The reference captures its decode step for buckets of 1, 2, 4 and 8 rows (runtime.py:55;
config.py caps max_live at 8), so batch-64 or batch-256 decode steps run eagerly.  Here a
bucket is captured for every size the caller asks for (16 ... 256 and beyond).  As in the
reference, each bucket owns static metadata tensors (ids, positions, tables, seqs, slots)
built for a padding-only plan, three warm-up steps run on a side stream, and one step is
captured.  Each replay then rewrites those static tensors in place on the device with
DeviceMetadata.build(plan, size, out=...) -- one packed host-to-device copy and one kernel
instead of the reference's per-tensor copies (runtime.py:75-78) -- and replays the graph.

Padding rows (bucket slots beyond the plan's rows) point at scratch page count + i, one
page per padding row (runtime.py:41-44), so the pool needs `max(sizes)` scratch pages after
the allocator's `count` pages (Cache(..., scratch_pages=...)).

The attention calls inside the captured step allocate nothing during capture: each
bucket's warm-up steps size the per-device workspace first, and a workspace replaced by a
larger bucket's stays alive for the graphs captured before it.
"""
from __future__ import annotations

import time
from typing import Any, Callable

from .kernel import KernelUnsupported

DEFAULT_SIZES = (1, 2, 4, 8, 16, 32, 64, 128, 256)


class DecodeGraphs:
    """Captured decode steps, one per bucket size.

    `forward(**data)` is the caller's decode step on the static metadata tensors `data`
    (ids, positions, tables, seqs, slots), e.g. `lambda **d: model.forward(cache=cache, **d)`
    as the reference does (runtime.py:62-71); its return value is the bucket's output.
    `meta` is the DeviceMetadata of the caller's allocator; `pool_pages` the pages of the KV
    pool (allocator count + scratch pages)."""

    def __init__(self, forward: Callable[..., Any], meta, device, pool_pages: int,
                 sizes=DEFAULT_SIZES, warmup: int = 3):
        import torch

        self.meta = meta
        self.device = torch.device(device)
        self.entries: dict = {}
        self.captures = 0
        self.replays = 0
        start = time.monotonic()
        for size in sorted(set(int(s) for s in sizes)):
            if meta.blocks.count + size > pool_pages:
                raise KernelUnsupported(
                    f"bucket {size} needs {size} scratch pages after the allocator's "
                    f"{meta.blocks.count} pages; the pool has {pool_pages}")
            data = meta.build({"rows": []}, size)
            data.pop("selected")
            stream = torch.cuda.Stream(device=self.device)
            stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(stream):
                for _ in range(warmup):
                    forward(**data)
            torch.cuda.current_stream(self.device).wait_stream(stream)
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = forward(**data)
            self.entries[size] = (graph, data, out)
            self.captures += 1
        self.startup_seconds = time.monotonic() - start

    def bucket(self, rows: int):
        """The smallest captured size holding `rows` rows (None when none does)."""
        return next((s for s in sorted(self.entries) if s >= rows), None)

    def run(self, plan: dict, size: int | None = None):
        """Builds `plan`'s metadata into the bucket's static tensors and replays its graph;
        returns the bucket's output (rows past the plan's are padding)."""
        size = size or self.bucket(len(plan["rows"]))
        if size not in self.entries:
            raise KernelUnsupported(f"no captured bucket holds {len(plan['rows'])} rows")
        graph, data, out = self.entries[size]
        self.meta.build(plan, size, out=data)
        graph.replay()
        self.replays += 1
        return out

    def close(self) -> None:
        """Releases the captured graphs (before a process group holding their collectives)."""
        self.entries.clear()
