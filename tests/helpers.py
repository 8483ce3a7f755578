"""Shared helpers for the tests: golden fixtures, case inputs as torch tensors."""
from __future__ import annotations

import json
import os
import sys

import numpy as np

import cases

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_blocks():
    """The reference's own logical page allocator class (shardserve/cache.py:6-35), from its
    offline install next to the repository (baseline/_ref) or the checkout named by
    SHARDSERVE_REFERENCE; None where neither is present."""
    for path in (os.environ.get("SHARDSERVE_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if path and os.path.isdir(os.path.join(path, "shardserve")) and path not in sys.path:
            sys.path.append(path)
    try:
        from shardserve.cache import Blocks
    except ImportError:
        return None
    return Blocks


class FreeListPages:
    """Test stand-in for the engine's page allocator where the reference is not installed:
    the attributes the device path's callers read (tables, count) and all-or-nothing
    reservations popping pages off the end of a free list, as the reference allocator does
    (shardserve/cache.py:14-30)."""

    def __init__(self, count):
        self.count = count
        self.free = list(range(count))
        self.tables = {}

    def reserve(self, requests):
        sizes = {key: (n + 15) // 16 for key, n in requests.items()}
        if sum(sizes.values()) > len(self.free):
            raise MemoryError("KV capacity exhausted")
        for key, n in sizes.items():
            self.tables[key] = [self.free.pop() for _ in range(n)]

    def release(self, key):
        self.free.extend(self.tables.pop(key))


def page_allocator():
    """The reference's allocator class where available, else the test stand-in."""
    return reference_blocks() or FreeListPages

# Parity bar for attention outputs (bf16 result vs fp32 reference), from the task contract.
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3


def load_golden(name: str) -> tuple[np.ndarray, dict]:
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return z["out_kernel"], json.loads(bytes(z["meta"]).decode())


def oracle_inputs(inp: dict):
    """Float32 arrays (bf16 values) of a case, with the append already applied."""
    import oracle

    kp = cases.as_f32(inp["k_pool"]).copy()
    vp = cases.as_f32(inp["v_pool"]).copy()
    if inp["append"]:
        oracle.kv_append(kp, vp, cases.as_f32(inp["k_new"]), cases.as_f32(inp["v_new"]),
                         inp["slots"])
    return cases.as_f32(inp["q"]), kp, vp


def bf16_tensor(bits: np.ndarray, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def bits_of(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
