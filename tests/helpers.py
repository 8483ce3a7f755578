"""Shared helpers for the tests: golden fixtures, case inputs as torch tensors."""
from __future__ import annotations

import json
import os

import numpy as np

import cases

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

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
