"""Generates tests/golden/<case>.npz by running the REFERENCE implementation itself.

For every case of cases.py this script imports ShardServe unchanged from the reference
checkout (the directory named by the SHARDSERVE_REFERENCE environment variable) and records:

* kpool_sha256 / vpool_sha256 — the bf16 pools after the reference's Cache.write
  (shardserve/cache.py:47-49, torch index_copy_), for the bit-exact append check;
* out_kernel — the reference Triton kernel `_ragged_paged_attention_kernel`
  (shardserve/kernel.py:85-166) executed by Triton's interpreter (TRITON_INTERPRET=1) on
  fp32 tensors holding the bf16 values, after the append;
* diag_vs_kernel — max |Cache.diagnostic - out_kernel| with fp32 pools (the reference's
  own CPU path, cache.py:51-61), recorded to show the two reference paths agree.

Run once in a container that has the reference (it is not needed afterwards):
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

REF = os.environ.get("SHARDSERVE_REFERENCE")
if not REF:
    sys.exit("set SHARDSERVE_REFERENCE to the reference checkout (its shardserve package)")
sys.path.insert(0, REF)
from shardserve import kernel as ref_kernel  # noqa: E402
from shardserve.cache import Cache as RefCache  # noqa: E402


def _t(bits: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(cases.as_f32(bits).copy()).to(dtype)


def _cache(kp: torch.Tensor, vp: torch.Tensor) -> RefCache:
    c = RefCache.__new__(RefCache)
    c.k = kp[None].clone()
    c.v = vp[None].clone()
    c.shape = tuple(c.k.shape)
    return c


def run_case(name: str) -> dict:
    inp = cases.build(name)
    H, KVH, D = inp["H"], inp["KVH"], inp["D"]
    bt = torch.from_numpy(inp["block_tables"])
    seqs = torch.from_numpy(inp["seq_ids"])
    pos = torch.from_numpy(inp["positions"])
    rec = {"name": name, "input_sha256": cases.input_digest(inp)}

    # (1) Append through the reference's Cache.write on bf16 pools: bit-exact target.
    kp16 = _t(inp["k_pool"], torch.bfloat16)
    vp16 = _t(inp["v_pool"], torch.bfloat16)
    c16 = _cache(kp16, vp16)
    if inp["append"]:
        c16.write(0, _t(inp["k_new"], torch.bfloat16), _t(inp["v_new"], torch.bfloat16),
                  torch.from_numpy(inp["slots"]))
    kbits = c16.k[0].contiguous().view(torch.int16).numpy().view(np.uint16)
    vbits = c16.v[0].contiguous().view(torch.int16).numpy().view(np.uint16)
    rec["kpool_sha256"] = cases.digest(kbits)
    rec["vpool_sha256"] = cases.digest(vbits)

    # (2) fp32 pools holding the same bf16 values, after the same append.
    c32 = _cache(_t(inp["k_pool"], torch.float32), _t(inp["v_pool"], torch.float32))
    if inp["append"]:
        c32.write(0, _t(inp["k_new"], torch.float32), _t(inp["v_new"], torch.float32),
                  torch.from_numpy(inp["slots"]))
    q32 = _t(inp["q"], torch.float32)
    out = torch.empty_like(q32)
    kp, vp = c32.k[0], c32.v[0]
    ref_kernel._ragged_paged_attention_kernel[(q32.shape[0], H)](
        q32, bt, seqs, pos, kp, vp, out, inp["scale"], H // KVH,
        *q32.stride(), *bt.stride(), *kp.stride(), *vp.stride(), *out.stride(),
        BLOCK=16, HEAD_DIM=D)
    diag = c32.diagnostic(0, q32, bt, seqs, pos)
    rec["diag_vs_kernel"] = float((diag - out).abs().max())
    rec["out_kernel"] = out.numpy()
    return rec


def main(selected: list[str]) -> None:
    for name in selected or cases.names():
        rec = run_case(name)
        meta = {k: v for k, v in rec.items() if k != "out_kernel"}
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), out_kernel=rec["out_kernel"],
                            meta=np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8))
        print(name, json.dumps(meta))


if __name__ == "__main__":
    main(sys.argv[1:])
