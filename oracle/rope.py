"""CPU oracle of rotary position embedding (RoPE) on bf16 q / k — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this module, and only as the checker.  The product path (shardserve_b200) never calls it.

Restates the reference's `apply_rope` (shardserve/math.py:28-38) as torch evaluates it on
bf16 tensors, one rounding per operation:

    c = bf16(cos[pos]), s = bf16(sin[pos])                    (math.py:36-37, `.to(q.dtype)`)
    rotate_half(x) = cat(-x[..., D/2:], x[..., :D/2])         (math.py:23-25)
    out = bf16( bf16(x * c) + bf16(rotate_half(x) * s) )      (math.py:38)

Each bf16 x bf16 product is exact in fp32 and rounded once to bf16 (round to nearest even);
the sum of the two bf16 terms is formed in fp32 (rounded there when their exponents differ
by more than 16) and rounded to bf16.  `cos` / `sin` are the caller's fp32 tables
(math.build_rope_cache, math.py:12-20) and are taken as given, so parity never depends on a
particular cos/sin implementation.  Pinned bit-exactly against the reference itself by
tests/golden/make_golden_rope.py.
"""
from __future__ import annotations

import numpy as np

from .ragged_attention import bf16_bits, bf16_to_f32


def apply_rope_bits(x_bits: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                    positions: np.ndarray) -> np.ndarray:
    """x_bits: bf16 bit patterns [T, heads, D]; cos / sin: fp32 [rows, D]; positions [T].
    Returns the rotated bf16 bit patterns (math.py:38, per-op bf16 rounding)."""
    x = bf16_to_f32(x_bits)
    pos = np.asarray(positions, dtype=np.int64)
    c = bf16_to_f32(bf16_bits(np.asarray(cos, dtype=np.float32)[pos]))[:, None, :]
    s = bf16_to_f32(bf16_bits(np.asarray(sin, dtype=np.float32)[pos]))[:, None, :]
    half = x.shape[-1] // 2
    rot = np.concatenate((-x[..., half:], x[..., :half]), axis=-1)
    a = bf16_to_f32(bf16_bits((x * c).astype(np.float32)))
    b = bf16_to_f32(bf16_bits((rot * s).astype(np.float32)))
    return bf16_bits((a + b).astype(np.float32))


def rope_tables(head_dim: int, max_len: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """fp32 cos / sin tables [max_len, head_dim] with the reference's layout (math.py:12-20:
    inverse frequencies theta^(-2i/D), angles pos * inv_freq, duplicated halves).  Values
    come from numpy's float32 math, so tests pass the same table to both sides."""
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                        / np.float32(head_dim)))).astype(np.float32)
    ang = np.arange(max_len, dtype=np.float32)[:, None] * inv[None, :]
    emb = np.concatenate((ang, ang), axis=-1).astype(np.float32)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
