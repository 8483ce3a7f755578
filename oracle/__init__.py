"""CPU oracle of the ShardServe attention path — test infrastructure, never product code.

Importable only from tests/, __graft_entry__.smoke() and bench.py (CPU baseline / reference
arm).  See ragged_attention.py for the restated reference functions and their citations.
"""
from .ragged_attention import (  # noqa: F401
    bf16_bits,
    bf16_round,
    bf16_to_f32,
    host_threads,
    kv_append,
    ragged_attention,
    token_slots,
)
from .rope import apply_rope_bits, rope_tables  # noqa: F401
