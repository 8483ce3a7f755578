"""shardserve_b200: B200-native ragged paged attention + slot-mapped KV append.

Drop-in for the hot path of ShardServe (shardserve/kernel.py, shardserve/cache.py):

    from shardserve_b200.kernel import ragged_attention_direct, KernelUnsupported
    from shardserve_b200.cache import Cache

Kernels are hand-written sm_100a CUDA in `libshardserve_b200.so` (C ABI in
include/shardserve_b200.h), bound with ctypes; PyTorch supplies device memory and streams.
"""
from .kernel import (  # noqa: F401
    KernelUnsupported,
    SUPPORTED_BLOCK_SIZE,
    SUPPORTED_RAGGED_HEAD_DIMS,
    kv_append,
    kv_append_attention,
    ragged_attention_direct,
    rope_kv_append,
)
from .cache import Cache  # noqa: F401
from .metadata import DeviceMetadata  # noqa: F401

__all__ = [
    "KernelUnsupported", "SUPPORTED_BLOCK_SIZE", "SUPPORTED_RAGGED_HEAD_DIMS", "kv_append",
    "kv_append_attention",
    "ragged_attention_direct", "rope_kv_append", "Cache", "DeviceMetadata",
]
