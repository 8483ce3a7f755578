"""Bindings of the in-tree sm_100a library `libshardserve_b200.so`.

The library is the product: every attention / append call goes through it.  `lib()` is its
ctypes binding (the whole C ABI); `ops()` is the torch-tensor binding of the per-layer hot
calls (`_shardserve_torch.so`, csrc/torch_binding.cpp), which calls the same library through
the entry-point addresses ctypes resolved.  There is no Python or CPU fallback; if either
file is missing these raise ImportError-like errors on first use, naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import threading

from ._build import BINDING_NAME, BINDING_PATH, LIB_PATH

_lock = threading.RLock()
_lib = None
_ops = None

_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p

SS_OK = 0
SS_ERR_INVALID = 1
SS_ERR_UNSUPPORTED = 2
SS_ERR_CUDA = 3
SS_ERR_WORKSPACE = 4

SS_DEVERR_PAGE = 0x1
SS_DEVERR_SEQ = 0x2
SS_DEVERR_POS = 0x4
SS_DEVERR_SLOT = 0x8
SS_DEVERR_TIMEOUT = 0x10

# Every symbol the header declares, with its ctypes signature.
SIGNATURES = {
    "ss_version": (ctypes.c_int, []),
    "ss_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ss_last_error_message": (ctypes.c_char_p, []),
    "ss_kv_append": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, ctypes.c_int,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _vp, _vp]),
    "ss_rope_kv_append": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, ctypes.c_int64,
        _vp, ctypes.c_int, _vp, _i64p, _vp, _i64p, _vp, ctypes.c_int, ctypes.c_int64,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _vp, _vp]),
    "ss_build_metadata": (ctypes.c_int, [
        _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp, _vp, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int64, ctypes.c_int64, _vp, _vp, _vp, _vp,
        _vp, _vp, _vp]),
    "ss_tp2_oproj_allreduce": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
        _vp, _vp, ctypes.c_int64, _vp, _vp, _vp]),
    "ss_device_alloc_zeroed": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "ss_device_free": (ctypes.c_int, [_vp]),
    "ss_ipc_handle": (ctypes.c_int, [_vp, _vp]),
    "ss_ipc_open": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "ss_ipc_close": (ctypes.c_int, [_vp]),
    "ss_attention_workspace_bytes": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_size_t)]),
    "ss_ragged_paged_attention": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _i64p, ctypes.c_int64,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_float, _vp,
        ctypes.c_size_t, _vp]),
    "ss_append_ragged_paged_attention": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, ctypes.c_int,
        _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _i64p, ctypes.c_int64,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_float, _vp,
        ctypes.c_size_t, _vp]),
    "ss_ragged_paged_attention_noalloc": (ctypes.c_int, [
        _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _i64p, ctypes.c_int64,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_float, _vp]),
    "ss_fetch_device_errors": (ctypes.c_int, [
        _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32), _vp]),
    "ss_noalloc_fetch_device_errors": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32), _vp]),
    "ss_last_attention_path": (ctypes.c_int, []),
    "ss_kernel_launch_count": (ctypes.c_ulonglong, []),
}


class NativeLibraryMissing(ImportError):
    pass


def lib() -> ctypes.CDLL:
    """Loads (once) and returns the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise NativeLibraryMissing(
                    f"{LIB_PATH} is missing; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` or "
                    "`python shardserve_b200/_build.py`")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().ss_last_error_message()
    return msg.decode() if msg else ""


def strides(seq) -> ctypes.Array:
    arr = (ctypes.c_int64 * len(seq))(*seq)
    return arr


_BOUND = ("ss_ragged_paged_attention", "ss_append_ragged_paged_attention", "ss_kv_append",
          "ss_rope_kv_append", "ss_attention_workspace_bytes", "ss_last_error_message")


def ops():
    """Loads (once), binds and returns the torch-tensor binding module."""
    global _ops
    if _ops is not None:
        return _ops
    with _lock:
        if _ops is None:
            import importlib.machinery
            import importlib.util

            import torch  # noqa: F401  (the binding links against the loaded libtorch)

            from .kernel import KernelUnsupported

            if not os.path.exists(BINDING_PATH):
                raise NativeLibraryMissing(
                    f"{BINDING_PATH} is missing; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` or "
                    "`python shardserve_b200/_build.py`")
            loader = importlib.machinery.ExtensionFileLoader(BINDING_NAME, BINDING_PATH)
            spec = importlib.util.spec_from_file_location(BINDING_NAME, BINDING_PATH,
                                                          loader=loader)
            mod = importlib.util.module_from_spec(spec)
            loader.exec_module(mod)
            handle = lib()
            addrs = {n: ctypes.cast(getattr(handle, n), ctypes.c_void_p).value for n in _BOUND}
            mod.bind(addrs, KernelUnsupported)
            _ops = mod
    return _ops
