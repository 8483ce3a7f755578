"""C ABI checks that need no GPU: the library loads, exports every declared entry point,
and rejects bad arguments before touching the device."""
import ctypes
import os
import re

import pytest

from shardserve_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "shardserve_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"SS_API\s+[\w\s\*]+?\b(ss_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for name in ("ss_kv_append", "ss_ragged_paged_attention", "ss_attention_workspace_bytes"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) <= set(_native.SIGNATURES)


def test_library_is_sm100a_only():
    # The fat binary carries sm_100a SASS only (cuobjdump is not used: the ELF note
    # section names the target architecture in the nvcc-written fatbin header).
    data = open(_native.LIB_PATH, "rb").read()
    assert b"sm_100a" in data


def test_status_strings():
    lib = _native.lib()
    assert lib.ss_status_string(0) == b"ok"
    assert lib.ss_status_string(_native.SS_ERR_WORKSPACE) == b"workspace too small"
    assert lib.ss_version() >= 100


def _attn(**over):
    args = dict(q=1, qs=(0, 0, 1), kp=1, ks=(0, 0, 0, 1), vp=1, vs=(0, 0, 0, 1), bt=1,
                bts=(1, 1), rows=1, cols=1, bt64=0, seq=1, seq64=0, pos=1, pos64=1, out=1,
                os=(0, 0, 1), T=1, H=8, KVH=1, D=128, N=1, scale=0.1, ws=1, wsb=1 << 20,
                stream=None)
    args.update(over)
    s = _native.strides
    return _native.lib().ss_ragged_paged_attention(
        args["q"], s(args["qs"]), args["kp"], s(args["ks"]), args["vp"], s(args["vs"]),
        args["bt"], s(args["bts"]), args["rows"], args["cols"], args["bt64"], args["seq"],
        args["seq64"], args["pos"], args["pos64"], args["out"], s(args["os"]), args["T"],
        args["H"], args["KVH"], args["D"], args["N"], args["scale"], args["ws"], args["wsb"],
        args["stream"])


@pytest.mark.parametrize("over,needle", [
    (dict(D=96), "64|128"),
    (dict(T=0), "empty"),
    (dict(H=6, KVH=4), "divisible"),
    (dict(rows=0), "block_tables"),
    (dict(N=0), "page"),
    (dict(q=None), "null"),
    (dict(scale=float("nan")), "finite"),
    (dict(qs=(-1, 0, 1)), "negative"),
])
def test_attention_rejects_invalid_arguments_on_host(over, needle):
    assert _attn(**over) == _native.SS_ERR_INVALID
    assert needle in _native.last_error()


def test_attention_requires_workspace():
    assert _attn(ws=None) == _native.SS_ERR_WORKSPACE
    assert _attn(wsb=16) == _native.SS_ERR_WORKSPACE


def test_append_rejects_invalid_arguments_and_accepts_empty():
    lib = _native.lib()
    s = _native.strides
    z3, z4 = s((0, 0, 1)), s((0, 0, 0, 1))
    assert lib.ss_kv_append(1, z3, 1, z3, 1, z4, 1, z4, 1, 1, 0, 1, 1, 128, None, None) == 0
    assert lib.ss_kv_append(1, z3, 1, z3, 1, z4, 1, z4, 1, 1, -1, 1, 1, 128, None, None) == 1
    assert lib.ss_kv_append(None, z3, 1, z3, 1, z4, 1, z4, 1, 1, 4, 1, 1, 128, None, None) == 1
    assert lib.ss_kv_append(1, z3, 1, z3, 1, z4, 1, z4, 1, 1, 4, 0, 1, 128, None, None) == 1


def test_fetch_errors_rejects_null():
    flags = ctypes.c_uint32(0)
    assert _native.lib().ss_fetch_device_errors(None, 0, ctypes.byref(flags), None) == 1
