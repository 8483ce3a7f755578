"""Builds the sm_100a shared library `libshardserve_b200.so` in-tree with nvcc.

The library exports the C ABI declared in include/shardserve_b200.h.  It is compiled for
B200 only (`-gencode arch=compute_100a,code=sm_100a`) and links the CUDA runtime
statically, so the single .so is all a GPU host needs next to this package.
"""
from __future__ import annotations

import concurrent.futures
import os
import shlex
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "libshardserve_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = ["capi.cu", "decode_attention.cu", "generic_attention.cu", "kv_append.cu", "noalloc.cu",
           "prefill_attention.cu", "rope_append.cu", "metadata.cu", "tp2_oproj.cu"]
HEADERS = ["attention.cuh", "ptx.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files.append(os.path.join(REPO_DIR, "include", "shardserve_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    built = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= built for f in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compiles every .cu source (in parallel) into LIB_PATH; returns the library path.
    Extra nvcc flags (for example -D overrides of tuning constants) come from the
    SS_NVCC_FLAGS environment variable."""
    if not force and not ptxas_info and up_to_date():
        return LIB_PATH
    nvcc = _nvcc()
    tmp_dir = os.path.join(PKG_DIR, "_build")
    os.makedirs(tmp_dir, exist_ok=True)
    extra = shlex.split(os.environ.get("SS_NVCC_FLAGS", ""))
    cmds = []
    for src in SOURCES:
        obj = os.path.join(tmp_dir, src.replace(".cu", ".o"))
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        cmds.append((cmd, obj))
    workers = max(1, min(len(cmds), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as ex:
        for f in [ex.submit(subprocess.run, cmd, check=True) for cmd, _ in cmds]:
            f.result()
    objs = [obj for _, obj in cmds]
    tmp_lib = LIB_PATH + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp_lib, *objs,
           "-Xcompiler", "-fPIC"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp_lib, LIB_PATH)
    return LIB_PATH


# ---- torch-tensor binding of the hot per-layer calls (host C++, torch headers) -------------
BINDING_NAME = "_shardserve_torch"
BINDING_SOURCE = os.path.join(CSRC, "torch_binding.cpp")
BINDING_PATH = os.path.join(PKG_DIR, BINDING_NAME + ".so")


def binding_up_to_date() -> bool:
    if not os.path.exists(BINDING_PATH):
        return False
    built = os.path.getmtime(BINDING_PATH)
    header = os.path.join(REPO_DIR, "include", "shardserve_b200.h")
    return all(os.path.getmtime(f) <= built for f in (BINDING_SOURCE, header))


def build_binding(force: bool = False, verbose: bool = False) -> str:
    """Compiles csrc/torch_binding.cpp against this interpreter's torch into BINDING_PATH
    (host code only: no GPU is needed to build it)."""
    if not force and binding_up_to_date():
        return BINDING_PATH
    from torch.utils import cpp_extension

    build_dir = os.path.join(PKG_DIR, "_build", "torch_binding")
    os.makedirs(build_dir, exist_ok=True)
    cpp_extension.load(name=BINDING_NAME, sources=[BINDING_SOURCE],
                       extra_include_paths=[os.path.join(REPO_DIR, "include")],
                       extra_cflags=["-O2", "-std=c++17"], build_directory=build_dir,
                       with_cuda=True, verbose=verbose)
    tmp = BINDING_PATH + ".tmp"
    shutil.copyfile(os.path.join(build_dir, BINDING_NAME + ".so"), tmp)
    os.replace(tmp, BINDING_PATH)
    return BINDING_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    build_binding(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
    print(BINDING_PATH)
