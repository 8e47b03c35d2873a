"""Builds libmhcpre_b200.so in place with nvcc for sm_100a.

The library is plain CUDA C++ behind the C ABI in include/mhc_pre.h: no torch
headers, cudart linked statically, the driver reached through
cudaGetDriverEntryPoint (so no -lcuda is needed at link time).

``build(trace=True)`` (``python -m mhcpre_review_b200.build --trace``) builds the
trace library libmhcpre_b200_trace.so instead: the same sources with -DMHC_TRACE,
which adds the stage stamps and mhcPreTraceRead (include/mhc_pre_trace.h).
``build(debug=True)`` (``--debug``) builds libmhcpre_b200_debug.so: -DMHC_DEBUG, the
kernels' bounds checks and include/mhc_pre_debug.h.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmhcpre_b200.so"
TRACE_LIB = PKG / "libmhcpre_b200_trace.so"
DEBUG_LIB = PKG / "libmhcpre_b200_debug.so"
SOURCES = ["mhc_pre_kernels.cu", "mhc_pre_api.cpp", "mhc_pre_noalloc.cu"]
HEADERS = ["ptx.cuh", "mhc_pre_internal.h", "mhc_pre_fused.cuh", "mhc_pre_decode.cuh", "mhc_pre_cluster.cuh",
           "mhc_pre_small.cuh", "mhc_pre_onepass.cuh", "mhc_pre_pair.cuh", "mhc_post.cuh", "mhc_post_pre.cuh",
           "trace.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    return os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def _inputs():
    return ([CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] +
            [ROOT / "include" / h for h in ("mhc_pre.h", "mhc_pre_trace.h", "mhc_pre_debug.h")])


def needs_build(lib: Path = LIB) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None, trace: bool = False,
          debug: bool = False) -> Path:
    assert not (trace and debug), "one variant at a time"
    lib = TRACE_LIB if trace else DEBUG_LIB if debug else LIB
    if not force and not needs_build(lib):
        return lib
    objs = []
    build_dir = PKG / "_build" / ("trace" if trace else "debug" if debug else "default")
    build_dir.mkdir(parents=True, exist_ok=True)
    flags = [*NVCC_FLAGS, *(["-DMHC_TRACE"] if trace else []), *(["-DMHC_DEBUG"] if debug else []), *(extra or [])]
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *flags, "-I", str(ROOT / "include"), "-c", str(CSRC / src), "-o", str(obj)]
        if src.endswith(".cpp"):
            cmd[1:1] = ["-x", "cu"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        objs.append(str(obj))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, trace="--trace" in sys.argv, debug="--debug" in sys.argv,
                extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None))
