"""Builds the sm_100a shared library ``laya_rust_b200/_lib/liblaya_b200.so``.

Ahead-of-time nvcc build for ``-gencode arch=compute_100a,code=sm_100a``
(no NVRTC, no JIT): every kernel and the host engine go into one shared
library exporting the C ABI of ``include/laya_b200.h``.  The CUDA runtime is
linked statically, so the library needs only the driver at run time.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIB_DIR, "liblaya_b200.so")
OBJ_DIR = os.path.join(ROOT, "_build", "obj")

SOURCES = ["gemm.cu", "attn_tc.cu", "attn_short.cu", "rownorm.cu", "tail.cu", "tail_static.cu", "engine.cpp",
           "gguf_reader.cpp", "json.cpp", "frontend.cpp", "serve.cpp"]
HEADERS = ["common.cuh", "kernels.h", "gguf_reader.h", "json.h", "unicode_tables.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", h)
                                                       for h in ("laya_b200.h", "laya_frontend.h", "laya_serve.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ_DIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [NVCC] + ARCH + FLAGS + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.check_call(cmd)
    if force or _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-lpthread"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
