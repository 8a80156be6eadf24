"""Builds oracle/_ref/libref_gpu.so: the reference's GPU schedule for timing
the reference's GPU algorithm on the same B200 (measurement infrastructure;
the product never loads it).

Recipe: the reference compiles the CUDA C source held in the SRC string of
laya-rust src/backend/cuda/kernels.rs with NVRTC at load time
(src/backend/cuda/mod.rs:83-101).  This script copies that string verbatim
from where it lies under the reference tree into oracle/_ref/ref_kernels.cuh
(not committed) and compiles it ahead of time with nvcc for sm_100a,
together with the C++ restatement of the host schedule
(oracle/ref_gpu_schedule.cu), linked to cuBLAS for the reference's FP32
SGEMMs.  Without the reference tree (the GPU box) it keeps an existing build.

The reference tree is given as an argument or by LAYA_REFERENCE_ROOT; with
neither, an existing build is kept and nothing is compiled.

Usage: python oracle/ref_gpu_build.py [reference-root]
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT, "libref_gpu.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def build(ref_root: str | None = None, force: bool = False) -> str | None:
    ref_root = ref_root or os.environ.get("LAYA_REFERENCE_ROOT")
    src = os.path.join(ref_root, "src", "backend", "cuda", "kernels.rs") if ref_root else ""
    if not src or not os.path.exists(src):
        return LIB if os.path.exists(LIB) else None
    text = open(src).read()
    a = text.index('r#"') + 3
    b = text.index('"#;', a)
    os.makedirs(OUT, exist_ok=True)
    kern = os.path.join(OUT, "ref_kernels.cuh")
    body = text[a:b]
    if not os.path.exists(kern) or open(kern).read() != body:
        with open(kern, "w") as f:
            f.write(body)
    host = os.path.join(HERE, "ref_gpu_schedule.cu")
    deps = [kern, host]
    if force or not os.path.exists(LIB) or any(os.path.getmtime(d) > os.path.getmtime(LIB) for d in deps):
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
               "-shared", f'-DREF_KERNELS="{kern}"', host, "-o", LIB, "-lcublas", "-cudart", "static",
               "-Xlinker", "-rpath=/usr/local/cuda/lib64", "-L/usr/local/cuda/lib64"]
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if a != "--force"]
    print(build(args[0] if args else None, force="--force" in sys.argv))
