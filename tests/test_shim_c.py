"""The Rust shim's call sequence through the C ABI, in a C program built with
gcc (tests/c/shim_sequence.c): laya_open_empty, one
laya_upload_weight_f32_graph per tensor with the values and dims the
reference's unchanged loader hands out (Tensors::f32 and Tensors::dims,
src/weights.rs:270-295: graph layout, the 120 matmul weights of
arch::transpose_names transposed), laya_finalize, laya_forward -- against
laya_open on the same GGUF.  The loader stand-in is write_graph_dump below
(gguf.rs decode + the arch.rs transpose)."""
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

from laya_rust_b200 import arch, gguf, modelgen

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c", "shim_sequence.c")
LIBDIR = os.path.join(ROOT, "laya_rust_b200", "_lib")


def build_program(out_dir):
    exe = os.path.join(out_dir, "shim_sequence")
    subprocess.check_call(["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), SRC,
                           "-o", exe, "-L", LIBDIR, "-llaya_b200", f"-Wl,-rpath,{LIBDIR}", "-lm"])
    return exe


def write_graph_dump(gguf_path, out_path):
    """What Tensors::f32 / Tensors::dims return for every tensor."""
    h = gguf.read(gguf_path)
    flip = set(arch.transpose_names())
    with open(out_path, "wb") as f:
        f.write(struct.pack("<I", len(h.tensors)))
        for t in h.tensors:
            v = h.f32(t.name)
            if t.name in flip and v.ndim == 2:
                v = np.ascontiguousarray(v.T)
            name = t.name.encode()
            f.write(struct.pack("<I", len(name)) + name + struct.pack("<I", v.ndim))
            f.write(np.asarray(v.shape, dtype="<i8").tobytes())
            f.write(np.ascontiguousarray(v, dtype="<f4").tobytes())


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no gcc")
def test_the_shim_program_builds_and_reports_a_missing_device(tmp_path):
    """Compiles and links against the library; without a usable GPU the first
    engine call returns a status (exit 3), never an abort."""
    import torch
    exe = build_program(str(tmp_path))
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU test covers the run")
    r = subprocess.run([exe, "none.dump", "none.gguf", "0"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 3, (r.returncode, r.stdout, r.stderr)
    assert "laya_open_empty failed" in r.stderr


@pytest.mark.gpu
def test_the_shim_sequence_matches_laya_open(tmp_path):
    exe = build_program(str(tmp_path))
    model = modelgen.cached_model(seed=0)
    dump = str(tmp_path / "graph.dump")
    write_graph_dump(model, dump)
    r = subprocess.run([exe, dump, model, "0"], capture_output=True, text=True, timeout=600)
    os.unlink(dump)
    print(r.stdout)
    assert r.returncode == 0, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    assert "identical outputs" in r.stdout
