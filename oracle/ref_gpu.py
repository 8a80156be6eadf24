"""TEST / MEASUREMENT INFRASTRUCTURE ONLY: Python handle on
oracle/_ref/libref_gpu.so, the reference's GPU schedule (its own CUDA
kernels from src/backend/cuda/kernels.rs and its cuBLAS FP32 op sequence of
src/backend/cuda/mod.rs:466-812, restated on the host in
oracle/ref_gpu_schedule.cu; built by oracle/ref_gpu_build.py).  Weights come
from a loaded OracleModel (f32, graph layout)."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import oracle as O
from .ref_gpu_build import LIB, build

_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)
_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build()
        if path is None or not os.path.exists(LIB):
            raise RuntimeError("oracle/_ref/libref_gpu.so is missing (built from the reference tree)")
        L = ctypes.CDLL(LIB)
        vp = ctypes.c_void_p
        L.rg_error.restype = ctypes.c_char_p
        L.rg_open.restype = vp
        L.rg_open.argtypes = [ctypes.c_int]
        L.rg_upload.argtypes = [vp, ctypes.c_char_p, _f32p, ctypes.c_size_t]
        L.rg_forward.argtypes = [vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64] + [_i64p] * 5 + [_f32p, _f32p]
        L.rg_time.argtypes = [vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64] + [_i64p] * 5 + \
            [ctypes.c_int, _f32p]
        L.rg_close.argtypes = [vp]
        L.rg_close.restype = None
        _lib = L
    return _lib


def available() -> bool:
    try:
        lib()
        return True
    except (RuntimeError, OSError):
        return False


class RefGpuSchedule:
    def __init__(self, model: "O.OracleModel", device: int = 0):
        L = lib()
        self._h = L.rg_open(device)
        if not self._h:
            raise RuntimeError(L.rg_error().decode())
        ol = O.lib()
        for i in range(ol.lo_weight_count()):
            name = ol.lo_weight_name(i)
            n = ctypes.c_size_t()
            ptr = ol.lo_weight_data(model._h, name, ctypes.byref(n))
            if not ptr:
                raise RuntimeError(f"oracle has no weight {name.decode()}")
            if L.rg_upload(self._h, name, ptr, n.value) != 0:
                raise RuntimeError(L.rg_error().decode())

    @staticmethod
    def _args(req_arrays):
        return [np.ascontiguousarray(a, np.int64).ctypes.data_as(_i64p) for a in req_arrays]

    def forward(self, n, l, k, ids, att, mpos, mmask, qtype):
        arrs = [np.ascontiguousarray(a, np.int64) for a in (ids, att, mpos, mmask, qtype)]
        logits = np.empty(n * k, np.float32)
        act = np.empty(n * 2, np.float32)
        rc = lib().rg_forward(self._h, n, l, k, *[a.ctypes.data_as(_i64p) for a in arrs],
                              logits.ctypes.data_as(_f32p), act.ctypes.data_as(_f32p))
        if rc:
            raise RuntimeError(lib().rg_error().decode())
        return logits, act

    def time(self, n, l, k, ids, att, mpos, mmask, qtype, iters: int) -> float:
        arrs = [np.ascontiguousarray(a, np.int64) for a in (ids, att, mpos, mmask, qtype)]
        ms = ctypes.c_float()
        rc = lib().rg_time(self._h, n, l, k, *[a.ctypes.data_as(_i64p) for a in arrs], iters, ctypes.byref(ms))
        if rc:
            raise RuntimeError(lib().rg_error().decode())
        return ms.value

    def close(self):
        if self._h:
            lib().rg_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
