"""Python host mirror of the reference's engine seam over the C ABI.

``Req``, ``Out``, ``EngineInfo`` and ``Engine.forward`` mirror laya-rust
``src/engine.rs:1-92``: a request of padded index arrays goes in, raw marker
logits ``[n*k]`` and act logits ``[n*2]`` come out in host memory.  Errors
raise :class:`LayaError` carrying the C status code (the reference panics).

The library is ``_lib/liblaya_b200.so`` built by ``build.py``; there is no
fallback: if it is missing or no B200 is visible, opening an engine fails.
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass

import numpy as np

from . import arch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "liblaya_b200.so")

LAYA_OK, LAYA_E_INVALID, LAYA_E_LOAD, LAYA_E_CUDA, LAYA_E_DEVICE_TIMEOUT, LAYA_E_STATE = range(6)

_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)
TAP_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, _f32p, ctypes.c_size_t)


class LayaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class _CReq(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int64), ("l", ctypes.c_int64), ("k", ctypes.c_int64),
                ("ids", _i64p), ("att", _i64p), ("mpos", _i64p), ("mmask", _i64p),
                ("qtype", _i64p)]


_lib = None


def lib():
    """Loads the shared library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LayaError(LAYA_E_STATE, f"{LIB_PATH} is missing: run laya_rust_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        vp = ctypes.c_void_p
        L.laya_last_error.restype = ctypes.c_char_p
        L.laya_open.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(vp)]
        L.laya_open_empty.argtypes = [ctypes.c_int, ctypes.POINTER(vp)]
        L.laya_upload_weight_f16.argtypes = [vp, ctypes.c_char_p, ctypes.c_void_p, _i64p, ctypes.c_int]
        L.laya_upload_weight_f32.argtypes = [vp, ctypes.c_char_p, _f32p, _i64p, ctypes.c_int]
        L.laya_upload_weight_f32_graph.argtypes = [vp, ctypes.c_char_p, _f32p, _i64p, ctypes.c_int]
        L.laya_finalize.argtypes = [vp]
        L.laya_forward.argtypes = [vp, ctypes.POINTER(_CReq), _f32p, _f32p]
        L.laya_forward_tapped.argtypes = [vp, ctypes.POINTER(_CReq), _f32p, _f32p, TAP_FN, vp]
        L.laya_info.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t]
        L.laya_close.argtypes = [vp]
        L.laya_close.restype = None
        L.laya_plan_create.argtypes = [vp, ctypes.POINTER(_CReq), ctypes.POINTER(vp)]
        L.laya_plan_run.argtypes = [vp, vp]
        L.laya_plan_outputs.argtypes = [vp, vp, _f32p, _f32p]
        L.laya_plan_capture.argtypes = [vp, vp]
        L.laya_plan_stats.argtypes = [vp, _i64p, _i64p, _i64p]
        L.laya_plan_profile.argtypes = [vp, vp, ctypes.c_int, ctypes.POINTER(ctypes.c_double), _i64p]
        L.laya_plan_destroy.argtypes = [vp]
        L.laya_plan_destroy.restype = None
        L.laya_plan_set_hidden.argtypes = [vp, vp, _f32p]
        L.laya_plan_run_layer.argtypes = [vp, vp, ctypes.c_int]
        L.laya_plan_hidden.argtypes = [vp, vp, _f32p]
        L.laya_stream.argtypes = [vp]
        L.laya_stream.restype = vp
        L.laya_decision_tail_static.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, vp, vp, vp, vp, vp, vp]
        L.laya_test_timeout_next.argtypes = [vp, ctypes.c_int, ctypes.c_uint64]
        L.laya_selftest_gemm.argtypes = [ctypes.c_int, vp, vp, _f32p, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int]
        L.laya_selftest_attention.argtypes = [ctypes.c_int, vp, ctypes.POINTER(ctypes.c_int32),
                                              ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int]
        L.laya_bench_gemm.argtypes = [ctypes.c_int] * 8 + [_f32p]
        _i32p = ctypes.POINTER(ctypes.c_int32)
        L.laya_plan_layout.argtypes = [ctypes.POINTER(_CReq), _i64p, _i64p, _i32p, ctypes.c_int64, _i64p, _i32p,
                                       ctypes.c_int64]
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != LAYA_OK:
        raise LayaError(rc, lib().laya_last_error().decode(errors="replace"))


@dataclass
class Req:
    """engine::Req (src/engine.rs:1-10)."""
    n: int
    l: int
    k: int
    ids: np.ndarray
    att: np.ndarray
    mpos: np.ndarray
    mmask: np.ndarray
    qtype: np.ndarray

    def __post_init__(self):
        for f in ("ids", "att", "mpos", "mmask", "qtype"):
            setattr(self, f, np.ascontiguousarray(np.asarray(getattr(self, f)).ravel(), dtype=np.int64))

    def _c(self) -> _CReq:
        p = lambda a: a.ctypes.data_as(_i64p)
        return _CReq(self.n, self.l, self.k, p(self.ids), p(self.att), p(self.mpos), p(self.mmask),
                     p(self.qtype))

    def real_tokens(self) -> int:
        return int((self.att.reshape(self.n, self.l) != 0).sum())


@dataclass
class Out:
    """engine::Out (src/engine.rs:12-17)."""
    n: int
    k: int
    logits: np.ndarray
    act: np.ndarray


@dataclass
class EngineInfo:
    """engine::EngineInfo (src/engine.rs:71-77)."""
    id: str
    device: str
    dtype: str
    layers: int
    calibration: dict


class Plan:
    """A request uploaded once to device memory (device-resident runs)."""

    def __init__(self, engine: "Engine", req: Req):
        self._e = engine
        self.req = req
        h = ctypes.c_void_p()
        _check(lib().laya_plan_create(engine._h, ctypes.byref(req._c()), ctypes.byref(h)))
        self._h = h

    def run(self) -> None:
        _check(lib().laya_plan_run(self._e._h, self._h))

    def capture(self) -> None:
        _check(lib().laya_plan_capture(self._e._h, self._h))

    def outputs(self) -> Out:
        r = self.req
        logits = np.empty(r.n * r.k, np.float32)
        act = np.empty(r.n * 2, np.float32)
        _check(lib().laya_plan_outputs(self._e._h, self._h, logits.ctypes.data_as(_f32p),
                                       act.ctypes.data_as(_f32p)))
        return Out(r.n, r.k, logits, act)

    def set_hidden(self, x: np.ndarray) -> None:
        """Residual stream of the real tokens, [real_tokens, 1024] f32."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        _check(lib().laya_plan_set_hidden(self._e._h, self._h, x.ctypes.data_as(_f32p)))

    def run_layer(self, layer: int) -> None:
        """Enqueues encoder layer `layer` (0..27) alone on the current residual
        stream (for layer 0: the embedding output, before the embedding norm)."""
        _check(lib().laya_plan_run_layer(self._e._h, self._h, layer))

    def hidden(self) -> np.ndarray:
        """Synchronizes and returns the residual stream, [real_tokens, 1024] f32."""
        x = np.empty((self.stats()[0], arch.H), np.float32)
        _check(lib().laya_plan_hidden(self._e._h, self._h, x.ctypes.data_as(_f32p)))
        return x

    PROF_KINDS = ["gemm_qkv", "gemm_attn_out", "gemm_ffn_in_geglu", "gemm_ffn_out", "gemm_head_scorer",
                  "attention", "row_norms", "tail"]

    def profile(self, steps: int) -> dict:
        """Device time (ms, summed over `steps` runs) and launch count per kernel kind."""
        ms = (ctypes.c_double * 8)()
        nl = (ctypes.c_int64 * 8)()
        _check(lib().laya_plan_profile(self._e._h, self._h, steps, ms, nl))
        return {k: (ms[i], nl[i]) for i, k in enumerate(self.PROF_KINDS)}

    def stats(self) -> tuple[int, int, int]:
        """(real tokens, kernel launches per run, host->device bytes per forward)."""
        rt, nl, ub = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        _check(lib().laya_plan_stats(self._h, ctypes.byref(rt), ctypes.byref(nl), ctypes.byref(ub)))
        return rt.value, nl.value, ub.value

    def close(self):
        if getattr(self, "_h", None):
            lib().laya_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


class Engine:
    """The B200 engine: Engine::forward over the C ABI (one per GPU)."""

    def __init__(self, gguf_path: str | None = None, device: int = 0):
        h = ctypes.c_void_p()
        if gguf_path is None:
            _check(lib().laya_open_empty(device, ctypes.byref(h)))
        else:
            _check(lib().laya_open(device, os.fsencode(gguf_path), ctypes.byref(h)))
        self._h = h
        self.device = device

    def upload_f16(self, name: str, data: np.ndarray) -> None:
        a = np.ascontiguousarray(data, dtype=np.float16)
        dims = np.asarray(a.shape, dtype=np.int64)
        _check(lib().laya_upload_weight_f16(self._h, name.encode(), a.ctypes.data, dims.ctypes.data_as(_i64p),
                                            a.ndim))

    def upload_f32(self, name: str, data: np.ndarray) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32)
        dims = np.asarray(a.shape, dtype=np.int64)
        _check(lib().laya_upload_weight_f32(self._h, name.encode(), a.ctypes.data_as(_f32p),
                                            dims.ctypes.data_as(_i64p), a.ndim))

    def upload_f32_graph(self, name: str, data: np.ndarray) -> None:
        """A tensor in graph layout (Tensors::f32 / Tensors::dims, weights.rs:270-295)."""
        a = np.ascontiguousarray(data, dtype=np.float32)
        dims = np.asarray(a.shape, dtype=np.int64)
        _check(lib().laya_upload_weight_f32_graph(self._h, name.encode(), a.ctypes.data_as(_f32p),
                                                  dims.ctypes.data_as(_i64p), a.ndim))

    def finalize(self) -> None:
        _check(lib().laya_finalize(self._h))

    def info(self) -> EngineInfo:
        buf = ctypes.create_string_buffer(4096)
        _check(lib().laya_info(self._h, buf, 4096))
        d = json.loads(buf.value.decode())
        return EngineInfo(d["id"], d["device"], d["dtype"], d["layers"], d["calibration"])

    def forward(self, req: Req, taps: dict | None = None) -> Out:
        logits = np.empty(req.n * req.k, np.float32)
        act = np.empty(req.n * 2, np.float32)
        c = req._c()
        if taps is None:
            _check(lib().laya_forward(self._h, ctypes.byref(c), logits.ctypes.data_as(_f32p),
                                      act.ctypes.data_as(_f32p)))
        else:
            def cb(_u, stage, data, count):
                taps[stage.decode()] = np.ctypeslib.as_array(data, shape=(count,)).copy()
            fn = TAP_FN(cb)
            _check(lib().laya_forward_tapped(self._h, ctypes.byref(c), logits.ctypes.data_as(_f32p),
                                             act.ctypes.data_as(_f32p), fn, None))
        return Out(req.n, req.k, logits, act)

    def plan(self, req: Req) -> Plan:
        return Plan(self, req)

    def decision_tail_static(self, x: int, n: int, k: int, cls_row: int, mk_row: int, mmask: int,
                             logits: int, act: int, stream: int = 0) -> None:
        """laya_decision_tail_static on caller-owned device buffers (raw device
        addresses): scorer, post and act head with no device allocation."""
        _check(lib().laya_decision_tail_static(self._h, x, n, k, cls_row, mk_row, mmask, logits, act,
                                               stream or None))

    def test_timeout_next(self, kind: int, limit_ns: int = 1_000_000) -> None:
        """Arms the next forward's first GEMM (kind 0) or attention launch
        (kind 1) to wait on a barrier nothing completes, bounded by limit_ns;
        that forward then raises LayaError(LAYA_E_DEVICE_TIMEOUT)."""
        _check(lib().laya_test_timeout_next(self._h, kind, limit_ns))

    def stream(self) -> int:
        return lib().laya_stream(self._h) or 0

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().laya_close(self._h)
            self._h = None

    def __del__(self):
        self.close()


def selftest_gemm(a: np.ndarray, w: np.ndarray, device: int = 0, tile_n: int = 256) -> np.ndarray:
    """out = a . w^T through the tcgen05 GEMM (f16 inputs, f32 result) on
    256 x tile_n tiles."""
    a = np.ascontiguousarray(a, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    m, k = a.shape
    n = w.shape[0]
    out = np.empty((m, n), np.float32)
    _check(lib().laya_selftest_gemm(device, a.ctypes.data, w.ctypes.data, out.ctypes.data_as(_f32p), m, n, k,
                                    tile_n))
    return out


def plan_layout(req: Req) -> tuple[int, np.ndarray, np.ndarray]:
    """laya_plan_layout: (real rows, tiles [T, 2], items [I, 4]) of the
    request's host plan, with no device; raises LayaError as laya_forward
    would for an invalid request."""
    c = req._c()
    rows, nt, ni = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    L = lib()
    _check(L.laya_plan_layout(ctypes.byref(c), ctypes.byref(rows), ctypes.byref(nt), None, 0, ctypes.byref(ni),
                              None, 0))
    tiles = np.zeros((nt.value, 2), np.int32)
    items = np.zeros((ni.value, 4), np.int32)
    i32p = ctypes.POINTER(ctypes.c_int32)
    _check(L.laya_plan_layout(ctypes.byref(c), ctypes.byref(rows), ctypes.byref(nt), tiles.ctypes.data_as(i32p),
                              nt.value, ctypes.byref(ni), items.ctypes.data_as(i32p), ni.value))
    return rows.value, tiles, items


def bench_gemm(m: int, n: int, k: int, epi: int, iters: int, device: int = 0, tile_n: int = 256,
               flush_l2: bool = True) -> float:
    """Mean device time (ms) of one launch of the tcgen05 GEMM with the
    forward's epilogue `epi` on [m, k] x [n, k]^T (operands of a fixed
    pattern; with flush_l2 a 256 MiB memset runs untimed before each launch)."""
    ms = ctypes.c_float(0.0)
    _check(lib().laya_bench_gemm(device, m, n, k, tile_n, epi, 1 if flush_l2 else 0, iters, ctypes.byref(ms)))
    return float(ms.value)


def selftest_attention(qkv: np.ndarray, lens, window: int, device: int = 0, impl: int = 1) -> np.ndarray:
    """Ragged attention on packed qkv [R, 3072] f16; returns [R, 1024] f32.
    impl 1: the tcgen05 kernel the forward uses (the only one)."""
    qkv = np.ascontiguousarray(qkv, dtype=np.float16)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    out = np.empty((qkv.shape[0], 1024), np.float32)
    _check(lib().laya_selftest_attention(device, qkv.ctypes.data,
                                         lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                         len(lens), window, out.ctypes.data_as(_f32p), impl))
    return out
