"""ctypes binding of the C oracle -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
reference arms may import this module.  It restates the laya-rust reference CPU
backend (``src/graph.rs`` + ``src/backend/cpu/mod.rs``); see laya_oracle.c for
the file:line map.  The shipped library never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblaya_oracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_sz = ctypes.c_size_t
TAP_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, _f32p, ctypes.c_size_t)


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "laya_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", HERE])
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        L.lo_open.restype = ctypes.c_void_p
        L.lo_open.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _sz]
        L.lo_close.argtypes = [ctypes.c_void_p]
        L.lo_forward_ex.restype = ctypes.c_int
        L.lo_forward_ex.argtypes = [ctypes.c_void_p, _sz, _sz, _sz, _i64p, _i64p, _i64p, _i64p,
                                    _i64p, _f32p, _f32p, TAP_FN, ctypes.c_void_p]
        L.lo_weight_data.restype = ctypes.POINTER(ctypes.c_float)
        L.lo_weight_data.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(_sz)]
        L.lo_encoder_layer.restype = ctypes.c_int
        L.lo_encoder_layer.argtypes = [ctypes.c_void_p, _sz, _sz, _i64p, ctypes.c_int, _f32p]
        L.lo_f2h.restype = ctypes.c_uint16
        L.lo_f2h.argtypes = [ctypes.c_float]
        L.lo_h2f.restype = ctypes.c_float
        L.lo_h2f.argtypes = [ctypes.c_uint16]
        L.lo_weight_name.restype = ctypes.c_char_p
        L.lo_weight_name.argtypes = [ctypes.c_int]
        L.lo_weight_transposed.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _p(a, t=_f32p):
    return a.ctypes.data_as(t)


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i(a):
    return np.ascontiguousarray(a, dtype=np.int64)


# ---- op-level API (cpu/mod.rs ops) --------------------------------------------------

def layernorm(x, w, b=None, eps=1e-5):
    x, w = _f(x), _f(w)
    rows, dim = x.shape
    out = np.empty_like(x)
    lib().lo_layernorm(_p(x), _sz(rows), _sz(dim), _p(w), _p(_f(b)) if b is not None else None,
                       ctypes.c_float(eps), _p(out))
    return out


def matmul(x, w):
    x, w = _f(x), _f(w)
    r, kk = x.shape
    assert w.shape[0] == kk, "matmul inner dim mismatch"
    y = np.empty((r, w.shape[1]), np.float32)
    lib().lo_matmul(_p(x), _sz(r), _sz(kk), _p(w), _sz(w.shape[1]), _p(y))
    return y


def matmul_order(x, w, tiled: bool):
    """matmul with the reference's traversal or the register-tiled one that
    LAYA_ORACLE_FAST selects, chosen explicitly."""
    x, w = _f(x), _f(w)
    r, kk = x.shape
    assert w.shape[0] == kk, "matmul inner dim mismatch"
    y = np.empty((r, w.shape[1]), np.float32)
    lib().lo_matmul_order(ctypes.c_int(1 if tiled else 0), _p(x), _sz(r), _sz(kk), _p(w), _sz(w.shape[1]), _p(y))
    return y


def matmul_t(x, w):
    x, w = _f(x), _f(w)
    r, kk = x.shape
    assert w.shape[1] == kk, "matmul_t inner dim mismatch"
    y = np.empty((r, w.shape[0]), np.float32)
    lib().lo_matmul_t(_p(x), _sz(r), _sz(kk), _p(w), _sz(w.shape[0]), _p(y))
    return y


def gelu(x):
    x = _f(x)
    out = np.empty_like(x)
    lib().lo_gelu(_p(x), _sz(x.size), _p(out))
    return out


def relu(x):
    x = _f(x)
    out = np.empty_like(x)
    lib().lo_relu(_p(x), _sz(x.size), _p(out))
    return out


def gelu_mul(x, half):
    x = _f(x)
    rows = x.shape[0]
    out = np.empty((rows, half), np.float32)
    lib().lo_gelu_mul(_p(x), _sz(rows), _sz(half), _p(out))
    return out


def split_qkv_rope(qkv, rope, scale, nh, hd, length):
    qkv = _f(qkv)
    rows = qkv.shape[0]
    n = rows // length
    q, k, v = (np.empty((n, nh, length, hd), np.float32) for _ in range(3))
    cs = _p(_f(rope[0])) if rope is not None else None
    sn = _p(_f(rope[1])) if rope is not None else None
    lib().lo_split_qkv_rope(_p(qkv), _sz(rows), cs, sn, ctypes.c_float(scale), _sz(nh), _sz(hd),
                            _sz(length), _p(q), _p(k), _p(v))
    return q, k, v


def attention(q, k, v, mask, nh, length):
    q, k, v, mask = _f(q), _f(k), _f(v), _f(mask)
    n, hd = q.shape[0], q.shape[3]
    out = np.empty((n * length, nh * hd), np.float32)
    lib().lo_attention(_p(q), _p(k), _p(v), _p(mask), _sz(n), _sz(nh), _sz(length), _sz(hd),
                       _p(out))
    return out


def window_mask(att, n, length, window=None):
    att = _i(att)
    m = np.empty((n, length, length), np.float32)
    lib().lo_window_mask(_p(att, _i64p), _sz(n), _sz(length),
                         ctypes.c_long(-1 if window is None else window), _p(m))
    return m


def add(a, b):
    a, b = _f(a), _f(b)
    assert a.size == b.size, "add shape mismatch"
    out = np.empty_like(a)
    lib().lo_add(_p(a), _p(b), _sz(a.size), _p(out))
    return out


def add_bias(x, b):
    x, b = _f(x), _f(b)
    out = np.empty_like(x)
    lib().lo_add_bias(_p(x), _sz(x.size), _p(b), _sz(b.size), _p(out))
    return out


def embedding(table, ids):
    table, ids = _f(table), _i(ids)
    dim = table.shape[1]
    out = np.empty((ids.size, dim), np.float32)
    lib().lo_embedding(_p(table), _sz(dim), _p(ids, _i64p), _sz(ids.size), _p(out))
    return out


def add_type(x, type_emb, qtype, length):
    x, type_emb, qtype = _f(x), _f(type_emb), _i(qtype)
    rows, dim = x.shape
    out = np.empty_like(x)
    lib().lo_add_type(_p(x), _sz(rows), _sz(dim), _p(type_emb), _p(qtype, _i64p), _sz(length),
                      _p(out))
    return out


def gather_markers(x, mpos, k):
    x, mpos = _f(x), _i(mpos)
    rows, dim = x.shape
    out = np.empty((mpos.size, dim), np.float32)
    lib().lo_gather_markers(_p(x), _sz(rows), _sz(dim), _p(mpos, _i64p), _sz(mpos.size), _sz(k),
                            _p(out))
    return out


def post(sc, mmask, k):
    sc, mmask = _f(sc), _i(mmask)
    n = sc.size // k
    logits = np.empty(sc.size, np.float32)
    feats = np.empty((n, 4), np.float32)
    lib().lo_post(_p(sc), _sz(sc.size), _p(mmask, _i64p), _sz(k), _p(logits), _p(feats))
    return logits, feats


def act_input(x, feats, length):
    x, feats = _f(x), _f(feats)
    dim = x.shape[1]
    n, nf = feats.shape
    out = np.empty((n, dim + nf), np.float32)
    lib().lo_act_input(_p(x), _sz(dim), _p(feats), _sz(n), _sz(nf), _sz(length), _p(out))
    return out


def f2h(x: float) -> int:
    return int(lib().lo_f2h(ctypes.c_float(x)))


def h2f(h: int) -> float:
    return float(np.float32(lib().lo_h2f(ctypes.c_uint16(h))))


def rope_freq(theta, half=32):
    out = np.empty(half, np.float32)
    lib().lo_rope_freq(ctypes.c_float(theta), _sz(half), _p(out))
    return out


def rope_tables(freq, length):
    freq = _f(freq)
    cs = np.empty((length, 32), np.float32)
    sn = np.empty((length, 32), np.float32)
    lib().lo_rope_tables(_p(freq), _sz(length), _p(cs), _p(sn))
    return cs, sn


# ---- whole model (graph.rs) ----------------------------------------------------------

class OracleModel:
    """The reference CPU engine (CpuEngine, cpu/mod.rs:468-501) over one GGUF."""

    def __init__(self, path: str):
        err = ctypes.create_string_buffer(512)
        self._h = lib().lo_open(path.encode(), err, 512)
        if not self._h:
            raise RuntimeError(err.value.decode())

    def close(self):
        if self._h:
            lib().lo_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward(self, n, l, k, ids, att, mpos, mmask, qtype, taps=None):
        """graph::forward; returns (logits [n*k], act [n*2]).  ``taps`` (a dict)
        receives the TapSink stages embed, enc.i, final, head.i, logits, act."""
        ids, att, mpos, mmask, qtype = (_i(a) for a in (ids, att, mpos, mmask, qtype))
        assert ids.size == n * l and att.size == n * l and mpos.size == n * k
        assert mmask.size == n * k and qtype.size == n
        logits = np.empty(n * k, np.float32)
        act = np.empty(n * 2, np.float32)
        if taps is not None:
            def cb(_u, stage, data, count):
                taps[stage.decode()] = np.ctypeslib.as_array(data, shape=(count,)).copy()
            fn = TAP_FN(cb)
        else:
            fn = TAP_FN()
        rc = lib().lo_forward_ex(self._h, n, l, k, _p(ids, _i64p), _p(att, _i64p),
                                 _p(mpos, _i64p), _p(mmask, _i64p), _p(qtype, _i64p),
                                 _p(logits), _p(act), fn, None)
        if rc != 0:
            raise RuntimeError("oracle forward rejected the request")
        return logits, act

    def encoder_layer(self, n, l, att, layer, x):
        """One encoder layer (0..27, graph.rs:104-123) on the padded residual
        stream x [n*l, 1024]; returns the new stream."""
        att = _i(att)
        y = np.ascontiguousarray(x, dtype=np.float32).reshape(n * l, 1024).copy()
        if lib().lo_encoder_layer(self._h, n, l, _p(att, _i64p), layer, _p(y)) != 0:
            raise RuntimeError("oracle encoder_layer rejected the arguments")
        return y
