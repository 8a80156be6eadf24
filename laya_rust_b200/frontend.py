"""ctypes binding of the request front end (include/laya_frontend.h): the
tokenizer (laya-rust src/tokenizer.rs), System One planning
(src/systemone.rs, src/main.rs:387-410), packing into forwards
(main.rs:448-500, and across requests), scoring and response JSON
(main.rs:502-557).  The work happens in the C++ library; this module only
moves arrays and strings across.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from .engine import LayaError, Req, _check, lib as _engine_lib

_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)
_bound = False


def lib():
    global _bound
    L = _engine_lib()
    if not _bound:
        vp = ctypes.c_void_p
        sz = ctypes.c_size_t
        L.laya_tokenizer_from_json.argtypes = [ctypes.c_char_p, sz, ctypes.POINTER(vp)]
        L.laya_tokenizer_from_gguf.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
        L.laya_tokenize.argtypes = [vp, ctypes.c_char_p, sz, ctypes.c_int, _i64p, sz, ctypes.POINTER(sz)]
        L.laya_tokenizer_specials.argtypes = [vp, _i64p]
        L.laya_tokenizer_close.argtypes = [vp]
        L.laya_tokenizer_close.restype = None
        L.laya_requests_plan.argtypes = [vp, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(sz), ctypes.c_int64,
                                         ctypes.c_int, ctypes.POINTER(vp)]
        L.laya_requests_error.argtypes = [vp, ctypes.c_int64]
        L.laya_requests_error.restype = ctypes.c_char_p
        L.laya_requests_questions.argtypes = [vp]
        L.laya_requests_questions.restype = ctypes.c_int64
        L.laya_requests_question.argtypes = [vp, ctypes.c_int64, _i64p, _i64p, _i64p, _i64p]
        L.laya_requests_question_tokens.argtypes = [vp, ctypes.c_int64, _i64p, _i64p]
        L.laya_requests_pack.argtypes = [vp, ctypes.c_int64, ctypes.c_int, _i64p]
        L.laya_requests_forward_shape.argtypes = [vp, ctypes.c_int64, _i64p, _i64p, _i64p]
        L.laya_requests_forward_batch.argtypes = [vp, ctypes.c_int64, _i64p, _i64p, _i64p, _i64p, _i64p]
        L.laya_requests_forward_questions.argtypes = [vp, ctypes.c_int64, _i64p]
        L.laya_requests_set_calibration.argtypes = [vp, _f32p, ctypes.c_char_p]
        L.laya_requests_score.argtypes = [vp, ctypes.c_int64, _f32p, _f32p]
        L.laya_requests_response.argtypes = [vp, ctypes.c_int64, ctypes.c_char_p, sz, ctypes.POINTER(sz)]
        L.laya_requests_merge.argtypes = [ctypes.POINTER(vp), ctypes.c_int64, ctypes.POINTER(vp)]
        L.laya_requests_pack_windows.argtypes = [vp, ctypes.c_int64, ctypes.c_int64, _i64p]
        L.laya_requests_close.argtypes = [vp]
        L.laya_requests_close.restype = None
        _bound = True
    return L


def _p64(a: np.ndarray):
    return a.ctypes.data_as(_i64p)


class Tokenizer:
    """Tokenizer (tokenizer.rs:120-265) from tokenizer.json text or from the
    copy embedded in a model file."""

    def __init__(self, json_text: str | None = None, gguf_path: str | None = None):
        self._h = ctypes.c_void_p()
        if (json_text is None) == (gguf_path is None):
            raise ValueError("give exactly one of json_text or gguf_path")
        if json_text is not None:
            b = json_text.encode("utf-8")
            _check(lib().laya_tokenizer_from_json(b, len(b), ctypes.byref(self._h)))
        else:
            _check(lib().laya_tokenizer_from_gguf(gguf_path.encode(), ctypes.byref(self._h)))

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        b = text.encode("utf-8")
        n = ctypes.c_size_t()
        cap = 4 * len(b) + 8
        out = np.empty(cap, np.int64)
        _check(lib().laya_tokenize(self._h, b, len(b), int(add_special_tokens), _p64(out), cap, ctypes.byref(n)))
        return out[:n.value].tolist()

    def specials(self) -> dict:
        ids = np.empty(5, np.int64)
        _check(lib().laya_tokenizer_specials(self._h, _p64(ids)))
        return dict(zip(["cls", "sep", "mask", "pad", "unk"], ids.tolist()))

    def close(self):
        if self._h:
            lib().laya_tokenizer_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Requests:
    """Planned requests: questions -> sequences (systemone.rs:156-198),
    forwards, scores and responses."""

    def __init__(self, tok: Tokenizer, requests: list, threads: int = 0):
        texts = [r if isinstance(r, (str, bytes)) else json.dumps(r) for r in requests]
        bs = [t.encode("utf-8") if isinstance(t, str) else t for t in texts]
        arr = (ctypes.c_char_p * len(bs))(*bs)
        lens = (ctypes.c_size_t * len(bs))(*[len(b) for b in bs])
        self._keep = bs
        self._tok = tok
        self._h = ctypes.c_void_p()
        _check(lib().laya_requests_plan(tok._h, arr, lens, len(bs), threads, ctypes.byref(self._h)))
        self.n_requests = len(bs)

    @classmethod
    def merge(cls, parts: list) -> "Requests":
        """laya_requests_merge: one object holding the requests of `parts`
        in order (the parts are left empty)."""
        arr = (ctypes.c_void_p * len(parts))(*[p._h for p in parts])
        h = ctypes.c_void_p()
        _check(lib().laya_requests_merge(arr, len(parts), ctypes.byref(h)))
        self = cls.__new__(cls)
        self._keep = [b for p in parts for b in p._keep]
        self._tok = parts[0]._tok if parts else None
        self._h = h
        self.n_requests = sum(p.n_requests for p in parts)
        for p in parts:
            p.n_requests = 0
        return self

    def error(self, request: int) -> str | None:
        e = lib().laya_requests_error(self._h, request)
        return None if e is None else e.decode()

    def questions(self) -> int:
        return int(lib().laya_requests_questions(self._h))

    def question(self, i: int) -> dict:
        req, ln, nm, qt = (ctypes.c_int64() for _ in range(4))
        _check(lib().laya_requests_question(self._h, i, ctypes.byref(req), ctypes.byref(ln), ctypes.byref(nm),
                                            ctypes.byref(qt)))
        seq = np.empty(ln.value, np.int64)
        mk = np.empty(max(nm.value, 1), np.int64)
        _check(lib().laya_requests_question_tokens(self._h, i, _p64(seq), _p64(mk)))
        return {"request": req.value, "seq": seq.tolist(), "markers": mk[:nm.value].tolist(), "qtype": qt.value}

    def question_shape(self, i: int) -> tuple[int, int, int, int]:
        """(request, seq_len, markers, qtype) of question i."""
        req, ln, nm, qt = (ctypes.c_int64() for _ in range(4))
        _check(lib().laya_requests_question(self._h, i, ctypes.byref(req), ctypes.byref(ln), ctypes.byref(nm),
                                            ctypes.byref(qt)))
        return req.value, ln.value, nm.value, qt.value

    def forward_questions(self, f: int) -> list[int]:
        n = ctypes.c_int64()
        _check(lib().laya_requests_forward_shape(self._h, f, ctypes.byref(n), None, None))
        q = np.empty(max(n.value, 1), np.int64)
        _check(lib().laya_requests_forward_questions(self._h, f, _p64(q)))
        return q[:n.value].tolist()

    def pack(self, max_tokens: int = 16384, across_requests: bool | int = False) -> int:
        """across_requests: 0/False per request (run_all), 1/True dispatch
        order across requests, 2 sorted by length across requests."""
        n = ctypes.c_int64()
        _check(lib().laya_requests_pack(self._h, max_tokens, int(across_requests), ctypes.byref(n)))
        return n.value

    def pack_windows(self, max_tokens: int = 16384, window: int = 64) -> int:
        """group_by_budget over each window of `window` consecutive requests."""
        n = ctypes.c_int64()
        _check(lib().laya_requests_pack_windows(self._h, max_tokens, window, ctypes.byref(n)))
        return n.value

    def batch(self, f: int) -> Req:
        n, l, k = (ctypes.c_int64() for _ in range(3))
        _check(lib().laya_requests_forward_shape(self._h, f, ctypes.byref(n), ctypes.byref(l), ctypes.byref(k)))
        n, l, k = n.value, l.value, k.value
        ids = np.empty(n * l, np.int64)
        att = np.empty(n * l, np.int64)
        mpos = np.empty(n * k, np.int64)
        mmask = np.empty(n * k, np.int64)
        qtype = np.empty(n, np.int64)
        _check(lib().laya_requests_forward_batch(self._h, f, _p64(ids), _p64(att), _p64(mpos), _p64(mmask),
                                                 _p64(qtype)))
        return Req(n, l, k, ids, att, mpos, mmask, qtype)

    def set_calibration(self, temperature=(1.0, 1.0, 1.0), by_options: dict | str | None = None) -> None:
        t = np.asarray(temperature, np.float32)
        bo = by_options if isinstance(by_options, str) or by_options is None else json.dumps(by_options)
        _check(lib().laya_requests_set_calibration(self._h, t.ctypes.data_as(_f32p),
                                                   None if bo is None else bo.encode()))

    def score(self, f: int, logits: np.ndarray, act: np.ndarray) -> None:
        lg = np.ascontiguousarray(logits, np.float32)
        ac = np.ascontiguousarray(act, np.float32)
        _check(lib().laya_requests_score(self._h, f, lg.ctypes.data_as(_f32p), ac.ctypes.data_as(_f32p)))

    def response_text(self, request: int) -> str:
        n = ctypes.c_size_t()
        _check(lib().laya_requests_response(self._h, request, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value + 1)
        _check(lib().laya_requests_response(self._h, request, buf, n.value, ctypes.byref(n)))
        return buf.raw[:n.value].decode("utf-8")

    def response(self, request: int) -> dict:
        return json.loads(self.response_text(request))

    def close(self):
        if self._h:
            lib().laya_requests_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def run_requests(engine, tok: Tokenizer, requests: list, max_tokens: int = 16384, across_requests: bool = False,
                 threads: int = 0, calibration: dict | None = None) -> list:
    """Requests in, responses out: plan (threads), pack, one laya_forward per
    forward, score, respond -- run_all (main.rs:520-557) for each request.
    Requests that fail to plan come back as {"error": message}."""
    rq = Requests(tok, requests, threads)
    if calibration:
        rq.set_calibration(calibration.get("temperature", (1.0, 1.0, 1.0)), calibration.get("by_options"))
    for f in range(rq.pack(max_tokens, across_requests)):
        out = engine.forward(rq.batch(f))
        rq.score(f, out.logits, out.act)
    res = []
    for i in range(rq.n_requests):
        e = rq.error(i)
        res.append({"error": e} if e is not None else rq.response(i))
    rq.close()
    return res
