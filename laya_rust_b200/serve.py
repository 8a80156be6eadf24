"""The System One HTTP service (include/laya_serve.h): ``laya serve`` of
laya-rust src/main.rs:996-1204.  The service itself (sockets, queue,
inference threads, planning, forwards, answers) runs in the C++ library; this
module binds it and gives it the reference's command line:

    python -m laya_rust_b200.serve -m MODEL.gguf [--addr 127.0.0.1:8080]
        [--endpoint /systemone] [--queue 64] [--connections 4]
        [--max-tokens 16384] [--devices 0,1,...] [--batch 1] [-v]

``--devices`` (one inference thread and engine per GPU, all serving one
queue) and ``--batch`` (an inference thread packs up to that many queued
requests into shared forwards) are this build's additions; the defaults are
the reference's single engine and per-request forwards.
"""
from __future__ import annotations

import argparse
import ctypes
import signal
import sys
import threading

import numpy as np

from .engine import LayaError, Req, _CReq, _check, lib as _engine_lib

FORWARD_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(_CReq),
                              ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float))
STATS = ("answered", "200", "400", "404", "405", "413", "422", "500", "503", "forwards", "queued")


class _Config(ctypes.Structure):
    _fields_ = [("model", ctypes.c_char_p), ("tokenizer_json", ctypes.c_char_p),
                ("tokenizer_json_len", ctypes.c_size_t), ("addr", ctypes.c_char_p),
                ("endpoint", ctypes.c_char_p), ("queue", ctypes.c_int64), ("connections", ctypes.c_int32),
                ("max_tokens", ctypes.c_int64), ("devices", ctypes.POINTER(ctypes.c_int32)),
                ("n_devices", ctypes.c_int32), ("batch", ctypes.c_int32), ("verbose", ctypes.c_int32),
                ("forward", FORWARD_FN), ("forward_user", ctypes.c_void_p)]


_bound = False


def lib():
    global _bound
    L = _engine_lib()
    if not _bound:
        vp = ctypes.c_void_p
        L.laya_serve_open.argtypes = [ctypes.POINTER(_Config), ctypes.POINTER(vp)]
        L.laya_serve_address.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t]
        L.laya_serve_stats.argtypes = [vp, ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
        L.laya_serve_stop.argtypes = [vp]
        L.laya_serve_wait.argtypes = [vp]
        L.laya_serve_close.argtypes = [vp]
        L.laya_serve_close.restype = None
        _bound = True
    return L


def _hook(fn):
    """Wraps fn(slot, Req) -> (logits, act) as a laya_serve_forward_fn."""

    def cb(_user, slot, creq, logits, act):
        try:
            c = creq.contents
            n, l, k = int(c.n), int(c.l), int(c.k)
            arr = lambda p, m: np.ctypeslib.as_array(p, shape=(max(m, 1),))[:m].copy()
            req = Req(n, l, k, arr(c.ids, n * l), arr(c.att, n * l), arr(c.mpos, n * k), arr(c.mmask, n * k),
                      arr(c.qtype, n))
            lg, ac = fn(int(slot), req)
            lg = np.ascontiguousarray(lg, np.float32).ravel()
            ac = np.ascontiguousarray(ac, np.float32).ravel()
            if lg.size != n * k or ac.size != n * 2:
                return 2
            ctypes.memmove(logits, lg.ctypes.data, lg.nbytes)
            ctypes.memmove(act, ac.ctypes.data, ac.nbytes)
            return 0
        except Exception:
            return 1

    return FORWARD_FN(cb)


class Server:
    """A running service.  With ``forward`` (fn(slot, Req) -> (logits, act))
    the service calls it instead of opening engines, one inference thread per
    entry of ``devices``; ``tokenizer_json`` then may replace the model."""

    def __init__(self, model: str | None = None, addr: str = "127.0.0.1:8080", endpoint: str = "/systemone",
                 queue: int = 64, connections: int = 4, max_tokens: int = 16384, devices=(0,), batch: int = 1,
                 verbose: bool = False, forward=None, tokenizer_json: str | None = None):
        devs = (ctypes.c_int32 * len(devices))(*devices)
        tj = tokenizer_json.encode() if tokenizer_json else None
        self._fn = _hook(forward) if forward is not None else FORWARD_FN()
        self._devs = devs
        cfg = _Config(model.encode() if model else None, tj, len(tj) if tj else 0, addr.encode(),
                      endpoint.encode(), queue, connections, max_tokens, devs, len(devices), batch,
                      1 if verbose else 0, self._fn, None)
        h = ctypes.c_void_p()
        _check(lib().laya_serve_open(ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h

    @property
    def address(self) -> str:
        buf = ctypes.create_string_buffer(64)
        _check(lib().laya_serve_address(self._h, buf, 64))
        return buf.value.decode()

    def stats(self) -> dict:
        out = (ctypes.c_int64 * len(STATS))()
        _check(lib().laya_serve_stats(self._h, out, len(STATS)))
        return dict(zip(STATS, (int(v) for v in out)))

    def stop(self) -> None:
        if self._h:
            _check(lib().laya_serve_stop(self._h))

    def wait(self) -> None:
        _check(lib().laya_serve_wait(self._h))

    def close(self) -> None:
        if self._h:
            lib().laya_serve_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="laya serve",
                                description="Serve the System One API over HTTP until interrupted")
    p.add_argument("--model", "-m", required=True, metavar="PATH", help="GGUF model")
    p.add_argument("--verbose", "-v", action="store_true", help="per-request status and timing on stderr")
    p.add_argument("--max-tokens", type=int, default=16384, metavar="N", help="padded-token budget per forward")
    p.add_argument("--addr", default="127.0.0.1:8080", metavar="ADDR", help="listen address")
    p.add_argument("--endpoint", default="/systemone", metavar="PATH", help="endpoint path (POST)")
    p.add_argument("--queue", type=int, default=64, metavar="N", help="queued requests before 503")
    p.add_argument("--connections", type=int, default=4, metavar="N", help="connection threads")
    p.add_argument("--devices", default="0", metavar="LIST", help="CUDA devices, one engine each (e.g. 0,1,2,3)")
    p.add_argument("--batch", type=int, default=1, metavar="N",
                   help="queued requests one engine packs into shared forwards")
    a = p.parse_args(argv)
    if a.queue < 1 or a.connections < 1:
        p.error("--queue and --connections must be at least 1")
    devices = [int(d) for d in a.devices.split(",") if d.strip()]
    try:
        srv = Server(a.model, a.addr, a.endpoint, a.queue, a.connections, a.max_tokens, devices, a.batch,
                     a.verbose)
    except LayaError as e:
        print(f"laya serve: {e}", file=sys.stderr)
        return 2
    print(f"laya serve: POST http://{srv.address}{a.endpoint} ({a.connections} connection thread(s), "
          f"queue {a.queue}, {len(devices)} engine(s))", file=sys.stderr)
    done = threading.Event()
    for sig in (signal.SIGINT, signal.SIGTERM):
        signal.signal(sig, lambda *_: done.set())
    while not done.wait(0.5):
        pass
    srv.stop()
    srv.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
