"""Load generator for the HTTP service (laya_rust_b200.serve): latency of
one System One request through HTTP against the library's own request path,
and throughput of a slice of the synthetic request stream from concurrent
keep-alive clients, for each --batch.

    python -m laya_rust_b200.serve_load [--model PATH] [--device 0]
        [--requests 512] [--clients 32] [--batch 1,32] [--out FILE]

Without --model it uses the seed-0 synthetic model (laya_rust_b200.modelgen).
Prints one JSON object.
"""
from __future__ import annotations

import argparse
import http.client
import json
import sys
import threading
import time

import numpy as np

from . import engine as E
from . import frontend as FE
from . import modelgen, tokgen, workloads
from . import serve as S


def _conn(addr: str) -> http.client.HTTPConnection:
    host, port = addr.split(":")
    return http.client.HTTPConnection(host, int(port), timeout=300)


def _sequential(addr: str, body: str, n: int, warm: int) -> list[float]:
    c = _conn(addr)
    lat = []
    for _ in range(n + warm):
        t = time.perf_counter()
        c.request("POST", "/systemone", body=body)
        r = c.getresponse()
        r.read()
        if r.status != 200:
            raise RuntimeError(f"status {r.status}")
        lat.append((time.perf_counter() - t) * 1e3)
    c.close()
    return lat[warm:]


def _stream(addr: str, bodies: list[str], clients: int) -> dict:
    lats = [0.0] * len(bodies)
    codes = [0] * len(bodies)

    def work(k):
        c = _conn(addr)
        for i in range(k, len(bodies), clients):
            t = time.perf_counter()
            c.request("POST", "/systemone", body=bodies[i])
            r = c.getresponse()
            r.read()
            lats[i] = (time.perf_counter() - t) * 1e3
            codes[i] = r.status
        c.close()

    t = time.perf_counter()
    ts = [threading.Thread(target=work, args=(k,)) for k in range(clients)]
    for x in ts:
        x.start()
    for x in ts:
        x.join()
    el = time.perf_counter() - t
    return {"requests_per_s": len(bodies) / el, "seconds": el, "p50_ms": float(np.percentile(lats, 50)),
            "p90_ms": float(np.percentile(lats, 90)), "ok": codes.count(200)}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="laya_rust_b200.serve_load")
    p.add_argument("--model", default=None)
    p.add_argument("--device", type=int, default=0)
    p.add_argument("--requests", type=int, default=512)
    p.add_argument("--clients", type=int, default=32)
    p.add_argument("--batch", default="1,32")
    p.add_argument("--sequential", type=int, default=50)
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    path = a.model or modelgen.cached_model(seed=0)
    words = workloads.vocab_words(tokgen.tokenizer_json(0))
    one = json.dumps(workloads.single_request_json(words, 0))
    stream = [json.dumps(r) for r in workloads.request_stream_json(words, a.requests, seed=4)]
    out = {"sequential": a.sequential, "requests": a.requests, "clients": a.clients}

    eng = E.Engine(path, a.device)
    tok = FE.Tokenizer(gguf_path=path)
    cal = eng.info().calibration
    lat = []
    for _ in range(a.sequential + 10):
        t = time.perf_counter()
        FE.run_requests(eng, tok, [one], calibration=cal, threads=1)
        lat.append((time.perf_counter() - t) * 1e3)
    out["library_p50_ms"] = float(np.percentile(lat[10:], 50))
    tok.close()
    eng.close()

    for batch in (int(b) for b in a.batch.split(",")):
        with S.Server(model=path, addr="127.0.0.1:0", devices=(a.device,), batch=batch, connections=a.clients,
                      queue=max(64, a.requests)) as s:
            lat = _sequential(s.address, one, a.sequential, 10)
            res = {"http_p50_ms": float(np.percentile(lat, 50)), "http_p90_ms": float(np.percentile(lat, 90))}
            f0 = s.stats()["forwards"]
            res["stream"] = _stream(s.address, stream, a.clients)
            res["stream"]["forwards"] = s.stats()["forwards"] - f0
            out[f"batch{batch}"] = res
    text = json.dumps(out)
    print(text)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
