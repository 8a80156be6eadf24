"""Generates tests/golden/fullsize_outputs.json: the C oracle's outputs (the
reference CPU backend restated, oracle/laya_oracle.c) on the benchmarked
workloads at their full size, so the GPU tests can compare the engine with
the reference algorithm on exactly what bench.py times.

Cases (all seeded, on the random-init f16 model of seed 0):
  forward-16k   workloads.forward_16k(0): 128 x 128 padded, 9872 real tokens
                (the bench's rank-0 batch of the default configuration)
  long-state    workloads.long_state(3): 8 x 512 (the bench's rank-0 batch)
  stream-32     the first 32 requests of the request stream (seed 4) as JSON,
                planned by the C++ front end and packed across requests into
                <=16384-token forwards as bench.py's stream configuration packs
                them; one entry per forward

Each entry keeps the oracle's logits and act and a SHA-256 of the request
arrays (ids, att, mpos, mmask, qtype as little-endian int64), so a test can
check it regenerated the same request before comparing.  The one-layer
configuration (32 x 256) is checked live by the GPU tests instead: its output
is a whole residual stream, and the oracle's layer call takes about a second.

Run from the repository root (8 host threads: about 15 minutes):
    python tests/golden/make_fullsize_fixtures.py [--only NAME]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
OUT = os.path.join(ROOT, "tests", "golden", "fullsize_outputs.json")
STREAM_REQUESTS = 32


def req_digest(req) -> str:
    h = hashlib.sha256()
    for a in (req.ids, req.att, req.mpos, req.mmask, req.qtype):
        h.update(np.ascontiguousarray(a, dtype="<i8").tobytes())
    h.update(f"{req.n},{req.l},{req.k}".encode())
    return h.hexdigest()


def stream_batches(n_requests: int = STREAM_REQUESTS):
    """The first n requests of configuration 4, packed across requests in
    dispatch order (bench.py run_stream with one GPU)."""
    from laya_rust_b200 import frontend as FE, modelgen, tokgen, workloads
    words = workloads.vocab_words(tokgen.tokenizer_json(0))
    texts = [json.dumps(r) for r in workloads.request_stream_json(words, n_requests, 4)]
    tok = FE.Tokenizer(gguf_path=modelgen.cached_model(seed=0))
    rq = FE.Requests(tok, texts, threads=0)
    nf = rq.pack(16384, True)
    out = [rq.batch(f) for f in range(nf)]
    rq.close()
    tok.close()
    return out


def cases():
    from laya_rust_b200 import workloads
    yield "forward-16k", [workloads.forward_16k(0)]
    yield "long-state", [workloads.long_state(3)]
    yield "stream-32", stream_batches()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    os.environ.setdefault("LAYA_ORACLE_FAST", "1")
    from laya_rust_b200 import modelgen
    from oracle.oracle import OracleModel
    data = json.load(open(OUT)) if os.path.exists(OUT) else {}
    m = OracleModel(modelgen.cached_model(seed=0))
    for name, reqs in cases():
        if args.only and name != args.only:
            continue
        entries = []
        for req in reqs:
            t = time.time()
            lg, act = m.forward(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype)
            entries.append({"n": req.n, "l": req.l, "k": req.k, "real_tokens": int((req.att != 0).sum()),
                            "sha256": req_digest(req),
                            "logits": [float(v) for v in lg], "act": [float(v) for v in act]})
            print(f"{name}: n={req.n} l={req.l} k={req.k} real={entries[-1]['real_tokens']} "
                  f"{time.time() - t:.1f} s", flush=True)
        data[name] = entries
        with open(OUT, "w") as f:
            json.dump(data, f, separators=(",", ":"))
    m.close()


if __name__ == "__main__":
    main()
