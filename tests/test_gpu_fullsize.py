"""Parity on the benchmarked workloads at their full size: the engine against
the C oracle of the reference CPU backend (graph.rs:86-186 over
backend/cpu/mod.rs) on exactly the batches bench.py times.

  forward-16k  128 x 128 padded, 9872 real tokens: nine 256-row blocks per
               GEMM wave, the multi-wave persistent tile walk, every epilogue
  long-state   8 x 512: the attention path for sequences over 128 tokens
  stream-32    the first 32 requests of the request stream through the C++
               front end, packed across requests (six forwards, up to 10259
               real tokens and rows of 512)
  layer        one encoder layer on 32 x 256 (layers 0 and 1, N(0,1) input
               rounded to f16), checked live against the oracle's layer call

The whole-forward outputs of the oracle are committed fixtures
(tests/golden/fullsize_outputs.json, made by make_fullsize_fixtures.py; each
entry carries a SHA-256 of its request arrays, checked first).  Tolerance and
argmax rule: tests/_parity.py (max-abs 2e-2, rel 1e-2, strict argmax).
"""
import json
import os
import sys

import numpy as np
import pytest

from laya_rust_b200 import engine as E
from laya_rust_b200 import modelgen, workloads

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from _parity import compare  # noqa: E402
from make_fullsize_fixtures import req_digest, stream_batches  # noqa: E402

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = json.load(open(os.path.join(HERE, "golden", "fullsize_outputs.json")))


@pytest.fixture(scope="module")
def engine():
    e = E.Engine(modelgen.cached_model(seed=0), device=0)
    yield e
    e.close()


def check_against(entry, req, out, name):
    assert entry["sha256"] == req_digest(req), f"{name}: the request differs from the one the fixture was made on"
    el, ea, margin = compare(req.n, req.k, req.mmask, out.logits, out.act, np.array(entry["logits"], np.float32),
                             np.array(entry["act"], np.float32), name)
    print(f"{name}: max|dlogit| {el:.3e} max|dact| {ea:.3e} smallest oracle top-2 margin {margin:.3e}")


@pytest.mark.parametrize("name,make", [("forward-16k", lambda: workloads.forward_16k(0)),
                                       ("long-state", lambda: workloads.long_state(3))])
def test_benchmarked_batch_matches_the_oracle(engine, name, make):
    """Through the public call (laya_forward) and through the plan path the
    bench times (CUDA graph replay): both against the oracle's outputs."""
    req = make()
    entry = FIX[name][0]
    check_against(entry, req, engine.forward(req), name + " laya_forward")
    p = engine.plan(req)
    p.capture()
    for _ in range(2):
        p.run()
    check_against(entry, req, p.outputs(), name + " graph replay")
    p.close()


def test_stream_slice_matches_the_oracle(engine):
    batches = stream_batches()
    assert len(batches) == len(FIX["stream-32"])
    for f, (req, entry) in enumerate(zip(batches, FIX["stream-32"])):
        check_against(entry, req, engine.forward(req), f"stream-32 forward {f}")


@pytest.fixture(scope="module")
def oracle():
    from oracle.oracle import OracleModel
    m = OracleModel(modelgen.cached_model(seed=0))
    yield m
    m.close()


@pytest.mark.parametrize("layer", [0, 1])
def test_layer_batch_matches_the_oracle_layer(engine, oracle, layer):
    """Configuration 1 at its size: 32 x 256 (4343 real tokens), the input
    the bench uses (N(0,1) rounded to f16), one layer against the oracle's
    lo_encoder_layer (graph.rs:104-123) on the padded layout."""
    req = workloads.layer_batch(1)
    real = (req.att.reshape(req.n, req.l) != 0).ravel()
    nreal = int(real.sum())
    xr = np.random.default_rng(1).standard_normal((nreal, 1024)).astype(np.float16).astype(np.float32)
    x = np.zeros((req.n * req.l, 1024), np.float32)
    x[real] = xr
    want = oracle.encoder_layer(req.n, req.l, req.att, layer, x).reshape(-1, 1024)[real]
    p = engine.plan(req)
    p.set_hidden(xr)
    p.run_layer(layer)
    got = p.hidden()
    p.close()
    rel = np.abs(got - want).max() / np.abs(want).max()
    print(f"layer {layer}: max relative error {rel:.3e}")
    assert rel < 1e-2, rel
