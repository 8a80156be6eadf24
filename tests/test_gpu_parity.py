"""Whole-forward parity: the B200 engine against the C oracle of the reference
CPU backend, on the same seeded random-init model and identical requests.

Tolerance (the contract's): final logits and act logits within max-abs 2e-2
and rel 1e-2 (``|got - want| <= 2e-2 + 1e-2 |want|`` with the max-abs bound
also enforced), masked logits exactly -10000, identical argmax over each row's
valid markers.  Requests: the request layouts of the reference's five golden
fixtures (six forwards) and seeded synthetic batches that reach the sliding
window (rows longer than 129 tokens) and the 512-token maximum.
"""
import json
import os

import numpy as np
import pytest

from laya_rust_b200 import arch, modelgen
from laya_rust_b200 import engine as E
from laya_rust_b200.engine import Req
from _parity import compare as shared_compare

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = json.load(open(os.path.join(HERE, "golden", "fixture_requests.json")))


@pytest.fixture(scope="module")
def model_path():
    return modelgen.cached_model(seed=0)


@pytest.fixture(scope="module")
def engine(model_path):
    e = E.Engine(model_path, device=0)
    yield e
    e.close()


@pytest.fixture(scope="module")
def oracle(model_path):
    from oracle.oracle import OracleModel
    m = OracleModel(model_path)
    yield m
    m.close()


def synthetic_req(seed, lens, k, l=None):
    rng = np.random.default_rng(seed)
    n = len(lens)
    l = l or max(lens)
    ids = np.zeros((n, l), np.int64)
    att = np.zeros((n, l), np.int64)
    mpos = np.zeros((n, k), np.int64)
    mmask = np.zeros((n, k), np.int64)
    for b, r in enumerate(lens):
        ids[b, :r] = rng.integers(0, 50280, r)
        ids[b, 0], ids[b, r - 1] = arch.CLS_ID, arch.SEP_ID
        att[b, :r] = 1
        nm = int(rng.integers(1, k + 1))
        pos = np.sort(rng.choice(np.arange(1, r - 1), size=min(nm, r - 2), replace=False))
        mpos[b, :len(pos)] = pos
        mmask[b, :len(pos)] = 1
        ids[b, pos] = arch.MASK_ID
    qtype = rng.integers(0, 3, n)
    return Req(n, l, k, ids, att, mpos, mmask, qtype)


SPLIT_LENS = [300, 40, 400, 128, 129, 77, 256, 200, 30, 390, 64, 100]


def fixture_reqs():
    out = []
    for fx in FIXTURES:
        for i, fw in enumerate(fx["forwards"]):
            out.append((f"{fx['name']}-{i}",
                        Req(fw["n"], fw["l"], fw["k"], fw["ids"], fw["att"], fw["mpos"], fw["mmask"],
                            fw["qtype"])))
    return out


CASES = fixture_reqs() + [
    ("window-3x200", synthetic_req(11, [200, 150, 70], 4)),
    ("maxlen-2x512", synthetic_req(12, [512, 300], 3)),
    ("ragged-8", synthetic_req(13, [24, 128, 77, 31, 128, 64, 65, 100], 5, l=128)),
    # >= 2048 real tokens: with LAYA_ROW_GROUPS=2 the batch runs as two row
    # groups on two streams
    ("two-groups-12", synthetic_req(14, SPLIT_LENS, 4, l=400)),
]


def compare(req, got, want_logits, want_act):
    el, ea, _ = shared_compare(req.n, req.k, req.mmask, got.logits, got.act, want_logits, want_act)
    return el, ea


@pytest.mark.parametrize("name,req", CASES, ids=[c[0] for c in CASES])
def test_forward_matches_oracle(name, req, engine, oracle):
    got = engine.forward(req)
    wl, wa = oracle.forward(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype)
    el, ea = compare(req, got, wl, wa)
    print(f"{name}: max|dlogit| {el:.3e} max|dact| {ea:.3e}")


def test_residual_stream_taps_track_the_oracle(engine, oracle):
    """TapSink localisation (ops.rs:1-3): real rows of enc.*, final and head.*."""
    req = CASES[0][1]
    taps_g, taps_w = {}, {}
    engine.forward(req, taps=taps_g)
    oracle.forward(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype, taps=taps_w)
    real = (req.att.reshape(req.n, req.l) != 0).ravel()
    for stage in ["enc.0", "enc.1", "enc.13", "enc.27", "final", "head.0", "head.1"]:
        g = taps_g[stage].reshape(-1, 1024)[real]
        w = taps_w[stage].reshape(-1, 1024)[real]
        rel = np.abs(g - w).max() / max(np.abs(w).max(), 1e-6)
        assert rel < 2e-2, (stage, rel)
    assert np.array_equal(taps_g["logits"], engine.forward(req).logits)


@pytest.mark.parametrize("layer,lens", [(0, [200, 150, 70]), (1, [200, 150, 70]), (3, [200, 150, 70]),
                                        (27, [200, 150, 70]), (0, SPLIT_LENS), (1, SPLIT_LENS)])
def test_single_layer_matches_the_oracle_layer(layer, lens, engine, oracle):
    """One encoder layer in isolation (the single-layer benchmark
    configuration): the oracle's residual stream before layer i goes in, the
    engine's after layer i must match the oracle's enc.{i} tap.  Rows longer
    than 129 tokens, so the local layers' window is active; the second
    request has two row groups."""
    req = synthetic_req(11, lens, 4, l=max(lens))
    taps = {}
    oracle.forward(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype, taps=taps)
    real = (req.att.reshape(req.n, req.l) != 0).ravel()
    x_in = taps[f"enc.{layer - 1}" if layer else "embed"].reshape(-1, 1024)[real]
    want = taps[f"enc.{layer}"].reshape(-1, 1024)[real]
    p = engine.plan(req)
    p.set_hidden(x_in)
    p.run_layer(layer)
    got = p.hidden()
    p.close()
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel < 1e-2, rel


# Split-K edges (the engine cuts the residual GEMMs' K loop when their
# 256 x 256 tiles fill at most half the clusters): 2304 rows is 9 row blocks,
# 2 parts filling the part region to its last row; 2305 rows is 10 row blocks,
# no split; 179 rows (one request) takes 4 parts.
LENS_2304 = SPLIT_LENS[:-1] + [290]
LENS_2305 = SPLIT_LENS[:-1] + [291]


@pytest.mark.parametrize("layer,lens", [(1, LENS_2304), (3, LENS_2304), (1, LENS_2305), (1, [85, 94]),
                                        (3, [85, 94])])
def test_single_layer_at_the_split_k_edges(layer, lens, engine, oracle):
    """One layer on an N(0,1) residual stream (configuration 1's input) at
    the row counts where split-K starts, fills its part region or stops:
    the engine's layer against the oracle's lo_encoder_layer."""
    assert sum(LENS_2304) == 2304 and sum(LENS_2305) == 2305
    req = synthetic_req(31, lens, 3, l=max(lens))
    rng = np.random.default_rng(layer)
    real = (req.att.reshape(req.n, req.l) != 0).ravel()
    x = np.zeros((req.n * req.l, 1024), np.float32)
    x[real] = rng.standard_normal((int(real.sum()), 1024)).astype(np.float32)
    want = oracle.encoder_layer(req.n, req.l, req.att, layer, x).reshape(-1, 1024)[real]
    p = engine.plan(req)
    p.set_hidden(x[real])
    p.run_layer(layer)
    got = p.hidden()
    p.close()
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel < 1e-2, rel


def test_single_layer_rejects_a_layer_out_of_range(engine):
    p = engine.plan(synthetic_req(12, [40], 2))
    for layer in (-1, 28):
        with pytest.raises(E.LayaError, match="layer"):
            p.run_layer(layer)
    p.close()


def test_plan_and_graph_replay_are_bitwise_identical(engine):
    req = CASES[-1][1]
    ref = engine.forward(req)
    p = engine.plan(req)
    p.run()
    a = p.outputs()
    p.capture()
    p.run()
    p.run()
    b = p.outputs()
    for o in (a, b):
        assert np.array_equal(o.logits, ref.logits) and np.array_equal(o.act, ref.act)
    real, launches, upload = p.stats()
    # 28 encoder layers of 4 GEMMs + attention, 2 head layers, the tail
    assert real == req.real_tokens() and launches >= 28 * 5 and upload > 0


@pytest.mark.parametrize("mutate,match", [
    (lambda r: r.att.__setitem__(5, 0), "prefix"),
    (lambda r: r.mpos.__setitem__(0, 10 ** 6), "outside"),
    (lambda r: r.qtype.__setitem__(0, 3), "qtype"),
    (lambda r: r.ids.__setitem__(0, 50368), "token id"),
])
def test_bad_requests_are_rejected_and_the_engine_recovers(engine, mutate, match):
    req = synthetic_req(21, [40, 30], 3)
    good = engine.forward(req)
    bad = synthetic_req(21, [40, 30], 3)
    mutate(bad)
    with pytest.raises(E.LayaError, match=match) as ei:
        engine.forward(bad)
    assert ei.value.code == E.LAYA_E_INVALID
    again = engine.forward(req)
    assert np.array_equal(again.logits, good.logits)


def test_marker_on_padding_is_rejected(engine):
    req = synthetic_req(22, [40, 30], 3, l=40)
    req.mpos[3] = 35   # row 1 has 30 real tokens
    req.mmask[3] = 1
    with pytest.raises(E.LayaError, match="padding"):
        engine.forward(req)


def test_info_reports_the_engine(engine):
    info = engine.info()
    assert info.id == "cuda" and info.layers == 28 and info.dtype == "fp16"
    assert info.calibration["temperature"] == [1.0, 1.0, 1.0]
