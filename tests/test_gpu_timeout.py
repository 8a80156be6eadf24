"""Failure detection without a GPU fault: every device-side wait of the
kernels is bounded.  laya_test_timeout_next makes the next forward's first
GEMM (or first attention launch) wait, before it issues any load, on an
mbarrier that nothing completes, bounded by 1 ms.  The wait expires, the
kernel records the error word, unwinds (its other roles see the abort flag
and leave their loops, the MMA thread drains, TMEM is freed) and returns.
The forward must report LAYA_E_DEVICE_TIMEOUT instead of hanging, and the
next forward on the same engine must match the oracle again -- the
reference's counterpart is a panic turned into a 500 (main.rs:1058-1059),
after which its service keeps serving."""
import numpy as np
import pytest

from laya_rust_b200 import engine as E
from laya_rust_b200 import modelgen
from _parity import compare
from test_gpu_parity import synthetic_req

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine():
    e = E.Engine(modelgen.cached_model(seed=0), device=0)
    yield e
    e.close()


@pytest.fixture(scope="module")
def want():
    from oracle.oracle import OracleModel
    req = synthetic_req(41, [200, 150, 70, 100], 4)
    m = OracleModel(modelgen.cached_model(seed=0))
    out = m.forward(req.n, req.l, req.k, req.ids, req.att, req.mpos, req.mmask, req.qtype)
    m.close()
    return req, out


@pytest.mark.parametrize("kind", [0, 1], ids=["gemm", "attention"])
def test_an_expired_device_wait_is_reported_and_the_engine_recovers(engine, want, kind):
    req, (wl, wa) = want
    engine.test_timeout_next(kind, 1_000_000)
    with pytest.raises(E.LayaError) as ei:
        engine.forward(req)
    assert ei.value.code == E.LAYA_E_DEVICE_TIMEOUT, ei.value
    got = engine.forward(req)
    compare(req.n, req.k, req.mmask, got.logits, got.act, wl, wa, "after the timeout")


def test_the_plan_path_reports_it_too(engine, want):
    req, (wl, wa) = want
    p = engine.plan(req)
    engine.test_timeout_next(0, 1_000_000)
    p.run()
    with pytest.raises(E.LayaError) as ei:
        p.outputs()
    assert ei.value.code == E.LAYA_E_DEVICE_TIMEOUT
    p.run()
    out = p.outputs()
    compare(req.n, req.k, req.mmask, out.logits, out.act, wl, wa, "plan after the timeout")
    p.close()


def test_bad_arguments_are_rejected(engine):
    for kind, lim in ((2, 1000), (0, 0), (1, 3_000_000_000)):
        with pytest.raises(E.LayaError) as ei:
            engine.test_timeout_next(kind, lim)
        assert ei.value.code == E.LAYA_E_INVALID
