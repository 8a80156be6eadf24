"""laya_decision_tail_static: the decision tail for callers that cannot
allocate device memory when they score (their GPU memory belongs to another
allocator's pool, or an allocation's device sync is not acceptable in their
loop).  It must give the same logits and act as the engine's own forward,
which ends with the same three kernels on arena scratch.

The test takes the final hidden rows from laya_forward_tapped (stage
"head.1"), hands them to the no-allocation entry point in buffers the test
owns, and compares with laya_forward's logits/act, on two calls in a row (a
different request in between, so stale scratch would show).  It runs last in
collection order so a failure here never hides the other tests.
"""
import numpy as np
import pytest
import torch

from laya_rust_b200 import engine as E
from laya_rust_b200 import modelgen, workloads

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def engine():
    e = E.Engine(modelgen.cached_model(seed=0), device=0)
    yield e
    e.close()


def compacted_inputs(req, taps):
    """Real rows of the final hidden state, packed back to back, and the row
    indices the tail reads (the engine's own layout)."""
    n, l, k = req.n, req.l, req.k
    lens = (req.att.reshape(n, l) != 0).sum(1)
    start = np.concatenate([[0], np.cumsum(lens)[:-1]])
    h = taps["head.1"].reshape(n, l, 1024)
    x = np.concatenate([h[b, :lens[b]] for b in range(n)]).astype(np.float32)
    mm = req.mmask.reshape(n, k) != 0
    mk = start[:, None] + np.where(mm, req.mpos.reshape(n, k), 0)
    dev = torch.device("cuda", 0)
    return (torch.from_numpy(x).to(dev), torch.from_numpy(start.astype(np.int32)).to(dev),
            torch.from_numpy(mk.astype(np.int32).ravel()).to(dev),
            torch.from_numpy(mm.astype(np.int8).ravel()).to(dev))


def run_static(engine, req, inputs):
    x, cls, mk, mm = inputs
    logits = torch.full((req.n * req.k,), float("nan"), device=x.device)
    act = torch.full((req.n * 2,), float("nan"), device=x.device)
    torch.cuda.synchronize()
    engine.decision_tail_static(x.data_ptr(), req.n, req.k, cls.data_ptr(), mk.data_ptr(), mm.data_ptr(),
                                logits.data_ptr(), act.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return logits.cpu().numpy(), act.cpu().numpy()


def check(got, want):
    for g, w in zip(got, want):
        err = np.abs(g - w)
        assert np.all(np.isfinite(g))
        assert err.max() <= ATOL and np.all(err <= ATOL + RTOL * np.abs(w)), float(err.max())


def test_static_tail_matches_the_forward_on_two_calls_in_a_row(engine):
    reqs = [workloads.forward_16k(seed=5), workloads.long_state(seed=6)]
    cases = []
    for req in reqs:
        taps = {}
        out = engine.forward(req, taps=taps)
        cases.append((req, compacted_inputs(req, taps), (out.logits, out.act)))
    for req, inputs, want in (cases[0], cases[1], cases[0]):
        check(run_static(engine, req, inputs), want)


def test_static_tail_rejects_more_rows_than_its_array_holds(engine):
    x = torch.zeros((4, 1024), device="cuda")
    idx = torch.zeros(4096, dtype=torch.int32, device="cuda")
    mm = torch.ones(4096, dtype=torch.int8, device="cuda")
    out = torch.zeros(4096, device="cuda")
    with pytest.raises(E.LayaError, match="LAYA_TAIL_STATIC_MAX_ROWS") as ei:
        engine.decision_tail_static(x.data_ptr(), 1, 4096, idx.data_ptr(), idx.data_ptr(), mm.data_ptr(),
                                    out.data_ptr(), out.data_ptr())
    assert ei.value.code == E.LAYA_E_INVALID


def test_static_tail_follows_a_weight_uploaded_again():
    """A weight uploaded after the first call (here the scorer's output bias)
    must reach the static tail too: it caches the engine's weight pointers and
    drops them on any upload.  Own engine, so the shared one keeps its weights."""
    eng = E.Engine(modelgen.cached_model(seed=0), device=0)
    try:
        req = workloads.forward_16k(seed=7)
        taps = {}
        eng.forward(req, taps=taps)
        inputs = compacted_inputs(req, taps)
        run_static(eng, req, inputs)                       # caches the pointers
        eng.upload_f32("scorer.3.bias", np.array([0.25], np.float32))
        out = eng.forward(req)
        got = run_static(eng, req, inputs)
        check(got, (out.logits, out.act))
        mm = req.mmask != 0
        assert np.all(got[0][~mm] == -10000.0)
    finally:
        eng.close()
