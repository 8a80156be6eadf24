"""The public forward's CUDA-graph cache (laya_forward): a request shape is
launched eagerly the first time, captured on its second call and replayed
after that.  A replay reads the request through the same device buffer, so
it must give bitwise the eager forward's logits and act -- for the request it
was captured on and for any other request of the same shape -- and a weight
uploaded again must retire the graph (it holds the old weight pointers).
Two engines given the same requests agree bit for bit."""
import numpy as np
import pytest

from laya_rust_b200 import engine as E
from laya_rust_b200 import modelgen
from test_gpu_parity import synthetic_req

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine():
    e = E.Engine(modelgen.cached_model(seed=0), device=0)
    yield e
    e.close()


def eager(engine, req):
    # a tapped forward always runs eagerly
    return engine.forward(req, taps={})


def same(a, b):
    return np.array_equal(a.logits, b.logits) and np.array_equal(a.act, b.act)


def test_replays_match_the_eager_forward_bitwise(engine):
    shapes = [[200, 150, 70, 100], [31, 77, 128, 64, 90, 12]]
    reqs = [synthetic_req(70 + i, lens, 4) for i, lens in enumerate(shapes)]
    want = [eager(engine, r) for r in reqs]
    for _ in range(3):   # first sight (eager), second (capture), then replays
        for r, w in zip(reqs, want):
            assert same(engine.forward(r), w)
    # another request of a captured shape: new ids, markers and question types
    other = synthetic_req(99, shapes[0], 4)
    assert not np.array_equal(other.ids, reqs[0].ids)
    assert same(engine.forward(other), eager(engine, other))


def test_a_weight_uploaded_again_retires_the_graph():
    eng = E.Engine(modelgen.cached_model(seed=0), device=0)
    try:
        req = synthetic_req(5, [120, 60, 33], 3)
        for _ in range(3):
            eng.forward(req)                 # captured and replayed
        eng.upload_f32("scorer.3.bias", np.array([0.5], np.float32))
        got = eng.forward(req)
        want = eager(eng, req)
        assert same(got, want)
        mm = req.mmask != 0
        before = E.Engine(modelgen.cached_model(seed=0), device=0)
        try:
            base = before.forward(req)
        finally:
            before.close()
        # scorer.3.bias is 0 in the model: every valid logit moved by 0.5
        assert np.allclose(got.logits[mm.ravel()], base.logits[mm.ravel()] + 0.5, atol=1e-5)
    finally:
        eng.close()


def test_a_longer_request_retires_the_graphs():
    """A request longer than any before grows the RoPE tables (reallocated);
    graphs captured over the old tables must not replay."""
    eng = E.Engine(modelgen.cached_model(seed=0), device=0)
    try:
        short = synthetic_req(11, [100, 80, 64], 3)
        for _ in range(3):
            eng.forward(short)               # captured and replayed
        eng.forward(synthetic_req(12, [600], 3))  # RoPE tables 512 -> 1024 rows
        for _ in range(3):                   # eager, captured again, replayed
            assert same(eng.forward(short), eager(eng, short))
    finally:
        eng.close()


def test_two_engines_agree_bitwise_through_arena_growth():
    """A forward that grows the arena clears the new buffers on the engine's
    own stream before its kernels run (a clear on the legacy default stream
    is not ordered before a non-blocking stream's kernels).  Two fresh
    engines fed the same requests of growing size -- every one of them grows
    the arena -- must agree bit for bit on each."""
    reqs = [synthetic_req(91, [94, 85], 2), synthetic_req(92, [371], 2), synthetic_req(93, [146] * 5, 5),
            synthetic_req(94, [300] * 6, 4), synthetic_req(95, [120] * 40, 3)]
    outs = []
    for _ in range(2):
        e = E.Engine(modelgen.cached_model(seed=0), device=0)
        try:
            outs.append([e.forward(r) for r in reqs])
        finally:
            e.close()
    for i, (a, b) in enumerate(zip(*outs)):
        assert same(a, b), f"request {i}"
