"""The HTTP service on a B200 with a real engine: 200 bodies equal to the
library's own request path (run_requests through laya_forward on a second
engine), the 422 contract through the engine-backed service, and
cross-request batching under concurrent clients (same questions, same
choices, probabilities within BATCH_TOL of the one-request-at-a-time
answers).  A batched forward has more rows, so its GEMMs take other tile
shapes and K splits (split-K parts and narrow tiles for one request, whole
256 x 256 tiles for a batch) and its rows sit in other attention tiles: the
f32 sums run in another order.  Each side is within the contract's logit
tolerance of the reference algorithm (the parity tests); against each other
the probabilities agree to a few 1e-3.

One request at a time the two paths run the same forwards and have given
byte-identical bodies in every run of this suite but one.  That run saw one
body's noul and act probabilities differ by 3e-4 and 8e-4, on the request
whose forward first grew both engines' arenas.  The engine then cleared a
grown arena on the legacy default stream, which is not ordered before its
non-blocking stream's kernels: a race at exactly such forwards, since fixed
(the clears and uploads run on the engine's stream; test_gpu_graphs checks
two engines bit for bit through arena growth).  This comparison still allows
SAME_TOL on the probabilities and requires everything else to be equal."""
import http.client
import json
import threading

import numpy as np
import pytest

from laya_rust_b200 import engine as E
from laya_rust_b200 import frontend as FE
from laya_rust_b200 import modelgen, tokgen, workloads
from laya_rust_b200 import serve as S

pytestmark = pytest.mark.gpu

BATCH_TOL = 5e-3
SAME_TOL = 2e-3


def assert_same_answers(a, b, tol):
    """Two response bodies (parsed JSON) with the same keys, strings and
    integers, and floats within `tol` of each other."""
    if isinstance(a, dict):
        assert isinstance(b, dict) and list(a) == list(b), (a, b)
        for k in a:
            assert_same_answers(a[k], b[k], tol)
    elif isinstance(a, list):
        assert isinstance(b, list) and len(a) == len(b), (a, b)
        for x, y in zip(a, b):
            assert_same_answers(x, y, tol)
    elif isinstance(a, float) or isinstance(b, float):
        assert abs(a - b) <= tol, (a, b)
    else:
        assert a == b, (a, b)


def bodies(n, seed):
    words = workloads.vocab_words(tokgen.tokenizer_json(0))
    rng = np.random.default_rng(seed)
    out = [workloads.single_request_json(words, 0)]
    out += [workloads.system_one_request_json(rng, words, int(rng.integers(20, 400)),
                                              workloads.random_questions(rng)[:int(rng.integers(1, 8))])
            for _ in range(n - 1)]
    return [json.dumps(b) for b in out]


def post(addr, body):
    host, port = addr.split(":")
    c = http.client.HTTPConnection(host, int(port), timeout=120)
    c.request("POST", "/systemone", body=body)
    r = c.getresponse()
    d = r.read()
    c.close()
    return r.status, d


@pytest.fixture(scope="module")
def direct():
    path = modelgen.cached_model(seed=0)
    eng = E.Engine(path, device=0)
    tok = FE.Tokenizer(gguf_path=path)
    info = eng.info()
    yield path, eng, tok, info.calibration
    tok.close()
    eng.close()


def test_served_bodies_equal_the_library_request_path(direct):
    path, eng, tok, cal = direct
    bs = bodies(6, 3)
    want = []
    for b in bs:
        rq = FE.Requests(tok, [b])
        rq.set_calibration(cal["temperature"], cal["by_options"])
        for f in range(rq.pack(16384)):
            out = eng.forward(rq.batch(f))
            rq.score(f, out.logits, out.act)
        want.append(rq.response_text(0))
        rq.close()
    with S.Server(model=path, addr="127.0.0.1:0", devices=(0,)) as s:
        for b, w in zip(bs, want):
            st, d = post(s.address, b)
            assert st == 200
            assert_same_answers(json.loads(d), json.loads(w), SAME_TOL)
        st, d = post(s.address, '{"state": "x", "questions": {}}')
        assert (st, json.loads(d)) == (422, {"error": "no questions"})


def test_batched_service_under_concurrent_clients(direct):
    path, eng, tok, cal = direct
    bs = bodies(24, 7)
    with S.Server(model=path, addr="127.0.0.1:0", devices=(0,)) as s:
        one = [post(s.address, b) for b in bs]
    res = [None] * len(bs)
    with S.Server(model=path, addr="127.0.0.1:0", devices=(0,), batch=16, connections=24) as s:
        ts = [threading.Thread(target=lambda i=i: res.__setitem__(i, post(s.address, bs[i])))
              for i in range(len(bs))]
        for t in ts:
            t.start()
        for t in ts:
            t.join(300)
        st = s.stats()
    assert st["200"] == len(bs) and st["forwards"] <= len(bs)
    for (s1, d1), (s2, d2) in zip(one, res):
        assert s1 == 200 and s2 == 200
        assert_same_answers(json.loads(d1), json.loads(d2), BATCH_TOL)
