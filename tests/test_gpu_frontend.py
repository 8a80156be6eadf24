"""Requests end to end on the GPU: request JSON -> C++ front end -> engine ->
scores -> response JSON, against the reference's run_all restated on the CPU
(oracle/frontend_ref.py around the C oracle's forward), for the reference's
fixture requests and a few synthetic ones.  Answers must agree: the same
questions in the same order, the same choices (strictly), probabilities within 2e-2
(the logits' tolerance, through a softmax), identical usage."""
import json
import os

import numpy as np
import pytest

from laya_rust_b200 import frontend as FE
from laya_rust_b200 import modelgen, tokgen, workloads
from laya_rust_b200 import engine as E

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "fixture_outputs.json")))


@pytest.fixture(scope="module")
def setup():
    from oracle import frontend_ref as F
    from oracle.oracle import OracleModel
    path = modelgen.cached_model(seed=0)
    eng = E.Engine(path, device=0)
    tok = FE.Tokenizer(gguf_path=path)
    otok = F.Tokenizer(tokgen.tokenizer_json(0))
    om = OracleModel(path)
    yield eng, tok, otok, om, F
    om.close()
    tok.close()
    eng.close()


def requests():
    reqs = [fx["request"] for fx in GOLD["fixtures"]]
    words = workloads.vocab_words(tokgen.tokenizer_json(0))
    rng = np.random.default_rng(11)
    reqs += [workloads.single_request_json(words, 0)]
    reqs += [workloads.system_one_request_json(rng, words, int(rng.integers(20, 60)),
                                               workloads.random_questions(rng)[:4]) for _ in range(3)]
    return reqs


@pytest.fixture(scope="module")
def reference_responses(setup):
    eng, tok, otok, om, F = setup
    return [F.run_all(om.forward, otok, F.loads(json.dumps(req)), 16384) for req in requests()]


def close_answers(got, want, name, ordered=True):
    if ordered:
        assert list(got) == list(want), name
    assert set(got) == set(want), name
    for qid in want:
        g, w = got[qid], want[qid]
        assert g["type"] == w["type"] and set(g) == set(w), (name, qid)
        if "choice" in w:
            # always the same choice; a disagreement reports the reference's
            # top-2 probability margin
            pw = np.sort(np.array(list(w["probabilities"].values())))
            margin = float(pw[-1] - pw[-2]) if len(pw) > 1 else float("inf")
            assert g["choice"] == w["choice"], (name, qid, "reference top-2 margin", margin)
        for key in ("probabilities",):
            if key in w:
                for k in w[key]:
                    assert abs(g[key][k] - w[key][k]) <= 2e-2, (name, qid, k)
        for key in ("noul", "score", "confidence"):
            if key in w:
                assert abs(g[key] - w[key]) <= 5e-2, (name, qid, key)
        assert abs(g["rl_agent"]["act_probability"] - w["rl_agent"]["act_probability"]) <= 2e-2


@pytest.mark.parametrize("across", [False, True])
def test_requests_end_to_end_match_the_cpu_reference(setup, reference_responses, across):
    """across=False is the reference's run_all per request (answers in its
    order); across=True packs questions of all requests together (answers in
    request order)."""
    eng, tok, otok, om, F = setup
    reqs = requests()
    got = FE.run_requests(eng, tok, reqs, max_tokens=16384, across_requests=across, threads=4)
    for i, want in enumerate(reference_responses):
        assert got[i]["usage"] == want["usage"], i
        close_answers(got[i]["answers"], want["answers"], i, ordered=not across)
