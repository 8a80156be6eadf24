"""Host packing around the hot path, pinned by the reference's golden fixtures.

The reference recorded its fixtures with ``--max-tokens 300``; each fixture
stores the padded index arrays of every forward it ran.  Rebuilding the items
(one per question, in request order) and packing them with the restated
``group_by_budget`` / ``build_batch`` must reproduce those forwards exactly:
row order, padding id 0, att, marker positions and masks, qtype, and the
budget split (e.g. many-questions -> 10 + 2).
"""
import json
import os

import numpy as np
import pytest

from laya_rust_b200 import arch
from laya_rust_b200.batching import Calibration, Item, build_batch, group_by_budget, score_row, temperature

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = json.load(open(os.path.join(HERE, "golden", "fixture_requests.json")))


def items_of(fx):
    found = {}
    for fw in fx["forwards"]:
        ids = np.array(fw["ids"]).reshape(fw["n"], fw["l"])
        att = np.array(fw["att"]).reshape(fw["n"], fw["l"])
        mpos = np.array(fw["mpos"]).reshape(fw["n"], fw["k"])
        for r, qid in enumerate(fw["rows"]):
            ln = int(att[r].sum())
            found[qid] = Item(list(ids[r, :ln]), list(mpos[r, :fw["markers"][r]]), fw["qtype"][r], qid)
    return [found[q] for q in fx["question_order"]]


@pytest.mark.parametrize("fx", FIXTURES, ids=[f["name"] for f in FIXTURES])
def test_budget_grouping_and_batches_match_the_fixture(fx):
    items = items_of(fx)
    groups = group_by_budget(items, fx["max_tokens"])
    assert len(groups) == len(fx["forwards"])
    for g, fw in zip(groups, fx["forwards"]):
        assert [items[i].id for i in g] == fw["rows"]
        req = build_batch(items, g)
        assert (req.n, req.l, req.k) == (fw["n"], fw["l"], fw["k"])
        for name in ("ids", "att", "mpos", "mmask", "qtype"):
            assert np.array_equal(getattr(req, name), np.array(fw[name], np.int64)), name


@pytest.mark.parametrize("fx", FIXTURES, ids=[f["name"] for f in FIXTURES])
def test_fixture_layout_invariants(fx):
    """[CLS] at 0, [SEP] closing each row, [MASK] at every marker, pad id 0."""
    for fw in fx["forwards"]:
        ids = np.array(fw["ids"]).reshape(fw["n"], fw["l"])
        att = np.array(fw["att"]).reshape(fw["n"], fw["l"])
        mpos = np.array(fw["mpos"]).reshape(fw["n"], fw["k"])
        mmask = np.array(fw["mmask"]).reshape(fw["n"], fw["k"])
        for r in range(fw["n"]):
            ln = int(att[r].sum())
            assert att[r, :ln].all() and not att[r, ln:].any()
            assert ids[r, 0] == arch.CLS_ID and ids[r, ln - 1] == arch.SEP_ID
            assert (ids[r, ln:] == arch.PAD_ID).all()
            for j in range(fw["k"]):
                if mmask[r, j]:
                    assert ids[r, mpos[r, j]] == arch.MASK_ID
                else:
                    assert mpos[r, j] == 0


def test_many_questions_splits_ten_and_two():
    fx = next(f for f in FIXTURES if f["name"] == "many-questions")
    groups = group_by_budget(items_of(fx), 300)
    assert [len(g) for g in groups] == [10, 2]


def test_temperature_lookup_by_option_count():
    """systemone.rs:200-216: option-count refinement falls back to the type."""
    cal = Calibration([1.5, 2.0, 3.0], [("choice:3-5", 0.75), ("noul:2", 1.25)])
    assert temperature(0, 3, cal) == 0.75
    assert temperature(0, 2, cal) == 1.5
    assert temperature(2, 2, cal) == 1.25
    assert temperature(1, 11, cal) == 2.0


def test_score_row_softmax_and_act_probability():
    logits = np.array([1.0, 2.0, -10000.0, 0.5, 0.5, 0.0], np.float32)
    act = np.array([0.0, 0.0, 2.0, 0.0], np.float32)
    p, a = score_row(logits, act, 0, 3, 2, 0, Calibration())
    assert np.allclose(p, [1 / (1 + np.e), np.e / (1 + np.e)], atol=1e-6)
    assert abs(a - 0.5) < 1e-7
    p, a = score_row(logits, act, 1, 3, 3, 0, Calibration())
    assert np.allclose(p.sum(), 1.0, atol=1e-6)
    assert abs(a - 1 / (1 + np.exp(-2.0))) < 1e-6
