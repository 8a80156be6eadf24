"""The request front end (C++, include/laya_frontend.h) against the Python
restatement of the reference's tokenizer.rs / systemone.rs / main.rs
(oracle/frontend_ref.py), and the scoring path against the reference's own
recorded answers (tests/golden/fixture_outputs.json).  CPU only."""
import json
import math
import os

import numpy as np
import pytest

from laya_rust_b200 import frontend as FE
from laya_rust_b200 import tokgen, workloads
from oracle import frontend_ref as F

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "fixture_outputs.json")))


@pytest.fixture(scope="module")
def tj():
    return tokgen.tokenizer_json(0)


@pytest.fixture(scope="module")
def tok(tj):
    t = FE.Tokenizer(tj)
    yield t
    t.close()


@pytest.fixture(scope="module")
def otok(tj):
    return F.Tokenizer(tj)


ALPHABET = (list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789") * 3 +
            list(" " * 30) + list(".,!?;:'\"()[]{}-_/@#$%^&*+=<>|\\~`") +
            ["\n", "\t", "\r", " ", "　", " ", "\x0b", "\x1c"] +
            list("éüßñçøÆΩλδЖжשאع数字日本語한국") + ["́", "٣", "Ⅷ", "½", "🙂", "€"] +
            ["'s", "'LL", "'re", "'ve", "'M", "'d", "'t"] + ["[MASK]", "[CLS]", " [MASK]", "[SEP] ", "[PAD]"])


def random_text(rng, n):
    return "".join(ALPHABET[int(i)] for i in rng.integers(0, len(ALPHABET), n))


def test_tokenizer_matches_the_restatement(tok, otok):
    rng = np.random.default_rng(0)
    for trial in range(400):
        s = random_text(rng, int(rng.integers(0, 80)))
        for special in (False, True):
            assert tok.encode(s, special) == otok.encode(s, special), repr(s)


def test_tokenizer_specials_and_gguf_copy(tok, tj):
    from laya_rust_b200 import modelgen
    assert tok.specials() == {"cls": 50281, "sep": 50282, "mask": 50284, "pad": 50283, "unk": 50280}
    g = FE.Tokenizer(gguf_path=modelgen.cached_model(seed=0))
    s = "choice question: Which team should handle this? [MASK] billing"
    assert g.encode(s) == tok.encode(s)
    g.close()


def test_tokenizer_rejects_bad_input(tj):
    with pytest.raises(FE.LayaError):
        FE.Tokenizer('{"model": {}}')
    t = FE.Tokenizer(tj)
    with pytest.raises(FE.LayaError, match="UTF-8"):
        n = FE.ctypes.c_size_t()
        FE._check(FE.lib().laya_tokenize(t._h, b"\xff\xfe", 2, 0, None, 0, FE.ctypes.byref(n)))
    t.close()


def edge_requests():
    long_opt = " ".join(["option"] * 80)
    return [
        {"state": "short", "questions": {"a": {"type": "choice", "instructions": "Pick [MASK] one.",
                                               "criteria": ["x", "y", "x", 3, None, True, 2.5]}}},
        {"state": {"k": [1, 2.0, -0.0, 1e21, 1.5e-7, "s\né"], "n": None},
         "questions": {"s": {"type": "score", "instructions": {"obj": [1, "two"]},
                             "criteria": ["low", {"mid": 1}, 3]}}},
        {"state": ["list", "state"], "questions": {"n": {"type": "noul", "instructions": "Is it?",
                                                         "criteria": {"true": "yes!", "false": None}}}},
        {"state": 42, "questions": {"c": {"type": "choice", "instructions": "x " * 300,
                                          "criteria": {f"o{i}": long_opt for i in range(6)}}}},
        {"state": " ".join(["state"] * 900), "questions": {"c": {"type": "choice", "instructions": "long state",
                                                                 "criteria": {"a": "A", "b": "B"}}}},
        {"questions": {"x": {"type": "noul", "instructions": "no state"}}},
    ]


def bad_requests():
    return [
        ('{"state": "s"}', 'missing "questions"'),
        ('{"questions": {"a": {"instructions": "i"}}}', 'question a: missing "type"'),
        ('{"questions": {"a": {"type": "rank", "instructions": "i"}}}', "question a: bad type rank"),
        ('{"questions": {"a": {"type": "noul"}}}', 'question a: missing "instructions"'),
        ('{"questions": {"a": {"type": "choice", "instructions": "i", "criteria": {'
         + ",".join(f'"c{i}": "{"word " * 40}"' for i in range(200)) + "}}}}", "options do not fit"),
        ('{"questions": ', "EOF"),
    ]


def all_requests():
    reqs = [fx["request"] for fx in GOLD["fixtures"]] + [s["request"] for s in GOLD["scenarios"]]
    reqs += edge_requests()
    rng = np.random.default_rng(7)
    words = workloads.vocab_words(tokgen.tokenizer_json(0))
    reqs += [workloads.system_one_request_json(rng, words, int(rng.integers(5, 300)),
                                               workloads.random_questions(rng)) for _ in range(30)]
    return reqs


def test_plan_matches_the_restatement(tok, otok):
    reqs = all_requests()
    rq = FE.Requests(tok, reqs, threads=4)
    qi = 0
    for r, req in enumerate(reqs):
        assert rq.error(r) is None, (r, rq.error(r))
        state, questions = F.parse_request(F.loads(json.dumps(req)))
        items = F.plan_items(otok, state, questions)
        for it in items:
            got = rq.question(qi)
            assert got["request"] == r and got["qtype"] == it.qtype
            assert got["seq"] == it.seq, (r, it.id)
            assert got["markers"] == it.markers, (r, it.id)
            qi += 1
    assert qi == rq.questions()
    rq.close()


def test_bad_requests_keep_the_reference_message(tok, otok):
    texts = [t for t, _ in bad_requests()]
    rq = FE.Requests(tok, texts + [json.dumps(GOLD["fixtures"][0]["request"])])
    for r, (text, want) in enumerate(bad_requests()):
        err = rq.error(r)
        assert err is not None and want in err, (err, want)
        if want != "EOF":
            with pytest.raises(F.RequestError) as ei:
                state, qs = F.parse_request(F.loads(text))
                F.plan_items(otok, state, qs)
            assert str(ei.value) == err
    assert rq.error(len(texts)) is None
    rq.close()


def test_threads_do_not_change_the_plan(tok):
    reqs = all_requests()
    a = FE.Requests(tok, reqs, threads=1)
    b = FE.Requests(tok, reqs, threads=8)
    assert a.questions() == b.questions()
    for i in range(a.questions()):
        assert a.question(i) == b.question(i)


def oracle_forwards(items_per_request, max_tokens, across):
    """Forwards as lists of (request, question) by the reference's rule."""
    out = []
    if across:
        order = [(r, i) for r, items in enumerate(items_per_request) for i in range(len(items))]
        cur, cur_max = [], 0
        for r, i in order:
            ln = len(items_per_request[r][i].seq)
            if cur and max(cur_max, ln) * (len(cur) + 1) > max_tokens:
                out.append(cur)
                cur, cur_max = [], 0
            cur_max = max(cur_max, ln)
            cur.append((r, i))
        if cur:
            out.append(cur)
    else:
        for r, items in enumerate(items_per_request):
            out += [[(r, i) for i in g] for g in F.group_by_budget(items, max_tokens)]
    return out


@pytest.mark.parametrize("max_tokens,across", [(300, False), (16384, False), (300, True), (2048, True)])
def test_packing_and_batches(tok, otok, max_tokens, across):
    reqs = all_requests()
    rq = FE.Requests(tok, reqs)
    per = []
    for req in reqs:
        state, qs = F.parse_request(F.loads(json.dumps(req)))
        per.append(F.plan_items(otok, state, qs))
    want = oracle_forwards(per, max_tokens, across)
    assert rq.pack(max_tokens, across) == len(want)
    for f, rows in enumerate(want):
        b = rq.batch(f)
        items = [per[r][i] for r, i in rows]
        n, l, k, ids, att, mpos, mmask, qtype = F.build_batch(items, list(range(len(items))))
        assert (b.n, b.l, b.k) == (n, l, k)
        for x, y in ((b.ids, ids), (b.att, att), (b.mpos, mpos), (b.mmask, mmask), (b.qtype, qtype)):
            assert np.array_equal(np.asarray(x).ravel(), y.ravel())
    rq.close()


def test_responses_match_the_restatement(tok, otok):
    """Random outputs scored by both: the response JSON text is identical
    (answers in scoring order, f32 arithmetic, ryu number layout)."""
    reqs = all_requests()
    rng = np.random.default_rng(3)
    cal = {"temperature": (1.3, 0.7, 2.0), "by_options": {"choice:3-5": 1.76, "noul:2": 1.98}}
    per = []
    for req in reqs:
        state, qs = F.parse_request(F.loads(json.dumps(req)))
        per.append(F.plan_items(otok, state, qs))
    fws = oracle_forwards(per, 16384, False)
    rq = FE.Requests(tok, reqs)
    rq.set_calibration(cal["temperature"], cal["by_options"])
    assert rq.pack(16384, False) == len(fws)
    outputs = []
    for f in range(len(fws)):
        b = rq.batch(f)
        lg = rng.standard_normal(b.n * b.k).astype(np.float32) * 3
        lg[np.asarray(b.mmask).ravel() == 0] = -10000.0
        ac = rng.standard_normal(b.n * 2).astype(np.float32) * 2
        rq.score(f, lg, ac)
        outputs.append((lg, ac))
    ocal = F.Calibration(cal["temperature"], sorted(cal["by_options"].items()))
    for r, req in enumerate(reqs):
        feed = iter([outputs[f] for f, rows in enumerate(fws) if rows[0][0] == r])
        want = F.run_all(lambda *a: next(feed), otok, F.loads(json.dumps(req)), 16384, ocal)
        assert rq.response_text(r) == F.to_json(want), r
    rq.close()


def _temperature_for(q, logits, act, want):
    """A temperature under which the restatement reproduces the reference's
    recorded answer exactly (the checkpoint's calibration is not recorded)."""
    ps = [1 - want["noul"], want["noul"]] if q.ty == "noul" else list(want["probabilities"].values())
    order = sorted(range(len(ps)), key=lambda i: -ps[i])
    i, j = order[0], order[1]
    t0 = (logits[i] - logits[j]) / math.log(ps[i] / ps[j]) if 0 < ps[j] < ps[i] else 1.0
    a = [np.float32(x) for x in act]
    mx = max(np.float32(np.finfo(np.float32).min), a[0], a[1])
    e0, e1 = F.expf(a[0] - mx), F.expf(a[1] - mx)
    act_p = np.float32(e0 / np.float32(e0 + e1))
    for d in np.linspace(-0.03, 0.03, 6001):
        t = np.float32(t0 * (1 + d))
        if t > 0 and F.answer(q, F.softmax_t([np.float32(x) for x in logits], t), act_p) == want:
            return float(t)
    return None


def test_scoring_reproduces_the_reference_answers(tok):
    """Each recorded answer (the reference's score_row + answer on its own
    logits and act) is reproduced exactly -- every printed number, the
    choice, the key order -- by the C++ scorer at a temperature the
    restatement finds; 19 answers over the 5 fixtures."""
    checked = 0
    for fx in GOLD["fixtures"]:
        state, qs = F.parse_request(fx["request"])
        byid = {q.id: q for q in qs}
        for fw in fx["forwards"]:
            k = fw["k"]
            for row_i, row in enumerate(fw["rows"]):
                q = byid[row["id"]]
                lg = fw["logits"][row_i * k: row_i * k + row["markers"]]
                ac = fw["act"][row_i * 2: row_i * 2 + 2]
                want = fx["answers"][row["id"]]
                t = _temperature_for(q, lg, ac, want)
                assert t is not None, (fx["name"], row["id"])
                one = {"state": fx["request"].get("state"), "questions": {q.id: fx["request"]["questions"][q.id]}}
                rq = FE.Requests(tok, [one])
                size = "2" if row["markers"] <= 2 else "3-5" if row["markers"] <= 5 else "6-10" \
                    if row["markers"] <= 10 else "11+"
                key = f"{['choice', 'score', 'noul'][q.qtype]}:{size}"
                rq.set_calibration((1.0, 1.0, 1.0), json.dumps({key: t}))
                assert rq.pack(16384, False) == 1
                b = rq.batch(0)
                lgp = np.full(b.k, -10000.0, np.float32)
                lgp[:len(lg)] = lg
                rq.score(0, lgp, np.asarray(ac, np.float32))
                got = json.loads(rq.response_text(0), parse_float=lambda t: {"f64": t})["answers"][q.id]
                # the same values printed as the same literal text
                assert got == fx["answers_literal"][q.id], (fx["name"], row["id"])
                assert list(got) == list(want)
                rq.close()
                checked += 1
    assert checked == 19


def test_number_formatting_follows_ryu():
    """The restatement's f64 printer against ryu's layout (serde_json); the
    C++ printer is checked through the serialised states of the plan test
    (1e21, 1.5e-7, -0.0, 2.0) and the answers above."""
    cases = {0.8366000056266785: "0.8366000056266785", 1.0: "1.0", 1e16: "1e16", 1e15: "1000000000000000.0",
             1.5e-5: "0.000015", 1e-6: "1e-6", 123.456: "123.456", -2.5e-300: "-2.5e-300", 4021.0: "4021.0",
             0.1: "0.1", 1.2345678901234568e20: "1.2345678901234568e20", -0.0: "-0.0", 5e-324: "5e-324"}
    for x, s in cases.items():
        assert F.fmt_f64(x) == s


def test_front_end_calls_reject_bad_arguments(tok):
    """Null pointers and out-of-range indices come back as a status and a
    message, never a crash (the engine ABI's convention)."""
    import ctypes
    L = FE.lib()
    h = ctypes.c_void_p()
    assert L.laya_tokenizer_from_json(None, 0, ctypes.byref(h)) != 0
    assert L.laya_tokenizer_from_gguf(b"/nonexistent.gguf", ctypes.byref(h)) != 0
    assert "nonexistent" in L.laya_last_error().decode()
    n = ctypes.c_size_t()
    assert L.laya_tokenize(None, b"x", 1, 0, None, 0, ctypes.byref(n)) != 0
    rq = FE.Requests(tok, [GOLD["fixtures"][0]["request"]])
    assert L.laya_requests_error(rq._h, 5) is not None          # out of range
    with pytest.raises(FE.LayaError):
        rq.question(10 ** 6)
    with pytest.raises(FE.LayaError):
        rq.batch(0)                                               # not packed yet
    rq.pack(16384)
    with pytest.raises(FE.LayaError):
        rq.batch(99)
    with pytest.raises(FE.LayaError, match="not scored"):
        rq.response_text(0)
    with pytest.raises(FE.LayaError):
        rq.set_calibration((1.0, 1.0, 1.0), "[1, 2]")             # not an object
    assert L.laya_requests_pack(rq._h, 0, 0, ctypes.byref(ctypes.c_int64())) != 0
    rq.close()


def test_long_pieces_match_and_stay_fast(tok, otok):
    """BPE on long single pieces (a letters-only run, a repeated pattern):
    the same tokens as the reference's merge loop, and a 50 000-character
    piece tokenizes in well under a second (the reference's loop is cubic
    in a piece's length)."""
    import time
    rng = np.random.default_rng(5)
    parts = ["the", "tion", "aaaa", "stand", "ing", "ou", "ea", "x"]
    for trial in range(200):
        w = "".join(parts[int(i)] for i in rng.integers(0, len(parts), int(rng.integers(1, 80))))
        s = ("" if trial % 2 else " ") + w
        assert tok.encode(s) == otok.encode(s, False), s
    s = "a" * 300 + "b" * 150 + "ab" * 150
    assert tok.encode(s) == otok.encode(s, False)
    t0 = time.perf_counter()
    ids = tok.encode("stand" * 10000)
    assert time.perf_counter() - t0 < 1.0 and len(ids) > 0


def test_merge_of_separately_planned_requests_equals_one_plan(tok, tj):
    """laya_requests_merge: requests planned one by one (as the HTTP service's
    connection threads do) pack, score and answer exactly like the same
    requests planned together; errors stay with their request."""
    words = workloads.vocab_words(tj)
    rng = np.random.default_rng(3)
    reqs = [workloads.system_one_request_json(rng, words, int(rng.integers(10, 120)),
                                              workloads.random_questions(rng)[:int(rng.integers(1, 6))])
            for _ in range(5)]
    reqs.insert(2, {"state": "x"})  # fails to plan
    texts = [json.dumps(r) for r in reqs]
    whole = FE.Requests(tok, texts)
    parts = [FE.Requests(tok, [t]) for t in texts]
    merged = FE.Requests.merge(parts)
    assert all(p.n_requests == 0 for p in parts)
    assert merged.n_requests == whole.n_requests == len(reqs)
    assert merged.questions() == whole.questions()
    for i in range(whole.questions()):
        assert merged.question(i) == whole.question(i)
    for across in (False, True):
        nf = whole.pack(4096, across)
        assert merged.pack(4096, across) == nf
        for f in range(nf):
            a, b = whole.batch(f), merged.batch(f)
            for name in ("ids", "att", "mpos", "mmask", "qtype"):
                assert np.array_equal(getattr(a, name), getattr(b, name))
            lg = np.sin(np.arange(a.n * a.k, dtype=np.float32))
            ac = np.cos(np.arange(a.n * 2, dtype=np.float32))
            whole.score(f, lg, ac)
            merged.score(f, lg, ac)
        for j in range(len(reqs)):
            assert merged.error(j) == whole.error(j)
            if whole.error(j) is None:
                assert merged.response_text(j) == whole.response_text(j)
    for p in parts:
        p.close()
    merged.close()
    whole.close()


def test_pack_sorted_across_requests_is_group_by_budget_over_the_set(tok, tj):
    """across_requests = 2: the reference's group_by_budget (main.rs:448-468)
    applied to every question of every request at once."""
    words = workloads.vocab_words(tj)
    rng = np.random.default_rng(8)
    reqs = [workloads.system_one_request_json(rng, words, int(rng.integers(10, 300)),
                                              workloads.random_questions(rng)[:int(rng.integers(1, 8))])
            for _ in range(12)]
    rq = FE.Requests(tok, reqs)
    lens = [rq.question_shape(i)[1] for i in range(rq.questions())]
    for budget in (2048, 16384):
        order = sorted(range(len(lens)), key=lambda i: lens[i])  # stable
        want, cur, cur_max = [], [], 0
        for i in order:
            if cur and max(cur_max, lens[i]) * (len(cur) + 1) > budget:
                want.append(cur)
                cur, cur_max = [], 0
            cur_max = max(cur_max, lens[i])
            cur.append(i)
        want.append(cur)
        nf = rq.pack(budget, 2)
        assert [rq.forward_questions(f) for f in range(nf)] == want
        assert nf <= rq.pack(budget, 1)
    with pytest.raises(FE.LayaError):
        rq.pack(16384, 3)
    rq.close()


def test_pack_windows_is_group_by_budget_per_window(tok, tj):
    """laya_requests_pack_windows: window 1 is run_all's per-request
    grouping (mode 0), a window over every request is mode 2, and in between
    each window of consecutive requests is grouped on its own."""
    words = workloads.vocab_words(tj)
    rng = np.random.default_rng(12)
    reqs = [workloads.system_one_request_json(rng, words, int(rng.integers(10, 300)),
                                              workloads.random_questions(rng)[:int(rng.integers(1, 8))])
            for _ in range(11)]
    rq = FE.Requests(tok, reqs)
    fw = lambda nf: [rq.forward_questions(f) for f in range(nf)]
    assert fw(rq.pack_windows(4096, 1)) == fw(rq.pack(4096, 0))
    assert fw(rq.pack_windows(4096, 11)) == fw(rq.pack(4096, 2))
    assert fw(rq.pack_windows(4096, 100)) == fw(rq.pack(4096, 2))
    got = fw(rq.pack_windows(4096, 4))
    owner = [rq.question_shape(i)[0] for i in range(rq.questions())]
    want = []
    for w0 in range(0, 11, 4):
        part = FE.Requests(tok, reqs[w0:w0 + 4])
        base = sum(1 for o in owner if o < w0)  # questions of the earlier requests
        for f in range(part.pack(4096, 2)):
            want.append([q + base for q in part.forward_questions(f)])
        part.close()
    assert got == want
    with pytest.raises(FE.LayaError):
        rq.pack_windows(4096, 0)
    rq.close()
