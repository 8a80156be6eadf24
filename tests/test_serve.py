"""The HTTP service (include/laya_serve.h, `laya serve` of laya-rust
src/main.rs:996-1204) on the CPU: the status-code contract of serve_request
(main.rs:1072-1138) and Service::run (:1029-1037), keep-alive, chunked and
100-continue bodies, the bounded queue's 503, several inference threads,
cross-request batching, and 200 bodies byte-identical to the reference's
run_all + response restated in oracle/frontend_ref.py.  A forward hook stands
in for the engine: per row, logits and act are a fixed function of the row's
real token ids, so answers do not depend on how rows are batched."""
import http.client
import json
import socket
import threading
import time

import numpy as np
import pytest

from laya_rust_b200 import frontend as FE
from laya_rust_b200 import serve as S
from laya_rust_b200 import tokgen, workloads
from oracle import frontend_ref as F


def row_outputs(n, l, k, ids, att):
    ids = np.asarray(ids, np.int64).reshape(n, l)
    att = np.asarray(att, np.int64).reshape(n, l)
    logits = np.zeros((n, k), np.float32)
    act = np.zeros((n, 2), np.float32)
    for r in range(n):
        real = ids[r][att[r] != 0]
        h = float((real * np.arange(1, real.size + 1)).sum() % 9973) / 97.0
        logits[r] = 3.0 * np.sin(h + np.arange(k))
        act[r] = [np.cos(h), np.sin(0.5 * h)]
    return logits.ravel(), act.ravel()


def hook(slot, req):
    return row_outputs(req.n, req.l, req.k, req.ids, req.att)


@pytest.fixture(scope="module")
def tj():
    return tokgen.tokenizer_json(0)


@pytest.fixture(scope="module")
def otok(tj):
    return F.Tokenizer(tj)


@pytest.fixture(scope="module")
def words(tj):
    return workloads.vocab_words(tj)


@pytest.fixture(scope="module")
def srv(tj):
    s = S.Server(addr="127.0.0.1:0", forward=hook, tokenizer_json=tj, connections=4)
    yield s
    s.close()


def request_bodies(words, n=6, seed=5):
    rng = np.random.default_rng(seed)
    out = [workloads.single_request_json(words, 0)]
    out += [workloads.system_one_request_json(rng, words, int(rng.integers(10, 80)),
                                              workloads.random_questions(rng)[:int(rng.integers(1, 6))])
            for _ in range(n - 1)]
    return [json.dumps(b) for b in out]


def expected(otok, body, max_tokens=16384):
    fwd = lambda n, l, k, ids, att, mpos, mmask, qtype: row_outputs(n, l, k, ids, att)
    return F.to_json(F.run_all(fwd, otok, F.loads(body), max_tokens))


def post(addr, body, path="/systemone", method="POST", headers=None):
    host, port = addr.split(":")
    c = http.client.HTTPConnection(host, int(port), timeout=30)
    c.request(method, path, body=body, headers=headers or {})
    r = c.getresponse()
    data = r.read()
    c.close()
    return r.status, r.getheader("Content-Type"), data


def raw(addr, payload: bytes, read_until_close=True) -> bytes:
    host, port = addr.split(":")
    s = socket.create_connection((host, int(port)), timeout=30)
    s.sendall(payload)
    if read_until_close:
        s.shutdown(socket.SHUT_WR)
    out = b""
    while True:
        d = s.recv(65536)
        if not d:
            break
        out += d
    s.close()
    return out


def test_200_bodies_match_the_reference_run_all(srv, otok, words):
    for body in request_bodies(words):
        st, ct, data = post(srv.address, body)
        assert st == 200 and ct == "application/json"
        assert data.decode() == expected(otok, body)


def test_status_codes_of_serve_request(srv):
    a = srv.address
    body = '{"state": "x", "questions": {"q": {"type": "noul", "instructions": "a"}}}'
    assert post(a, body, path="/other")[0] == 404
    assert post(a, body, path="/systemone?x=1")[0] == 404          # the target is compared byte for byte
    assert post(a, None, path="/systemone", method="GET")[:3:2] == (405, b'{"error":"use POST"}')
    assert post(a, body, method="PUT")[0] == 405
    st, _, d = post(a, "{not json")
    assert st == 400 and json.loads(d)["error"].startswith("invalid json: ")
    st, _, d = post(a, "")
    assert st == 400 and json.loads(d)["error"].startswith("invalid json: ")
    st, _, d = post(a, b'{"state": "\xff"}')
    assert (st, json.loads(d)) == (400, {"error": "body: stream did not contain valid UTF-8"})
    st, _, d = post(a, '{"state": "x", "questions": {}}')
    assert (st, json.loads(d)) == (422, {"error": "no questions"})
    st, _, d = post(a, '{"state": "x"}')
    assert st == 422 and "questions" in json.loads(d)["error"]
    st, _, d = post(a, '{"state": "x", "questions": {"q": {"type": "essay", "instructions": "a"}}}')
    assert st == 422 and "bad type" in json.loads(d)["error"]
    assert post(a, body)[0] == 200


def test_413_is_answered_before_the_body(srv):
    head = (b"POST /systemone HTTP/1.1\r\nHost: x\r\nContent-Length: %d\r\n\r\n" % (8 * 1024 * 1024 + 1))
    out = raw(srv.address, head)
    assert out.startswith(b"HTTP/1.1 413 ") and out.endswith(b'{"error":"body too large"}')
    # exactly 8 MiB is allowed through to the JSON check
    big = b" " * (8 * 1024 * 1024 - 2) + b"{}"
    st, _, d = post(srv.address, big)
    assert st == 422


def test_truncated_body_is_a_400(srv):
    out = raw(srv.address, b"POST /systemone HTTP/1.1\r\nContent-Length: 100\r\n\r\n{\"state\"")
    assert out.startswith(b"HTTP/1.1 400 ") and b'"error":"body: ' in out


def test_keep_alive_chunked_and_expect_100(srv, otok, words):
    bodies = request_bodies(words, 3, seed=9)
    host, port = srv.address.split(":")
    c = http.client.HTTPConnection(host, int(port), timeout=30)
    for b in bodies:  # one connection, three requests
        c.request("POST", "/systemone", body=b)
        r = c.getresponse()
        assert r.status == 200 and r.read().decode() == expected(otok, b)
        assert r.getheader("Connection") == "keep-alive"
    c.close()
    b = bodies[0].encode()
    chunks = b"".join(b"%x;ext=1\r\n%s\r\n" % (len(b[i:i + 7]), b[i:i + 7]) for i in range(0, len(b), 7))
    out = raw(srv.address, b"POST /systemone HTTP/1.1\r\nTransfer-Encoding: chunked\r\nConnection: close\r\n\r\n" +
              chunks + b"0\r\nX-Trailer: y\r\n\r\n")
    assert out.startswith(b"HTTP/1.1 200 ") and out.split(b"\r\n\r\n", 1)[1].decode() == expected(otok, bodies[0])
    s = socket.create_connection((host, int(port)), timeout=30)
    s.sendall(b"POST /systemone HTTP/1.1\r\nExpect: 100-continue\r\nConnection: close\r\nContent-Length: %d\r\n\r\n"
              % len(b))
    assert s.recv(64) == b"HTTP/1.1 100 Continue\r\n\r\n"
    s.sendall(b)
    out = b""
    while (d := s.recv(65536)):
        out += d
    s.close()
    assert out.startswith(b"HTTP/1.1 200 ") and b"Connection: close" in out


def test_forward_failure_is_a_500(tj):
    def bad(slot, req):
        raise RuntimeError("device lost")
    with S.Server(addr="127.0.0.1:0", forward=bad, tokenizer_json=tj) as s:
        body = '{"state": "x", "questions": {"q": {"type": "noul", "instructions": "a"}}}'
        st, _, d = post(s.address, body)
        assert st == 500 and json.loads(d)["error"].startswith("inference failed: ")
        assert s.stats()["500"] == 1


def test_full_queue_answers_503_and_queued_requests_are_served(tj, otok, words):
    gate, entered = threading.Event(), threading.Event()

    def slow(slot, req):
        entered.set()
        gate.wait(30)
        return hook(slot, req)

    bodies = request_bodies(words, 3, seed=13)
    with S.Server(addr="127.0.0.1:0", forward=slow, tokenizer_json=tj, queue=1, connections=4) as s:
        res = {}
        ta = threading.Thread(target=lambda: res.__setitem__("a", post(s.address, bodies[0])))
        ta.start()
        assert entered.wait(30)                       # the inference thread holds request a
        tb = threading.Thread(target=lambda: res.__setitem__("b", post(s.address, bodies[1])))
        tb.start()
        for _ in range(300):                          # request b waits in the queue
            if s.stats()["queued"] == 1:
                break
            time.sleep(0.01)
        assert s.stats()["queued"] == 1
        st, _, d = post(s.address, bodies[2])
        assert (st, json.loads(d)) == (503, {"error": "server busy"})
        gate.set()
        ta.join(30)
        tb.join(30)
        assert res["a"][0] == 200 and res["a"][2].decode() == expected(otok, bodies[0])
        assert res["b"][0] == 200 and res["b"][2].decode() == expected(otok, bodies[1])
        st = s.stats()
        assert (st["200"], st["503"], st["queued"]) == (2, 1, 0)


def run_clients(addr, bodies, threads=8):
    out = [None] * len(bodies)

    def work(i0):
        for i in range(i0, len(bodies), threads):
            out[i] = post(addr, bodies[i])
    ts = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(120)
    return out


def test_several_inference_threads_share_the_queue(tj, otok, words):
    seen = set()
    lock = threading.Lock()

    def slotted(slot, req):
        with lock:
            seen.add(slot)
        time.sleep(0.02)  # long enough that both threads take work
        return hook(slot, req)

    bodies = request_bodies(words, 16, seed=21)
    with S.Server(addr="127.0.0.1:0", forward=slotted, tokenizer_json=tj, devices=(0, 1), connections=8) as s:
        out = run_clients(s.address, bodies)
        assert seen == {0, 1}
    for (st, _, d), b in zip(out, bodies):
        assert st == 200 and d.decode() == expected(otok, b)


def test_batching_packs_queued_requests_into_shared_forwards(tj, otok, words):
    gate = threading.Event()
    rows = []

    def gated(slot, req):
        gate.wait(30)
        rows.append(req.n)
        return hook(slot, req)

    bodies = request_bodies(words, 12, seed=31)
    with S.Server(addr="127.0.0.1:0", forward=gated, tokenizer_json=tj, batch=16, queue=64, connections=12) as s:
        res = {}
        ts = [threading.Thread(target=lambda i=i: res.__setitem__(i, post(s.address, bodies[i])))
              for i in range(len(bodies))]
        for t in ts:
            t.start()
        for _ in range(500):  # the first request is in the hook, the rest queue up
            if s.stats()["queued"] == len(bodies) - 1:
                break
            time.sleep(0.01)
        gate.set()
        for t in ts:
            t.join(60)
        forwards = s.stats()["forwards"]
    assert forwards < len(bodies)  # the 11 queued requests went through shared forwards
    assert max(rows) > 6
    for i, b in enumerate(bodies):
        st, _, d = res[i]
        assert st == 200 and d.decode() == expected(otok, b)  # same answers as one request at a time


def test_stop_and_open_failures(tj):
    s = S.Server(addr="127.0.0.1:0", forward=hook, tokenizer_json=tj)
    a = s.address
    s.stop()
    s.wait()
    with pytest.raises(OSError):
        post(a, "{}")
    s.close()
    with S.Server(addr="127.0.0.1:0", forward=hook, tokenizer_json=tj) as busy:
        with pytest.raises(S.LayaError):  # the port is taken
            S.Server(addr=busy.address, forward=hook, tokenizer_json=tj)
    with pytest.raises(S.LayaError):
        S.Server(model="/nonexistent.gguf", addr="127.0.0.1:0")
    with pytest.raises(S.LayaError):  # no model and no tokenizer
        S.Server(addr="127.0.0.1:0", forward=hook)
    with pytest.raises(S.LayaError):
        S.Server(addr="no-port", forward=hook, tokenizer_json=tj)


def test_cli_rejects_bad_flags(capsys):
    with pytest.raises(SystemExit):
        S.main(["--model", "x.gguf", "--queue", "0"])
    assert S.main(["--model", "/nonexistent.gguf", "--addr", "127.0.0.1:0"]) == 2


def test_http_framing_edge_cases(srv, otok, words):
    a = srv.address
    body = request_bodies(words, 1, seed=41)[0].encode()
    want = expected(otok, body.decode()).encode()
    req = b"POST /systemone HTTP/1.1\r\nContent-Length: %d\r\n\r\n%s" % (len(body), body)
    # two pipelined requests on one connection, then close
    out = raw(a, req + req[:-len(body)].replace(b"HTTP/1.1\r\n", b"HTTP/1.1\r\nConnection: close\r\n") + body)
    assert out.count(b"HTTP/1.1 200 ") == 2 and out.count(want) == 2
    # HTTP/1.0 closes after the answer unless asked to keep the connection
    out = raw(a, req.replace(b"HTTP/1.1", b"HTTP/1.0"))
    assert out.startswith(b"HTTP/1.1 200 ") and b"Connection: close" in out and out.endswith(want)
    # malformed request line, unknown version, oversized head: 400 and close
    for bad in (b"POST\r\n\r\n", b"POST /systemone HTTP/2.0\r\n\r\n",
                b"POST /systemone HTTP/1.1\r\nX: " + b"y" * (70 * 1024) + b"\r\n\r\n",
                b"POST /systemone HTTP/1.1\r\nContent-Length: 1x\r\n\r\n"):
        out = raw(a, bad)
        assert out.startswith(b"HTTP/1.1 400 ") and b"Connection: close" in out, bad[:40]
    # a 404 without a body keeps the connection open for the next request
    out = raw(a, b"GET /nope HTTP/1.1\r\n\r\n" + req.replace(b"HTTP/1.1\r\n", b"HTTP/1.1\r\nConnection: close\r\n"))
    assert out.startswith(b"HTTP/1.1 404 ") and out.count(b"HTTP/1.1 200 ") == 1 and out.endswith(want)
