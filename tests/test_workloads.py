"""Host-side logic of the benchmark workloads: the System One sequence layout,
the request stream, its greedy assignment to GPUs and cross-request packing
into token-budget forwards."""
import numpy as np

from laya_rust_b200 import arch, batching, workloads


def test_single_request_has_the_config0_shape():
    items = workloads.single_request(0)
    assert len(items) == 2 and all(len(it.seq) <= 128 for it in items)
    for it in items:
        assert it.seq[0] == arch.CLS_ID and it.seq[-1] == arch.SEP_ID
        assert all(it.seq[m] == arch.MASK_ID for m in it.markers)
    assert [it.qtype for it in items] == [0, 2] and [len(it.markers) for it in items] == [2, 2]


def test_question_items_are_cut_to_the_maximum_length():
    rng = np.random.default_rng(0)
    items = workloads.system_one_request(rng, 2000, [("choice", [60, 5], 8), ("noul", 30)])
    for it in items:
        assert len(it.seq) == arch.MAX_LEN and it.seq[-1] == arch.SEP_ID
        assert all(m < arch.MAX_LEN and it.seq[m] == arch.MASK_ID for m in it.markers)
    # options are cut to 48 tokens: the second marker follows the first by 49
    assert items[0].markers[1] - items[0].markers[0] == 49


def test_request_stream_is_seeded():
    a = workloads.request_stream(16, 4)
    b = workloads.request_stream(16, 4)
    assert [[it.seq for it in r] for r in a] == [[it.seq for it in r] for r in b]
    assert all(1 <= len(r) <= 16 for r in a)


def test_greedy_assignment_partitions_and_balances():
    reqs = workloads.request_stream(200, 4)
    for world in (1, 2, 3, 8):
        parts = workloads.assign_requests(reqs, world)
        assert sorted(i for p in parts for i in p) == list(range(len(reqs)))
        cost = [sum(len(it.seq) for i in p for it in reqs[i]) for p in parts]
        biggest = max(sum(len(it.seq) for it in r) for r in reqs)
        assert max(cost) - min(cost) <= biggest


def test_packing_respects_the_budget_and_keeps_order():
    reqs = workloads.request_stream(64, 4)
    fws = workloads.pack_stream(reqs, 16384)
    seen = [ids for _, idl in fws for ids in idl]
    assert seen == [(r, i) for r, items in enumerate(reqs) for i in range(len(items))]
    for items, _ in fws:
        assert max(len(it.seq) for it in items) * len(items) <= 16384
        req = batching.build_batch(items, list(range(len(items))))
        assert req.n * req.l <= 16384


def test_long_state_has_a_32_token_head():
    req = workloads.long_state()
    ids = req.ids.reshape(req.n, req.l)
    assert req.n == 8 and req.l == 512 and workloads.real_tokens(req) == 8 * 512
    for b in range(req.n):
        assert ids[b, 32] == arch.SEP_ID
        assert np.all(req.mpos.reshape(req.n, req.k)[b] > 32)


def test_assignment_by_cost_partitions_and_balances():
    rng = np.random.default_rng(3)
    costs = [int(c) for c in rng.integers(20, 1100, 1024)]
    for world in (1, 2, 4, 8):
        parts = workloads.assign_by_cost(costs, world)
        assert sorted(i for p in parts for i in p) == list(range(len(costs)))
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(costs)
        for p in parts:
            assert p == sorted(p)   # each GPU keeps dispatch order
