"""The host side of the engine's plan, with no device (laya_plan_layout):
the request validation laya_forward applies (the reference asserts n, l,
k > 0 at graph.rs:93 and panics on out-of-range ids, markers and question
types, cpu/mod.rs:145-153, 372-398; here each is an error status), the
compaction of the real tokens, and the attention work split -- tiles that
pack whole consecutive sequences of at most 128 tokens, and flash items of
up to 128 query rows for longer sequences, longest first.  Every real row
must be a query row of exactly one tile or item: a row in none would keep
a stale context, a row in two would be written twice."""
import numpy as np
import pytest

from laya_rust_b200 import arch
from laya_rust_b200 import engine as E
from laya_rust_b200 import workloads

Q = 128   # query rows per attention tile / flash item


def req_of(lens, k=4, l=None, seed=0):
    rng = np.random.default_rng(seed)
    n = len(lens)
    l = l or max(lens)
    ids = np.zeros((n, l), np.int64)
    att = np.zeros((n, l), np.int64)
    mpos = np.zeros((n, k), np.int64)
    mmask = np.zeros((n, k), np.int64)
    for b, r in enumerate(lens):
        ids[b, :r] = rng.integers(0, 50280, r)
        att[b, :r] = 1
        m = min(k, r)
        mpos[b, :m] = np.sort(rng.choice(r, size=m, replace=False))
        mmask[b, :m] = 1
    return E.Req(n, l, k, ids, att, mpos, mmask, rng.integers(0, 3, n))


def check_layout(lens, rows, tiles, items):
    lens = np.asarray(lens)
    start = np.concatenate([[0], np.cumsum(lens)[:-1]])
    assert rows == int(lens.sum())
    seq_at = {int(s): b for b, s in enumerate(start)}
    ends = set(int(s + n) for s, n in zip(start, lens))
    cover = np.zeros(rows, np.int32)
    tile_of = {}
    for t, (r0, nr) in enumerate(tiles.tolist()):
        assert 0 < nr <= Q and r0 in seq_at and r0 + nr in ends, (r0, nr)
        b = seq_at[r0]
        while start[b] < r0 + nr:       # whole consecutive short sequences
            assert lens[b] <= Q
            tile_of[b] = t
            b += 1
            if b == len(lens):
                break
        cover[r0:r0 + nr] += 1
    prev = None
    for q0, qr, s0, sl in items.tolist():
        assert s0 in seq_at and lens[seq_at[s0]] == sl and sl > Q
        assert (q0 - s0) % Q == 0 and 0 <= q0 - s0 < sl and qr == min(Q, sl - (q0 - s0))
        cover[q0:q0 + qr] += 1
        if prev is not None:           # longest sequences first, ties in order
            assert prev[1] > sl or (prev[1] == sl and prev[0] <= s0)
        prev = (s0, sl)
    assert np.all(cover == 1), np.flatnonzero(cover != 1)[:8]
    # greedy packing: a short sequence opens a new tile only when it does not
    # fit in the previous short sequence's tile
    for b in range(1, len(lens)):
        if lens[b] <= Q and lens[b - 1] <= Q and tile_of[b] != tile_of[b - 1]:
            r0, nr = tiles[tile_of[b - 1]]
            assert nr + lens[b] > Q, (b, nr, lens[b])


@pytest.mark.parametrize("seed", range(12))
def test_every_real_row_is_in_exactly_one_tile_or_item(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 40))
    if seed % 3 == 0:
        lens = rng.integers(1, 129, n)                     # short only
    elif seed % 3 == 1:
        lens = rng.integers(129, 513, n)                   # long only
    else:
        lens = np.where(rng.random(n) < 0.5, rng.integers(1, 129, n), rng.integers(129, 513, n))
    lens = [int(x) for x in lens]
    rows, tiles, items = E.plan_layout(req_of(lens, seed=seed))
    check_layout(lens, rows, tiles, items)


def test_edges_of_the_tile_and_item_sizes():
    for lens in ([128], [129], [1], [1] * 200, [127, 1, 128, 129, 256, 257, 512, 64, 64, 1], [512] * 3):
        rows, tiles, items = E.plan_layout(req_of(lens, k=1))
        check_layout(lens, rows, tiles, items)


def test_the_benchmark_batches():
    fw = workloads.forward_16k(0)
    lens = (fw.att.reshape(fw.n, fw.l) != 0).sum(1).tolist()
    rows, tiles, items = E.plan_layout(fw)
    check_layout(lens, rows, tiles, items)
    assert rows == 9872 and len(items) == 0 and len(tiles) == 104
    ls = workloads.long_state(3)
    lens = (ls.att.reshape(ls.n, ls.l) != 0).sum(1).tolist()
    rows, tiles, items = E.plan_layout(ls)
    check_layout(lens, rows, tiles, items)
    assert len(tiles) == 0 and len(items) == 8 * 4


def invalid(req, words):
    with pytest.raises(E.LayaError) as ei:
        E.plan_layout(req)
    assert ei.value.code == E.LAYA_E_INVALID and words in str(ei.value), str(ei.value)


def test_invalid_requests_get_the_forward_s_errors():
    good = lambda: req_of([10, 20], k=2)
    r = good()
    r.att[5] = 0                                   # a hole: row 0 keeps a real token after padding
    invalid(r, "att is not a prefix of ones")
    r = good()
    r.att[20:40] = 0                               # row 1 has no real token
    invalid(r, "row 1 has no real tokens")
    r = good()
    r.ids[3] = arch.NVOCAB
    invalid(r, "token id")
    r = good()
    r.qtype[1] = arch.QTYPES
    invalid(r, "qtype")
    r = good()
    r.mpos[1] = 15                                 # row 0 is 10 tokens long, padded to 20
    invalid(r, "points at padding")
    r = good()
    r.mpos[2] = 20
    invalid(r, "outside [0, 20)")
    r = good()
    invalid(E.Req(0, r.l, r.k, r.ids, r.att, r.mpos, r.mmask, r.qtype), "n, l, k > 0")
    # a marker switched off may sit on padding: its logit is -10000 anyway
    r = good()
    r.mpos[1], r.mmask[1] = 15, 0
    rows, tiles, items = E.plan_layout(r)
    assert rows == 30
