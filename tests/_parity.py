"""Comparison of engine outputs with the oracle's (the reference CPU backend
restated), shared by the GPU parity tests and written to the contract's
tolerance: logits and act within max-abs 2e-2 and |got - want| <= 2e-2 +
1e-2 |want|; masked markers exactly -10000; the same argmax over every row's
valid markers, strictly.  An argmax disagreement is reported with the
oracle's top-2 margin for that row."""
import numpy as np

ATOL, RTOL = 2e-2, 1e-2


def compare(n, k, mmask, got_logits, got_act, want_logits, want_act, name=""):
    """Returns (max |dlogit|, max |dact|, smallest oracle top-2 margin)."""
    mm = np.asarray(mmask).reshape(n, k) != 0
    gl = np.asarray(got_logits, np.float32).reshape(n, k)
    wl = np.asarray(want_logits, np.float32).reshape(n, k)
    ga = np.asarray(got_act, np.float32)
    wa = np.asarray(want_act, np.float32)
    assert np.all(gl[~mm] == -10000.0) and np.all(wl[~mm] == -10000.0), name
    for what, g, w in (("logits", gl[mm], wl[mm]), ("act", ga, wa)):
        err = np.abs(g - w)
        assert np.all(np.isfinite(g)), (name, what)
        assert err.max() <= ATOL, (name, what, float(err.max()))
        assert np.all(err <= ATOL + RTOL * np.abs(w)), (name, what, float((err - RTOL * np.abs(w)).max()))
    min_margin = float("inf")
    bad = []
    for b in range(n):
        v = np.flatnonzero(mm[b])
        if len(v) < 2:
            continue
        top = np.sort(wl[b, v])
        margin = float(top[-1] - top[-2])
        min_margin = min(min_margin, margin)
        if np.argmax(gl[b, v]) != np.argmax(wl[b, v]):
            bad.append((b, margin, gl[b, v].tolist(), wl[b, v].tolist()))
    assert not bad, (name, "argmax differs (row, oracle top-2 margin, got, want)", bad)
    return float(np.abs(gl[mm] - wl[mm]).max()), float(np.abs(ga - wa).max()), min_margin
