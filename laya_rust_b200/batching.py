"""Request packing around the engine call.

Restates the host side of laya-rust ``src/main.rs`` that feeds the hot path:
``group_by_budget`` (main.rs:448-468), ``build_batch`` (main.rs:470-500),
``score_row`` (main.rs:502-518) and ``run_all`` (main.rs:520-549), plus the
calibration helpers they call (systemone.rs:200-233).  An ``Item`` is one
tokenized question: its sequence ids, marker positions and question type.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .engine import Req


@dataclass
class Item:
    seq: list
    markers: list
    qtype: int
    id: str = ""


@dataclass
class Calibration:
    temperature: list = field(default_factory=lambda: [1.0, 1.0, 1.0])
    by_options: list = field(default_factory=list)   # [(key, value)], sorted by key


def group_by_budget(items: list[Item], max_tokens: int) -> list[list[int]]:
    """main.rs:448-468: stable sort by length, then greedy groups while
    max_len * (count + 1) <= max_tokens."""
    order = sorted(range(len(items)), key=lambda i: len(items[i].seq))
    groups, cur, cur_max = [], [], 0
    for i in order:
        ln = len(items[i].seq)
        new_max = max(cur_max, ln)
        if cur and new_max * (len(cur) + 1) > max_tokens:
            groups.append(cur)
            cur, cur_max = [], 0
        cur_max = max(cur_max, ln)
        cur.append(i)
    if cur:
        groups.append(cur)
    return groups


def build_batch(items: list[Item], idxs: list[int]) -> Req:
    """main.rs:470-500: pad with id 0 / att 0; markers left-aligned with mmask."""
    n = len(idxs)
    l = max(len(items[i].seq) for i in idxs)
    k = max(len(items[i].markers) for i in idxs)
    ids = np.zeros((n, l), np.int64)
    att = np.zeros((n, l), np.int64)
    mpos = np.zeros((n, k), np.int64)
    mmask = np.zeros((n, k), np.int64)
    qtype = np.zeros(n, np.int64)
    for r, i in enumerate(idxs):
        it = items[i]
        ids[r, :len(it.seq)] = it.seq
        att[r, :len(it.seq)] = 1
        mpos[r, :len(it.markers)] = it.markers
        mmask[r, :len(it.markers)] = 1
        qtype[r] = it.qtype
    return Req(n, l, k, ids, att, mpos, mmask, qtype)


def qname(q: int) -> str:
    return {0: "choice", 1: "score"}.get(q, "noul")


def temperature(qtype: int, k: int, cal: Calibration) -> float:
    """systemone.rs:200-216."""
    size = "2" if k <= 2 else "3-5" if k <= 5 else "6-10" if k <= 10 else "11+"
    key = f"{qname(qtype)}:{size}"
    for kk, v in cal.by_options:
        if kk == key:
            return float(np.float32(v))
    return float(np.float32(cal.temperature[qtype]))


def softmax_t(logits, t: float) -> np.ndarray:
    """systemone.rs:218-224 (f32)."""
    z = np.asarray(logits, np.float32) / np.float32(t)
    e = np.exp(z - z.max()).astype(np.float32)
    return (e / e.sum(dtype=np.float32)).astype(np.float32)


def score_row(logits: np.ndarray, act: np.ndarray, row: int, k: int, markers: int, qtype: int,
              cal: Calibration):
    """main.rs:502-518: calibrated option probabilities and the act probability."""
    raw = logits[row * k: row * k + markers]
    probs = softmax_t(raw, temperature(qtype, markers, cal))
    a = act[row * 2: row * 2 + 2].astype(np.float32)
    m = a.max()
    e0, e1 = np.exp(a[0] - m), np.exp(a[1] - m)
    return probs, float(e0 / (e0 + e1))


def run_all(engine, items: list[Item], max_tokens: int = 16384, cal: Calibration | None = None):
    """main.rs:520-549 without answer shaping: returns, per item, the calibrated
    probabilities and act probability, plus the executed batches."""
    cal = cal or Calibration()
    results = [None] * len(items)
    forwards = []
    for g in group_by_budget(items, max_tokens):
        req = build_batch(items, g)
        out = engine.forward(req)
        for row, i in enumerate(g):
            results[i] = score_row(out.logits, out.act, row, req.k, len(items[i].markers),
                                   items[i].qtype, cal)
        forwards.append((g, req, out))
    return results, forwards
