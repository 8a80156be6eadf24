"""Seeded synthetic requests with the shapes of the benchmark configurations.

No public dataset is involved; the real tokenizer and checkpoint are absent, so
token ids are drawn uniformly from the non-special vocabulary [0, 50280) and
laid out the way the reference's sequence builder lays them out
(systemone.rs:156-198): [CLS] at 0, a [SEP] closing the question head, one
[MASK] per option marker, the state, and a closing [SEP]; padding id 0.
"""
from __future__ import annotations

import numpy as np

from . import arch
from .engine import Req

NON_SPECIAL = 50280


def _row(rng, r, n_markers, head=None):
    """One sequence of length r with n_markers [MASK] markers after the [SEP]
    closing a question head of `head` tokens (default r // 3)."""
    ids = rng.integers(0, NON_SPECIAL, r)
    ids[0] = arch.CLS_ID
    ids[r - 1] = arch.SEP_ID
    head = max(2, min(r // 3 if head is None else head, r - n_markers - 3))
    ids[head] = arch.SEP_ID
    pos = np.sort(rng.choice(np.arange(head + 1, r - 1), size=n_markers, replace=False))
    ids[pos] = arch.MASK_ID
    return ids, pos


def padded_batch(rng, lens, l, markers_lo=2, markers_hi=6, qtypes=None, head=None) -> Req:
    n = len(lens)
    nms = [int(rng.integers(markers_lo, markers_hi + 1)) for _ in lens]
    k = max(nms)
    ids = np.zeros((n, l), np.int64)
    att = np.zeros((n, l), np.int64)
    mpos = np.zeros((n, k), np.int64)
    mmask = np.zeros((n, k), np.int64)
    for b, (r, nm) in enumerate(zip(lens, nms)):
        row, pos = _row(rng, r, nm, head)
        ids[b, :r] = row
        att[b, :r] = 1
        mpos[b, :nm] = pos
        mmask[b, :nm] = 1
    qtype = np.asarray(qtypes if qtypes is not None else rng.integers(0, 3, n), np.int64)
    return Req(n, l, k, ids, att, mpos, mmask, qtype)


def forward_16k(seed: int = 0) -> Req:
    """Config 2: the default --max-tokens 16384 budget as 128 sequences x 128
    padded tokens, real lengths uniform in [24, 128]."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(24, 129, 128)
    return padded_batch(rng, lens, 128)


def long_state(seed: int = 3) -> Req:
    """Config 3: 8 sequences at the maximum position length (512), i.e. two
    requests of 4 choice questions: a 32-token question head, 3 criteria
    markers after it, the state filling the rest."""
    rng = np.random.default_rng(seed)
    return padded_batch(rng, [512] * 8, 512, markers_lo=3, markers_hi=3, qtypes=[0] * 8, head=32)


def layer_batch(seed: int = 1) -> Req:
    """Config 1 (one encoder layer in isolation): 32 sequences padded to 256,
    real lengths uniform in [16, 256]."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(16, 257, 32)
    return padded_batch(rng, lens, 256)


# ---- System One requests at the token level -----------------------------------------
# The real tokenizer is not available, so a word is one token drawn from the
# non-special vocabulary; the sequence layout is the reference's
# (systemone.rs:156-198): [CLS] head [SEP] ([MASK] option)* [SEP] state [SEP],
# options cut to 48 tokens, the whole sequence to 512.

NOUL_FALSE_TOKENS = 9   # " false: no, the statement does not hold"
NOUL_TRUE_TOKENS = 7    # " true: yes, the statement holds"


def _words(rng, n):
    return list(rng.integers(0, NON_SPECIAL, int(n)))


def question_item(rng, state, qtype, instr_words, options):
    """One question -> Item(seq, markers, qtype) (systemone.rs:156-198)."""
    from .batching import Item
    head = _words(rng, 3 + instr_words)              # "<type> question: <instructions>"
    ids = [arch.CLS_ID] + head + [arch.SEP_ID]
    markers = []
    for opt in options:
        markers.append(len(ids))
        ids += [arch.MASK_ID] + opt[:48]
    ids.append(arch.SEP_ID)
    room = max(0, arch.MAX_LEN - (len(ids) + 1))
    ids += state[:room]
    ids.append(arch.SEP_ID)
    ids = ids[:arch.MAX_LEN]
    markers = [m for m in markers if m < arch.MAX_LEN]
    return Item(ids, markers, qtype)


def system_one_request(rng, state_words, questions):
    """questions: list of ("choice", criteria_word_counts, instr_words) or
    ("noul", instr_words)."""
    state = _words(rng, state_words)
    items = []
    for q in questions:
        if q[0] == "choice":
            opts = [_words(rng, c) for c in q[1]]
            items.append(question_item(rng, state, 0, q[2], opts))
        else:
            opts = [_words(rng, NOUL_FALSE_TOKENS), _words(rng, NOUL_TRUE_TOKENS)]
            items.append(question_item(rng, state, 2, q[1], opts))
    return items


def single_request(seed: int = 0):
    """Config 0: a 48-word state, one choice question with 2 criteria of 6
    words, one noul question with 12-word instructions."""
    rng = np.random.default_rng(seed)
    return system_one_request(rng, 48, [("choice", [6, 6], 8), ("noul", 12)])


def request_stream(n_requests: int = 4096, seed: int = 4):
    """Config 4: per request, state length lognormal (median 96 tokens,
    sigma 0.8, capped at 1024), 1..16 questions, choice (2..6 criteria of
    3..8 tokens) and noul 1:1, instructions 8..16 tokens."""
    rng = np.random.default_rng(seed)
    reqs = []
    for _ in range(n_requests):
        state = int(min(1024, round(float(rng.lognormal(np.log(96.0), 0.8)))))
        qs = []
        for _ in range(int(rng.integers(1, 17))):
            instr = int(rng.integers(8, 17))
            if rng.random() < 0.5:
                qs.append(("choice", list(rng.integers(3, 9, int(rng.integers(2, 7)))), instr))
            else:
                qs.append(("noul", instr))
        reqs.append(system_one_request(rng, state, qs))
    return reqs


def assign_requests(requests, world: int):
    """Greedy assignment of requests (in dispatch order) to `world` GPUs: each
    request goes to the GPU with the least padded-token cost so far, its cost
    being the sum of its sequence lengths.  Returns the request indices per GPU."""
    load = [0] * world
    out = [[] for _ in range(world)]
    for ri, items in enumerate(requests):
        g = min(range(world), key=lambda i: (load[i], i))
        out[g].append(ri)
        load[g] += sum(len(it.seq) for it in items)
    return out


def assign_by_cost(costs, world: int):
    """The same greedy rule over plain per-request token costs (in dispatch
    order, ties to the lowest rank): the request indices per GPU."""
    load = [0] * world
    out = [[] for _ in range(world)]
    for ri, c in enumerate(costs):
        g = min(range(world), key=lambda i: (load[i], i))
        out[g].append(ri)
        load[g] += c
    return out


def pack_stream(requests, max_tokens: int = 16384):
    """Cross-request packing in dispatch order: items join the current forward
    while max_len * count stays within the budget (the budget rule of
    main.rs:448-468, applied across requests).  Returns [(items, [(request,
    item index)])] per forward."""
    forwards, cur, cur_ids, cur_max = [], [], [], 0
    for ri, items in enumerate(requests):
        for ii, it in enumerate(items):
            ln = len(it.seq)
            if cur and max(cur_max, ln) * (len(cur) + 1) > max_tokens:
                forwards.append((cur, cur_ids))
                cur, cur_ids, cur_max = [], [], 0
            cur.append(it)
            cur_ids.append((ri, ii))
            cur_max = max(cur_max, ln)
    if cur:
        forwards.append((cur, cur_ids))
    return forwards


# ---- System One requests as JSON text (through the C++ front end) ------------------
# Words are the letter-only entries of the model's tokenizer vocabulary (a
# space-prefixed entry "Gword" stands for " word"), drawn uniformly, so the
# text tokenizes to about one token per word as real text does with a real
# vocabulary.

def vocab_words(tokenizer_json: str) -> list[str]:
    import json as _json
    from .tokgen import bytes_to_unicode
    inv = {c: b for b, c in bytes_to_unicode().items()}
    words = []
    for tok in _json.loads(tokenizer_json)["model"]["vocab"]:
        try:
            text = bytes(inv[c] for c in tok).decode("ascii")
        except (KeyError, UnicodeDecodeError):
            continue
        if text.startswith(" ") and len(text) > 2 and text[1:].isalpha():
            words.append(text[1:])
    return sorted(set(words))


def _text(rng, words, n) -> str:
    return " ".join(words[int(i)] for i in rng.integers(0, len(words), int(n)))


def random_questions(rng) -> list:
    """Config 4's question mix: 1..16 questions, choice (2..6 criteria of 3..8
    words) and noul 1:1, instructions 8..16 words."""
    qs = []
    for _ in range(int(rng.integers(1, 17))):
        instr = int(rng.integers(8, 17))
        if rng.random() < 0.5:
            qs.append(("choice", [int(c) for c in rng.integers(3, 9, int(rng.integers(2, 7)))], instr))
        else:
            qs.append(("noul", instr))
    return qs


def system_one_request_json(rng, words, state_words, questions) -> dict:
    """A request object as the reference's API takes it (systemone.rs:74-118):
    {"state": text, "questions": {id: {"type", "instructions", "criteria"}}}."""
    qs = {}
    for i, q in enumerate(questions):
        if q[0] == "choice":
            crit = {}
            for j, c in enumerate(q[1]):
                crit[f"{words[int(rng.integers(0, len(words)))]}_{j}"] = _text(rng, words, max(1, c - 1))
            qs[f"q{i}"] = {"type": "choice", "instructions": _text(rng, words, q[2]), "criteria": crit}
        else:
            qs[f"q{i}"] = {"type": "noul", "instructions": _text(rng, words, q[1])}
    return {"state": _text(rng, words, state_words), "questions": qs}


def single_request_json(words, seed: int = 0) -> dict:
    """Config 0 as request JSON: a 48-word state, a choice question with 2
    criteria of 6 words, a noul question with 12-word instructions."""
    rng = np.random.default_rng(seed)
    return system_one_request_json(rng, words, 48, [("choice", [6, 6], 8), ("noul", 12)])


def request_stream_json(words, n_requests: int = 4096, seed: int = 4) -> list[dict]:
    """Config 4 as request JSON: state length lognormal (median 96 words,
    sigma 0.8, capped at 1024), questions as random_questions."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_requests):
        state = int(min(1024, round(float(rng.lognormal(np.log(96.0), 0.8)))))
        out.append(system_one_request_json(rng, words, max(1, state), random_questions(rng)))
    return out


def real_tokens(req: Req) -> int:
    return int((req.att != 0).sum())


def padded_tokens(req: Req) -> int:
    return req.n * req.l


def gemm_flops(req: Req) -> float:
    """Algorithmic GEMM FLOPs of one forward on real tokens (scorer included)."""
    R = real_tokens(req)
    p_enc = 28 * (1024 * 3072 + 1024 * 1024 + 1024 * 5248 + 2624 * 1024)
    p_head = 2 * (3072 * 1024 + 1024 * 1024 + 2 * 1024 * 4096)
    return 2.0 * R * (p_enc + p_head) + 2.0 * req.n * req.k * 1024 * 1024


def attention_flops(req: Req) -> float:
    """4*H per visible (query, key) pair: 10 global + 18 windowed encoder
    layers and 2 global head layers, real tokens only."""
    lens = (req.att.reshape(req.n, req.l) != 0).sum(1)
    g = float((lens.astype(np.float64) ** 2).sum())
    band = 0.0
    for r in lens:
        i = np.arange(r)
        band += float((np.minimum(i + 64, r - 1) - np.maximum(i - 64, 0) + 1).sum())
    return 4.0 * 1024 * (10 * g + 18 * band + 2 * g)
