"""TEST INFRASTRUCTURE ONLY: a pure-Python restatement of the laya-rust
request front end, the checker for the C++ front end in
laya_rust_b200/csrc/frontend.cpp.  Nothing in the product imports it.

What it restates (paths inside the zerodegress/laya-rust project):
  - src/tokenizer.rs:16-37     byte -> unicode map of byte-level BPE
  - src/tokenizer.rs:51-116    pre-tokenisation (contractions, letter /
                               number / other runs with an optional leading
                               space, whitespace runs)
  - src/tokenizer.rs:120-170   tokenizer.json loading (vocab, merge ranks,
                               added tokens sorted by length)
  - src/tokenizer.rs:172-265   BPE by merge rank, chunk encoding, added-token
                               splitting with lstrip
  - src/systemone.rs:30-296    request parsing, option rendering, sequence
                               layout with the head budget, temperatures,
                               softmax, confidence, answer objects
  - src/main.rs:387-549        plan_items, group_by_budget, build_batch,
                               score_row, run_all
  - serde_json / ryu           number and string formatting of serialised
                               values (ryu's shortest digits with its
                               "pretty" layout; compact separators)

Character classes: letters are Unicode general categories L* and Nl (Rust's
`is_alphabetic` also includes the Other_Alphabetic marks, which Python's
unicodedata does not list; both implementations here use the same tables),
numbers are categories N*, whitespace is the White_Space property.

f32 arithmetic follows the reference: numpy float32 scalars for + - * /,
glibc expf / logf through ctypes for exp and ln.

Parity status: the real tokenizer.json is absent, so real-vocabulary ids are
unpinned; the sequence layout is pinned by the reference's fixtures
(tests/fixtures/*.json, index arrays) where the token counts allow.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import json
import math
import unicodedata

import numpy as np

MAX_LEN = 512          # systemone.rs:4
HEAD_MAX_LEN = 192     # systemone.rs:5
CONTRACTIONS = ["'s", "'t", "'re", "'ve", "'m", "'ll", "'d"]   # tokenizer.rs:49

_libm = ctypes.CDLL(ctypes.util.find_library("m"))
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
_libm.logf.restype = ctypes.c_float
_libm.logf.argtypes = [ctypes.c_float]
F32 = np.float32


def expf(x) -> np.float32:
    return F32(_libm.expf(float(x)))


def logf(x) -> np.float32:
    return F32(_libm.logf(float(x)))


# ---- character classes ----------------------------------------------------------
WHITE_SPACE = set([0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000]
                  + list(range(0x2000, 0x200B)))


def is_letter(c: str) -> bool:
    cat = unicodedata.category(c)
    return cat[0] == "L" or cat == "Nl"


def is_number(c: str) -> bool:
    return unicodedata.category(c)[0] == "N"


def is_space(c: str) -> bool:
    return ord(c) in WHITE_SPACE


def bytes_to_unicode() -> dict[int, str]:
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    out = {b: chr(b) for b in keep}
    n = 0
    for b in range(256):
        if b not in out:
            out[b] = chr(256 + n)
            n += 1
    return out


def pre_tokenize(text: str) -> list[str]:
    """tokenizer.rs:51-116."""
    ch = list(text)
    out = []
    i = 0
    n = len(ch)
    while i < n:
        lower = "".join(ch[i:i + 3]).lower()
        matched = None
        for c in CONTRACTIONS:
            if lower.startswith(c):
                matched = len(c)
                break
        if matched is not None:
            out.append("".join(ch[i:i + matched]))
            i += matched
            continue
        j = i + 1 if ch[i] == " " else i
        if j < n and is_letter(ch[j]):
            k = j
            while k < n and is_letter(ch[k]):
                k += 1
            out.append("".join(ch[i:k]))
            i = k
            continue
        if j < n and is_number(ch[j]):
            k = j
            while k < n and is_number(ch[k]):
                k += 1
            out.append("".join(ch[i:k]))
            i = k
            continue
        other = lambda c: not is_space(c) and not is_letter(c) and not is_number(c)
        if j < n and other(ch[j]):
            k = j
            while k < n and other(ch[k]):
                k += 1
            out.append("".join(ch[i:k]))
            i = k
            continue
        if is_space(ch[i]):
            k = i
            while k < n and is_space(ch[k]):
                k += 1
            if k < n and k - i > 1:
                k -= 1
            out.append("".join(ch[i:k]))
            i = k
            continue
        out.append(ch[i])
        i += 1
    return out


class Tokenizer:
    """tokenizer.rs:120-265."""

    def __init__(self, text: str):
        v = json.loads(text)
        self.vocab = dict(v["model"]["vocab"])
        self.ranks = {}
        for i, m in enumerate(v["model"]["merges"]):
            pair = f"{m[0]} {m[1]}" if isinstance(m, list) else m
            self.ranks[pair] = i
        added = [(a["content"], int(a["id"]), bool(a.get("lstrip", False))) for a in v["added_tokens"]]
        # stable sort by byte length, longest first (tokenizer.rs:147)
        self.added = sorted(added, key=lambda a: -len(a[0].encode("utf-8")))

        def spec(name):
            for a in v["added_tokens"]:
                if a["content"] == name:
                    return int(a["id"])
            raise KeyError(name)
        self.cls, self.sep, self.mask = spec("[CLS]"), spec("[SEP]"), spec("[MASK]")
        self.pad, self.unk = spec("[PAD]"), spec("[UNK]")
        self.bmap = bytes_to_unicode()

    def bpe(self, word: str) -> list[str]:
        syms = list(word)
        if len(syms) < 2:
            return syms
        while True:
            best = None
            for i in range(len(syms) - 1):
                r = self.ranks.get(f"{syms[i]} {syms[i + 1]}")
                if r is not None and (best is None or r < best[0]):
                    best = (r, i)
            if best is None:
                break
            at = best[1]
            a, b = syms[at], syms[at + 1]
            nxt = []
            i = 0
            while i < len(syms):
                if i + 1 < len(syms) and syms[i] == a and syms[i + 1] == b:
                    nxt.append(a + b)
                    i += 2
                else:
                    nxt.append(syms[i])
                    i += 1
            syms = nxt
            if len(syms) == 1:
                break
        return syms

    def encode_chunk(self, text: str, out: list[int]) -> None:
        for piece in pre_tokenize(text):
            mapped = "".join(self.bmap[b] for b in piece.encode("utf-8"))
            for s in self.bpe(mapped):
                out.append(self.vocab.get(s, self.unk))

    def encode(self, text: str, add_special_tokens: bool) -> list[int]:
        ch = list(text)
        ids = []
        buf = []
        i = 0
        while i < len(ch):
            hit = None
            for content, tid, lstrip in self.added:
                n = len(content)
                if n > 0 and i + n <= len(ch) and "".join(ch[i:i + n]) == content:
                    hit = (tid, lstrip, n)
                    break
            if hit is not None:
                tid, lstrip, n = hit
                if lstrip:
                    while buf and is_space(buf[-1]):
                        buf.pop()
                self.encode_chunk("".join(buf), ids)
                buf = []
                ids.append(tid)
                i += n
            else:
                buf.append(ch[i])
                i += 1
        self.encode_chunk("".join(buf), ids)
        if add_special_tokens:
            return [self.cls] + ids + [self.sep]
        return ids


# ---- serde_json-compatible formatting ----------------------------------------------
def fmt_f64(x: float) -> str:
    """ryu's shortest digits in its layout (as serde_json prints an f64)."""
    if x == 0.0:
        return "-0.0" if math.copysign(1.0, x) < 0 else "0.0"
    s = repr(abs(float(x)))
    mant, _, exp = s.partition("e")
    e = int(exp) if exp else 0
    if "." in mant:
        ip, fp = mant.split(".")
    else:
        ip, fp = mant, ""
    digits = (ip + fp).lstrip("0")
    lead = len(ip.lstrip("0")) if ip.strip("0") else -(len(fp) - len(fp.lstrip("0")))
    # decimal exponent of the position after the first digit
    kk = lead + e
    digits = digits.rstrip("0") or "0"
    length = len(digits)
    k = kk - length
    sign = "-" if x < 0 else ""
    if 0 <= k and kk <= 16:
        out = digits + "0" * k + ".0"
    elif 0 < kk <= 16:
        out = digits[:kk] + "." + digits[kk:]
    elif -5 < kk <= 0:
        out = "0." + "0" * (-kk) + digits
    elif length == 1:
        out = digits + "e" + str(kk - 1)
    else:
        out = digits[0] + "." + digits[1:] + "e" + str(kk - 1)
    return sign + out


def fmt_num(v) -> str:
    if isinstance(v, bool):
        raise TypeError
    if isinstance(v, int):
        return str(v)
    return fmt_f64(v)


def json_str(s: str) -> str:
    out = ['"']
    for c in s:
        o = ord(c)
        if c == '"':
            out.append('\\"')
        elif c == "\\":
            out.append("\\\\")
        elif c == "\n":
            out.append("\\n")
        elif c == "\r":
            out.append("\\r")
        elif c == "\t":
            out.append("\\t")
        elif c == "\b":
            out.append("\\b")
        elif c == "\f":
            out.append("\\f")
        elif o < 0x20:
            out.append("\\u%04x" % o)
        else:
            out.append(c)
    out.append('"')
    return "".join(out)


def to_json(v) -> str:
    """serde_json::to_string (compact)."""
    if v is None:
        return "null"
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, (int, float)):
        return fmt_num(v)
    if isinstance(v, str):
        return json_str(v)
    if isinstance(v, list):
        return "[" + ",".join(to_json(x) for x in v) + "]"
    return "{" + ",".join(json_str(k) + ":" + to_json(x) for k, x in v.items()) + "}"


def loads(text: str):
    """serde_json with preserve_order: objects keep key order; integer
    literals that fit i64/u64 stay integers, everything else is f64."""
    def num_int(s):
        v = int(s)
        if v == 0 and s.startswith("-"):
            return -0.0          # "-0" is the float -0.0
        return v if -(1 << 63) <= v < (1 << 64) else float(v)
    return json.loads(text, parse_int=num_int)


def py_str(v) -> str:
    """systemone.rs:48-69."""
    if isinstance(v, str):
        return v
    if v is None:
        return "None"
    if isinstance(v, bool):
        return "True" if v else "False"
    if isinstance(v, (int, float)):
        return fmt_num(v)
    if isinstance(v, list):
        return "[" + ", ".join(py_str(x) for x in v) + "]"
    return "{" + ", ".join(f"'{k}': {py_str(x)}" for k, x in v.items()) + "}"


# ---- System One (systemone.rs) ------------------------------------------------------
class Question:
    def __init__(self, qid, ty, instructions, crit):
        self.id, self.ty, self.instructions, self.crit = qid, ty, instructions, crit
        self.qtype = {"choice": 0, "score": 1}.get(ty, 2)


class RequestError(ValueError):
    pass


def parse_request(req) -> tuple[object, list[Question]]:
    """systemone.rs:74-118."""
    state = req.get("state") if isinstance(req, dict) else None
    qs = req.get("questions") if isinstance(req, dict) else None
    if not isinstance(qs, dict):
        raise RequestError('missing "questions"')
    out = []
    for qid, q in qs.items():
        ty = q.get("type") if isinstance(q, dict) else None
        if not isinstance(ty, str):
            raise RequestError(f'question {qid}: missing "type"')
        if ty not in ("choice", "score", "noul"):
            raise RequestError(f"question {qid}: bad type {ty}")
        ins = q.get("instructions")
        if isinstance(ins, str):
            instructions = ins
        elif ins is None:
            raise RequestError(f'question {qid}: missing "instructions"')
        else:
            instructions = to_json(ins)
        crit = q.get("criteria")
        if ty == "choice" and isinstance(crit, list):
            m = {}
            for c in crit:
                m[py_str(c)] = None
            crit = m
        out.append(Question(qid, ty, instructions, crit))
    return state, out


def render_options(q: Question) -> list[str]:
    """systemone.rs:120-154."""
    if q.ty == "choice":
        if isinstance(q.crit, dict):
            return [k if v is None else f"{k}: {py_str(v)}" for k, v in q.crit.items()]
        return []
    if q.ty == "score":
        if isinstance(q.crit, list):
            return [f"level {i}: {py_str(c)}" for i, c in enumerate(q.crit)]
        return []
    m = q.crit if isinstance(q.crit, dict) else None

    def get(k, d):
        if m is not None and m.get(k) is not None:
            return py_str(m[k])
        return d
    return [f"false: {get('false', 'no, the statement does not hold')}",
            f"true: {get('true', 'yes, the statement holds')}"]


def serialize_state(state) -> str:
    return state if isinstance(state, str) else to_json(state)


def build_sequence(tok: Tokenizer, state, q: Question) -> tuple[list[int], list[int]]:
    """systemone.rs:156-198."""
    opts = render_options(q)
    ins = q.instructions.replace("[MASK]", " ")
    head_ids = tok.encode(f"{q.ty} question: {ins}", False)
    opt_ids = []
    for o in opts:
        ids = tok.encode(" " + o.replace("[MASK]", " "), False)[:48]
        opt_ids.append([tok.mask] + ids)
    total = lambda: sum(len(o) for o in opt_ids)
    budget = HEAD_MAX_LEN - total()
    if budget < 16:
        per = max(4, (HEAD_MAX_LEN - 16) // max(1, len(opt_ids)))
        opt_ids = [o[:per] for o in opt_ids]
        budget = HEAD_MAX_LEN - total()
    keep = max(8, budget)
    ids = [tok.cls] + head_ids[:keep] + [tok.sep]
    markers = []
    for o in opt_ids:
        markers.append(len(ids))
        ids += o
    ids.append(tok.sep)
    room = max(0, MAX_LEN - (len(ids) + 1))
    st = tok.encode(serialize_state(state).replace("[MASK]", " "), False)
    ids += st[:room]
    ids.append(tok.sep)
    ids = ids[:MAX_LEN]
    markers = [m for m in markers if m < MAX_LEN]
    return ids, markers


class Calibration:
    def __init__(self, temperature=(1.0, 1.0, 1.0), by_options=()):
        self.temperature = [F32(t) for t in temperature]
        self.by_options = [(k, F32(v)) for k, v in by_options]


def temperature(qtype: int, k: int, cal: Calibration) -> np.float32:
    """systemone.rs:200-218."""
    size = "2" if k <= 2 else "3-5" if k <= 5 else "6-10" if k <= 10 else "11+"
    key = f"{['choice', 'score', 'noul'][min(qtype, 2)]}:{size}"
    for kk, v in cal.by_options:
        if kk == key:
            return v
    return cal.temperature[qtype]


def softmax_t(logits, t) -> list:
    """systemone.rs:220-226 in f32."""
    z = [F32(x) / F32(t) for x in logits]
    m = F32(np.finfo(np.float32).min)
    for x in z:
        m = max(m, x)
    e = [expf(x - m) for x in z]
    s = F32(0.0)
    for x in e:
        s = F32(s + x)
    return [F32(x / s) for x in e]


def confidence(p) -> np.float32:
    """systemone.rs:228-235."""
    k = len(p)
    if k < 2:
        return F32(1.0)
    ent = F32(0.0)
    for x in p:
        ent = F32(ent + F32(-x * logf(max(x, F32(1e-12)))))
    return max(F32(1.0) - ent / logf(F32(k)), F32(0.0))


def r4(x) -> np.float32:
    """systemone.rs:237-239: f32 round half away from zero."""
    y = F32(F32(x) * F32(10000.0))
    r = F32(math.floor(abs(float(y)) + 0.5))
    r = F32(math.copysign(float(r), float(y)))
    return F32(r / F32(10000.0))


def f32_json(x) -> float:
    """An f32 as serde_json stores it: widened to f64."""
    return float(np.float32(x))


def answer(q: Question, p, act_prob) -> dict:
    """systemone.rs:241-296."""
    conf = f32_json(r4(confidence(p)))
    ext = {"act_probability": f32_json(r4(act_prob))}
    if q.ty == "choice":
        keys = list(q.crit.keys()) if isinstance(q.crit, dict) else []
        best = 0
        for i in range(len(p)):
            if p[i] >= p[best]:
                best = i            # max_by keeps the last of equal maxima
        probs = {k: f32_json(r4(v)) for k, v in zip(keys, p)}
        return {"type": "choice", "choice": keys[best] if best < len(keys) else "",
                "probabilities": probs, "confidence": conf, "rl_agent": ext}
    if q.ty == "score":
        desc = q.crit if isinstance(q.crit, list) else []
        score = F32(0.0)
        for i, v in enumerate(p):
            score = F32(score + F32(F32(i) * v))
        return {"type": "score", "score": f32_json(r4(score)),
                "legend": {str(i): py_str(c) for i, c in enumerate(desc)},
                "probabilities": {str(i): f32_json(r4(v)) for i, v in enumerate(p)},
                "confidence": conf, "rl_agent": ext}
    return {"type": "noul", "noul": f32_json(r4(p[1] if len(p) > 1 else F32(0.0))), "rl_agent": ext}


# ---- planning, batching, scoring (main.rs:387-549) -----------------------------------
class Item:
    def __init__(self, qid, seq, markers, qtype):
        self.id, self.seq, self.markers, self.qtype = qid, seq, markers, qtype


def plan_items(tok: Tokenizer, state, questions) -> list[Item]:
    items = []
    for q in questions:
        seq, markers = build_sequence(tok, state, q)
        expect = len(render_options(q))
        if len(markers) != expect:
            raise RequestError(f"question {q.id}: {expect} options do not fit in head budget "
                               f"({len(markers)} markers)")
        items.append(Item(q.id, seq, markers, q.qtype))
    return items


def group_by_budget(items, max_tokens: int) -> list[list[int]]:
    order = sorted(range(len(items)), key=lambda i: len(items[i].seq))   # stable
    groups, cur, cur_max = [], [], 0
    for i in order:
        ln = len(items[i].seq)
        if cur and max(cur_max, ln) * (len(cur) + 1) > max_tokens:
            groups.append(cur)
            cur, cur_max = [], 0
        cur_max = max(cur_max, ln)
        cur.append(i)
    if cur:
        groups.append(cur)
    return groups


def build_batch(items, idxs):
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
    return n, l, k, ids, att, mpos, mmask, qtype


def score_row(logits, act, row, k, markers, qtype, cal):
    raw = [F32(x) for x in logits[row * k: row * k + markers]]
    probs = softmax_t(raw, temperature(qtype, markers, cal))
    a = [F32(act[row * 2]), F32(act[row * 2 + 1])]
    m = max(F32(np.finfo(np.float32).min), a[0], a[1])
    e0, e1 = expf(a[0] - m), expf(a[1] - m)
    return probs, F32(e0 / F32(e0 + e1))


def run_all(forward, tok: Tokenizer, request, max_tokens=16384, cal=None) -> dict:
    """main.rs:520-556: the response object; `forward(n, l, k, ids, att, mpos,
    mmask, qtype) -> (logits, act)`."""
    cal = cal or Calibration()
    state, questions = parse_request(request)
    items = plan_items(tok, state, questions)
    answers = {}
    tokens = 0
    for g in group_by_budget(items, max_tokens):
        tokens += sum(len(items[i].seq) for i in g)
        n, l, k, ids, att, mpos, mmask, qtype = build_batch(items, g)
        logits, act = forward(n, l, k, ids, att, mpos, mmask, qtype)
        for row, i in enumerate(g):
            it = items[i]
            probs, act_p = score_row(logits, act, row, k, len(it.markers), it.qtype, cal)
            answers[it.id] = answer(questions[i], probs, act_p)
    return {"model": "laya", "answers": answers, "usage": {"input_tokens": tokens, "output_tokens": 0}}
