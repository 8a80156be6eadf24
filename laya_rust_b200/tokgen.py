"""Seeded synthetic byte-level BPE tokenizer in the HuggingFace
``tokenizer.json`` layout the reference loads (laya-rust src/tokenizer.rs:
120-170: ``model.vocab``, ``model.merges``, ``added_tokens`` with
``lstrip``).

The real ModernBERT ``tokenizer.json`` is not available, so the model files
carry this one instead, embedded under ``tokenizer.huggingface.json`` as the
reference's converter embeds the real one (src/convert.rs:188-223) and reads
it back (src/lib.rs:47-57).  Its merges are learned by plain BPE training on a
seeded corpus of pseudo-words (consonant-vowel syllables, capitalised and
space-prefixed forms, digits and punctuation), so encoding exercises every
path of the reference's algorithm: pre-tokenisation classes, multi-step merges
by rank, unknown-free byte fallback.  Special tokens have ModernBERT's ids:
[UNK] 50280, [CLS] 50281, [SEP] 50282, [PAD] 50283, [MASK] 50284 ([MASK] with
``lstrip``).  Ordinary ids are below 50280.
"""
from __future__ import annotations

import collections
import functools
import json

import numpy as np

SPECIALS = [("[UNK]", 50280, False), ("[CLS]", 50281, False), ("[SEP]", 50282, False),
            ("[PAD]", 50283, False), ("[MASK]", 50284, True)]


def bytes_to_unicode() -> dict[int, str]:
    """The byte -> printable character map of byte-level BPE
    (tokenizer.rs:16-37): printable Latin-1 bytes map to themselves, the
    other 68 bytes to U+0100 onwards in byte order."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    out = {b: chr(b) for b in keep}
    n = 0
    for b in range(256):
        if b not in out:
            out[b] = chr(256 + n)
            n += 1
    return out


# Common English words, so that English text (instructions, options, states)
# encodes to realistic lengths.
ENGLISH = """the of and to a in is it you that he was for on are with as his they be at one have this
from or had by hot word but what some we can out other were all there when up use your how said an
each she which do their time if will way about many then them write would like so these her long
make thing see him two has look more day could go come did number sound no most people my over know
water than call first who may down side been now find any new work part take get place made live
where after back little only round man year came show every good me give our under name very through
just form sentence great think say help low line differ turn cause much mean before move right boy
old too same tell does set three want air well also play small end put home read hand port large
spell add even land here must big high such follow act why ask men change went light kind off need
house picture try us again animal point mother world near build self earth father head stand own page
should country found answer school grow study still learn plant cover food sun four between state
keep eye never last let thought city tree cross farm hard start might story saw far sea draw left late
run while press close night real life few north open seem together next white children begin got walk
example ease paper group always music those both mark often letter until mile river car feet care
second book carry took science eat room friend began idea fish mountain stop once base hear horse cut
sure watch color face wood main enough plain girl usual young ready above ever red list though feel
talk bird soon body dog family direct pose leave song measure door product black short numeral class
wind question happen complete ship area half rock order fire south problem piece told knew pass since
top whole king space heard best hour better true during hundred five remember step early hold west
ground interest reach fast verb sing listen six table travel less morning ten simple several vowel
toward war lay against pattern slow center love person money serve appear road map rain rule govern
pull cold notice voice unit power town fine certain fly fall lead cry dark machine note wait plan
figure star box noun field rest correct able pound done beauty drive stood contain front teach week
final gave green oh quick develop ocean warm free minute strong special mind behind clear tail produce
fact street inch multiply nothing course stay wheel full force blue object decide surface deep moon
island foot system busy test record boat common gold possible plane stead dry wonder laugh thousand
ago ran check game shape equate miss brought heat snow tire bring yes distant fill east paint language
among customer ticket payment invoice refund account billing technical sales support urgent issue
error failed failing pending order delivery price upgrade team handle route message request status
""".split()


def _corpus(rng) -> collections.Counter:
    """Pre-tokenised pieces with frequencies: pseudo-words (Zipf-distributed),
    their space-prefixed and capitalised forms, common English words, numbers
    and punctuation."""
    onsets = ["", "b", "c", "d", "f", "g", "h", "j", "k", "l", "m", "n", "p", "r", "s", "t", "v", "w", "z",
              "st", "tr", "pl", "gr", "ch", "sh", "th", "br", "cl"]
    vowels = ["a", "e", "i", "o", "u", "ea", "ou", "ai", "y"]
    codas = ["", "", "n", "r", "s", "t", "l", "nd", "ng", "ck", "st", "m"]
    words = []
    seen = set()
    while len(words) < 1600:
        w = "".join(rng.choice(onsets) + rng.choice(vowels) + rng.choice(codas)
                    for _ in range(int(rng.integers(1, 4))))
        if w and w not in seen:
            seen.add(w)
            words.append(w)
    freq = 1.0 / np.arange(1, len(words) + 1) ** 1.05
    counts = rng.multinomial(60000, freq / freq.sum())
    c = collections.Counter()
    for w, k in zip(words, counts):
        if k == 0:
            continue
        c[" " + w] += int(k)
        c[w] += int(k) // 3 + 1
        c[" " + w.capitalize()] += int(k) // 4 + 1
    for w in ENGLISH:
        c[" " + w] += 200
        c[" " + w.capitalize()] += 40
        c[w.capitalize()] += 20
        c[w] += 20
    for d in range(200):
        c[" " + str(d)] += 20
        c[str(d)] += 10
    for p in [".", ",", "!", "?", ":", ";", "'", "\"", "(", ")", "[", "]", "{", "}", "-", "_", "/", "@",
              " -", " (", " \"", "\n", "\n\n", "  ", "'s", "'t", "'re", ":", "\":", "\",", "},", "],"]:
        c[p] += 50
    return c


def _pairs(sym):
    return [(sym[i], sym[i + 1]) for i in range(len(sym) - 1)]


def _train(pieces: collections.Counter, n_merges: int, bmap: dict[int, str]) -> list[tuple[str, str]]:
    """Plain BPE training: repeatedly merge the most frequent adjacent pair
    (ties: the larger pair string), with incremental pair counts."""
    words = [[tuple(bmap[b] for b in p.encode("utf-8")), f] for p, f in sorted(pieces.items())]
    counts = collections.Counter()
    where = collections.defaultdict(set)
    for wi, (sym, f) in enumerate(words):
        for pr in _pairs(sym):
            counts[pr] += f
            where[pr].add(wi)
    merges = []
    for _ in range(n_merges):
        if not counts:
            break
        best = max(counts.items(), key=lambda kv: (kv[1], kv[0]))[0]
        merges.append(best)
        a, b = best
        for wi in sorted(where.pop(best, ())):
            sym, f = words[wi]
            for pr in _pairs(sym):
                counts[pr] -= f
                if counts[pr] <= 0:
                    del counts[pr]
            out = []
            i = 0
            while i < len(sym):
                if i + 1 < len(sym) and sym[i] == a and sym[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(sym[i])
                    i += 1
            sym = tuple(out)
            words[wi][0] = sym
            for pr in _pairs(sym):
                counts[pr] += f
                where[pr].add(wi)
        counts.pop(best, None)
    return merges


@functools.lru_cache(maxsize=4)
def tokenizer_json(seed: int = 0, n_merges: int = 4000) -> str:
    """The tokenizer as a tokenizer.json string (deterministic for a seed)."""
    rng = np.random.default_rng(seed)
    bmap = bytes_to_unicode()
    merges = _train(_corpus(rng), n_merges, bmap)
    vocab = {}
    for b in range(256):
        vocab[bmap[b]] = len(vocab)
    for a, b in merges:
        if a + b not in vocab:
            vocab[a + b] = len(vocab)
    assert len(vocab) < 50280
    added = [{"id": i, "content": c, "single_word": False, "lstrip": ls, "rstrip": False,
              "normalized": False, "special": True} for c, i, ls in SPECIALS]
    doc = {"version": "1.0", "added_tokens": added,
           "model": {"type": "BPE", "vocab": vocab, "merges": [f"{a} {b}" for a, b in merges]}}
    return json.dumps(doc, ensure_ascii=False)
