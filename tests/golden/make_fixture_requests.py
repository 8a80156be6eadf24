"""Extracts the reference's golden fixtures for the tests.

Reads laya-rust ``tests/fixtures/*.json`` (recorded by the reference's
``golden`` command with ``--max-tokens 300``) and ``tests/scenarios.json``.

``fixture_requests.json``: per fixture the padded index arrays of each
forward (ids, att, mpos, mmask, qtype), the question ids of each row and the
request's question order -- the request layout, which does not depend on the
real checkpoint.

``fixture_outputs.json``: per fixture the request JSON (key order kept), each
forward's rows with the reference's recorded logits and act, and the answers
object the reference computed from them.  Logits and act come from the real
checkpoint, but the scoring that turns them into answers (score_row,
softmax_t, confidence, answer; main.rs:502-518, systemone.rs:200-296) does
not, so these pin the front end's scoring and number formatting.  Also the
scenario requests of scenarios.json.

Usage: python tests/golden/make_fixture_requests.py <reference-root>
"""
import glob
import json
import os
import sys


def main(ref_root: str) -> None:
    out = []
    for path in sorted(glob.glob(os.path.join(ref_root, "tests", "fixtures", "*.json"))):
        d = json.load(open(path))
        fws = []
        for fw in d["forwards"]:
            fws.append({key: fw[key] for key in ("n", "l", "k", "ids", "att", "mpos", "mmask", "qtype")}
                       | {"rows": [r["id"] for r in fw["rows"]],
                          "markers": [r["markers"] for r in fw["rows"]]})
        out.append({"name": d["name"], "max_tokens": 300,
                    "question_order": list(d["request"]["questions"].keys()),
                    "forwards": fws})
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fixture_requests.json")
    with open(dst, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(dst, len(out), "fixtures")

    outs = []
    for path in sorted(glob.glob(os.path.join(ref_root, "tests", "fixtures", "*.json"))):
        text = open(path).read()
        d = json.loads(text)
        # the answers with every float kept as the literal text the reference
        # printed (serde_json / ryu), to pin the number formatting too
        raw = json.loads(text, parse_float=lambda t: {"f64": t})["answers"]
        outs.append({"name": d["name"], "request": d["request"],
                     "forwards": [{"rows": fw["rows"], "k": fw["k"], "logits": fw["logits"], "act": fw["act"]}
                                  for fw in d["forwards"]],
                     "answers": d["answers"], "answers_literal": raw})
    scen = json.load(open(os.path.join(ref_root, "tests", "scenarios.json")))
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fixture_outputs.json")
    with open(dst, "w") as f:
        json.dump({"fixtures": outs, "scenarios": [{"name": s["name"], "request": s["request"]}
                                                   for s in scen["scenarios"]]}, f, separators=(",", ":"))
    print(dst, len(outs), "fixtures,", len(scen["scenarios"]), "scenarios")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LAYA_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_fixture_requests.py REFERENCE_ROOT (or set LAYA_REFERENCE_ROOT)")
    main(root)
