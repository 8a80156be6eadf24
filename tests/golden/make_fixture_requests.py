"""Extracts the request layout of the reference's golden fixtures.

Reads laya-rust ``tests/fixtures/*.json`` (recorded by the reference's ``golden``
command with ``--max-tokens 300``) and keeps only what does not depend on the
real checkpoint: per forward the padded index arrays (ids, att, mpos, mmask,
qtype), the question ids of each row, and the request's question order.  The
logits/act/answers in those files need the real weights and are dropped.

Usage: python tests/golden/make_fixture_requests.py <reference-root>
Writes tests/golden/fixture_requests.json.
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


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
