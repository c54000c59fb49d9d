"""Lexical audit of dev vs validation splits (the reference's `tools/weight-space/split_audit.py:13-83`
role). Every cross-split question pair is compared under a fixed profile:

  normalised   NFKC, casefold, whitespace collapsed
  masked       every number replaced by NUMBER
  shingles     5-token windows over word / punctuation tokens of the masked text

A pair is flagged when the normalised texts are equal, the masked texts are equal, or the shingle
Jaccard similarity is >= 0.80. The report carries ids and scores only, never question text.

    python -m dllm_qwen38_b200.weight_space.split_audit --dev dev.json --validation val.json --output A.json
"""

from __future__ import annotations

import argparse
import hashlib
import json
import pathlib
import re
import unicodedata

PROFILE = "nfkc-casefold-numbermask-shingle5-jaccard0.80/v1"
JACCARD = 0.80
_NUM = re.compile(r"\d+(?:\.\d+)?")
_TOK = re.compile(r"\w+|[^\w\s]")


def _normalise(text: str) -> str:
    return " ".join(unicodedata.normalize("NFKC", text).casefold().split())


def fingerprint(text: str):
    norm = _normalise(text)
    masked = _NUM.sub("NUMBER", norm)
    toks = _TOK.findall(masked)
    shingles = frozenset(tuple(toks[i:i + 5]) for i in range(len(toks) - 4))
    return norm, masked, shingles


def pair_flags(a, b):
    """(flags, jaccard) for two fingerprints."""
    union = len(a[2] | b[2])
    jac = len(a[2] & b[2]) / union if union else 0.0
    flags = []
    if a[0] == b[0]:
        flags.append("normalised_exact")
    if a[1] == b[1]:
        flags.append("number_masked_exact")
    if jac >= JACCARD:
        flags.append("shingle5_jaccard_ge_0.80")
    return flags, jac


def _load(path, role: str, index: int):
    raw = pathlib.Path(path).read_bytes()
    doc = json.loads(raw)
    cases = doc.get("cases") or []
    if not cases or len({c["id"] for c in cases}) != len(cases):
        raise ValueError(f"{path}: empty split or duplicate case ids")
    if any(not isinstance(c.get("question"), str) or not c["question"].strip() for c in cases):
        raise ValueError(f"{path}: a case without a question")
    if doc.get("split") != role:
        raise ValueError(f"{path}: split label {doc.get('split')!r} is not {role!r}")
    meta = {"file": pathlib.Path(path).name, "sha256": hashlib.sha256(raw).hexdigest(), "split": role,
            "index": index, "n": len(cases)}
    return [(index, c["id"], fingerprint(c["question"])) for c in cases], meta


def audit(dev_paths, validation_paths) -> dict:
    metas, groups = [], []
    for role, paths in (("dev", dev_paths), ("validation", validation_paths)):
        rows = []
        for i, p in enumerate(paths):
            r, m = _load(p, role, i)
            rows += r
            metas.append(m)
        groups.append(rows)
    flagged, best, count = [], 0.0, 0
    for di, did, df in groups[0]:
        for vi, vid, vf in groups[1]:
            count += 1
            flags, jac = pair_flags(df, vf)
            best = max(best, jac)
            if flags:
                flagged.append({"dev_input": di, "dev_id": did, "validation_input": vi, "validation_id": vid,
                                "reasons": flags, "jaccard": jac})
    return {"profile": PROFILE, "inputs": metas, "cross_split_pair_count": count,
            "flagged_pair_count": len(flagged), "flagged_pairs": flagged,
            "maximum_shingle5_jaccard": best,
            "limitations": ["a fixed lexical heuristic: not semantic equivalence, not a contamination proof",
                            "only the given files are compared", "the report authorises no split change"]}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--dev", nargs="+", required=True)
    p.add_argument("--validation", nargs="+", required=True)
    p.add_argument("--output", required=True)
    a = p.parse_args(argv)
    res = audit(a.dev, a.validation)
    with open(a.output, "x") as f:
        json.dump(res, f, indent=2)
        f.write("\n")
    print(json.dumps({k: res[k] for k in ("profile", "cross_split_pair_count", "flagged_pair_count")}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
