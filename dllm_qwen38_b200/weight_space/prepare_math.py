"""Hard MATH-train integer-answer subset from local parquet files (the reference's
`tools/weight-space/prepare_math.py:21-62` role; no download: the parquet files are given).

    python -m dllm_qwen38_b200.weight_space.prepare_math --source DIR --output OUT [--size 32]

DIR holds the train parquet files (any depth; `problem`, `level`, `solution` columns). Kept:
Level 4 and Level 5 problems whose solution has exactly one \\boxed{} holding a plain integer;
duplicates (by problem hash) dropped; ordered by problem hash; the first `size` are `dev`, the
next `size` `validation`. Test splits are never read (files with "test" in the path are refused).
"""

from __future__ import annotations

import argparse
import json
import pathlib
import re

import pyarrow.parquet as pq

from .common import canonical, digest, write_new

_BOX_INT = re.compile(r"\\boxed\{\s*(-?\d[\d,]*)\s*\}")


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--source", required=True, type=pathlib.Path)
    p.add_argument("--output", required=True, type=pathlib.Path)
    p.add_argument("--size", type=int, default=32)
    a = p.parse_args(argv)
    if a.size < 1:
        raise ValueError("size must be positive")
    files = sorted(a.source.rglob("*.parquet"))
    if not files:
        raise ValueError("no parquet files")
    if any("test" in str(f.relative_to(a.source)).lower() for f in files):
        raise ValueError("test split files are not read")
    sources, cases, seen = [], [], set()
    for f in files:
        sources.append({"file": str(f.relative_to(a.source)), "sha256": digest(f)})
        subject = f.parent.name if f.parent != a.source else f.stem
        for row in pq.read_table(f).to_pylist():
            if row.get("level") not in ("Level 4", "Level 5"):
                continue
            boxed = _BOX_INT.findall(row["solution"])
            if len(boxed) != 1 or len(re.findall(r"\\boxed\s*\{", row["solution"])) != 1:
                continue
            key = canonical(row["problem"])
            if key in seen:
                continue
            seen.add(key)
            cases.append({"id": key[:20], "question": row["problem"], "answer": boxed[0].replace(",", ""),
                          "subject": row.get("type", subject), "level": row["level"]})
    cases.sort(key=lambda c: c["id"])
    if len(cases) < 2 * a.size:
        raise ValueError("not enough eligible problems")
    a.output.mkdir(parents=True, exist_ok=True)
    for split, part in (("dev", cases[: a.size]), ("validation", cases[a.size: 2 * a.size])):
        write_new(a.output / f"{split}.json", {
            "schema": "bdllm.ws.math-integer-mini/v1", "sources": sources, "split": split,
            "selection": "train only; level 4/5; one plain integer boxed answer; problem SHA-256 ascending",
            "cases": part})
    print(json.dumps({"eligible": len(cases), "size_per_split": a.size,
                      "qualification": "a selected development subset, not MATH accuracy"}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
