"""Digests, canonical hashing and exclusive JSON writes shared by the weight-space tools
(the reference's `tools/weight-space/bench.py:21-36` helpers, same roles)."""

from __future__ import annotations

import hashlib
import json
import pathlib

CHUNK = 16 << 20


def digest(path) -> str:
    """SHA-256 of a file's bytes, streamed."""
    h = hashlib.sha256()
    with pathlib.Path(path).open("rb") as f:
        while True:
            b = f.read(CHUNK)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def digest_tree(path) -> str:
    """SHA-256 over a file, or over a directory's regular files (sorted relative names and their
    digests), so a model directory has one identity."""
    p = pathlib.Path(path)
    if p.is_file():
        return digest(p)
    h = hashlib.sha256()
    for f in sorted(x for x in p.rglob("*") if x.is_file()):
        h.update(str(f.relative_to(p)).encode() + b"\0" + digest(f).encode() + b"\n")
    return h.hexdigest()


def canonical(value) -> str:
    """SHA-256 of the sorted-key JSON encoding of a value."""
    return hashlib.sha256(json.dumps(value, sort_keys=True).encode()).hexdigest()


def write_new(path, value) -> None:
    """Write JSON to a path that must not exist yet."""
    with pathlib.Path(path).open("x") as f:
        json.dump(value, f, ensure_ascii=False, indent=2)
        f.write("\n")


def read_jsonl(path) -> list:
    p = pathlib.Path(path)
    if not p.exists():
        return []
    return [json.loads(line) for line in p.read_text().splitlines() if line.strip()]
