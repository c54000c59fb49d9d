"""Projection edits on MLP down projections of a copy of a safetensors checkpoint (the
reference's `tools/weight-space/surgery.py:20-160` role, for this framework's safetensors files instead
of GGUF).

    python -m dllm_qwen38_b200.weight_space.surgery --source model.safetensors --source-sha256 H
           --output edited.safetensors --spec spec.json

spec.json: {"hypothesis": str, "edits": [{"tensor": "<prefix>layers.N.mlp.down_proj.weight",
            "direction": "direction-N.npy", "strength": s}]}  (paths relative to the spec)
For each edit, with d the unit direction over the projection's output (hidden) dimension:
    W <- W - s * d (d^T W),   0 <= s <= 1
which removes the fraction s of every column's component along d (s = 1 projects d out; s = 0 is
a true no-op that keeps the stored bytes). The source is copied to a new file first; only the
edited tensors' byte ranges are rewritten in the copy, and the run fails unless the source still
hashes to its declared digest and every byte outside the edited ranges is identical in both
files. A journal `<output>.edit.json` records the plan, per-edit statistics (values changed,
relative change, projection norm before / after) and the outcome, also on failure.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import mmap
import pathlib
import re
import shutil
import struct

import numpy as np
import torch

from .common import CHUNK, digest

_NAME = re.compile(r"(model\.language_model\.|model\.|text_model\.)?layers\.\d+\.mlp\.down_proj\.weight")
_DT = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}


def read_header(path) -> tuple[dict, int]:
    """(tensor table, byte offset of the data section)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        if n <= 0 or n > 100 << 20:
            raise ValueError("not a safetensors file")
        hdr = json.loads(f.read(n))
    hdr.pop("__metadata__", None)
    return hdr, 8 + n


def checksums(path, excluded) -> tuple[str, str]:
    """(digest of the whole file, digest of the bytes outside the sorted `excluded` ranges)."""
    whole, outside = hashlib.sha256(), hashlib.sha256()
    pos = 0
    with open(path, "rb") as f:
        while True:
            chunk = f.read(CHUNK)
            if not chunk:
                break
            whole.update(chunk)
            mv, end, cur = memoryview(chunk), pos + len(chunk), pos
            for lo, hi in excluded:
                if hi <= cur or lo >= end:
                    continue
                outside.update(mv[cur - pos:max(cur, lo) - pos])
                cur = min(end, hi)
            outside.update(mv[cur - pos:])
            pos = end
    return whole.hexdigest(), outside.hexdigest()


def _to_f32(raw: bytes, dtype: str, shape) -> np.ndarray:
    t = torch.frombuffer(bytearray(raw), dtype=_DT[dtype]).reshape(shape)
    return t.to(torch.float32).numpy().astype(np.float64)


def _encode(w: np.ndarray, dtype: str) -> bytes:
    t = torch.from_numpy(w.astype(np.float32)).to(_DT[dtype]).contiguous()
    return t.view(torch.uint8).numpy().tobytes()


def apply(source, source_sha256: str, output, spec_path) -> dict:
    source, output, spec_path = pathlib.Path(source), pathlib.Path(output), pathlib.Path(spec_path)
    if output.exists() or source.resolve() == output.resolve():
        raise ValueError("the output must be a new file")
    if digest(source) != source_sha256:
        raise ValueError("source checksum mismatch")
    spec = json.loads(spec_path.read_text())
    if not spec.get("hypothesis") or not spec.get("edits"):
        raise ValueError("an explicit hypothesis and edits are required")
    table, base = read_header(source)
    plans, names = [], set()
    for e in spec["edits"]:
        name = e["tensor"]
        if not _NAME.fullmatch(name) or name in names or name not in table:
            raise ValueError(f"{name}: only distinct MLP down projections present in the file can be edited")
        names.add(name)
        meta = table[name]
        if meta["dtype"] not in _DT or len(meta["shape"]) != 2:
            raise ValueError(f"{name}: unsupported dtype or shape")
        dpath = (spec_path.parent / e["direction"]).resolve()
        d = np.load(dpath, allow_pickle=False).astype(np.float64)
        if d.shape != (meta["shape"][0],) or not np.isfinite(d).all():
            raise ValueError(f"{name}: the direction must be a finite vector over the output dimension")
        dn = float(np.linalg.norm(d))
        if not np.isfinite(dn) or dn == 0.0:
            raise ValueError(f"{name}: zero direction")
        s = float(e["strength"])
        if not np.isfinite(s) or not 0.0 <= s <= 1.0:
            raise ValueError(f"{name}: strength must be in [0, 1]")
        lo, hi = (base + meta["data_offsets"][0], base + meta["data_offsets"][1])
        plans.append((name, meta, d / dn, s, digest(dpath), lo, hi))
    journal_path = pathlib.Path(str(output) + ".edit.json")
    journal = {"state": "preparing", "source_sha256": source_sha256, "spec_sha256": digest(spec_path),
               "hypothesis": spec["hypothesis"], "edits": []}
    with journal_path.open("x") as f:
        json.dump(journal, f, indent=2)
    try:
        with source.open("rb") as src, output.open("xb") as dst:
            shutil.copyfileobj(src, dst, length=CHUNK)
        if source.stat().st_ino == output.stat().st_ino and source.stat().st_dev == output.stat().st_dev:
            raise ValueError("the copy is the original file")
        ranges = []
        with output.open("r+b") as f, mmap.mmap(f.fileno(), 0) as mm:
            for name, meta, d, s, dhash, lo, hi in plans:
                w = _to_f32(mm[lo:hi], meta["dtype"], meta["shape"])
                if not np.isfinite(w).all() or np.linalg.norm(w) == 0.0:
                    raise ValueError(f"{name}: the stored tensor is not finite and nonzero")
                before = d @ w
                if s == 0.0:
                    enc = bytes(mm[lo:hi])  # a true no-op keeps the stored bytes
                else:
                    enc = _encode(w - s * np.outer(d, before), meta["dtype"])
                if len(enc) != hi - lo:
                    raise ValueError(f"{name}: encoded size changed")
                mm[lo:hi] = enc
                back = _to_f32(enc, meta["dtype"], meta["shape"])
                delta = back - w
                journal["edits"].append({
                    "tensor": name, "dtype": meta["dtype"], "shape": meta["shape"], "strength": s,
                    "direction_sha256": dhash, "operation": "no_op" if s == 0.0 else "projection",
                    "parameters_touched": int(w.size), "values_changed": int(np.count_nonzero(delta)),
                    "delta_l2": float(np.linalg.norm(delta)),
                    "relative_delta_l2": float(np.linalg.norm(delta) / np.linalg.norm(w)),
                    "projection_norm_before": float(np.linalg.norm(before)),
                    "projection_norm_after": float(np.linalg.norm(d @ back)), "byte_range": [lo, hi]})
                ranges.append((lo, hi))
            mm.flush()
        ranges.sort()
        src_whole, src_out = checksums(source, ranges)
        out_whole, out_out = checksums(output, ranges)
        if src_whole != source_sha256 or src_out != out_out:
            raise ValueError("the source changed, or bytes outside the edited tensors differ")
        journal.update(state="complete", candidate_sha256=out_whole, unchanged_ranges_sha256=src_out,
                       original_preserved=True, bytes_outside_edited_tensors_equal=True)
    except BaseException as exc:
        journal.update(state="incomplete", error=str(exc))
        raise
    finally:
        journal_path.write_text(json.dumps(journal, indent=2) + "\n")
    return journal


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--source", required=True)
    p.add_argument("--source-sha256", required=True)
    p.add_argument("--output", required=True)
    p.add_argument("--spec", required=True)
    a = p.parse_args(argv)
    print(json.dumps(apply(a.source, a.source_sha256, a.output, a.spec), indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
