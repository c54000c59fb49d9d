"""Collect completed launched runs under an explicit comparison plan into one verified bundle
(the role of the reference's `tools/weight-space/collect.py:13-99`; no inference, no regrading).

    python -m dllm_qwen38_b200.weight_space.collect PLAN.json --output BUNDLE.json

PLAN: {"qualification": str, "conditions": [{"name", "run": RUN_DIR relative to the plan}],
       "paired": [[baseline, candidate], ...], "no_op": [[baseline, candidate], ...]}

A bundle is only as good as the runs under it, so each run is admitted by `admit_run`, which
fails on the first of these it finds: the run did not complete or its server is still up; the
launch configuration and the manifest name different models or backends; the dataset moved or
changed; the results are not the manifest's full case list in order; the stored summary is not
the one the results give. Paired runs must also share the scorer revision and the engine's
identity and arguments. Every file the collector reads goes through one `Ledger` that records its
digest; the ledger is checked again at the end, so a run that changes during collection fails it.
"""

from __future__ import annotations

import argparse
import json
import math
import pathlib

from . import bench
from .common import digest, read_jsonl, write_new

RUN_FILES = ("manifest.json", "launch.json", "process-status.json", "results.jsonl", "summary.json")
ENGINE_KEYS = ("tokenizer", "block", "threshold", "sub_block", "n_ctx", "backend_commit")
LIMITATIONS = ["stored grades and timings are aggregated; no new inference or regrading",
               "model files are not re-hashed by the collector (the launcher checked them)",
               "small or selected development subsets do not establish a held-out improvement"]


class Ledger:
    """Digests of every file read, for the end-of-collection re-check."""

    def __init__(self):
        self.seen = {}

    def note(self, path, expected: str | None = None) -> str:
        h = digest(path)
        if expected is not None and h != expected:
            raise ValueError(f"{path}: checksum differs from the manifest's")
        self.seen[pathlib.Path(path)] = h
        return h

    def verify(self) -> None:
        changed = [str(p) for p, h in self.seen.items() if digest(p) != h]
        if changed:
            raise ValueError(f"a run changed while it was being collected: {changed[:3]}")


def _same_summary(stored: dict, recomputed: dict) -> str | None:
    """The first summary key whose stored value disagrees with the recomputed one (floats to a
    relative 1e-10 / absolute 1e-8), or None."""
    for k, v in recomputed.items():
        s = stored.get(k)
        ok = (isinstance(s, (int, float)) and math.isclose(v, s, rel_tol=1e-10, abs_tol=1e-8)) \
            if isinstance(v, float) else s == v
        if not ok:
            return k
    return None


def admit_run(name: str, root: pathlib.Path, ledger: Ledger) -> dict:
    """Verify one run directory and return its bundle entry plus what the pairing needs."""
    files = {f: root / f for f in RUN_FILES}
    hashes = {f: ledger.note(p) for f, p in files.items()}
    status = json.loads(files["process-status.json"].read_text())
    if not (status.get("state") == "completed" and status.get("engine_stopped")
            and type(status.get("engine_exit_code")) is int):
        raise ValueError(f"{name}: run not completed with its server stopped")
    ident = json.loads(files["manifest.json"].read_text())["identity"]
    launch = json.loads(files["launch.json"].read_text())
    cfg = launch["config"]
    if not launch.get("engine_sha256") or (cfg.get("model_sha256"), cfg.get("backend_commit")) != (
            ident["model_sha256"], ident["backend_commit"]):
        raise ValueError(f"{name}: launch and manifest provenance disagree")
    data = pathlib.Path(cfg["data"])
    if not data.is_absolute():
        raise ValueError(f"{name}: dataset path not absolute")
    try:
        ledger.note(data, ident["data_sha256"])
    except ValueError:
        raise ValueError(f"{name}: dataset checksum changed") from None
    rows = read_jsonl(files["results.jsonl"])
    if not rows or [r["id"] for r in rows] != ident["case_ids"]:
        raise ValueError(f"{name}: incomplete or reordered results")
    recomputed = bench.summary(rows)
    bad = _same_summary(json.loads(files["summary.json"].read_text()), recomputed)
    if bad is not None:
        raise ValueError(f"{name}: stored summary differs at {bad}")
    if not ident.get("bench_sha256"):
        raise ValueError(f"{name}: scorer revision missing")
    entry = {"identity": ident, "summary": recomputed, "artifact_sha256": hashes,
             "engine": {"engine_sha256": launch["engine_sha256"], **{k: cfg.get(k) for k in ENGINE_KEYS}},
             "engine_exit_code": status["engine_exit_code"], "engine_stopped": True}
    return {"entry": entry, "root": root, "rows": rows}


def collect(plan_path) -> dict:
    plan_path = pathlib.Path(plan_path).resolve()
    plan = json.loads(plan_path.read_text())
    ledger = Ledger()
    admitted = {}
    for cond in plan["conditions"]:
        if cond["name"] in admitted:
            raise ValueError(f"duplicate condition {cond['name']}")
        admitted[cond["name"]] = admit_run(cond["name"], (plan_path.parent / cond["run"]).resolve(), ledger)
    entries = {k: v["entry"] for k, v in admitted.items()}
    paired = []
    for base, cand in plan["paired"]:
        if entries[base]["identity"]["bench_sha256"] != entries[cand]["identity"]["bench_sha256"]:
            raise ValueError(f"{base}/{cand}: scorer revisions differ")
        if entries[base]["engine"] != entries[cand]["engine"]:
            raise ValueError(f"{base}/{cand}: engine identity or arguments differ")
        paired.append({"baseline": base, "candidate": cand,
                       "result": bench.compare_runs(admitted[base]["root"], admitted[cand]["root"])})
    no_ops = []
    for base, cand in plan.get("no_op", []):
        if [base, cand] not in plan["paired"]:
            raise ValueError("a no-op pair must also be a paired comparison")
        bi, ci = entries[base]["identity"], entries[cand]["identity"]
        if bi["case_ids"] != ci["case_ids"]:
            raise ValueError("no-op case lists differ")
        same_text = sum(x["response"]["content"] == y["response"]["content"]
                        for x, y in zip(admitted[base]["rows"], admitted[cand]["rows"]))
        no_ops.append({"baseline": base, "candidate": cand,
                       "checkpoint_hash_equal": bi["model_sha256"] == ci["model_sha256"],
                       "exact_response_text_matches": same_text, "n": len(admitted[base]["rows"])})
    ledger.verify()
    return {"schema": "bdllm.ws.bundle/v1", "plan_sha256": digest(plan_path), "collector_sha256": digest(__file__),
            "comparison_code_sha256": digest(bench.__file__), "qualification": plan["qualification"], "runs": entries,
            "paired": paired, "no_op": no_ops, "limitations": LIMITATIONS}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("plan", type=pathlib.Path)
    p.add_argument("--output", required=True, type=pathlib.Path)
    a = p.parse_args(argv)
    res = collect(a.plan)
    write_new(a.output, res)
    print(json.dumps({k: r["summary"] for k, r in res["runs"].items()}, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
