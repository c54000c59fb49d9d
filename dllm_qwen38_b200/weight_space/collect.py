"""Collect completed launched runs under an explicit comparison plan into one verified bundle
(the reference's `tools/weight-space/collect.py` role; no inference, no regrading).

    python -m dllm_qwen38_b200.weight_space.collect PLAN.json --output BUNDLE.json

PLAN: {"qualification": str, "conditions": [{"name", "run": RUN_DIR relative to the plan}],
       "paired": [[baseline, candidate], ...], "no_op": [[baseline, candidate], ...]}
Each run must be completed with its server stopped; its launch config and manifest must agree
on the model digest and backend; its dataset must still hash to the manifest's digest; its
results must be the manifest's full case list in order; its stored summary must equal the one
recomputed from the results. Paired runs must share the scorer revision and the engine identity
and arguments. Every file read is hashed, and re-hashed at the end: a run that changes while it
is collected fails the collection.
"""

from __future__ import annotations

import argparse
import contextlib
import io
import json
import math
import pathlib

from . import bench
from .common import digest, read_jsonl, write_new

FILES = ("manifest.json", "launch.json", "process-status.json", "results.jsonl", "summary.json")
ENGINE_KEYS = ("tokenizer", "block", "threshold", "sub_block", "n_ctx", "backend_commit")


def collect(plan_path) -> dict:
    plan_path = pathlib.Path(plan_path).resolve()
    plan = json.loads(plan_path.read_text())
    runs, ids, launches, records, roots, frozen = {}, {}, {}, {}, {}, {}
    for item in plan["conditions"]:
        name = item["name"]
        if name in runs:
            raise ValueError(f"duplicate condition {name}")
        root = (plan_path.parent / item["run"]).resolve()
        paths = [root / f for f in FILES]
        hashes = {p.name: digest(p) for p in paths}
        proc = json.loads(paths[2].read_text())
        if proc.get("state") != "completed" or not proc.get("engine_stopped") or type(
                proc.get("engine_exit_code")) is not int:
            raise ValueError(f"{name}: run not completed with its server stopped")
        ident = json.loads(paths[0].read_text())["identity"]
        launch = json.loads(paths[1].read_text())
        lcfg = launch["config"]
        if (lcfg.get("model_sha256") != ident["model_sha256"] or lcfg.get("backend_commit") != ident["backend_commit"]
                or not launch.get("engine_sha256")):
            raise ValueError(f"{name}: launch and manifest provenance disagree")
        data = pathlib.Path(lcfg["data"])
        if not data.is_absolute() or digest(data) != ident["data_sha256"]:
            raise ValueError(f"{name}: dataset path not absolute or its checksum changed")
        frozen[data] = ident["data_sha256"]
        rows = read_jsonl(paths[3])
        if not rows or [r["id"] for r in rows] != ident["case_ids"]:
            raise ValueError(f"{name}: incomplete or reordered results")
        got, stored = bench.summary(rows), json.loads(paths[4].read_text())
        for k, v in got.items():
            sv = stored.get(k)
            if isinstance(v, float):
                if not isinstance(sv, (int, float)) or not math.isclose(v, sv, rel_tol=1e-10, abs_tol=1e-8):
                    raise ValueError(f"{name}: stored summary differs at {k}")
            elif sv != v:
                raise ValueError(f"{name}: stored summary differs at {k}")
        if not ident.get("bench_sha256"):
            raise ValueError(f"{name}: scorer revision missing")
        roots[name], ids[name], launches[name], records[name] = root, ident, launch, rows
        runs[name] = {"identity": ident, "summary": got, "artifact_sha256": hashes,
                      "engine": {"engine_sha256": launch["engine_sha256"],
                                 **{k: lcfg.get(k) for k in ENGINE_KEYS}},
                      "engine_exit_code": proc["engine_exit_code"], "engine_stopped": True}
        frozen.update({p: hashes[p.name] for p in paths})
    paired = []
    for left, right in plan["paired"]:
        if ids[left]["bench_sha256"] != ids[right]["bench_sha256"]:
            raise ValueError(f"{left}/{right}: scorer revisions differ")
        if runs[left]["engine"] != runs[right]["engine"]:
            raise ValueError(f"{left}/{right}: engine identity or arguments differ")
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            res = bench.compare(argparse.Namespace(baseline=str(roots[left]), candidate=str(roots[right]), output=None))
        paired.append({"baseline": left, "candidate": right, "result": res})
    no_ops = []
    for left, right in plan.get("no_op", []):
        if [left, right] not in plan["paired"]:
            raise ValueError("a no-op pair must also be a paired comparison")
        if ids[left]["case_ids"] != ids[right]["case_ids"]:
            raise ValueError("no-op case lists differ")
        a, b = records[left], records[right]
        no_ops.append({"baseline": left, "candidate": right,
                       "checkpoint_hash_equal": ids[left]["model_sha256"] == ids[right]["model_sha256"],
                       "exact_response_text_matches": sum(x["response"]["content"] == y["response"]["content"]
                                                          for x, y in zip(a, b)), "n": len(a)})
    if any(digest(p) != h for p, h in frozen.items()):
        raise ValueError("a run changed while it was being collected")
    return {"schema": "bdllm.ws.bundle/v1", "plan_sha256": digest(plan_path), "collector_sha256": digest(__file__),
            "comparison_code_sha256": digest(bench.__file__), "qualification": plan["qualification"], "runs": runs,
            "paired": paired, "no_op": no_ops,
            "limitations": ["stored grades and timings are aggregated; no new inference or regrading",
                            "model files are not re-hashed by the collector (the launcher checked them)",
                            "small or selected development subsets do not establish a held-out improvement"]}


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
