"""GSM8K-train development runs against a loopback completion server, and the paired comparison
of two runs (the role of the reference's `tools/weight-space/bench.py:39-185`; this one drives this
framework's `server.py` instead of llama-server and reads the data from a local file).

    python -m dllm_qwen38_b200.weight_space.bench prepare --source train.jsonl --output DIR [--size 32]
    python -m dllm_qwen38_b200.weight_space.bench run --data DIR/dev.json --model MODEL
           --model-sha256 H --backend-commit C --condition NAME --output RUN [--server URL]
           [--thinking on|off] [--max-tokens 1024] [--limit 0] [--seed 42] [--timeout 600]
    python -m dllm_qwen38_b200.weight_space.bench compare RUN_A RUN_B [--output OUT.json]

Three stages, three file kinds:

* ``prepare`` writes two disjoint case lists (dev, validation) chosen deterministically from the
  GSM8K train file, so two people who prepare from the same file get the same cases.
* ``run`` owns one run directory: ``manifest.json`` pins what the run is (data digest, case ids,
  generation settings, server context, model digest, this file's digest); ``results.jsonl``
  grows by one graded case at a time, so an interrupted run resumes where it stopped, and only
  when its manifest is unchanged; ``summary.json`` is rewritten after every case.
* ``compare`` reads two complete runs over the same cases and settings and reports the paired
  accuracy delta with a bootstrap interval and the exact McNemar p-value.

Contracts kept with the reference so that results mean the same in both code bases: the answer
line `FINAL: <number>` and its parser, the selection order (SHA-256 of the question, dev then
validation), the bootstrap (10,000 resamples from `random.Random(797)`, 2.5 / 97.5 % order
statistics) and the McNemar test.
"""

from __future__ import annotations

import argparse
import collections
import datetime
import decimal
import hashlib
import json
import math
import pathlib
import random
import re
import time
import urllib.parse
import urllib.request

from .common import canonical, digest, digest_tree, read_jsonl, write_new

BOOT_N, BOOT_SEED = 10000, 797
ANSWER_LINE = re.compile(r"\s*FINAL:\s*([-+]?(?:\d[\d,]*)(?:\.\d+)?)\s*[.!]?\s*", re.IGNORECASE)
INSTRUCTION = "\nGive your final answer on its own line as FINAL: <number>."
PAIRED_KEYS = ("data_sha256", "case_ids", "split", "settings", "thinking", "backend_commit", "server_context",
               "decoder")
QUALIFICATION = "development diagnostic: small n and selected candidates do not establish a held-out improvement"


def canonical_number(text: str) -> str:
    """The normalised decimal string of a number with thousands separators removed ('1,234.50' ->
    '1234.5', '100' -> '1E+2'), as both code bases store it; raises decimal.InvalidOperation on
    anything but a number."""
    return str(decimal.Decimal(text.replace(",", "")).normalize())


# ----------------------------------------------------------------------------- prepare


def mini_splits(rows: list, size: int) -> tuple:
    """(dev, validation): the 2 * size questions with the smallest SHA-256, in that order."""
    if size < 1:
        raise ValueError("size must be positive")
    ranked = sorted(rows, key=lambda r: canonical(r["question"]))[: 2 * size]
    if len(ranked) < 2 * size:
        raise ValueError("not enough questions for two splits")
    if len({r["question"] for r in ranked}) < len(ranked):
        raise ValueError("duplicate questions")
    return ranked[:size], ranked[size:]


def _case(row: dict) -> dict:
    answer = row["answer"].rsplit("####", 1)[1].strip()
    canonical_number(answer)  # the gold answer must parse as a number
    return {"id": canonical(row["question"])[:20], "question": row["question"], "answer": answer}


def prepare(args) -> dict:
    src = pathlib.Path(args.source)
    raw = src.read_bytes()
    sha = hashlib.sha256(raw).hexdigest()
    rows = [json.loads(line) for line in raw.splitlines() if line.strip()]
    out = pathlib.Path(args.output)
    out.mkdir(parents=True, exist_ok=True)
    for split, part in zip(("dev", "validation"), mini_splits(rows, args.size)):
        write_new(out / f"{split}.json", {"schema": "bdllm.ws.gsm8k-mini/v1", "source": src.name, "source_sha256": sha,
                                          "split": split,
                                          "selection": "question SHA-256 ascending; dev then validation",
                                          "cases": [_case(r) for r in part]})
    res = {"size_per_split": args.size, "source_sha256": sha}
    print(json.dumps(res))
    return res


# ----------------------------------------------------------------------------- grading


def final_number(text: str):
    """The number on the single `FINAL: <number>` line after the reasoning, canonicalised; None
    when the reasoning never closed, or when there is no such line or more than one."""
    if "<think>" in text and "</think>" not in text:
        return None
    visible = text.split("</think>")[-1]
    hits = [m.group(1) for m in map(ANSWER_LINE.fullmatch, visible.splitlines()) if m]
    return canonical_number(hits[0]) if len(hits) == 1 else None


def repeated_fourgram_fraction(text: str) -> float:
    """Share of word 4-grams that repeat an earlier one (a degeneration signal)."""
    w = text.split()
    counts = collections.Counter(tuple(w[i : i + 4]) for i in range(len(w) - 3))
    total = sum(counts.values())
    return sum(c - 1 for c in counts.values()) / total if total else 0.0


def summary(records) -> dict:
    """Aggregate of graded records (the summary.json schema)."""
    agg = collections.Counter()
    for r in records:
        resp = r["response"]
        agg["correct"] += bool(r["correct"])
        agg["tokens"] += resp.get("tokens_predicted", 0)
        agg["limit"] += resp.get("stop_type") == "limit" or bool(resp.get("stopped_limit"))
        agg["no_final"] += r["predicted"] is None
    n, right = len(records), agg["correct"]
    secs = sum(r["wall_seconds"] for r in records)
    per = (lambda x: x / right) if right else (lambda x: None)  # noqa: E731
    return {"n": n, "correct": right, "accuracy": right / n if n else None, "wall_seconds": secs,
            "generated_tokens": agg["tokens"], "seconds_per_correct": per(secs),
            "tokens_per_correct": per(agg["tokens"]), "limit_hits": agg["limit"], "no_final_answer": agg["no_final"]}


# ----------------------------------------------------------------------------- run


class LoopbackClient:
    """JSON over HTTP to a server on this machine only."""

    def __init__(self, base: str):
        u = urllib.parse.urlparse(base)
        if u.scheme != "http" or u.hostname not in {"127.0.0.1", "localhost", "::1"}:
            raise ValueError("only an explicit loopback server is supported")
        self.base = base

    def call(self, path: str, payload=None, timeout: float = 30):
        data = None if payload is None else json.dumps(payload).encode()
        req = urllib.request.Request(self.base + path, data=data, headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=timeout) as r:
            return json.load(r)


def request(server: str, endpoint: str, payload=None, timeout: float = 30):
    """One JSON call to a loopback server."""
    return LoopbackClient(server).call(endpoint, payload, timeout)


def render_prompt(question: str, thinking: str) -> str:
    """Qwen chat turn asking for the FINAL line; with thinking off the think block is pre-closed."""
    opener = "<think>\n" if thinking == "on" else "<think>\n</think>\n\n"
    return f"<|im_start|>user\n{question}{INSTRUCTION}<|im_end|>\n<|im_start|>assistant\n{opener}"


class RunDir:
    """A run directory: the manifest that pins it, the append-only results, the summary."""

    def __init__(self, path, identity: dict, extra: dict):
        self.path = pathlib.Path(path)
        self.path.mkdir(parents=True, exist_ok=True)
        man = self.path / "manifest.json"
        if man.exists():
            if json.loads(man.read_text())["identity"] != identity:
                raise ValueError("resume manifest mismatch")
        else:
            write_new(man, {"identity": identity, **extra})
        self.rows = self.path / "results.jsonl"
        self.records = read_jsonl(self.rows)
        if [r["id"] for r in self.records] != identity["case_ids"][: len(self.records)]:
            raise ValueError("results are not a prefix of the manifest's cases")

    def append(self, rec: dict) -> dict:
        with self.rows.open("a") as f:
            f.write(json.dumps(rec, ensure_ascii=False) + "\n")
            f.flush()
        self.records.append(rec)
        s = summary(self.records)
        (self.path / "summary.json").write_text(json.dumps(s, indent=2) + "\n")
        return s


def run(args) -> dict:
    if args.limit < 0 or args.max_tokens < 1 or args.timeout <= 0:
        raise ValueError("invalid limit, token budget or timeout")
    client = LoopbackClient(args.server)
    if digest_tree(args.model) != args.model_sha256:
        raise ValueError("model checksum mismatch")
    data = json.loads(pathlib.Path(args.data).read_text())
    cases = data["cases"][: args.limit] if args.limit else data["cases"]
    ids = [c["id"] for c in cases]
    if not cases or len(set(ids)) < len(ids):
        raise ValueError("empty or duplicate cases")
    props = client.call("/props")
    served = props.get("model_path")
    if served is None or pathlib.Path(served).resolve() != pathlib.Path(args.model).resolve():
        raise ValueError(f"the server runs {served}, not the requested model")
    settings = {"n_predict": args.max_tokens, "temperature": 0.0, "seed": args.seed, "stream": False}
    identity = {"schema": "bdllm.ws.run/v1", "data_sha256": digest(args.data), "case_ids": ids,
                "split": data["split"], "settings": settings, "thinking": args.thinking,
                "backend_commit": args.backend_commit,
                "server_context": props.get("default_generation_settings", {}).get("n_ctx"),
                "decoder": props.get("decoder"), "model_sha256": args.model_sha256, "condition": args.condition,
                "bench_sha256": digest(__file__)}
    rd = RunDir(args.output, identity, {"model_path": str(pathlib.Path(args.model).resolve()), "server_props": props,
                                        "started_utc": datetime.datetime.now(datetime.timezone.utc).isoformat()})
    for case in cases[len(rd.records):]:
        prompt = render_prompt(case["question"], args.thinking)
        t0 = time.monotonic()
        resp = client.call("/completion", {**settings, "prompt": prompt}, timeout=args.timeout)
        elapsed = time.monotonic() - t0
        text = resp["content"]
        pred = final_number(("<think>\n" + text) if args.thinking == "on" else text)  # the opener is in the prompt
        want = canonical_number(case["answer"])
        s = rd.append({"id": case["id"], "prompt_sha256": canonical(prompt), "expected": want, "predicted": pred,
                       "correct": pred == want, "wall_seconds": elapsed,
                       "repeated_fourgram_fraction": repeated_fourgram_fraction(text), "response": resp})
        print(json.dumps({"completed": len(rd.records), **s}), flush=True)
    return summary(rd.records)


# ----------------------------------------------------------------------------- compare


def mcnemar_exact(wins: int, losses: int) -> float:
    """Two-sided exact McNemar p-value: the binomial(wins + losses, 1/2) tail at the smaller
    count, doubled and capped at 1."""
    d = wins + losses
    if d == 0:
        return 1.0
    k = min(wins, losses)
    return min(1.0, 2.0 * sum(math.comb(d, i) for i in range(k + 1)) / 2 ** d)


def bootstrap_interval(diff: list, n_resamples: int = BOOT_N, seed: int = BOOT_SEED) -> list:
    """Percentile interval of the mean paired difference: `n_resamples` resamples with
    replacement from `random.Random(seed)`, the 2.5 % and 97.5 % order statistics."""
    rng, n = random.Random(seed), len(diff)
    means = sorted(sum(rng.choices(diff, k=n)) / n for _ in range(n_resamples))
    return [means[int(0.025 * n_resamples)], means[int(0.975 * n_resamples) - 1]]


def compare_runs(baseline, candidate) -> dict:
    """Paired report of two complete run directories over the same cases and settings."""
    dirs = [pathlib.Path(baseline), pathlib.Path(candidate)]
    base_id, cand_id = (json.loads((d / "manifest.json").read_text())["identity"] for d in dirs)
    differing = [k for k in PAIRED_KEYS if base_id.get(k) != cand_id.get(k)]
    if differing:
        raise ValueError(f"not a paired comparison: {differing[0]} differs")
    base, cand = (read_jsonl(d / "results.jsonl") for d in dirs)
    if [r["id"] for r in base] != base_id["case_ids"] or [r["id"] for r in cand] != base_id["case_ids"]:
        raise ValueError("a paired comparison needs two complete runs over the same cases")
    diff = [int(c["correct"]) - int(b["correct"]) for b, c in zip(base, cand)]
    wins, losses = diff.count(1), diff.count(-1)
    return {"baseline": summary(base), "candidate": summary(cand), "paired_accuracy_delta": sum(diff) / len(diff),
            "bootstrap_95_interval": bootstrap_interval(diff), "wins": wins, "losses": losses,
            "mcnemar_exact_two_sided_p": mcnemar_exact(wins, losses), "qualification": QUALIFICATION}


def compare(args) -> dict:
    res = compare_runs(args.baseline, args.candidate)
    print(json.dumps(res, indent=2))
    if getattr(args, "output", None):
        write_new(args.output, res)
    return res


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="command", required=True)
    q = sub.add_parser("prepare")
    q.add_argument("--source", required=True, help="local GSM8K train JSONL")
    q.add_argument("--output", required=True)
    q.add_argument("--size", type=int, default=32)
    q.set_defaults(func=prepare)
    q = sub.add_parser("run")
    for flag in ("data", "model", "model-sha256", "backend-commit", "condition", "output"):
        q.add_argument("--" + flag, required=True)
    q.add_argument("--server", default="http://127.0.0.1:17977")
    q.add_argument("--thinking", choices=("on", "off"), default="off")
    q.add_argument("--max-tokens", type=int, default=1024)
    q.add_argument("--limit", type=int, default=0)
    q.add_argument("--seed", type=int, default=42)
    q.add_argument("--timeout", type=float, default=600)
    q.set_defaults(func=run)
    q = sub.add_parser("compare")
    q.add_argument("baseline")
    q.add_argument("candidate")
    q.add_argument("--output")
    q.set_defaults(func=compare)
    a = p.parse_args(argv)
    a.func(a)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
