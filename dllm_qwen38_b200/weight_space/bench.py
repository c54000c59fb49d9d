"""Small, resumable GSM8K-train development runs against a loopback completion server, and
paired comparison of two runs (the reference's `tools/weight-space/bench.py` role, driving this
framework's `server.py` instead of llama-server).

    python -m dllm_qwen38_b200.weight_space.bench prepare --source train.jsonl --output DIR [--size 32]
    python -m dllm_qwen38_b200.weight_space.bench run --data DIR/dev.json --model MODEL
           --model-sha256 H --backend-commit C --condition NAME --output RUN [--server URL]
           [--thinking on|off] [--max-tokens 1024] [--limit 0] [--seed 42] [--timeout 600]
    python -m dllm_qwen38_b200.weight_space.bench compare RUN_A RUN_B [--output OUT.json]

prepare: the local GSM8K train JSONL (no network) is ordered by the SHA-256 of each question;
the first `size` questions are `dev`, the next `size` are `validation`.
run: every case is asked once, greedily, with "FINAL: <number>" as the answer contract; the
manifest pins the data, case ids, settings, model digest and this file's digest, and a rerun
resumes only when all of that matches; results.jsonl is appended one case at a time.
compare: the two runs must share data, cases, settings and server context; the report has the
paired accuracy delta, a seeded 10,000-resample bootstrap interval and the exact two-sided
McNemar p-value over the discordant pairs.
"""

from __future__ import annotations

import argparse
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

NUMBER = r"[-+]?(?:\d[\d,]*)(?:\.\d+)?"
BOOT_N, BOOT_SEED = 10000, 797


def _norm_number(s: str) -> str:
    return str(decimal.Decimal(s.replace(",", "")).normalize())


def prepare(args) -> dict:
    src = pathlib.Path(args.source)
    raw = src.read_bytes()
    rows = [json.loads(x) for x in raw.splitlines() if x.strip()]
    if args.size < 1:
        raise ValueError("size must be positive")
    rows.sort(key=lambda r: canonical(r["question"]))
    chosen = rows[: 2 * args.size]
    if len(chosen) != 2 * args.size:
        raise ValueError("not enough questions for two splits")
    if len({r["question"] for r in chosen}) != len(chosen):
        raise ValueError("duplicate questions")
    out = pathlib.Path(args.output)
    out.mkdir(parents=True, exist_ok=True)
    sha = hashlib.sha256(raw).hexdigest()
    for split, part in (("dev", chosen[: args.size]), ("validation", chosen[args.size:])):
        cases = []
        for r in part:
            ans = r["answer"].rsplit("####", 1)[1].strip()
            _norm_number(ans)  # must be a number
            cases.append({"id": canonical(r["question"])[:20], "question": r["question"], "answer": ans})
        write_new(out / f"{split}.json", {"schema": "bdllm.ws.gsm8k-mini/v1", "source": src.name,
                                          "source_sha256": sha, "split": split,
                                          "selection": "question SHA-256 ascending; dev then validation",
                                          "cases": cases})
    res = {"size_per_split": args.size, "source_sha256": sha}
    print(json.dumps(res))
    return res


def final_number(text: str):
    """The one `FINAL: <number>` line after any reasoning; None when missing, repeated, or when
    the reasoning is unfinished."""
    if "<think>" in text and "</think>" not in text:
        return None
    tail = text.rsplit("</think>", 1)[-1]
    found = re.findall(r"(?im)^\s*FINAL:\s*(" + NUMBER + r")\s*[.!]?\s*$", tail)
    return _norm_number(found[0]) if len(found) == 1 else None


def repeated_fourgram_fraction(text: str) -> float:
    w = text.split()
    grams = list(zip(w, w[1:], w[2:], w[3:]))
    return (len(grams) - len(set(grams))) / len(grams) if grams else 0.0


def request(server: str, endpoint: str, payload=None, timeout: float = 30):
    body = None if payload is None else json.dumps(payload).encode()
    req = urllib.request.Request(server + endpoint, data=body, headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.load(r)


def summary(records) -> dict:
    n = len(records)
    right = sum(bool(r["correct"]) for r in records)
    secs = sum(r["wall_seconds"] for r in records)
    toks = sum(r["response"].get("tokens_predicted", 0) for r in records)
    return {"n": n, "correct": right, "accuracy": right / n if n else None, "wall_seconds": secs,
            "generated_tokens": toks, "seconds_per_correct": secs / right if right else None,
            "tokens_per_correct": toks / right if right else None,
            "limit_hits": sum(r["response"].get("stop_type") == "limit" or bool(r["response"].get("stopped_limit"))
                              for r in records),
            "no_final_answer": sum(r["predicted"] is None for r in records)}


def _model_digest(path: str) -> str:
    return digest_tree(path)


def run(args) -> dict:
    if args.limit < 0 or args.max_tokens < 1 or args.timeout <= 0:
        raise ValueError("invalid limit, token budget or timeout")
    u = urllib.parse.urlparse(args.server)
    if u.scheme != "http" or u.hostname not in {"127.0.0.1", "localhost", "::1"}:
        raise ValueError("only an explicit loopback server is supported")
    if _model_digest(args.model) != args.model_sha256:
        raise ValueError("model checksum mismatch")
    data = json.loads(pathlib.Path(args.data).read_text())
    cases = data["cases"][: args.limit] if args.limit else data["cases"]
    if not cases or len({c["id"] for c in cases}) != len(cases):
        raise ValueError("empty or duplicate cases")
    props = request(args.server, "/props")
    loaded = props.get("model_path")
    if loaded is None or pathlib.Path(loaded).resolve() != pathlib.Path(args.model).resolve():
        raise ValueError(f"the server runs {loaded}, not the requested model")
    settings = {"n_predict": args.max_tokens, "temperature": 0.0, "seed": args.seed, "stream": False}
    identity = {"schema": "bdllm.ws.run/v1", "data_sha256": digest(args.data), "case_ids": [c["id"] for c in cases],
                "split": data["split"], "settings": settings, "thinking": args.thinking,
                "backend_commit": args.backend_commit,
                "server_context": props.get("default_generation_settings", {}).get("n_ctx"),
                "decoder": props.get("decoder"), "model_sha256": args.model_sha256, "condition": args.condition,
                "bench_sha256": digest(__file__)}
    out = pathlib.Path(args.output)
    out.mkdir(parents=True, exist_ok=True)
    man = out / "manifest.json"
    if man.exists():
        if json.loads(man.read_text())["identity"] != identity:
            raise ValueError("resume manifest mismatch")
    else:
        write_new(man, {"identity": identity, "model_path": str(pathlib.Path(args.model).resolve()),
                        "server_props": props,
                        "started_utc": datetime.datetime.now(datetime.timezone.utc).isoformat()})
    rows_path = out / "results.jsonl"
    records = read_jsonl(rows_path)
    if [r["id"] for r in records] != identity["case_ids"][: len(records)]:
        raise ValueError("results are not a prefix of the manifest's cases")
    for case in cases[len(records):]:
        user = case["question"] + "\nGive your final answer on its own line as FINAL: <number>."
        opener = "<think>\n" if args.thinking == "on" else "<think>\n</think>\n\n"
        prompt = "<|im_start|>user\n" + user + "<|im_end|>\n<|im_start|>assistant\n" + opener
        t0 = time.monotonic()
        resp = request(args.server, "/completion", {**settings, "prompt": prompt}, timeout=args.timeout)
        dt = time.monotonic() - t0
        content = resp["content"]
        judged = ("<think>\n" + content) if args.thinking == "on" else content
        pred = final_number(judged)
        want = _norm_number(case["answer"])
        rec = {"id": case["id"], "prompt_sha256": canonical(prompt), "expected": want, "predicted": pred,
               "correct": pred == want, "wall_seconds": dt,
               "repeated_fourgram_fraction": repeated_fourgram_fraction(content), "response": resp}
        with rows_path.open("a") as f:
            f.write(json.dumps(rec, ensure_ascii=False) + "\n")
            f.flush()
        records.append(rec)
        print(json.dumps({"completed": len(records), **summary(records)}), flush=True)
        (out / "summary.json").write_text(json.dumps(summary(records), indent=2) + "\n")
    return summary(records)


def mcnemar_exact(wins: int, losses: int) -> float:
    """Two-sided exact McNemar p-value: binomial(wins + losses, 1/2) tail, doubled, capped at 1."""
    d = wins + losses
    if d == 0:
        return 1.0
    tail = sum(math.comb(d, i) for i in range(min(wins, losses) + 1))
    return min(1.0, 2.0 * tail / 2 ** d)


def compare(args) -> dict:
    roots = [pathlib.Path(x) for x in (args.baseline, args.candidate)]
    ids = [json.loads((r / "manifest.json").read_text())["identity"] for r in roots]
    for key in ("data_sha256", "case_ids", "split", "settings", "thinking", "backend_commit", "server_context",
                "decoder"):
        if ids[0].get(key) != ids[1].get(key):
            raise ValueError(f"not a paired comparison: {key} differs")
    recs = [read_jsonl(r / "results.jsonl") for r in roots]
    if any([r["id"] for r in rows] != ids[0]["case_ids"] for rows in recs):
        raise ValueError("a paired comparison needs two complete runs over the same cases")
    diff = [int(b["correct"]) - int(a["correct"]) for a, b in zip(*recs)]
    n = len(diff)
    rng = random.Random(BOOT_SEED)
    boot = sorted(sum(rng.choices(diff, k=n)) / n for _ in range(BOOT_N))
    wins, losses = diff.count(1), diff.count(-1)
    res = {"baseline": summary(recs[0]), "candidate": summary(recs[1]), "paired_accuracy_delta": sum(diff) / n,
           "bootstrap_95_interval": [boot[int(0.025 * BOOT_N)], boot[int(0.975 * BOOT_N) - 1]],
           "wins": wins, "losses": losses, "mcnemar_exact_two_sided_p": mcnemar_exact(wins, losses),
           "qualification": "development diagnostic: small n and selected candidates do not establish a "
                            "held-out improvement"}
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
