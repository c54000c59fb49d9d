"""Local launcher: the reference's Modal entry points (`modal_app.py:22-317`) as subcommands that run
on this node's GPUs, tee their output to a log and extract a report.

    python -m dllm_qwen38_b200.launch equivalence [-- args]
    python -m dllm_qwen38_b200.launch train [-- args]              # single device
    python -m dllm_qwen38_b200.launch fsdp --gpus 8 [-- args]      # torchrun, one rank per GPU
    python -m dllm_qwen38_b200.launch levers [-- args]
    python -m dllm_qwen38_b200.launch eval [-- args]               # GSM8K
    python -m dllm_qwen38_b200.launch decode --gpus N [-- args]    # decode benchmark (TP when N > 1)
    python -m dllm_qwen38_b200.launch bench --gpus N [-- args]     # flagship training benchmark

Every run writes `<log-dir>/<name>-<UTC time>.log` and, when the program printed a `REPORT\\t{json}`
line or a final JSON line, `<name>-<UTC time>.report.json` (the reference kept the same pair under
`reports/modal/`). Multi-GPU runs use torchrun with the rendezvous on 127.0.0.1 and an outer
`timeout -k` bound; the child's exit code is returned.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

MODULES = {
    "equivalence": "dllm_qwen38_b200.equivalence",
    "train": "dllm_qwen38_b200.train.single",
    "fsdp": "dllm_qwen38_b200.train.fsdp_train",
    "levers": "dllm_qwen38_b200.bench.levers",
    "eval": "dllm_qwen38_b200.eval.gsm8k",
    "decode": "dllm_qwen38_b200.bench.decode",
    "bench": None,  # bench.py at the repository root
}


def command(name: str, gpus: int, port: int, timeout_s: int, args: list) -> list:
    target = ["-m", MODULES[name]] if MODULES[name] else [os.path.join(ROOT, "bench.py")]
    if name == "bench":
        args = ["--gpus", str(gpus)] + args
    if gpus > 1:
        return ["timeout", "-k", "60", str(timeout_s), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                f"--nproc-per-node={gpus}", "--master-addr", "127.0.0.1", "--master-port", str(port)] + target + args
    return ["timeout", "-k", "60", str(timeout_s), sys.executable] + target + args


def extract_report(lines: list):
    for ln in reversed(lines):
        if ln.startswith("REPORT\t"):
            try:
                return json.loads(ln.split("\t", 1)[1])
            except json.JSONDecodeError:
                continue
    for ln in reversed(lines):
        s = ln.strip()
        if s.startswith("{") and s.endswith("}"):
            try:
                return json.loads(s)
            except json.JSONDecodeError:
                continue
    return None


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="dllm_qwen38_b200.launch", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("name", choices=sorted(MODULES))
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--port", type=int, default=29541)
    p.add_argument("--timeout", type=int, default=24 * 3600, help="outer bound in seconds (timeout -k 60)")
    p.add_argument("--log-dir", default="runs")
    p.add_argument("--dry-run", action="store_true")
    argv = list(sys.argv[1:] if argv is None else argv)
    cut = argv.index("--") if "--" in argv else len(argv)
    a = p.parse_args(argv[:cut])
    args = argv[cut + 1:]
    if a.name in ("equivalence", "train", "levers", "eval") and a.gpus > 1:
        raise SystemExit(f"{a.name} runs on one device")
    cmd = command(a.name, a.gpus, a.port, a.timeout, args)
    if a.dry_run:
        print(" ".join(cmd))
        return 0
    os.makedirs(a.log_dir, exist_ok=True)
    stamp = datetime.datetime.now(datetime.timezone.utc).strftime("%Y%m%d-%H%M%S")
    base = os.path.join(a.log_dir, f"{a.name}-{stamp}")
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    lines = []
    with open(base + ".log", "w") as log:
        log.write(" ".join(cmd) + "\n")
        proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, env=env, cwd=ROOT)
        for ln in proc.stdout:
            sys.stdout.write(ln)
            log.write(ln)
            lines.append(ln.rstrip("\n"))
        rc = proc.wait()
    rep = extract_report(lines)
    if rep is not None:
        with open(base + ".report.json", "w") as f:
            json.dump({"name": a.name, "gpus": a.gpus, "rc": rc, "command": cmd, "report": rep}, f, indent=1)
    return rc


if __name__ == "__main__":
    raise SystemExit(main())
