"""Run one JSON-configured bench: start this framework's completion server on a loopback port,
run `bench.run` against it, and stop only the server this run started (the reference's
`tools/weight-space/launch.py:14-91` role, for our server instead of llama-server).

    python -m dllm_qwen38_b200.weight_space.launch CONFIG.json

CONFIG: {"model": HF_DIR, "model_sha256": H, "output": RUN_DIR, "data": SPLIT.json, "condition": NAME,
         "backend_commit": C, "port": 17977, "tokenizer": HF_DIR|"bytes", "block": 32, "threshold": 0.9,
         "sub_block": 0, "n_ctx": 8192, "limit": 0, "max_tokens": 1024, "thinking": "off", "seed": 42,
         "request_timeout": 600, "startup_timeout": 300, "engine_sha256": optional}
The engine identity is the SHA-256 over the server module and the loaded native extension; when
the config names one it must match. RUN_DIR/launch.json pins the config (a changed config needs a
new directory); RUN_DIR/process-status.json records the state, the server's exit code and that it
was stopped; RUN_DIR/engine.log holds the server's output.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import socket
import subprocess
import sys
import time

from . import bench
from .common import canonical, digest, digest_tree, write_new


def engine_identity() -> str:
    root = pathlib.Path(__file__).resolve().parent.parent
    parts = {"server": digest(pathlib.Path(__file__).with_name("server.py"))}
    for so in sorted(root.glob("_C*.so")):
        parts[so.name] = digest(so)
    return canonical(parts)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("config", type=pathlib.Path)
    a = p.parse_args(argv)
    cfg = json.loads(a.config.read_text())
    eng = engine_identity()
    if cfg.get("engine_sha256") and cfg["engine_sha256"] != eng:
        raise ValueError("engine checksum mismatch")
    if digest_tree(cfg["model"]) != cfg["model_sha256"]:
        raise ValueError("model checksum mismatch")
    port = int(cfg.get("port", 17977))
    with socket.socket() as sk:  # the port must be free before anything starts
        sk.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        sk.bind(("127.0.0.1", port))
    out = pathlib.Path(cfg["output"])
    out.mkdir(parents=True, exist_ok=True)
    lf = out / "launch.json"
    if lf.exists():
        if json.loads(lf.read_text())["config"] != cfg:
            raise ValueError("launch config changed; use a new output directory")
    else:
        write_new(lf, {"config": cfg, "engine_sha256": eng, "launcher_sha256": digest(__file__)})
    cmd = [sys.executable, "-m", "dllm_qwen38_b200.weight_space.server", "--model", cfg["model"], "--port", str(port),
           "--tokenizer", cfg.get("tokenizer", cfg["model"]), "--block", str(cfg.get("block", 32)),
           "--threshold", str(cfg.get("threshold", 0.9)), "--sub-block", str(cfg.get("sub_block", 0)),
           "--n-ctx", str(cfg.get("n_ctx", 8192))]
    base = f"http://127.0.0.1:{port}"
    status = {"started_utc": datetime.datetime.now(datetime.timezone.utc).isoformat(), "command": cmd,
              "state": "starting", "engine_sha256": eng}
    sf = out / "process-status.json"

    def save():
        sf.write_text(json.dumps(status, indent=2) + "\n")

    env = dict(os.environ, PYTHONPATH=str(pathlib.Path(__file__).resolve().parents[2]) + os.pathsep +
               os.environ.get("PYTHONPATH", ""))
    with (out / "engine.log").open("a") as log:
        proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, env=env)
        status["pid"] = proc.pid
        save()
        try:
            deadline = time.monotonic() + float(cfg.get("startup_timeout", 300))
            while True:
                if proc.poll() is not None:
                    raise RuntimeError(f"server exited {proc.returncode}; see engine.log")
                try:
                    bench.request(base, "/health", timeout=2)
                    break
                except Exception:  # noqa: BLE001
                    if time.monotonic() >= deadline:
                        raise TimeoutError("server startup deadline; see engine.log") from None
                    time.sleep(0.5)
            status["state"] = "running"
            save()
            bench.run(argparse.Namespace(
                server=base, model=cfg["model"], model_sha256=cfg["model_sha256"], backend_commit=cfg["backend_commit"],
                condition=cfg["condition"], data=cfg["data"], output=str(out), limit=cfg.get("limit", 0),
                max_tokens=cfg.get("max_tokens", 1024), thinking=cfg.get("thinking", "off"), seed=cfg.get("seed", 42),
                timeout=cfg.get("request_timeout", 600)))
            status["state"] = "completed"
        except BaseException as e:
            status["state"] = "incomplete"
            status["error"] = str(e)
            raise
        finally:
            proc.terminate()
            try:
                proc.wait(timeout=15)
            except subprocess.TimeoutExpired:
                proc.kill()
                proc.wait()
            status.update(engine_exit_code=proc.returncode, engine_stopped=True,
                          ended_utc=datetime.datetime.now(datetime.timezone.utc).isoformat())
            save()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
