"""Run the boxed-answer scorer in a child process with a wall-clock deadline (the reference's
`tools/weight-space/symbolic_process.py` role): a pathological prediction can cost at most
`timeout_seconds`, after which the case is "grader_unavailable" (correct None), never "wrong".
Only the scorer's fixed result fields cross the process boundary."""

from __future__ import annotations

import json
import math
import subprocess
import sys

from .symbolic_score import MAX_GOLD, MAX_PRED, PROFILE, score

_FIELDS = {"profile", "status", "correct", "error_type", "reason"}


def _unavailable(reason: str) -> dict:
    return {"profile": PROFILE, "status": "grader_unavailable", "correct": None, "reason": reason}


def score_isolated(gold: str, content: str, *, thinking_open: bool = False, timeout_seconds: float = 20.0) -> dict:
    if not isinstance(gold, str) or not gold or len(gold.encode()) > MAX_GOLD:
        raise ValueError("invalid_reference_size")
    if not isinstance(content, str):
        raise ValueError("invalid_prediction_type")
    if len(content.encode()) > MAX_PRED:
        return {"profile": PROFILE, "status": "prediction_too_long", "correct": False}
    if not isinstance(thinking_open, bool):
        raise ValueError("invalid_thinking_state")
    if not isinstance(timeout_seconds, (int, float)) or not math.isfinite(timeout_seconds) or not (
            0 < timeout_seconds <= 60):
        raise ValueError("invalid_timeout")
    req = json.dumps({"gold": gold, "content": content, "thinking_open": thinking_open})
    cmd = [sys.executable, "-m", "dllm_qwen38_b200.weight_space.symbolic_process", "--worker"]
    with subprocess.Popen(cmd, stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                          text=True) as child:
        try:
            out, _ = child.communicate(req, timeout=timeout_seconds)
        except subprocess.TimeoutExpired:
            child.kill()
            child.communicate()
            return _unavailable("process_timeout")
        if child.returncode:
            return _unavailable("process_exit")
    try:
        res = json.loads(out)
        if set(res) - _FIELDS or res["profile"] != PROFILE or not isinstance(res["status"], str) or not (
                res["correct"] is None or type(res["correct"]) is bool):
            raise ValueError
    except (ValueError, KeyError, TypeError):
        return _unavailable("invalid_process_result")
    return res


def _worker() -> None:
    try:
        req = json.loads(sys.stdin.read(MAX_PRED * 4 + MAX_GOLD * 4 + 1024))
        res = score(req["gold"], req["content"], thinking_open=req["thinking_open"])
    except Exception as e:  # noqa: BLE001
        res = _unavailable("worker_exception")
        res["error_type"] = type(e).__name__
    print(json.dumps(res))


if __name__ == "__main__":
    if sys.argv[1:] != ["--worker"]:
        raise SystemExit("use score_isolated(); this entry point is the scorer's child process")
    _worker()
