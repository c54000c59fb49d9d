"""The boxed-answer scorer behind a process boundary with a per-case deadline (the role of the
reference's `tools/weight-space/symbolic_process.py:12-74`).

A symbolic comparison can run away on a hostile prediction, so the scorer runs in a separate
process. One long-lived child serves every case of a run through a pipe (starting a Python
process per case would dominate a bench's scoring time); when a case overruns its deadline the
child is killed and the next case starts a fresh one. A case that overruns, or whose child dies
or answers with anything but the scorer's fixed result fields, is reported as
"grader_unavailable" with correct None, never as wrong. The validation codes and result fields
are the reference's contract (`invalid_reference_size`, `invalid_prediction_type`,
`invalid_thinking_state`, `invalid_timeout`; `process_timeout`, `process_exit`,
`invalid_process_result`, `worker_exception`).
"""

from __future__ import annotations

import math
import multiprocessing as mp
import threading

from .symbolic_score import MAX_GOLD, MAX_PRED, PROFILE, score

RESULT_FIELDS = frozenset({"profile", "status", "correct", "error_type", "reason"})


def _unavailable(reason: str, **extra) -> dict:
    return {"profile": PROFILE, "status": "grader_unavailable", "correct": None, "reason": reason, **extra}


def _serve(conn) -> None:
    """Child loop: one request dict in, one result dict out, until the pipe closes."""
    while True:
        try:
            req = conn.recv()
        except (EOFError, OSError):
            return
        try:
            res = score(req["gold"], req["content"], thinking_open=req["thinking_open"])
        except Exception as e:  # noqa: BLE001 - any scorer failure is the case's, not the run's
            res = _unavailable("worker_exception", error_type=type(e).__name__)
        conn.send(res)


def _well_formed(res) -> bool:
    return (isinstance(res, dict) and not (set(res) - RESULT_FIELDS) and res.get("profile") == PROFILE
            and isinstance(res.get("status"), str) and (res.get("correct") is None or type(res["correct"]) is bool))


def _request_error(gold, content, thinking_open, timeout_seconds):
    """The contract's argument checks, in order: the first failing check's code, or None."""
    if not isinstance(gold, str) or not gold or len(gold.encode()) > MAX_GOLD:
        return "invalid_reference_size"
    if not isinstance(content, str):
        return "invalid_prediction_type"
    if len(content.encode()) > MAX_PRED:
        return "prediction_too_long"  # a result, not an error
    if not isinstance(thinking_open, bool):
        return "invalid_thinking_state"
    if isinstance(timeout_seconds, bool) or not isinstance(timeout_seconds, (int, float)) or \
            not math.isfinite(timeout_seconds) or not 0 < timeout_seconds <= 60:
        return "invalid_timeout"
    return None


class IsolatedScorer:
    """A scorer child process reused across cases, restarted after a timeout or a crash."""

    def __init__(self):
        self._ctx = mp.get_context("spawn")
        self._proc = None
        self._conn = None
        self._lock = threading.Lock()

    def _ensure(self) -> None:
        if self._proc is not None and self._proc.is_alive():
            return
        self.close()
        parent, child = self._ctx.Pipe()
        self._proc = self._ctx.Process(target=_serve, args=(child,), daemon=True)
        self._proc.start()
        child.close()
        self._conn = parent

    def close(self) -> None:
        if self._proc is not None:
            if self._proc.is_alive():
                self._proc.kill()
            self._proc.join(5)
        if self._conn is not None:
            self._conn.close()
        self._proc = self._conn = None

    def score(self, gold: str, content: str, *, thinking_open: bool = False, timeout_seconds: float = 20.0) -> dict:
        code = _request_error(gold, content, thinking_open, timeout_seconds)
        if code == "prediction_too_long":
            return {"profile": PROFILE, "status": code, "correct": False}
        if code is not None:
            raise ValueError(code)
        with self._lock:
            self._ensure()
            try:
                self._conn.send({"gold": gold, "content": content, "thinking_open": thinking_open})
                if not self._conn.poll(timeout_seconds):
                    self.close()  # the runaway case takes its child with it
                    return _unavailable("process_timeout")
                res = self._conn.recv()
            except (EOFError, OSError):
                self.close()
                return _unavailable("process_exit")
        return res if _well_formed(res) else _unavailable("invalid_process_result")


_SHARED = IsolatedScorer()


def score_isolated(gold: str, content: str, *, thinking_open: bool = False, timeout_seconds: float = 20.0) -> dict:
    """Score one case in the shared child process with a deadline of `timeout_seconds` (0 < t <= 60)."""
    return _SHARED.score(gold, content, thinking_open=thinking_open, timeout_seconds=timeout_seconds)
