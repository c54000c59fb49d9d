"""NVTX ranges around layers, fused collectives and decode steps (`BDLLM_NVTX=1`), for Nsight
timelines; a no-op otherwise (no per-call cost beyond one dict lookup). The reference has no
ranges of its own: it times loops with the host clock (`src/dllm_qwen38/train.py:145,165-166`)."""

from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("BDLLM_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx(name: str):
    if not ENABLED or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
