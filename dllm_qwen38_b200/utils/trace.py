"""NVTX ranges around layers, fused collectives and decode steps (`BDLLM_NVTX=1`), for Nsight
timelines; a no-op otherwise (no per-call cost beyond one dict lookup)."""

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
