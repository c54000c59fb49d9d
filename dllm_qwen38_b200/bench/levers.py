"""One-lever-at-a-time training benchmark (the reference's lever bench, `modal_app.py:95-163`,
`README.md:105-125`): the same model, data and step, with one change per leg.

    python -m dllm_qwen38_b200.bench.levers [--model 0.8b] [--batch 4] [--seq-len 512] [--steps 8]

Legs: all native kernels; each native kernel family swapped for its torch path on the device
(`ops.torch_on_cuda`: GEMMs -> cuBLAS, attention -> SDPA with a boolean mask, GDN core / conv /
norms -> torch); activation checkpointing off; batch x2. Each leg prints one LEG line with
seq-tok/s (device-timed with CUDA events) and peak memory, then one JSON summary.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

LEGS = [
    ("native", (), {}),
    ("gemm->cublas", ("linear", "mlp", "masked_ce"), {}),
    ("attention->sdpa", ("attention",), {}),
    ("gdn_core->torch", ("gdn_core",), {}),
    ("conv->torch", ("conv",), {}),
    ("norms->torch", ("rmsnorm", "gated_rmsnorm", "qk_norm_rope"), {}),
    ("no-checkpointing", (), {"checkpointing": False}),
    ("batch-x2", (), {"batch_mult": 2}),
]


def run_leg(a, ops_off, opts):
    from dllm_qwen38_b200 import ops
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model
    from dllm_qwen38_b200.train.trainer import Trainer

    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    cfg = preset(a.model, layers=a.layers)
    model = build_model(cfg, seed=0, device="cuda", dtype=torch.bfloat16)
    tr = Trainer(model, block=a.block, mask_id=cfg.mask_id, lr=1e-5, checkpointing=opts.get("checkpointing", True),
                 seed=0)
    B = a.batch * opts.get("batch_mult", 1)
    g = torch.Generator().manual_seed(0)
    x = torch.randint(0, cfg.mask_id, (B, a.seq_len), generator=g)
    pl = torch.zeros(B, dtype=torch.long)
    vl = torch.full((B,), a.seq_len, dtype=torch.long)
    with ops.torch_on_cuda(*ops_off):
        for _ in range(a.warmup):
            tr.step(x, pl, vl)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            tr.step(x, pl, vl)
        e1.record()
        torch.cuda.synchronize()
        impl = ops.last_impl()
    s = e0.elapsed_time(e1) / 1e3
    res = {"seq_tok_s": round(B * a.seq_len * a.steps / s, 1), "ms_per_step": round(1e3 * s / a.steps, 2),
           "peak_gib": round(torch.cuda.max_memory_allocated() / 2**30, 2), "batch": B,
           "torch_paths": sorted(k for k, v in impl.items() if v == "torch-cuda")}
    del tr, model
    return res


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="0.8b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--legs", default=",".join(name for name, _, _ in LEGS))
    a = p.parse_args(argv)
    sys.path.insert(0, ROOT)
    want = set(a.legs.split(","))
    out = {}
    for name, ops_off, opts in LEGS:
        if name not in want:
            continue
        try:
            r = run_leg(a, ops_off, opts)
        except torch.OutOfMemoryError as e:
            r = {"oom": str(e).splitlines()[0]}
            torch.cuda.empty_cache()
        out[name] = r
        print(f"LEG\t{name}\t{json.dumps(r)}", flush=True)
    print(json.dumps({"bench": "levers", "model": a.model, "seq_len": a.seq_len, "legs": out}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
