"""Where a training step's device time goes: one step of the flagship configuration under the torch
profiler (CUPTI kernel records, no replay), kernel times summed by name and by family.

    python -m dllm_qwen38_b200.bench.step_profile [--layers 16] [--seq-len 4096] [--top 40]

The step is the sharded engine's (`FSDPTrainer`, one rank), after three warm-up steps (the first
one decides which layers keep their GEMM outputs). Kernel times under the profiler are a share
breakdown, not a benchmark: `bench.py` times the step.
"""

from __future__ import annotations

import argparse
import collections
import sys
import time

import torch

# kernel-name fragments -> family (first match wins)
FAMILIES = (
    ("gemm", "GEMM (tcgen05)"),
    ("gdn", "state-fork GDN"),
    ("attn", "attention"),
    ("adamw", "AdamW"),
    ("norm", "norms"),
    ("conv", "causal conv"),
    ("swiglu", "SwiGLU element-wise"),
    ("ce_rows", "CE rows"),
    ("embed", "embedding"),
    ("gates", "GDN gates"),
    ("sumsq", "clip sum of squares"),
    ("colsum", "norms"),
    ("group_sum", "state-fork GDN"),
    ("out_gate", "attention"),
    ("at::native", "torch element-wise / copies"),
    ("Memcpy", "copies"),
)


def family(name: str) -> str:
    for frag, fam in FAMILIES:
        if frag in name:
            return fam
    return "other"


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="27b")
    p.add_argument("--layers", type=int, default=16)
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--top", type=int, default=40)
    a = p.parse_args(argv)

    from ..config import preset
    from ..models.qwen35 import build_model
    from ..parallel.fsdp import FSDPTrainer

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset(a.model, layers=a.layers)
    model = build_model(cfg, seed=0, device=dev, dtype=torch.bfloat16)
    tr = FSDPTrainer(model, block=a.block, mask_id=cfg.mask_id, lr=1e-5)
    del model
    torch.cuda.empty_cache()
    g = torch.Generator().manual_seed(0)
    x = torch.randint(0, cfg.mask_id, (1, a.seq_len), generator=g).pin_memory()
    pl = torch.zeros(1, dtype=torch.long).pin_memory()
    vl = torch.full((1,), a.seq_len, dtype=torch.long).pin_memory()
    for _ in range(a.warmup):
        tr.step(x, pl, vl, n_targets=a.seq_len)
    torch.cuda.synchronize()

    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        t0 = time.perf_counter()
        tr.step(x, pl, vl, n_targets=a.seq_len)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    by_name = collections.defaultdict(lambda: [0.0, 0])
    by_fam = collections.defaultdict(float)
    for e in evs:
        us = e.time_range.end - e.time_range.start
        rec = by_name[e.name]
        rec[0] += us
        rec[1] += 1
        by_fam[family(e.name)] += us
    total = sum(v[0] for v in by_name.values())
    span = (max(e.time_range.end for e in evs) - min(e.time_range.start for e in evs)) if evs else 0.0
    print(f"{a.model}, {a.layers} layers, seq {a.seq_len}: wall {wall * 1e3:.1f} ms, device span {span / 1e3:.1f} ms, "
          f"kernel time {total / 1e3:.1f} ms over {len(evs)} device records; GEMM outputs kept for "
          f"{tr.engine.save_gemms} layers ('1' = all)")
    print("\nby family:")
    for fam, us in sorted(by_fam.items(), key=lambda kv: -kv[1]):
        print(f"  {us / 1e3:9.2f} ms  {100 * us / max(total, 1e-9):5.1f} %  {fam}")
    print(f"\ntop {a.top} kernels:")
    for name, (us, n) in sorted(by_name.items(), key=lambda kv: -kv[1][0])[: a.top]:
        print(f"  {us / 1e3:9.2f} ms  {100 * us / max(total, 1e-9):5.1f} %  {n:5d}x  {name[:120]}")
    tr.engine.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
