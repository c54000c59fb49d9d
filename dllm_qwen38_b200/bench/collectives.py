"""Fused collective paths over 27B layer shapes, as fractions of their roofline (one rank per GPU).
They replace the reference's FSDP2 per-unit all-gather and fp32 reduce-scatter
(`src/dllm_qwen38/fsdp_train.py:133-171`), which NCCL runs as separate calls.

    torchrun --nproc-per-node N -m dllm_qwen38_b200.bench.collectives [--iters 10]

For each 27B layer weight (GDN in-proj 16480x5120, attention qkv 14336x5120, MLP gate|up
34816x5120, down 5120x17408) and a unit-sized gradient (one GDN layer, ~383M elements):

  ag_gemm     fused all-gather -> GEMM (`_C.gemm_ag`): y = x W^T with W gathered from the peers'
              shards inside the GEMM, x = 8192 rows (seq 4096, both streams)
  ag_nccl     baseline: NCCL all_gather_into_tensor of the same shard, then the same GEMM
  rs_adam     fused reduce-scatter -> fp32 cast / scale -> AdamW (`_C.peer_reduce_scatter` with
              the optimizer state; the no-clip variant) of a bf16 flat gradient
  rs_nccl     baseline: NCCL reduce_scatter_tensor (fp32, AVG, as FSDP2 runs it) + AdamW launch

Roofline of a fused path = max(FLOPs / measured bf16 GEMM peak, bytes that must cross NVLink per
GPU / 770 GB/s (the measured per-direction peer copy bandwidth)); achieved fraction = roofline /
measured time. Times are CUDA-event device times per rank, max over ranks, median of `--iters`.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
NVLINK_GBS = 770.0

WEIGHTS = {"gdn_in_proj": (16480, 5120), "attn_qkv": (14336, 5120), "mlp_gate_up": (34816, 5120),
           "mlp_down": (5120, 17408)}


def _peak_flops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]) * 1e12
    except Exception:  # noqa: BLE001
        return 1.59e15


def _time(fn, iters):
    ts = []
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    t = torch.tensor([statistics.median(ts)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--rows", type=int, default=8192)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--unit", type=int, default=383_000_000, help="gradient elements of one unit")
    a = p.parse_args(argv)
    sys.path.insert(0, ROOT)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    W, r = dist.get_world_size(), dist.get_rank()
    from dllm_qwen38_b200.ops import cuda as Cu
    from dllm_qwen38_b200.parallel.peer import SymmetricHeap

    C = Cu._C
    dev = torch.device("cuda", local)
    peak = _peak_flops()
    biggest = max(n * k for n, k in WEIGHTS.values())
    shard_max = -(-biggest // W)
    shard_max = -(-shard_max // 64) * 64
    ushard = -(-a.unit // W)
    ushard = -(-ushard // 64) * 64
    heap = SymmetricHeap(shard_max * 2 + ushard * W * 2 + ushard * 2 + (1 << 20), dev)
    wshard, woff = heap.alloc(shard_max, torch.bfloat16)
    grad, goff = heap.alloc(ushard * W, torch.bfloat16)
    pshard, _ = heap.alloc(ushard, torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(r)
    wshard.normal_(generator=g)
    grad.normal_(generator=g)
    torch.cuda.synchronize()
    dist.barrier()
    x = torch.randn(a.rows, 5120, device=dev).bfloat16()
    gathered = torch.empty(shard_max * W, dtype=torch.bfloat16, device=dev)
    ready = torch.zeros(8192 + 64, dtype=torch.int32, device=dev)
    claim = torch.zeros(1, dtype=torch.int32, device=dev)
    seq = [0]
    rows = []
    for name, (n, k) in WEIGHTS.items():
        xk = x if k == 5120 else torch.randn(a.rows, k, device=dev).bfloat16()
        numel = n * k
        sb = -(-numel // W)
        sb = -(-sb // 64) * 64 * 2  # bytes of this weight's shard
        w = gathered[:numel].view(n, k)
        out = torch.empty(a.rows, n, dtype=torch.bfloat16, device=dev)

        def fused():
            seq[0] += 1
            C.gemm_ag(xk, w, out, 0, None, heap.ptrs, r, woff, sb, gathered, ready, claim, seq[0], 0, 0, 60.0)

        def nccl():
            dist.all_gather_into_tensor(gathered[: sb // 2 * W], wshard[: sb // 2])
            Cu.gemm_nt(xk, w, out=out)

        flops = 2.0 * a.rows * n * k
        link = sb * (W - 1) / 1e9 / NVLINK_GBS * 1e3  # ms: this rank pulls W-1 shards
        roof = max(flops / peak * 1e3, link)
        tf, tn = _time(fused, a.iters), _time(nccl, a.iters)
        rows.append({"path": "ag_gemm", "weight": name, "ms": round(tf, 3), "roofline_ms": round(roof, 3),
                     "frac_roofline": round(roof / tf, 3), "baseline_ms": round(tn, 3),
                     "speedup_vs_nccl": round(tn / tf, 3)})
    # reduce-scatter -> AdamW of one unit
    master = torch.randn(ushard, device=dev)
    m = torch.zeros(ushard, device=dev)
    v = torch.zeros(ushard, device=dev)
    gout = torch.empty(ushard, device=dev)
    sq = torch.zeros(1, device=dev)
    hp = (1e-5, 0.9, 0.95, 1e-8, 0.0, 0.1, 0.05)

    blocks = [2 * torch.cuda.get_device_properties(dev).multi_processor_count]

    def rs_fused():
        heap.reduce_scatter(goff, ushard, False, gout, 1.0 / W, sq, max_blocks=blocks[0],
                            adam=((master, m, v, pshard), hp))

    def rs_nccl():
        dist.reduce_scatter_tensor(gout, grad.float(), op=dist.ReduceOp.AVG)
        Cu.adamw_flat(master, pshard, gout, m, v, *hp[:5], 1.0, hp[5], hp[6])

    link = ushard * 2 * (W - 1) / 1e9 / NVLINK_GBS * 1e3
    # local HBM traffic: read+write fp32 master/m/v, write bf16 p, read this rank's own grad slice
    hbm = ushard * (24 + 2 + 2) / 6.5e12 * 1e3
    roof = max(link, hbm)
    tf, tn = _time(rs_fused, a.iters), _time(rs_nccl, a.iters)
    blocks[0] = 64  # the engine's setting: leaves most SMs to the overlapped backward
    t64 = _time(rs_fused, a.iters)
    rows.append({"path": "rs_adam", "unit_elems": a.unit, "ms": round(tf, 3), "roofline_ms": round(roof, 3),
                 "frac_roofline": round(roof / tf, 3), "baseline_ms": round(tn, 3),
                 "speedup_vs_nccl": round(tn / tf, 3), "ms_64_ctas_overlapped_setting": round(t64, 3)})
    C.read_error_word(False)
    if r == 0:
        for row in rows:
            print(json.dumps({"n_gpus": W, **row}), flush=True)
    heap.close()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
