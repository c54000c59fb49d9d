"""Flagship benchmark: block-diffusion training throughput on the 27B-shape hybrid.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Metric: unique sequence tokens per second (batch x L per step; neither the two complementary
views nor the x_t||x_0 doubling counted, the reference's unit), whole job, plus MFU.
Config: 27B-shape hybrid (hidden 5120, FFN 17408, GDN 16/48 heads of 128, attention 24/4 of 256,
vocab 248320). Depth per N (`--layers`, default `auto`): all 64 layers (48 GDN + 16 attention) at
N = 8, the full 27B configuration; 16 layers (12 GDN + 4 attention) at N = 1, 2 and 4, a 3:1
truncation that fits one GPU (27B parameters need 378 GB of fp32 master weights, AdamW moments and
bf16 shards, more than one GPU holds), so N = 1 -> 4 is a clean weak-scaling curve at fixed
per-GPU work and N = 8 is the headline configuration. Seq 4096 per stream (x_t||x_0 = 8192),
block 32, micro-batch 1 sequence per GPU (global batch = N), activation checkpointing, AdamW, bf16
compute, random init, synthetic uniform token ids.

Timing: W untimed warm-up steps; then K steps between a barrier + synchronize on both sides,
timed with CUDA events on the compute stream; the reported time is the max over ranks. L2 is
flushed (a 256 MiB write) before every timed step. Clocks and throttle reasons are sampled with
nvidia-smi during the timed region. A second loop of K steps measures the same metric end to end
through the public API (`Trainer.step`): each step copies its inputs host->device from pinned
memory and reads the loss back, timed by the host clock.

The reference arm runs the unmodified reference package from baseline/_ref through its own
FSDP trainer (`build_and_shard` + `train_fsdp`, `fsdp_train.py:133-171,544-716`) on the same
config, with two environment adapters and no edit of the reference: transformers 5.5 here ships
`causal_conv1d_fn = None` where the reference's pinned transformers (>= 5.17) provides a callable,
so a torch depthwise conv + SiLU is installed as that callable; and torch 2.11 names one FSDP
state attribute differently from the torch the reference was written against (see
`_install_fsdp_state_adapter`).
"""

from __future__ import annotations

import argparse
import datetime
import faulthandler
import json
import os
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
BASELINE_SEQ_TOK_S = 1233.12  # the reference's published 27B FSDP production run (8 x H200, full 64 layers)
METRIC = "block-diff train tok/s & MFU, 27B FSDP 1/2/4/8 B200"


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops_sustained"]) * 1e12, "measured-sustained"
    except Exception:  # noqa: BLE001
        return 1.4e15, "fallback"


def _dist_setup(n: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1 or os.environ.get("MASTER_ADDR"):
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, local


def _barrier():
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(x: float) -> float:
    if dist.is_initialized():
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def model_flops_per_step(cfg, L: int, seqs: int) -> float:
    """Model FLOPs (no recompute) per optimizer step for `seqs` sequences of length L: dense
    layers over 4 token streams per sequence (2 views x {x_t, x_0}), masked-row lm_head over L
    rows per sequence, complementary-mask attention (about L^2 allowed pairs per view), fwd+bwd."""
    dense = cfg.param_count(embeddings=False)
    tokens = 4 * L * seqs
    f = 6.0 * dense * tokens
    f += 6.0 * cfg.hidden_size * cfg.vocab_size * L * seqs
    n_attn = sum(1 for t in cfg.layer_types if t == "full_attention")
    f += 12.0 * cfg.head_dim * cfg.num_attention_heads * (L * L) * 2 * seqs * n_attn
    return f


# ----------------------------------------------------------------------------- native arm


def run_native(a, rank, world):
    sys.path.insert(0, ROOT)
    from dllm_qwen38_b200 import ops
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model
    from dllm_qwen38_b200.ops import cuda as C
    from dllm_qwen38_b200.train.trainer import Trainer

    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = preset(a.model, layers=a.layers)
    model = build_model(cfg, seed=a.seed, device=dev, dtype=torch.bfloat16)
    if a.engine == "fsdp":
        from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

        trainer = FSDPTrainer(model, block=a.block, mask_id=cfg.mask_id, lr=a.lr)
        del model
        parallel = f"fsdp{world}"
    elif world > 1:
        from dllm_qwen38_b200.parallel.dp import ReplicatedDP

        trainer = ReplicatedDP(model, block=a.block, mask_id=cfg.mask_id, lr=a.lr, checkpointing=not a.no_ckpt,
                               seed=a.seed, rank=rank, world=world)
        parallel = f"dp{world}-replicated"
    else:
        trainer = Trainer(model, block=a.block, mask_id=cfg.mask_id, lr=a.lr, checkpointing=not a.no_ckpt,
                          seed=a.seed, rank=rank)
        parallel = "single"
    torch.cuda.empty_cache()
    g = torch.Generator().manual_seed(a.seed + rank)
    B, L = a.micro_batch, a.seq_len
    host_x = [torch.randint(0, cfg.mask_id, (B, L), generator=g).pin_memory() for _ in range(2)]
    pl = torch.zeros(B, dtype=torch.long).pin_memory()
    vl = torch.full((B,), L, dtype=torch.long).pin_memory()
    n_t = B * L
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)

    for i in range(a.warmup):
        trainer.step(host_x[i % 2], pl, vl, n_targets=n_t)
    torch.cuda.synchronize()
    C.check_errors()

    from dllm_qwen38_b200.utils.clocks import ClockSampler

    sampler = ClockSampler(gpu=torch.cuda.current_device()).start()
    _barrier()
    C.LAUNCHES[0] = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    losses = []
    ev0.record()
    for i in range(a.steps):
        flush.fill_(i & 0xFF)
        losses.append(trainer.step(host_x[i % 2], pl, vl, n_targets=n_t))
    ev1.record()
    _barrier()
    launches = C.LAUNCHES[0]
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1) / a.steps
    ms = _max_over_ranks(ms)
    C.check_errors()
    loss_last = float(losses[-1])

    # end-to-end: host clock, pinned H2D of inputs and a D2H loss read every step
    _barrier()
    t0 = time.perf_counter()
    for i in range(a.steps):
        loss = trainer.step(host_x[i % 2], pl, vl, n_targets=n_t)
        loss_host = float(loss.to("cpu"))
    _barrier()
    e2e_s = _max_over_ranks((time.perf_counter() - t0) / a.steps)
    del loss_host
    if dist.is_initialized():  # each rank's loss is its share of the global mean CE
        t = torch.tensor([loss_last], device="cuda", dtype=torch.float64)
        dist.all_reduce(t)
        loss_last = float(t.item())
    ckpt_policy = "per layer" if not a.no_ckpt else "off"
    if hasattr(trainer, "engine"):
        eng = trainer.engine
        kept = ["GDN core outputs and block states", "attention outputs and LSE"] if eng.save_cores else []
        sg = getattr(eng, "save_gemms", "0")
        mlp = "MLP gate|up and activation" if getattr(eng, "keep_act", False) else \
            "MLP gate|up (activation rebuilt in the backward)"
        if sg == "1":
            kept.append(f"projection GEMM outputs and {mlp}")
        elif sg.isdigit() and sg != "0":
            kept.append(f"projection GEMM outputs and {mlp} of the first {sg} of {len(eng.layers)} layers")
        if kept:
            ckpt_policy = "per layer; the forward keeps " + ", ".join(kept) + " for the backward"
        eng.close()
    h2d = host_x[0].numel() * host_x[0].element_size() + pl.numel() * 8 + vl.numel() * 8
    return {
        "ms_per_step": ms, "e2e_s_per_step": e2e_s, "launches": launches, "clocks": clocks, "cfg": cfg,
        "parallel": parallel, "loss_last": loss_last, "h2d": h2d, "d2h": 4, "impl": ops.last_impl(),
        "ckpt_policy": ckpt_policy,
        "peak_mem_gib": round(torch.cuda.max_memory_allocated() / 2**30, 2),
    }


# ----------------------------------------------------------------------------- reference arm


def _install_conv_adapter(gdn_mod):
    import torch.nn.functional as F

    def causal_conv1d_fn(x, weight, bias=None, activation=None, **_):
        # x [B, C, T], weight [C, K]: depthwise causal conv (+ SiLU), the transformers>=5.17 fallback
        K = weight.shape[-1]
        y = F.conv1d(F.pad(x, (K - 1, 0)), weight[:, None, :].to(x.dtype), bias, groups=x.shape[1])
        return F.silu(y) if activation in ("silu", "swish") else y

    gdn_mod.causal_conv1d_fn = causal_conv1d_fn


def _install_fsdp_state_adapter():
    """The reference reads `FSDPState._fsdp_param_groups` (a list; torch 2.14 per its own
    docstring, `fsdp_train.py:13-14`); torch 2.11 here keeps one optional `_fsdp_param_group`.
    A read-only property maps one onto the other; nothing of the reference is edited."""
    from torch.distributed.fsdp._fully_shard._fsdp_state import FSDPState

    if not hasattr(FSDPState, "_fsdp_param_groups"):
        FSDPState._fsdp_param_groups = property(
            lambda self: [self._fsdp_param_group] if self._fsdp_param_group is not None else [])


def _install_reference(ref_root: str, rank: int) -> None:
    """Offline install of the reference package into `ref_root` when it is missing and its source
    tree is named by BDLLM_REFERENCE_SRC: pip from a scratch copy (the build writes into its
    source tree), no index, no dependency resolution (every dependency is already importable).
    Rank 0 installs; the other ranks wait for its marker file."""
    src = os.environ.get("BDLLM_REFERENCE_SRC", "")
    if not src or not os.path.isfile(os.path.join(src, "pyproject.toml")):
        return
    done = ref_root + ".installed"
    if rank == 0:
        import shutil
        import subprocess
        import tempfile

        with tempfile.TemporaryDirectory() as tmp:
            copy = os.path.join(tmp, "src")
            shutil.copytree(src, copy)
            cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                   "--find-links", "/opt/wheelhouse", "--target", ref_root, copy]
            rc = subprocess.run(cmd, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, text=True).returncode
        with open(done, "w") as f:
            f.write(str(rc))
    else:
        for _ in range(600):
            if os.path.exists(done):
                break
            time.sleep(1.0)


def run_reference(a, rank, world):
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "dllm_qwen38")):
        _install_reference(ref_root, rank)
    if not os.path.isdir(os.path.join(ref_root, "dllm_qwen38")):
        return {"unavailable": "baseline/_ref not installed (pip install --no-deps --target baseline/_ref)"}
    sys.path.insert(0, ref_root)
    import dllm_qwen38.gdn as rgdn
    from dllm_qwen38 import fsdp_train as ft
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

    _install_conv_adapter(rgdn)
    _install_fsdp_state_adapter()
    rgdn.set_impl("torch")  # the reference's fsdp default (`--gdn torch`)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29534")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    sys.path.insert(0, ROOT)
    from dllm_qwen38_b200.config import preset

    c = preset(a.model, layers=a.layers)
    hc = Qwen3_5TextConfig(
        vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
        num_hidden_layers=c.num_hidden_layers, layer_types=list(c.layer_types),
        num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim,
        linear_num_key_heads=c.linear_num_key_heads, linear_num_value_heads=c.linear_num_value_heads,
        linear_key_head_dim=c.linear_key_head_dim, linear_value_head_dim=c.linear_value_head_dim,
        linear_conv_kernel_dim=c.linear_conv_kernel_dim, rms_norm_eps=c.rms_norm_eps, max_position_embeddings=8192,
        rope_parameters={"rope_type": "default", "rope_theta": c.rope_theta, "mrope_section": [11, 11, 10],
                         "partial_rotary_factor": c.partial_rotary_factor},
        attn_implementation="sdpa",
    )
    torch.manual_seed(a.seed)
    with torch.device("cuda"):
        text_model = Qwen3_5TextModel(hc).to(torch.bfloat16)
        lm_head = torch.nn.Linear(c.hidden_size, c.vocab_size, bias=False).to(torch.bfloat16)
    steps = ft.build_and_shard(text_model, None)
    uniq, names = ft._unique_params(text_model, lm_head)
    for p in uniq:
        p.requires_grad_(True)
    opt = torch.optim.AdamW(uniq, lr=a.lr, betas=(0.9, 0.95), weight_decay=0.0, foreach=False)
    L = a.seq_len

    def batches():
        g = torch.Generator().manual_seed(a.seed)
        while True:
            yield (torch.randint(0, c.mask_id, (world * a.micro_batch, L), generator=g),
                   torch.zeros(world * a.micro_batch, dtype=torch.long),
                   torch.full((world * a.micro_batch,), L, dtype=torch.long))

    it = batches()
    quiet = lambda *_a, **_k: None  # noqa: E731
    ft.train_fsdp(text_model, lm_head, steps, it, opt=opt, uniq=uniq, uniq_names=names, block=a.block,
                  mask_id=c.mask_id, n_steps=a.warmup, start_step=0, checkpointing=not a.no_ckpt, log=quiet,
                  log_every=10**9)
    from dllm_qwen38_b200.utils.clocks import ClockSampler

    sampler = ClockSampler(gpu=torch.cuda.current_device()).start()
    _barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    rep = ft.train_fsdp(text_model, lm_head, steps, it, opt=opt, uniq=uniq, uniq_names=names, block=a.block,
                        mask_id=c.mask_id, n_steps=a.steps, start_step=a.warmup, checkpointing=not a.no_ckpt,
                        log=quiet, log_every=10**9)
    ev1.record()
    _barrier()
    clocks = sampler.stop()
    ms = _max_over_ranks(ev0.elapsed_time(ev1) / a.steps)
    return {"ms_per_step": ms, "e2e_s_per_step": _max_over_ranks(rep["seconds"] / a.steps), "launches": None,
            "clocks": clocks, "cfg": c, "parallel": f"fsdp{world}", "loss_last": rep["loss_last"],
            "h2d": L * 8 * world * a.micro_batch + 16, "d2h": 4, "impl": {"gdn": rep["gdn_impl"]},
            "peak_mem_gib": rep["peak_mem_gib"]}


# ----------------------------------------------------------------------------- main


def main(argv=None) -> int:
    faulthandler.enable()  # a fatal signal in any rank prints every thread's Python stack
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--model", default="27b")
    p.add_argument("--layers", default="auto",
                   help="decoder layers: an int, or auto = 64 at 8 GPUs, else 16 (27b model)")
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--micro-batch", type=int, default=1)
    p.add_argument("--lr", type=float, default=1e-5)
    p.add_argument("--no-ckpt", action="store_true")
    p.add_argument("--engine", default="fsdp", choices=["fsdp", "module"],
                   help="native arm: the sharded engine (default, every N) or the module trainer")
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    if a.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if a.layers == "auto":
        a.layers = (64 if a.gpus >= 8 else 16) if a.model == "27b" else None
    else:
        a.layers = int(a.layers)
    rank, world, _ = _dist_setup(a.gpus)
    try:
        r = run_reference(a, rank, world) if a.impl == "reference" else run_native(a, rank, world)
    except torch.OutOfMemoryError as e:
        r = {"unavailable": f"out of memory: {str(e).splitlines()[0][:160]}"}
    if "unavailable" in r:
        if rank == 0:
            print(json.dumps({"impl": a.impl, "unavailable": r["unavailable"]}), flush=True)
        if dist.is_initialized():
            dist.destroy_process_group()
        return 0
    cfg = r["cfg"]
    seqs = world * a.micro_batch
    value = seqs * a.seq_len / (r["ms_per_step"] / 1e3)
    peak, peak_src = _peaks()
    mfu = model_flops_per_step(cfg, a.seq_len, seqs) / (r["ms_per_step"] / 1e3) / (peak * world)
    proxy_mfu = 24 * cfg.param_count() * value / (world * peak)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "seq-tok/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(r["ms_per_step"], 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(value / BASELINE_SEQ_TOK_S, 4) if (cfg.num_hidden_layers == 64 and world == 8) else None,
        "dtype": "bf16",
        "data": "synthetic uniform token ids, random-init weights (seed 0)",
        "config": {
            "model": f"27b-shape hybrid, {cfg.num_hidden_layers} of 64 layers" if a.model == "27b" else a.model,
            "depth_per_n": "64 layers at 8 GPUs, 16 at 1, 2 and 4 (per-GPU work grows 4x at 8 GPUs)",
            "global_batch": seqs, "seq_len": a.seq_len, "block": a.block, "micro_batch_per_gpu": a.micro_batch,
            "parallelism": r["parallel"], "activation_checkpointing": r.get("ckpt_policy", not a.no_ckpt), "optimizer": "AdamW lr 1e-5",
            "l2": "flushed (256 MiB write) before every timed step; step working set >> L2",
        },
        "mfu": round(mfu, 4), "proxy_mfu_24N": round(proxy_mfu, 4), "peak_flops_source": peak_src,
        "clocks": r["clocks"],
        "e2e": {"value": round(seqs * a.seq_len / r["e2e_s_per_step"], 2), "unit": "seq-tok/s",
                "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
        "gpu_launches": r["launches"],
        "loss_last": r["loss_last"],
        "peak_mem_gib": r["peak_mem_gib"],
        "paths": r["impl"],
    }
    if a.impl == "reference":
        line["impl"] = "reference"
        line["vs_baseline"] = None
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
