"""Sharded (FSDP) block-diffusion training CLI — the reference's `fsdp_train.main` contract
(`fsdp_train.py:719-901`) on this framework's engine.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m dllm_qwen38_b200.train.fsdp_train \\
        --model 27b --data random --seq-len 4096 --batch 8 --steps 100 --ckpt-dir /ckpt

* Every rank draws the same GLOBAL batch iterator and keeps rows [rank*b, (rank+1)*b)
  (`fsdp_train.py:600-606`); masks are seeded per (global step, rank).
* Windowed resume: `--resume` loads the latest committed checkpoint, verifies its fingerprints
  (fails closed: a restore that cannot be proven bit-exact refuses to train, exit 1), replays the
  data stream by draining `step` batches, and continues the global step numbering.
* `--resume-selftest`: an uninterrupted window with a mid-window save, then a cold rebuild that
  resumes from the midpoint; the gate is fingerprint match + seq_tokens continuity + the resumed
  losses inside a 5e-3 band of the uninterrupted ones (`fsdp_train.py:375,822-883`).
* Weight-spread probe: fp64 checksums of every gathered parameter, MIN/MAX over ranks; exit 0 only
  with a finite loss and zero spread (`fsdp_train.py:667-692,891`).
Exit codes: 0 ok, 1 a gate failed, 2 could not measure.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time

import torch
import torch.distributed as dist

from .. import ops
from ..io import ckpt
from ..utils import mem

RESUME_LOSS_BAND = 5e-3


def _init_dist():
    if "RANK" in os.environ and not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def _device():
    return f"cuda:{torch.cuda.current_device()}" if torch.cuda.is_available() else "cpu"


def make_batches(data: str, tok, cfg, batch: int, seq_len: int, block: int, seed: int, split: str = "chat"):
    from .single import chat_batches, random_batches, synthetic_batches

    if data == "synthetic":
        return synthetic_batches(batch, seq_len, cfg.vocab_size if tok is None else len(tok), block, seed)
    if data == "random":
        return random_batches(batch, seq_len, cfg.mask_id, seed)
    if tok is None:
        raise ValueError("a chat dataset needs a tokenizer (HF checkpoint directory)")
    return chat_batches(data, split, tok, batch, seq_len, block, seed)


def weight_spread(engine) -> tuple[float, list]:
    """Max over parameters of (max - min) across ranks of the fp64 checksum of the gathered value."""
    state = engine.full_state()
    names = sorted(state)
    cks = torch.stack([state[n].double().sum() for n in names])
    if dist.is_initialized() and dist.get_world_size() > 1:
        lo, hi = cks.clone(), cks.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        sp = hi - lo
    else:
        sp = torch.zeros_like(cks)
    bad = [(names[i], float(sp[i])) for i in (sp > 0).nonzero().flatten().tolist()]
    return float(sp.max()) if len(sp) else 0.0, bad


def train_window(trainer, batches, *, n_steps: int, start_step: int, seq_tokens_start: int, ckpt_dir, ckpt_every: int,
                 fingerprint_saves: str, log_every: int, mem_history: bool, log=print) -> dict:
    rank, world = trainer.rank, trainer.world
    engine = trainer.engine
    first, last = start_step + 1, start_step + n_steps
    trainer.gstep = start_step
    local = None
    losses, seq_tok, skipped = [], 0, 0
    t0 = time.time()
    if torch.cuda.is_available():
        torch.cuda.reset_peak_memory_stats()
    if mem_history and rank == 0:
        mem.start_history()
    for gstep in range(first, last + 1):
        local_step = gstep - start_step
        if mem_history and rank == 0 and local_step == 4:
            mem.stop_history()
        x0, pl, vl = next(batches)
        if local is None:
            if x0.shape[0] % world:
                raise ValueError(f"global batch {x0.shape[0]} not divisible by world {world}")
            local = x0.shape[0] // world
        sl = slice(rank * local, (rank + 1) * local)
        xr, pr, vr = x0[sl], pl[sl], vl[sl]
        n_local = int((vr - pr).clamp(min=0).sum())
        counts = torch.tensor([float(n_local)], device=engine.device)
        if world > 1:
            dist.all_reduce(counts)
        n_global = int(counts.item())
        if n_global == 0:  # every rank skips together (`fsdp_train.py:624-629`)
            skipped += 1
            trainer.gstep += 1
            continue
        try:  # a rank with no local target still steps (zero loss, zero gradients, same collectives)
            contrib = trainer.step(xr, pr, vr, n_targets=n_local, n_global=n_global)
        except torch.OutOfMemoryError:
            mem.on_oom(engine, rank, mem_history and rank == 0)
            raise
        loss = contrib.detach().float().reshape(1)
        if world > 1:
            dist.all_reduce(loss)
        losses.append(float(loss))
        seq_tok += xr.numel() * world
        if rank == 0 and local_step == 1:
            log(mem.mem_line("after step 1"))
        if ckpt_dir and ((ckpt_every and gstep % ckpt_every == 0) or gstep == last):
            ckpt.save_engine(engine, ckpt_dir, gstep, seq_tokens_start + seq_tok,
                             fingerprint_save=(gstep == last) or fingerprint_saves == "all")
        if rank == 0 and (local_step % log_every == 0 or local_step == n_steps):
            el = time.time() - t0
            log(f"step {gstep}\tloss {losses[-1]:.4f}\ttargets {n_global}\tseq-tok/s {seq_tok / el:.0f}\telapsed {el:.0f}s")
    el = time.time() - t0
    spread, bad = weight_spread(engine)
    if bad and rank == 0:
        log(f"WEIGHT-SPREAD\tdivergent {len(bad)}\t{bad[:8]}")
    peak = torch.tensor([float(torch.cuda.max_memory_allocated()) if torch.cuda.is_available() else 0.0],
                        device=engine.device)
    if world > 1:
        dist.all_reduce(peak, op=dist.ReduceOp.MAX)
    return {
        "steps": n_steps, "start_step": start_step, "skipped_steps": skipped, "world": world,
        "loss_first": losses[0] if losses else None, "loss_last": losses[-1] if losses else None,
        "loss_mean_last10": sum(losses[-10:]) / max(1, len(losses[-10:])), "losses": losses,
        "seq_tokens": seq_tokens_start + seq_tok, "seq_tokens_window": seq_tok,
        "seq_tokens_per_s": seq_tok / el if el else 0.0, "seconds": el,
        "peak_mem_gib": round(float(peak) / 2**30, 2), "weight_spread": spread, "divergent_params": bad[:8],
    }


def build(a, rank):
    from ..io.hf_load import load_model
    from ..parallel.fsdp import FSDPTrainer

    dtype = torch.bfloat16 if torch.cuda.is_available() else torch.float32
    model, tok = load_model(a.model, dtype=dtype, device=_device(), layers=a.layers, seed=a.seed)
    cfg = model.config
    mask_id = cfg.mask_id if tok is None else len(tok)
    trainer = FSDPTrainer(model, block=a.block, mask_id=mask_id, lr=a.lr)
    return trainer, tok, cfg


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="27b")
    p.add_argument("--data", default="random", help="'random', 'synthetic' or an HF chat dataset id")
    p.add_argument("--split", default="chat")
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--batch", type=int, default=4, help="GLOBAL rows per step, sliced across ranks")
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--lr", type=float, default=1e-5)
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--grad-checkpoint", action="store_true", help="accepted for compatibility: always on")
    p.add_argument("--mem-history", action="store_true")
    p.add_argument("--gdn", default="native", choices=["native", "auto", "torch", "fla"],
                   help="GDN core: native (= auto) runs the sm_100a kernels; torch runs the fp32 torch "
                        "chunked rule on the device (the reference's default path, for comparison); fla is "
                        "not part of this framework")
    p.add_argument("--attn", default="native", choices=list(ops.ATTN_CHOICES),
                   help="masked attention: native runs the sm_100a kernels; sdpa / eager run torch's "
                        "attention over the boolean mask on the device (for comparison)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--out", default=None)
    p.add_argument("--ckpt-dir", default=None)
    p.add_argument("--ckpt-every", type=int, default=0)
    p.add_argument("--resume", action="store_true")
    p.add_argument("--resume-selftest", action="store_true")
    p.add_argument("--ckpt-fingerprint", action="store_true")
    p.add_argument("--log-every", type=int, default=10)
    a = p.parse_args(argv)
    if a.seq_len % a.block:
        print("COULD-NOT-MEASURE seq-len must be a multiple of block", file=sys.stderr)
        return 2
    if a.resume_selftest and not a.ckpt_dir:
        print("COULD-NOT-MEASURE --resume-selftest needs --ckpt-dir", file=sys.stderr)
        return 2
    if a.gdn == "fla":
        print("COULD-NOT-MEASURE --gdn fla: fla's Triton kernel is not part of this framework (the native "
              "tcgen05 kernel replaces it); use --gdn native, or --gdn torch for the torch chunked rule",
              file=sys.stderr)
        return 2
    # the chosen GDN / attention paths for the whole run
    with ops.torch_paths(a.gdn, a.attn):
        return _run(a)


def _run(a) -> int:
    rank, world = _init_dist()
    say = print if rank == 0 else (lambda *_a, **_k: None)
    try:
        trainer, tok, cfg = build(a, rank)
    except Exception as e:  # noqa: BLE001
        print(f"COULD-NOT-MEASURE model build failed: {type(e).__name__}: {e}", file=sys.stderr)
        return 2
    say(mem.mem_line("after shard"))
    start_step, seq_tokens_start = 0, 0
    if a.resume:
        last = ckpt.latest_checkpoint(a.ckpt_dir) if a.ckpt_dir else None
        if last is None:
            print("COULD-NOT-MEASURE --resume found no committed checkpoint", file=sys.stderr)
            return 2
        info = ckpt.load_engine(trainer.engine, a.ckpt_dir, last, verify=True)
        if not info["fp_ok"]:
            print("CKPT-FP\trestore failed fingerprint verification -- refusing to train on it", file=sys.stderr)
            return 1
        start_step, seq_tokens_start = last, info["seq_tokens"]
        say(f"RESUME\tfrom step {start_step}\tseq_tokens {seq_tokens_start}")
    batches = make_batches(a.data, tok, cfg, a.batch, a.seq_len, a.block, a.seed, a.split)
    for _ in range(start_step):  # exact data replay
        next(batches)
    rep = train_window(trainer, batches, n_steps=a.steps, start_step=start_step, seq_tokens_start=seq_tokens_start,
                       ckpt_dir=a.ckpt_dir, ckpt_every=(a.steps // 2) if a.resume_selftest else a.ckpt_every,
                       fingerprint_saves="all" if a.resume_selftest else "window_end", log_every=a.log_every,
                       mem_history=a.mem_history, log=say)
    rep.update({"model": a.model, "data": a.data, "block": a.block, "seq_len": a.seq_len, "batch": a.batch,
                "lr": a.lr, "layers": a.layers, "engine": "fsdp", "world": world,
                "gdn": ops.last_impl("gdn_core"), "attn": ops.last_impl("attention")})  # the paths that ran
    ok = rep["loss_last"] is not None and math.isfinite(rep["loss_last"]) and rep["weight_spread"] == 0.0
    if a.resume_selftest:
        mid = a.steps // 2
        trainer2, _, _ = build(a, rank)
        info = ckpt.load_engine(trainer2.engine, a.ckpt_dir, mid, verify=True)
        b2 = make_batches(a.data, tok, cfg, a.batch, a.seq_len, a.block, a.seed, a.split)
        for _ in range(mid):
            next(b2)
        rep2 = train_window(trainer2, b2, n_steps=a.steps - mid, start_step=mid, seq_tokens_start=info["seq_tokens"],
                            ckpt_dir=None, ckpt_every=0, fingerprint_saves="window_end", log_every=a.log_every,
                            mem_history=False, log=say)
        ref, got = rep["losses"][mid:], rep2["losses"]
        diffs = [abs(x - y) for x, y in zip(ref, got)] if len(ref) == len(got) else None
        max_abs = max(diffs) if diffs else float("nan")
        st = {"fp_match": info["fp_ok"], "loss_band_ok": diffs is not None and max_abs <= RESUME_LOSS_BAND,
              "band": RESUME_LOSS_BAND, "n": len(got), "max_abs_diff": max_abs,
              "seq_tokens_match": rep["seq_tokens"] == rep2["seq_tokens"]}
        rep["resume_selftest"] = st
        say(f"SELFTEST\tfp_match {st['fp_match']}\tn {st['n']}\tmax_abs_diff {max_abs:.3g} (band {RESUME_LOSS_BAND:.1e})"
            f"\tseq_tokens_match {st['seq_tokens_match']}")
        ok = ok and st["fp_match"] and st["loss_band_ok"] and st["seq_tokens_match"]
    if rank == 0:
        say(f"TRAIN\tsteps {rep['steps']}\tskipped {rep['skipped_steps']}\tloss {rep['loss_first']} -> {rep['loss_last']}"
            f"\tseq-tok/s {rep['seq_tokens_per_s']:.0f}\tpeak_mem_gib {rep['peak_mem_gib']}\tweight_spread "
            f"{rep['weight_spread']:.3g}\t{rep['seconds']:.0f}s")
        if a.out:
            os.makedirs(a.out, exist_ok=True)
            with open(os.path.join(a.out, "report.json"), "w") as f:
                json.dump(rep, f, indent=1, default=str)
        say("REPORT\t" + json.dumps({k: v for k, v in rep.items() if k != "losses"}, default=str))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
