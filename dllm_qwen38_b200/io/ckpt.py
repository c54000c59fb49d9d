"""Checkpoints: resumable sharded saves of the FSDP engine, exports and imports.

Resumable save (`save_engine` / `load_engine`), the reference's contract (`fsdp_train.py:352-517`):
  * directory ``<ckpt_dir>/step-%08d`` written by torch.distributed.checkpoint (every rank writes
    its own shards into ``step-N.tmp``); after a barrier rank 0 renames it to ``step-N`` (the rename
    is the commit point: a run killed mid-save leaves only a ``.tmp``), then keeps the last two;
  * contents: {"model": flat bf16 parameter shards, "optim": fp32 master + AdamW moments + step,
    "step", "seq_tokens"}; each unit's shard is stored as a DTensor sharded on dim 0 over the
    world, so a checkpoint written at one world size loads at another (DCP reshards);
  * optional per-rank SHA256 fingerprints of the model and optimizer shards, written to
    ``fingerprints/step-N.tsv`` as ``rank \\t model-fp \\t opt-fp`` at save and verified at load;
    a missing or unparseable file fails closed (all-reduced, identical on every rank);
  * no RNG state: masks are a pure function of (global step, rank), so a resumed window replays
    the uninterrupted run's masks (`fsdp_train.py:418-422,607`).

Exports/imports:
  * `export_safetensors`: full parameters under our keys (``text_model.<HF text key>``,
    ``lm_head.weight``) -- the reference's single-device layout (`train.py:270-276`);
  * `reference_dcp_tensors` + `plain_fqn`: read a reference FSDP checkpoint (per-parameter
    DTensors named ``text_model.layers.N.layer.<...>``, `gsm8k_eval.py:249-285`) as plain tensors;
  * `convert_to_reference`: rewrite one of this engine's checkpoints in the reference's layout
    (`fsdp_train.py:408-464`) so the reference's tools (`gsm8k_eval.py:264-328`) read it.

    python -m dllm_qwen38_b200.io.ckpt to-reference <step dir> <out dir> --model 27b [--layers N]
"""

from __future__ import annotations

import hashlib
import os
import re
import shutil

import torch
import torch.distributed as dist


def ckpt_path(ckpt_dir: str, gstep: int) -> str:
    return os.path.join(ckpt_dir, f"step-{gstep:08d}")


def latest_checkpoint(ckpt_dir: str) -> int | None:
    """Highest committed step-N (a `.tmp` left by an interrupted save does not count)."""
    try:
        entries = os.listdir(ckpt_dir)
    except FileNotFoundError:
        return None
    ns = []
    for e in entries:
        if e.startswith("step-") and not e.endswith(".tmp"):
            try:
                ns.append(int(e.split("-")[1]))
            except ValueError:
                pass
    return max(ns) if ns else None


def fingerprint(tensors: dict) -> str:
    """SHA256 over the raw bytes of a flat {name: tensor} map (sorted), first 16 hex digits."""
    h = hashlib.sha256()
    for k in sorted(tensors):
        t = tensors[k]
        h.update(f"{k}\x1f".encode())
        if torch.is_tensor(t):
            u = t.detach().contiguous().cpu()
            h.update(f"{tuple(u.shape)}\x1f{u.dtype}\x1f".encode())
            h.update(u.reshape(-1).view(torch.uint8).numpy().tobytes())
        else:
            h.update(repr(t).encode())
    return h.hexdigest()[:16]


def _world():
    return (dist.get_world_size(), dist.get_rank()) if dist.is_initialized() else (1, 0)


def _barrier():
    if dist.is_initialized():
        dist.barrier()


def _local_maps(engine):
    model = {f"{u.name}": u.p for u in engine.units}
    optim = {}
    for u in engine.units:
        optim[f"{u.name}.master"] = u.master
        optim[f"{u.name}.exp_avg"] = u.m
        optim[f"{u.name}.exp_avg_sq"] = u.v
    return model, optim


def _as_dtensor(t: torch.Tensor, world: int):
    """Wrap this rank's dim-0 shard as a DTensor over all ranks (single-process: plain tensor)."""
    if world == 1 or not dist.is_initialized():
        return t
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import DTensor, Shard

    mesh = init_device_mesh(t.device.type, (world,))
    return DTensor.from_local(t, mesh, [Shard(0)], run_check=False, shape=torch.Size([t.numel() * world]),
                              stride=(1,))


def save_engine(engine, ckpt_dir: str, gstep: int, seq_tokens: int, *, fingerprint_save: bool = True,
                keep: int = 2) -> str:
    """Collective: every rank writes its shards, rank 0 commits by rename and prunes."""
    import torch.distributed.checkpoint as dcp

    world, rank = _world()
    model, optim = _local_maps(engine)
    if fingerprint_save:
        fp = f"{fingerprint(model)} {fingerprint(optim)}"
        fps = [None] * world
        if world > 1:
            dist.all_gather_object(fps, fp)
        else:
            fps = [fp]
        if rank == 0:
            os.makedirs(os.path.join(ckpt_dir, "fingerprints"), exist_ok=True)
            with open(os.path.join(ckpt_dir, "fingerprints", f"step-{gstep}.tsv"), "w") as f:
                for r, s in enumerate(fps):
                    mfp, ofp = s.split()
                    f.write(f"{r}\t{mfp}\t{ofp}\n")
    state = {
        "model": {k: _as_dtensor(v, world) for k, v in model.items()},
        "optim": {**{k: _as_dtensor(v, world) for k, v in optim.items()},
                  "step": torch.tensor(engine.step_count, dtype=torch.int64)},
        "step": torch.tensor(gstep, dtype=torch.int64),
        "seq_tokens": torch.tensor(seq_tokens, dtype=torch.int64),
    }
    tmp = ckpt_path(ckpt_dir, gstep) + ".tmp"
    dcp.save(state, checkpoint_id=tmp, no_dist=not dist.is_initialized())
    _barrier()
    if rank == 0:
        final = ckpt_path(ckpt_dir, gstep)
        if os.path.exists(final):
            shutil.rmtree(final)
        os.rename(tmp, final)
        kept = sorted((int(e.split("-")[1]), e) for e in os.listdir(ckpt_dir)
                      if e.startswith("step-") and not e.endswith(".tmp"))
        for _, e in kept[:-keep]:
            shutil.rmtree(os.path.join(ckpt_dir, e))
    _barrier()
    return ckpt_path(ckpt_dir, gstep)


def load_engine(engine, ckpt_dir: str, gstep: int, *, verify: bool = True) -> dict:
    """Restore shards in place. Returns {"seq_tokens", "step", "fp_ok"}; fp_ok is False on every
    rank when any rank's restored state fails (or cannot be) verified against the saved
    fingerprints (fail closed)."""
    import torch.distributed.checkpoint as dcp

    world, rank = _world()
    model, optim = _local_maps(engine)
    state = {
        "model": {k: _as_dtensor(v, world) for k, v in model.items()},
        "optim": {**{k: _as_dtensor(v, world) for k, v in optim.items()},
                  "step": torch.zeros((), dtype=torch.int64)},
        "step": torch.zeros((), dtype=torch.int64),
        "seq_tokens": torch.zeros((), dtype=torch.int64),
    }
    dcp.load(state, checkpoint_id=ckpt_path(ckpt_dir, gstep), no_dist=not dist.is_initialized())
    engine.step_count = int(state["optim"]["step"])
    engine.invalidate()
    fp_ok = True
    if verify:
        got = f"{fingerprint(model)} {fingerprint(optim)}"
        expected = None
        fp_file = os.path.join(ckpt_dir, "fingerprints", f"step-{gstep}.tsv")
        if os.path.exists(fp_file):
            for ln in open(fp_file):
                parts = ln.rstrip("\n").split("\t")
                if len(parts) >= 3 and parts[0] == str(rank):
                    expected = parts[1] + " " + parts[2]
        bad = expected is None or expected != got
        flag = torch.tensor([1.0 if bad else 0.0], device=engine.device)
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        fp_ok = float(flag) == 0.0
    return {"seq_tokens": int(state["seq_tokens"]), "step": int(state["step"]), "fp_ok": fp_ok}


# ----------------------------------------------------------------------------- exports / imports


@torch.no_grad()
def export_safetensors(engine_or_model, path: str) -> None:
    """Full parameters under `text_model.*` / `lm_head.weight` (collective for an engine; rank 0
    writes)."""
    from safetensors.torch import save_file

    if hasattr(engine_or_model, "full_state"):
        state = engine_or_model.full_state()
        if engine_or_model.tied and "lm_head.weight" not in state:
            state["lm_head.weight"] = state["text_model.embed_tokens.weight"]
    else:
        m = engine_or_model
        state = {f"text_model.{k}": v for k, v in m.text_model.state_dict().items()}
        state["lm_head.weight"] = m.lm_head.weight
    _, rank = _world()
    if rank == 0:
        save_file({k: v.detach().cpu().contiguous().clone() for k, v in state.items()}, path)
    _barrier()


def plain_fqn(dcp_fqn: str) -> str | None:
    """Reference checkpoint FQN -> our key; None = not a model key. Strips the LayerStep `.layer.`
    hop: `text_model.layers.7.layer.mlp.x` -> `text_model.layers.7.mlp.x` (`gsm8k_eval.py:249-261`)."""
    if dcp_fqn.startswith("text_model."):
        m = re.match(r"^text_model\.(layers\.\d+)\.layer\.(.+)$", dcp_fqn)
        return f"text_model.{m.group(1)}.{m.group(2)}" if m else dcp_fqn
    if dcp_fqn.startswith("lm_head."):
        return dcp_fqn
    return None


def reference_dcp_tensors(path: str) -> tuple[dict, int, int]:
    """The 'model' half of a reference FSDP checkpoint as plain CPU tensors (resharding read with
    no process group), plus (step, seq_tokens)."""
    from torch.distributed.checkpoint import FileSystemReader, load as dcp_load

    reader = FileSystemReader(path)
    md = reader.read_metadata()
    model = {}
    for key, meta in md.state_dict_metadata.items():
        if not key.startswith("model."):
            continue
        if not hasattr(meta, "size"):
            raise ValueError(f"{path}: non-tensor entry under 'model': {key}")
        model[key[len("model."):]] = torch.empty(tuple(meta.size), dtype=meta.properties.dtype)
    step, seq = torch.zeros((), dtype=torch.int64), torch.zeros((), dtype=torch.int64)
    dcp_load({"model": model, "step": step, "seq_tokens": seq}, storage_reader=reader, no_dist=True)
    return model, int(step), int(seq)


def engine_unit_layout(cfg) -> dict:
    """{unit name: [(our key, shape, offset, numel)]} of the sharded engine's flat units, in the
    engine's flat order (`parallel.fsdp.flat_order`: small non-GEMM parameters first, shared
    parameters once)."""
    from ..models.qwen35 import BlockDiffusionLM

    with torch.device("meta"):
        m = BlockDiffusionLM(cfg)
    tm = m.text_model
    units = [("embed", "text_model.embed_tokens.", tm.embed_tokens)]
    units += [(f"layers.{i}", f"text_model.layers.{i}.", layer) for i, layer in enumerate(tm.layers)]
    head = {"norm": tm.norm} if cfg.tie_word_embeddings else {"norm": tm.norm, "lm_head": m.lm_head}
    units.append(("head", "", torch.nn.ModuleDict(head)))
    from ..parallel.fsdp import flat_order

    out = {}
    for name, prefix, mod in units:
        off, ent = 0, []
        for n, p in flat_order(mod):
            key = prefix + n
            if name == "head" and n.startswith("norm."):
                key = "text_model." + n
            ent.append((key, tuple(p.shape), off, p.numel()))
            off += p.numel()
        out[name] = ent
    return out


def any_dcp_tensors(path: str, cfg) -> tuple[dict, int, int]:
    """Full parameters {our or reference key: tensor} from either checkpoint kind: this
    repository's engine (flat per-unit shards under 'model.<unit>') or the reference's FSDP
    layout (per-parameter entries under 'model.text_model...' / 'model.lm_head...')."""
    from torch.distributed.checkpoint import FileSystemReader, load as dcp_load

    md = FileSystemReader(path).read_metadata()
    keys = [k for k in md.state_dict_metadata if k.startswith("model.")]
    if any(k.startswith("model.text_model.") or k.startswith("model.lm_head.") for k in keys):
        return reference_dcp_tensors(path)
    flat = {}
    for k in keys:
        meta = md.state_dict_metadata[k]
        flat[k[len("model."):]] = torch.empty(tuple(meta.size), dtype=meta.properties.dtype)
    step, seq = torch.zeros((), dtype=torch.int64), torch.zeros((), dtype=torch.int64)
    dcp_load({"model": flat, "step": step, "seq_tokens": seq}, storage_reader=FileSystemReader(path), no_dist=True)
    out = {}
    for unit, entries in engine_unit_layout(cfg).items():
        if unit not in flat:
            raise ValueError(f"{path}: unit {unit} missing (checkpoint of another model shape?)")
        buf = flat[unit]
        need = sum(e[3] for e in entries)
        if buf.numel() < need:
            raise ValueError(f"{path}: unit {unit} holds {buf.numel()} elements, the model needs {need}")
        for key, shape, off, n in entries:
            out[key] = buf[off : off + n].view(shape).clone()
    return out, int(step), int(seq)


def restore_into(model, tensors: dict, ctx: str = "ckpt") -> None:
    """Load {reference or our FQN: tensor} into a `BlockDiffusionLM`; any missing, unexpected or
    foreign key raises (a partial restore would score silently wrong, `gsm8k_eval.py:306-328`)."""
    own = dict(model.named_parameters(remove_duplicate=False))
    seen, bad = set(), []
    for fqn, t in tensors.items():
        k = plain_fqn(fqn)
        if k is None:
            bad.append("ckpt?" + fqn)
            continue
        if k not in own:
            bad.append("model?" + k)
            continue
        with torch.no_grad():
            own[k].copy_(t.to(own[k].dtype))
        seen.add(k)
    tied = model.config.tie_word_embeddings
    missing = [k for k in own if k not in seen and not (tied and k == "lm_head.weight")]
    bad += ["model:" + k for k in missing]
    if bad:
        raise ValueError(f"{ctx}: restore incomplete ({len(bad)} problems, first 10: {bad[:10]})")


def reference_fqn(key: str) -> str:
    """Our key -> the reference's checkpoint FQN: decoder-layer parameters sit under the
    reference's per-layer wrapper (`text_model.layers.N.layer.<...>`); the rest is unchanged."""
    m = re.match(r"^text_model\.(layers\.\d+)\.(.+)$", key)
    return f"text_model.{m.group(1)}.layer.{m.group(2)}" if m else key


def _optimizer_tensors(path: str, cfg) -> tuple[dict, int]:
    """{our key: (master fp32, exp_avg fp32, exp_avg_sq fp32)} and the AdamW step count of one of
    this engine's checkpoints."""
    from torch.distributed.checkpoint import FileSystemReader, load as dcp_load

    md = FileSystemReader(path).read_metadata()
    flat = {}
    for k, meta in md.state_dict_metadata.items():
        if k.startswith("optim.") and hasattr(meta, "size") and k != "optim.step":
            flat[k[len("optim."):]] = torch.empty(tuple(meta.size), dtype=meta.properties.dtype)
    step = torch.zeros((), dtype=torch.int64)
    dcp_load({"optim": {**flat, "step": step}}, storage_reader=FileSystemReader(path), no_dist=True)
    out = {}
    for unit, entries in engine_unit_layout(cfg).items():
        parts = [flat.get(f"{unit}.{x}") for x in ("master", "exp_avg", "exp_avg_sq")]
        if any(t is None for t in parts):
            raise ValueError(f"{path}: optimizer state of unit {unit} missing")
        for key, shape, off, n in entries:
            out[key] = tuple(t[off : off + n].view(shape).clone() for t in parts)
    return out, int(step)


@torch.no_grad()
def convert_to_reference(src: str, dst: str, cfg, *, lr: float = 1e-5, betas=(0.9, 0.95), eps: float = 1e-8,
                         weight_decay: float = 0.0) -> dict:
    """Write checkpoint `src` of this engine as a checkpoint in the reference's layout at `dst`.

    Layout written (`fsdp_train.py:408-464` there): {"model": {FQN: bf16}, "optim": {"state":
    {FQN: {"exp_avg", "exp_avg_sq": bf16, "step": fp32}}, "param_groups": [AdamW hyper-parameters
    with the FQN list]}, "step", "seq_tokens"}, FQNs as `reference_fqn` spells them. The reference
    trains bf16 parameters with bf16 moments and no master copy, so the fp32 master weights are
    rounded to bf16 for "model" and the fp32 moments to bf16 for "optim". A tied head is written
    as its own `lm_head.weight` entry too (the reference's restore requires the key). Single
    process; the full model passes through host memory once."""
    import torch.distributed.checkpoint as dcp

    params, step, seq = any_dcp_tensors(src, cfg)
    opt, adam_step = _optimizer_tensors(src, cfg)
    if cfg.tie_word_embeddings and "lm_head.weight" not in params:
        params["lm_head.weight"] = params["text_model.embed_tokens.weight"]
    model, state = {}, {}
    for key, t in params.items():
        fqn = reference_fqn(key)
        src_key = "text_model.embed_tokens.weight" if (key == "lm_head.weight" and key not in opt) else key
        master, m, v = opt[src_key]
        model[fqn] = master.to(torch.bfloat16)
        state[fqn] = {"exp_avg": m.to(torch.bfloat16), "exp_avg_sq": v.to(torch.bfloat16),
                      "step": torch.tensor(float(adam_step))}
    groups = [{"lr": lr, "betas": list(betas), "eps": eps, "weight_decay": weight_decay, "amsgrad": False,
               "foreach": False, "maximize": False, "capturable": False, "differentiable": False, "fused": None,
               "params": sorted(model)}]
    dcp.save({"model": model, "optim": {"state": state, "param_groups": groups},
              "step": torch.tensor(step, dtype=torch.int64), "seq_tokens": torch.tensor(seq, dtype=torch.int64)},
             checkpoint_id=dst, no_dist=True)
    return {"params": len(model), "step": step, "seq_tokens": seq}


def main(argv=None) -> int:
    import argparse

    import json

    from ..config import PRESETS, ModelConfig, preset

    p = argparse.ArgumentParser(description="checkpoint conversion")
    sub = p.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("to-reference", help="rewrite an engine checkpoint in the reference's DCP layout")
    c.add_argument("src")
    c.add_argument("dst")
    c.add_argument("--model", default="27b", help="preset name or HF checkpoint directory (its config.json)")
    c.add_argument("--layers", type=int, default=None)
    c.add_argument("--lr", type=float, default=1e-5)
    a = p.parse_args(argv)
    if a.model in PRESETS:
        cfg = preset(a.model, layers=a.layers)
    else:
        with open(os.path.join(a.model, "config.json")) as f:
            cfg = ModelConfig.from_hf_dict(json.load(f)).truncated(a.layers)
    rep = convert_to_reference(a.src, a.dst, cfg, lr=a.lr)
    print(f"CONVERTED\t{a.src} -> {a.dst}\tparams {rep['params']}\tstep {rep['step']}\tseq_tokens {rep['seq_tokens']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
