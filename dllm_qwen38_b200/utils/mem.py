"""Memory observability: MEM lines, allocation-history snapshots on OOM, engine buffer census.

Mirrors the reference's diagnostics (`fsdp_train.py:255-323,585-658`): `MEM` lines after the
first forward/backward, a bounded ring of allocation stacks recorded for the first steps on rank 0,
and, on an out-of-memory error, a census of live engine buffers printed first (fast) followed by
the top live allocations grouped by their allocation stack (slow, under SIGTERM ignored because a
launcher tears the other ranks down shortly after the first exit).
"""

from __future__ import annotations

import signal

import torch


def mem_line(tag: str) -> str:
    if not torch.cuda.is_available():
        return f"MEM\t{tag}\tcpu"
    return (f"MEM\t{tag}\tallocated {torch.cuda.memory_allocated() / 2**30:.2f} GiB\t"
            f"reserved {torch.cuda.memory_reserved() / 2**30:.2f} GiB")


def start_history(max_entries: int = 60000) -> None:
    if torch.cuda.is_available():
        torch.cuda.memory._record_memory_history(max_entries=max_entries)


def stop_history() -> None:
    if torch.cuda.is_available():
        torch.cuda.memory._record_memory_history(None)


def engine_census(engine) -> str:
    """Live storage held by the sharded engine (shards, gathered buffers, gradient buffers)."""
    def gib(ts):
        return sum(t.numel() * t.element_size() for t in ts) / 2**30

    shards = [t for u in engine.units for t in (u.p, u.master, u.m, u.v, u.g)]
    bufs = list(engine.bufs) + list(engine.grads) + ([engine.table_grad] if engine.table_grad is not None else [])
    owners = [o.name if o is not None else "-" for o in engine.owner]
    return (f"MEMCENSUS\tshards_gib={gib(shards):.2f}\tbuffers_gib={gib(bufs):.2f}\t"
            f"gathered_slots={owners}")


def dump_history(rank: int, top: int = 25, out=print) -> None:
    """Aggregate live blocks of the recorded snapshot by their last three frames."""
    try:
        snap = torch.cuda.memory._snapshot()
    except Exception as e:  # never mask the error being reported
        out(f"[MEMHIST rank {rank}] snapshot failed: {e!r}")
        return
    live: dict[str, list[int]] = {}
    for seg in snap.get("segments", []):
        for b in seg.get("blocks", []):
            if b.get("state") != "active_allocated":
                continue
            frames = b.get("frames") or []
            key = " <- ".join(f["name"].split("/")[-1] for f in frames[-3:]) or "<no stack>"
            ent = live.setdefault(key, [0, 0])
            ent[0] += int(b["size"])
            ent[1] += 1
    tot = sum(v[0] for v in live.values())
    out(f"[MEMHIST rank {rank}] live {tot / 2**30:.2f} GiB in {sum(v[1] for v in live.values())} blocks")
    for key, (nbytes, n) in sorted(live.items(), key=lambda kv: -kv[1][0])[:top]:
        out(f"[MEMHIST rank {rank}] {nbytes / 2**20:9.1f} MiB n={n:5d} {key}")


def on_oom(engine, rank: int, with_history: bool, out=print) -> None:
    out(mem_line("at OOM"))
    if engine is not None:
        out(engine_census(engine))
    if with_history:
        signal.signal(signal.SIGTERM, signal.SIG_IGN)
        out(f"[MEMHIST rank {rank}] OOM caught; snapshotting allocation stacks (SIGTERM ignored)")
        dump_history(rank, out=out)
