"""Out-of-memory diagnostics on the host (CPU): MEM lines, the engine buffer census and the
allocation-stack aggregation of a memory snapshot."""

import torch

from dllm_qwen38_b200.utils import mem


def test_mem_line_on_a_host_without_cuda(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    assert mem.mem_line("after shard") == "MEM\tafter shard\tcpu"


def test_engine_census_counts_shards_and_buffers():
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model
    from dllm_qwen38_b200.parallel.fsdp import FSDPEngine

    eng = FSDPEngine(build_model(preset("tiny_ref", layers=2), seed=0, device="cpu", dtype=torch.float32))
    line = mem.engine_census(eng)
    assert line.startswith("MEMCENSUS\tshards_gib=") and "gathered_slots=['-', '-']" in line
    shard_bytes = sum(t.numel() * t.element_size() for u in eng.units for t in (u.p, u.master, u.m, u.v, u.g))
    assert f"shards_gib={shard_bytes / 2**30:.2f}" in line


def test_history_dump_groups_live_blocks_by_their_last_frames(monkeypatch):
    def frames(*names):
        return [{"name": f"/src/{n}"} for n in names]

    snap = {"segments": [{"blocks": [
        {"state": "active_allocated", "size": 3 << 20, "frames": frames("a.py", "b.py", "gemm.py")},
        {"state": "active_allocated", "size": 1 << 20, "frames": frames("a.py", "b.py", "gemm.py")},
        {"state": "inactive", "size": 64 << 20, "frames": frames("x.py")},
        {"state": "active_allocated", "size": 2 << 20, "frames": []},
    ]}]}
    monkeypatch.setattr(torch.cuda.memory, "_snapshot", lambda: snap)
    lines = []
    mem.dump_history(0, out=lines.append)
    assert lines[0] == "[MEMHIST rank 0] live 0.01 GiB in 3 blocks"
    assert "4.0 MiB n=    2 a.py <- b.py <- gemm.py" in lines[1]  # largest group first
    assert "2.0 MiB n=    1 <no stack>" in lines[2]


def test_history_dump_reports_a_failed_snapshot(monkeypatch):
    def boom():
        raise RuntimeError("no allocator")

    monkeypatch.setattr(torch.cuda.memory, "_snapshot", boom)
    lines = []
    mem.dump_history(1, out=lines.append)
    assert lines == ["[MEMHIST rank 1] snapshot failed: RuntimeError('no allocator')"]
