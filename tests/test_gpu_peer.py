"""Peer-memory collectives (csrc/peer.cu) and the FSDP engine over them.

One GPU: a wait on a flag that nothing sets runs out after its short limit and reports
ERR_COMM_WAIT through the error word; the context stays usable. Two GPUs (skipped otherwise):
all-gather / reduce-scatter / all-reduce against fp32 torch references, and the FSDP engine with
peer collectives against the same engine over NCCL."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ERR_COMM_WAIT = 4


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_peer_wait_times_out_and_reports():
    from dllm_qwen38_b200.ops import _native
    from dllm_qwen38_b200.parallel.peer import SymmetricHeap

    C = _native.require()
    torch.cuda.set_device(0)
    store = dist.TCPStore("127.0.0.1", _port(), 1, True)
    dist.init_process_group("gloo", store=store, rank=0, world_size=1)
    try:
        heap = SymmetricHeap(1 << 20, torch.device("cuda", 0))
        shard, off = heap.alloc(4096, torch.bfloat16)
        shard.copy_(torch.arange(4096, device="cuda").to(torch.bfloat16))
        out = torch.empty(4096, dtype=torch.bfloat16, device="cuda")
        C.read_error_word(True)
        heap.timeout = 1.0
        heap.all_gather(off, 4096 * 2, out, epoch=heap.epoch + 7)  # nobody publishes that epoch
        torch.cuda.synchronize()
        assert C.read_error_word(True) == ERR_COMM_WAIT
        heap.all_gather(off, 4096 * 2, out)  # the context is still usable
        torch.cuda.synchronize()
        assert C.read_error_word(False) == 0
        assert torch.equal(out, shard)
        g, goff = heap.alloc(4096, torch.float32)
        g.normal_()
        res = torch.empty(4096, dtype=torch.float32, device="cuda")
        sq = torch.zeros(1, dtype=torch.float32, device="cuda")
        heap.reduce_scatter(goff, 4096, True, res, 0.5, sq)
        torch.cuda.synchronize()
        assert C.read_error_word(False) == 0
        torch.testing.assert_close(res, 0.5 * g)
        torch.testing.assert_close(sq[0], (0.5 * g).pow(2).sum(), rtol=1e-5, atol=1e-5)
        heap.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("N,K,M,wide", [(1536, 1024, 300, "1"), (4096, 1024, 4096, "1"), (4096, 1024, 4096, "0")])
def test_fused_allgather_gemm_single_rank(N, K, M, wide, monkeypatch):
    """gemm_ag with one rank: the copy warps fill the whole gathered buffer from the (own) shard
    while the tiles wait per chunk; result and buffer against torch. M 300 runs the one-CTA kernel,
    M 4096 the two-CTA kernel in both tile widths."""
    from dllm_qwen38_b200.ops import _native
    from dllm_qwen38_b200.parallel.peer import SymmetricHeap

    monkeypatch.setenv("BDLLM_GEMM_WIDE", wide)
    C = _native.require()
    torch.cuda.set_device(0)
    store = dist.TCPStore("127.0.0.1", _port(), 1, True)
    dist.init_process_group("gloo", store=store, rank=0, world_size=1)
    try:
        extra = 777 * 64
        numel = 4096 + N * K + extra  # [something | W | the rest of a unit]
        heap = SymmetricHeap(numel * 2 + (1 << 20), torch.device("cuda", 0))
        shard, off = heap.alloc(numel, torch.bfloat16)
        shard.copy_(torch.randn(numel, device="cuda").to(torch.bfloat16) * 0.1)
        gathered = torch.zeros(numel, dtype=torch.bfloat16, device="cuda")
        w = gathered[4096 : 4096 + N * K].view(N, K)
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        ready = torch.zeros(8192 + 64, dtype=torch.int32, device="cuda")
        claim = torch.zeros(1, dtype=torch.int32, device="cuda")
        for seq in (1, 2):
            gathered.zero_()
            C.read_error_word(True)
            C.gemm_ag(x, w, out, 0, None, heap.ptrs, 0, off, numel * 2, gathered, ready, claim, seq, 0, 0, 10.0)
            torch.cuda.synchronize()
            assert C.read_error_word(False) == 0
            assert torch.equal(gathered, shard)
            want = x.float() @ shard[4096 : 4096 + N * K].view(N, K).float().t()
            assert float((out.float() - want).abs().max()) < 2e-2 * float(want.abs().max())
        heap.close()
    finally:
        dist.destroy_process_group()


def _collectives_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from dllm_qwen38_b200.ops import _native
        from dllm_qwen38_b200.parallel.peer import SymmetricHeap

        C = _native.require()
        dev = torch.device("cuda", rank)
        heap = SymmetricHeap(64 << 20, dev)
        heap.timeout = 20.0
        S = 1 << 16
        shard, soff = heap.alloc(S, torch.bfloat16)
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        shard.copy_(torch.randn(S, device=dev, generator=gen).to(torch.bfloat16))
        full = [torch.empty(S, dtype=torch.bfloat16, device=dev) for _ in range(world)]
        torch.cuda.synchronize()
        dist.all_gather(full, shard)
        dist.barrier()
        out = torch.empty(S * world, dtype=torch.bfloat16, device=dev)
        heap.all_gather(soff, S * 2, out)
        torch.cuda.synchronize()
        ok_ag = torch.equal(out, torch.cat(full))
        errs = []
        for dt, f32 in ((torch.bfloat16, False), (torch.float32, True)):
            g, goff = heap.alloc(S * world, dt)
            for it in range(3):  # the sequence flags advance every call
                torch.cuda.synchronize()
                gg = torch.Generator(device=dev).manual_seed(1000 * it + rank)
                g.copy_(torch.randn(S * world, device=dev, generator=gg).to(dt))
                allg = [torch.empty_like(g) for _ in range(world)]
                dist.all_gather(allg, g)
                ref = torch.stack([a.float() for a in allg]).sum(0)[rank * S : (rank + 1) * S] / world
                res = torch.empty(S, dtype=torch.float32, device=dev)
                sq = torch.zeros(1, dtype=torch.float32, device=dev)
                heap.reduce_scatter(goff, S, f32, res, 1.0 / world, sq)
                torch.cuda.synchronize()
                errs.append(float((res - ref).abs().max()))
                errs.append(abs(float(sq[0]) - float(ref.pow(2).sum())) / float(ref.pow(2).sum()))
        vals = torch.tensor([1.0 + rank, 2.0 * rank], device=dev)
        outv = torch.empty(2, device=dev)
        for _ in range(3):
            heap.allreduce_f32(vals, outv)
        torch.cuda.synchronize()
        ok_ar = torch.allclose(outv, torch.tensor([sum(1.0 + r for r in range(world)),
                                                    sum(2.0 * r for r in range(world))], device=dev))
        heap.publish_epoch(1)
        heap.all_gather(soff, S * 2, out, epoch=1)
        torch.cuda.synchronize()
        q.put((rank, ok_ag, max(errs), ok_ar, C.read_error_word(False)))
        heap.close()
    finally:
        dist.destroy_process_group()


def _spawn(fn, world, timeout=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=timeout) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_collectives_two_gpus():
    for rank, ok_ag, err, ok_ar, word in _spawn(_collectives_worker, 2):
        assert ok_ag, rank
        assert err < 1e-5, (rank, err)
        assert ok_ar, rank
        assert word == 0, (rank, word)


def _engine_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from dllm_qwen38_b200.config import preset
        from dllm_qwen38_b200.models.qwen35 import build_model
        from dllm_qwen38_b200.ops import cuda as C
        from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

        dev = torch.device("cuda", rank)
        cfg = preset("tiny", hidden_size=256, intermediate_size=512, linear_key_head_dim=64, linear_value_head_dim=64,
                     head_dim=64)
        runs = {}
        for comm, fused, clip in (("nccl", "0", 1.0), ("peer", "0", 1.0), ("peer", "1", 1.0), ("nccl", "0", 0.0),
                                  ("peer", "1", 0.0)):
            os.environ["BDLLM_COMM"] = comm
            os.environ["BDLLM_FUSED_AG"] = fused
            model = build_model(cfg, seed=0, device=dev, dtype=torch.bfloat16)
            tr = FSDPTrainer(model, block=32, mask_id=cfg.mask_id, lr=1e-4, grad_clip=clip)
            assert (tr.engine.peer is not None) == (comm == "peer")
            assert tr.engine.__dict__.get("fused_ag", False) == (comm == "peer" and fused == "1")
            comm = comm + ("-fused" if fused == "1" else "") + ("-noclip" if clip == 0 else "")
            g = torch.Generator().manual_seed(7)
            losses = []
            for _ in range(3):
                x0 = torch.randint(0, cfg.mask_id, (2 * world, 128), generator=g)[rank * 2 : rank * 2 + 2]
                loss = tr.step(x0, torch.zeros(2, dtype=torch.long), torch.full((2,), 128, dtype=torch.long))
                losses.append(float(loss))
            state = {k: v.float().cpu() for k, v in tr.engine.full_state().items()}
            runs[comm] = (losses, state, float(tr.engine.last_grad_norm))
            tr.engine.close()
        C.check_errors()
        (la, sa, na) = runs["nccl"]
        dl = dp = dn = 0.0
        for base, other in (("nccl", "peer"), ("nccl", "peer-fused"), ("nccl-noclip", "peer-fused-noclip")):
            la, sa, na = runs[base]
            lb, sb, nb = runs[other]
            dl = max(dl, max(abs(a - b) / max(1.0, abs(a)) for a, b in zip(la, lb)))
            dp = max(dp, max(float((sa[k] - sb[k]).abs().max()) for k in sa))
            dn = max(dn, abs(na - nb) / max(1e-6, na))
        q.put((rank, dl, dp, dn))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fsdp_peer_collectives_match_nccl_two_gpus():
    for rank, dl, dp, dn in _spawn(_engine_worker, 2):
        assert dl < 1e-3, (rank, dl)
        assert dp < 2e-3, (rank, dp)
        assert dn < 1e-3, (rank, dn)
