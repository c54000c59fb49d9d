"""FSDP engine on CPU: world 1 against the single-device trainer, world 2 (gloo ranks) against
replicated data parallelism with the same masks and reduction semantics."""

import copy
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.models.qwen35 import build_model


def _batches(B, L, vocab, seed, n=3):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randint(0, vocab - 1, (B, L), generator=g), torch.zeros(B, dtype=torch.long),
             torch.full((B,), L, dtype=torch.long)) for _ in range(n)]


def _flat(sd):
    return {k: v.detach().float().cpu() for k, v in sd.items()}


@pytest.mark.parametrize("name", ["tiny_ref", "tiny"])  # untied head / tied head
def test_world1_fsdp_matches_single_device_trainer(name):
    from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer
    from dllm_qwen38_b200.train.trainer import Trainer

    torch.manual_seed(0)
    cfg = preset(name)
    m1 = build_model(cfg, seed=0)
    m2 = copy.deepcopy(m1)
    if cfg.tie_word_embeddings:
        m2.lm_head.weight = m2.text_model.embed_tokens.weight
    t1 = Trainer(m1, block=8, mask_id=cfg.mask_id, lr=1e-3, checkpointing=False)
    t2 = FSDPTrainer(m2, block=8, mask_id=cfg.mask_id, lr=1e-3)
    for x0, pl, vl in _batches(2, 32, cfg.vocab_size, 1):
        l1 = t1.step(x0, pl, vl)
        l2 = t2.step(x0, pl, vl)
        assert abs(float(l1) - float(l2)) < 1e-4 * max(1.0, abs(float(l1)))
    ref = _flat({f"text_model.{k}" if not k.startswith("lm_head") else k: v
                 for k, v in {**{("text_model." + k)[len("text_model."):]: v for k, v in m1.text_model.state_dict().items()},
                              "lm_head.weight": m1.lm_head.weight}.items()})
    got = _flat(t2.engine.full_state())
    for k, v in got.items():
        assert k in ref, k
        assert float((v - ref[k]).abs().max()) < 1e-4, k


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dllm_qwen38_b200.parallel.dp import ReplicatedDP
        from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

        torch.manual_seed(0)
        cfg = preset("tiny_ref")
        m1 = build_model(cfg, seed=0)
        m2 = copy.deepcopy(m1)
        dp = ReplicatedDP(m1, block=8, mask_id=cfg.mask_id, lr=1e-3, checkpointing=False, rank=rank, world=world)
        fs = FSDPTrainer(m2, block=8, mask_id=cfg.mask_id, lr=1e-3)
        losses = []
        for x0, pl, vl in _batches(2 * world, 32, cfg.vocab_size, 2):
            sl = slice(rank * 2, (rank + 1) * 2)
            a = dp.step(x0[sl], pl[sl], vl[sl])
            b = fs.step(x0[sl], pl[sl], vl[sl])
            losses.append((float(a), float(b)))
        got = _flat(fs.engine.full_state())
        ref = {("text_model." + k): v.detach().float() for k, v in m1.text_model.state_dict().items()}
        ref["lm_head.weight"] = m1.lm_head.weight.detach().float()
        worst = max(float((v - ref[k]).abs().max()) for k, v in got.items())
        out.put((rank, losses, worst))
    finally:
        dist.destroy_process_group()


def test_world2_fsdp_matches_replicated_dp_on_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 2000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, losses, worst in res:
        for a, b in losses:
            assert abs(a - b) < 1e-4 * max(1.0, abs(a)), (rank, losses)
        assert worst < 1e-4, (rank, worst)


def test_partial_gemm_saving_policy():
    """gemm_saved: "1" every layer, "0" none, "<n>" the first n layers."""
    from dllm_qwen38_b200.parallel.fsdp import FSDPEngine

    e = object.__new__(FSDPEngine)
    for s, want in (("1", [True] * 4), ("0", [False] * 4), ("2", [True, True, False, False])):
        e.save_gemms = s
        assert [e.gemm_saved(i) for i in range(4)] == want, s


def test_saved_layer_choice_keeps_the_activation_only_when_everything_fits():
    from dllm_qwen38_b200.parallel.fsdp import choose_saved_layers

    gib = 1 << 30
    per, per_act = [2 * gib] * 4, [3 * gib] * 4
    # 0.92 * (20 - 3) = 15.6 GiB: all four with the activation (12 GiB)
    assert choose_saved_layers(per, per_act, 20 * gib) == (4, 12 * gib, True)
    # 0.92 * (14 - 3) = 10.1 GiB: not all with it (12), so gate|up only: all four (8 GiB)
    assert choose_saved_layers(per, per_act, 14 * gib) == (4, 8 * gib, False)
    # 0.92 * (9 - 3) = 5.5 GiB: two layers of gate|up
    assert choose_saved_layers(per, per_act, 9 * gib) == (2, 4 * gib, False)
    assert choose_saved_layers(per, per_act, gib)[0] == 0
    # several ranks (no rerun after an out-of-memory error): 0.85 * (9 - 2) = 5.95 GiB, two layers
    assert choose_saved_layers(per, per_act, 9 * gib, frac=0.85, reserve=2 * gib) == (2, 4 * gib, False)
    # 0.85 * (16 - 2) = 11.9 GiB: all four, gate|up only (12 GiB with the activation does not fit)
    assert choose_saved_layers(per, per_act, 16 * gib, frac=0.85, reserve=2 * gib) == (4, 8 * gib, False)


def test_one_rank_out_of_memory_retries_with_fewer_kept_layers():
    """An out-of-memory error before the update, after the probe chose the kept layers, reruns
    the step with two layers fewer; a second failure, or one after the update, propagates."""
    from dllm_qwen38_b200.parallel.fsdp import FSDPEngine

    class Store:
        cleared = 0

        @classmethod
        def clear(cls):
            cls.cleared += 1

    e = object.__new__(FSDPEngine)
    e.world, e.layers, e.save_gemms, e._auto_saved, e.step_count = 1, [0] * 6, "5", True, 3
    e.act_store = Store
    calls = []

    def failing_once(*a, **k):
        calls.append(e.save_gemms)
        e._updated = False
        e.step_count += 1
        if len(calls) == 1:
            raise torch.cuda.OutOfMemoryError("test")
        return "loss"

    e._step = failing_once
    kw = dict(block=8, mask_id=0, n_local=1, n_global=1, gstep=1)
    assert e.step(None, None, None, **kw) == "loss"
    assert calls == ["5", "3"] and e.save_gemms == "3" and e.step_count == 4 and Store.cleared == 1

    def always_failing(*a, **k):
        e._updated = False
        raise torch.cuda.OutOfMemoryError("test")

    e._step = always_failing
    with pytest.raises(torch.cuda.OutOfMemoryError):
        e.step(None, None, None, **kw)

    def failing_after_update(*a, **k):
        e._updated = True
        raise torch.cuda.OutOfMemoryError("test")

    e._step, e.save_gemms = failing_after_update, "5"
    with pytest.raises(torch.cuda.OutOfMemoryError):
        e.step(None, None, None, **kw)
    assert e.save_gemms == "5"


def _zero_target_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

        cfg = preset("tiny_ref")
        fs = FSDPTrainer(build_model(cfg, seed=0), block=8, mask_id=cfg.mask_id, lr=1e-3, grad_clip=0.0)
        losses = []
        for x0, pl, vl in _batches(2 * world, 32, cfg.vocab_size, 3):
            sl = slice(rank * 2, (rank + 1) * 2)
            pr = pl[sl].clone()
            if rank == 1:
                pr[:] = 32  # every row of this rank is prompt: no scored target here
            n_local = int((vl[sl] - pr).clamp(min=0).sum())
            counts = torch.tensor([float(n_local)])
            dist.all_reduce(counts)
            loss = fs.step(x0[sl], pr, vl[sl], n_targets=n_local, n_global=int(counts.item()))
            t = loss.detach().float().reshape(1)
            dist.all_reduce(t)
            losses.append(float(t))
        # numpy copies travel by value (a tensor would be shared by a handle that dies with the rank)
        out.put((rank, losses, {k: v.numpy().copy() for k, v in _flat(fs.engine.full_state()).items()}))
    finally:
        dist.destroy_process_group()


def test_world2_rank_with_zero_targets_keeps_collectives_in_step():
    """Rank 1 holds only prompt rows. It must still run the step (a graph-connected zero loss, zero
    gradients, the same gathers and reduce-scatters), and the result must equal training on rank
    0's rows alone with the loss divided by twice its target count (the world-2 gradient average
    halves rank 0's gradient)."""
    from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + (os.getpid() + 777) % 2000
    procs = [ctx.Process(target=_zero_target_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = preset("tiny_ref")
    solo = FSDPTrainer(build_model(cfg, seed=0), block=8, mask_id=cfg.mask_id, lr=1e-3, grad_clip=0.0)
    want = []
    for x0, pl, vl in _batches(4, 32, cfg.vocab_size, 3):
        n = int((vl[:2] - pl[:2]).clamp(min=0).sum())
        # divided by twice the count: the gradient AdamW sees is then the world-2 average exactly
        want.append(2 * float(solo.step(x0[:2], pl[:2], vl[:2], n_targets=n, n_global=2 * n)))
    ref = _flat(solo.engine.full_state())
    res = [(r, ls, {k: torch.from_numpy(v) for k, v in st.items()}) for r, ls, st in res]
    for rank, losses, state in res:
        for a, b in zip(losses, want):
            assert abs(a - b) < 1e-4 * max(1.0, abs(b)), (rank, losses, want)
        worst = max(float((v - ref[k]).abs().max()) for k, v in state.items())
        assert worst < 1e-4, (rank, worst)
    assert all(torch.equal(res[0][2][k], res[1][2][k]) for k in res[0][2])
