"""Failure detection on the host (gloo ranks on CPU): a rank that dies between steps or never
joins is seen by the survivor as an error from its next collective (short process-group timeout),
never as a hang; a checkpoint whose fingerprint file is missing fails closed."""

import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_dies(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model
    from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

    torch.manual_seed(0)
    cfg = preset("tiny_ref")
    tr = FSDPTrainer(build_model(cfg, seed=0), block=8, mask_id=cfg.mask_id, lr=1e-3)
    x = torch.randint(0, cfg.mask_id, (2, 32), generator=torch.Generator().manual_seed(rank))
    pl, vl = torch.zeros(2, dtype=torch.long), torch.full((2,), 32, dtype=torch.long)
    tr.step(x, pl, vl)  # one good step on both ranks
    if rank == 1:
        q.put((rank, "exited"))
        q.close()
        q.join_thread()  # the message is out before the process ends
        os._exit(0)  # leaves between steps, nothing in flight
    t0 = time.time()
    try:
        tr.step(x, pl, vl)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def test_survivor_errors_when_a_rank_dies_between_steps():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank_dies, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res[1] == "exited"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 60


def _never_joins(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1:
        q.put((rank, "never joined"))
        return
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        dist.barrier()
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error after {time.time() - t0:.1f}s"))


def test_rank_that_never_joins_is_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_never_joins, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res[1] == "never joined" and res[0].startswith("error after"), res


def test_checkpoint_without_fingerprints_fails_closed(tmp_path):
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.io import ckpt
    from dllm_qwen38_b200.models.qwen35 import build_model
    from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

    cfg = preset("tiny_ref")
    tr = FSDPTrainer(build_model(cfg, seed=0), block=8, mask_id=cfg.mask_id, lr=1e-3)
    ckpt.save_engine(tr.engine, str(tmp_path), 3, 96)
    assert ckpt.load_engine(tr.engine, str(tmp_path), 3)["fp_ok"]
    os.remove(tmp_path / "fingerprints" / "step-3.tsv")
    assert not ckpt.load_engine(tr.engine, str(tmp_path), 3)["fp_ok"]
    with open(tmp_path / "fingerprints" / "step-3.tsv", "w") as f:
        f.write("0\tdeadbeef\tdeadbeef\n")
    assert not ckpt.load_engine(tr.engine, str(tmp_path), 3)["fp_ok"]
