"""Tensor-parallel decoding on 2 GPUs (skipped with fewer): fused all-gather -> GEMM and
GEMM -> reduce-scatter kernels over peer memory against single-GPU decoding of the same model."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model

    cfg = preset("tiny", hidden_size=256, intermediate_size=512, linear_key_head_dim=64, linear_value_head_dim=64,
                 head_dim=64)
    return build_model(cfg, seed=0, device="cuda", dtype=torch.bfloat16)


def _worker(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from dllm_qwen38_b200.infer.engine import DecodeEngine
        from dllm_qwen38_b200.infer.tp import TPDecodeEngine
        from dllm_qwen38_b200.ops import cuda as Cu

        model = _model()
        cfg = model.config
        prompts = torch.randint(0, cfg.mask_id, (2, 40), generator=torch.Generator().manual_seed(5)).tolist()
        # one denoise step from the same state: confidence and picks against one GPU
        tp = TPDecodeEngine(model, 2, 256, 32, graphs=False, timeout_s=20)
        single = DecodeEngine(model, 2, 256, 32, graphs=False)
        cur = torch.tensor(prompts, device="cuda")
        for eng in (tp, single):
            eng.masked.zero_()
            eng.ids.copy_(cur[:, :32])
            eng._set_block(0)
            eng._run("commit")
            blk = torch.full((2, 32), cfg.mask_id, dtype=torch.long, device="cuda")
            blk[:, :8] = cur[:, 32:40]
            eng.ids.copy_(blk)
            eng.masked.zero_()
            eng.masked[:, 8:] = True
            eng._set_block(32)
            eng.fw.zero_()
            eng._run("step")
        torch.cuda.synchronize()
        conf_err = float(((tp.conf - single.conf).abs() / single.conf.abs().clamp_min(1e-6)).max())
        pick_eq = float((tp.pick == single.pick).float().mean())
        ids_eq = bool(torch.equal(tp.ids, single.ids))
        # graphs reproduce eager exactly, and every rank holds the same tokens
        outs = []
        for graphs in (False, True):
            eng = TPDecodeEngine(model, 2, 256, 32, sub_block=8, graphs=graphs, timeout_s=20)
            tr = eng.generate(prompts, n_blocks=3)
            outs.append([t.tokens for t in tr] + [[t.forwards for t in tr]])
            eng.close()
        tp.close()
        Cu.check_errors()
        q.put((rank, conf_err, pick_eq, ids_eq, outs[0] == outs[1], outs[0]))
    finally:
        dist.destroy_process_group()


def test_tp2_decode_matches_single_gpu_and_graphs():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=400) for _ in procs])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, conf_err, pick_eq, ids_eq, same, _ in res:
        assert conf_err < 5e-2, (rank, conf_err)
        assert pick_eq > 0.9, (rank, pick_eq)
        assert same, rank
    assert res[0][5] == res[1][5]  # both ranks decoded the same tokens
