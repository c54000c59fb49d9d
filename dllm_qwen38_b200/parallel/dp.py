"""Replicated data parallelism over NCCL (the all-reduce baseline).

Every rank holds the full model and its own micro-batch; after backward each gradient is
all-reduced and divided by the world size; the clip uses the (identical) global norm. The loss
on each rank is its local CE sum over the GLOBAL target count (`fsdp_train.py:39-44,618-630`),
and the all-reduce averages over ranks (the reference's FSDP reduce-scatter averages, and its
replicated grads are divided by world, `fsdp_train.py:207-221`), so the optimizer sees the same
(1/world) * grad(global mean CE) the reference's does.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..train.trainer import Trainer


class ReplicatedDP(Trainer):
    def __init__(self, model, *, world: int, **kw):
        super().__init__(model, **kw)
        self.world = world
        with torch.no_grad():  # identical start on every rank
            for p in self.params:
                dist.broadcast(p.data, 0)
            for i, p in enumerate(self.params):
                if self.opt.master[i] is not None:
                    self.opt.master[i].copy_(p.data)

    def loss_divisor(self, n_local: int) -> float:
        t = torch.tensor([float(n_local)], device=self.device)
        dist.all_reduce(t)
        return float(t.item())

    def reduce_grads(self) -> None:
        for p in self.params:
            if p.grad is not None:
                dist.all_reduce(p.grad)
                p.grad.div_(self.world)
