"""Public training-step API: `Trainer.step(x0, prompt_len, valid_len)`.

One call = one optimizer step of the block-diffusion objective on this process's rows:
complementary masks (pure function of (global step, rank), `fsdp_train.py:607`), state-fork
forward with per-layer activation checkpointing, masked CE over the 248k vocab on masked rows
only, backward, global-norm clip, AdamW.

The forward, the loss and the backward never synchronise the host with the device: the number
of scored targets is known on the host before any kernel runs, because the two complementary
views together mask every scorable position exactly once (n = sum(valid_len - prompt_len)); the
masked-row gather uses that count (`nonzero_static`) instead of reading it back. The one host read
per step is the global gradient norm, from which `MasterAdamW` computes the clip coefficient (the
sharded engine, `parallel/fsdp.py`, keeps that coefficient on the device). The returned loss is a
device tensor; reading it is the caller's choice.
"""

from __future__ import annotations

import torch

from .. import ops
from ..models.blockdiff import block_diffusion_forward
from .objective import complementary_step_inputs
from .optim import MasterAdamW


class Trainer:
    def __init__(self, model, *, block: int, mask_id: int, lr: float = 1e-5, grad_clip: float = 1.0,
                 checkpointing: bool = True, seed: int = 0, rank: int = 0):
        self.model = model
        self.block, self.mask_id, self.grad_clip = block, mask_id, grad_clip
        self.checkpointing, self.seed, self.rank = checkpointing, seed, rank
        self.params = model.unique_parameters()
        for p in self.params:
            p.requires_grad_(True)
        self.opt = MasterAdamW(self.params, lr=lr, betas=(0.9, 0.95), weight_decay=0.0)
        self.device = next(model.parameters()).device
        self.gstep = 0

    def step(self, x0: torch.Tensor, prompt_len: torch.Tensor, valid_len: torch.Tensor,
             n_targets: int | None = None) -> torch.Tensor:
        """x0 [B, L] token ids (any device; moved here non-blocking), prompt_len/valid_len [B].
        n_targets: the host-known scored-target count (computed from the host copies when the
        inputs are on the host). Returns the mean masked CE as a 0-d device tensor."""
        self.gstep += 1
        if n_targets is None:
            if x0.is_cuda:
                raise ValueError("pass n_targets when the inputs are already on the device")
            n_targets = int((valid_len - prompt_len).clamp(min=0).sum())  # both views together
        dev = self.device
        x0 = x0.to(dev, non_blocking=True)
        prompt_len = prompt_len.to(dev, non_blocking=True)
        valid_len = valid_len.to(dev, non_blocking=True)
        gen = torch.Generator(device=dev).manual_seed(self.gstep * 1000 + self.rank)
        x0_2, xt_2, m_2 = complementary_step_inputs(x0, prompt_len, self.block, self.mask_id, gen, valid_len,
                                                    seed=self.gstep * 1000 + self.rank)
        ht, _ = block_diffusion_forward(self.model, x0_2, xt_2, self.block, output="hidden",
                                        checkpointing=self.checkpointing)
        if n_targets == 0:
            return torch.zeros((), device=dev)
        idx = torch.nonzero_static(m_2.reshape(-1), size=n_targets).squeeze(1)
        rows = ht.reshape(-1, ht.shape[-1]).index_select(0, idx)
        tgt = x0_2.reshape(-1).index_select(0, idx)
        loss = ops.masked_ce_sum(rows, self.model.lm_head.weight, tgt) / self.loss_divisor(n_targets)
        self.opt.zero_grad()
        loss.backward()
        self.reduce_grads()
        self.opt.step(clip=self.grad_clip, total_norm=self.global_grad_norm())
        return loss.detach()

    # hooks for data-parallel subclasses
    def loss_divisor(self, n_local: int) -> float:
        return float(n_local)

    def reduce_grads(self) -> None:
        pass

    def global_grad_norm(self):
        return self.opt.grad_norm()
