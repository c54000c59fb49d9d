"""AdamW with fp32 master weights and a global-norm clip.

Semantics match the reference's optimizer (`train.py:140`: AdamW betas (0.9, 0.95), weight decay
0; `train.py:160` clip_grad_norm_ 1.0; clip coefficient max_norm / (total + 1e-6) clamped at 1,
`fsdp_train.py:224-252`). Differences by design: bf16 parameters get an fp32 master copy and
fp32 moments (the reference steps bf16 params with bf16 moments); on CUDA each parameter's update
(clip scale, moments, master step, bf16 write-back) is one fused kernel (``csrc/misc.cu``,
``adamw_step``); the sharded engine runs the same kernel once per unit over its flat shard.
"""

from __future__ import annotations

import torch

from .. import ops


class MasterAdamW:
    def __init__(self, params, lr: float, betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0):
        self.params = [p for p in params]
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.step_count = 0
        self.master = [p.detach().float().clone() if p.dtype != torch.float32 else None for p in self.params]
        self.exp_avg = [torch.zeros_like(p, dtype=torch.float32) for p in self.params]
        self.exp_avg_sq = [torch.zeros_like(p, dtype=torch.float32) for p in self.params]

    def zero_grad(self):
        for p in self.params:
            p.grad = None

    def grad_norm(self) -> torch.Tensor:
        sq = [p.grad.float().pow(2).sum() for p in self.params if p.grad is not None]
        if not sq:
            return torch.zeros(())
        return torch.stack(sq).sum().sqrt()

    @torch.no_grad()
    def step(self, clip: float | None = 1.0, total_norm: torch.Tensor | None = None) -> float:
        """Clip by the global 2-norm (computed here unless given), then AdamW. Returns the norm."""
        if total_norm is None:
            total_norm = self.grad_norm()
        tn = float(total_norm)
        coef = 1.0 if clip is None else min(1.0, clip / (tn + 1e-6))
        self.step_count += 1
        b1, b2 = self.betas
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        for i, p in enumerate(self.params):
            if p.grad is None:
                continue
            w = self.master[i] if self.master[i] is not None else p.data
            native = getattr(ops._nat(), "adamw_step", None) if p.is_cuda else None
            if native is not None:
                native(w, p.data, p.grad, self.exp_avg[i], self.exp_avg_sq[i], self.lr, b1, b2,
                                         self.eps, self.wd, coef, bc1, bc2)
                continue
            g = p.grad.float() * coef
            if self.wd:
                w.mul_(1 - self.lr * self.wd)
            self.exp_avg[i].mul_(b1).add_(g, alpha=1 - b1)
            self.exp_avg_sq[i].mul_(b2).addcmul_(g, g, value=1 - b2)
            denom = (self.exp_avg_sq[i] / bc2).sqrt_().add_(self.eps)
            w.addcdiv_(self.exp_avg[i], denom, value=-self.lr / bc1)
            if self.master[i] is not None:
                p.data.copy_(w)
        return tn

    def state_dict(self) -> dict:
        return {
            "step": self.step_count,
            "exp_avg": [t.clone() for t in self.exp_avg],
            "exp_avg_sq": [t.clone() for t in self.exp_avg_sq],
            "master": [None if t is None else t.clone() for t in self.master],
        }

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        for dst, src in zip(self.exp_avg, sd["exp_avg"]):
            dst.copy_(src)
        for dst, src in zip(self.exp_avg_sq, sd["exp_avg_sq"]):
            dst.copy_(src)
        for dst, src in zip(self.master, sd["master"]):
            if dst is not None and src is not None:
                dst.copy_(src)
