"""Python half of the native tools (`capture`, `meter`): the engine calls they make (the
reference's tools make llama.cpp calls instead: `tools/weight-space/capture.cpp:27-57,124`,
`tools/weight-space/meter.cpp:180-198`).

The C++ programs own argument handling, limits, file formats, timing and accounting; these
functions are the only way they touch the model:

  load(spec, layers)                  model from a preset name (random init, seed 0) or an HF dir
  capture(model, ids, layers)         {layer: float32 [T, D]} residual stream after each chosen
                                      layer for one prompt (clean, block-causal stream), plus the
                                      number of layer visits
  Session(model, block, ...)          a stateful cached decoder for the meter:
      prefill(ids) -> passes          commit the prompt's whole blocks
      begin_block() -> masked         start the next block (prompt tail kept)
      step() -> remaining             one denoise step (one block pass + commit rule)
      commit() -> new token ids       commit the finished block (one block pass)
      passes                          block passes run so far (the meter's "graph visits")
"""

from __future__ import annotations

import os

import numpy as np
import torch


def _device():
    return "cuda" if torch.cuda.is_available() else "cpu"


def load(spec: str, layers: int = 0):
    from ..config import preset
    from ..models.qwen35 import build_model

    dev = _device()
    dtype = torch.bfloat16 if dev == "cuda" else torch.float32
    if os.path.isdir(spec):
        from ..io.hf_load import load_model

        model, _ = load_model(spec, dtype=dtype, device=dev, layers=layers or None)
        return model
    cfg = preset(spec, layers=layers or None)
    return build_model(cfg, seed=0, device=dev, dtype=dtype)


@torch.no_grad()
def capture(model, ids, layers, block: int = 32):
    """Residual stream after each layer in `layers` (0-based) for the clean stream of `ids`
    (block-causal: a token sees its own block and the blocks before it). The prompt is padded with
    [MASK] to a whole number of blocks; tokens of the last partial block therefore also see the
    padding of their block. Returns ({layer: float32 [T, D]}, layer visits)."""
    from .. import ops
    from ..models.blockdiff import layer_step, rope_tables

    cfg = model.config
    dev = model.text_model.embed_tokens.weight.device
    n = len(ids)
    T = -(-n // block) * block
    x = torch.full((1, T), cfg.mask_id, dtype=torch.long, device=dev)
    x[0, :n] = torch.tensor(list(ids), dtype=torch.long, device=dev)
    want = sorted(set(int(i) for i in layers))
    if not want or want[-1] >= cfg.num_hidden_layers or want[0] < 0:
        raise ValueError(f"layers must be within [0, {cfg.num_hidden_layers})")
    # two-stream layout with x_t = x_0: the clean half is the stream being captured
    h = ops.embedding(torch.cat([x, x], 1), model.text_model.embed_tokens.weight)
    cos, sin = rope_tables(cfg, T, h.dtype, dev)
    out, visits = {}, 0
    for i in range(want[-1] + 1):
        h = layer_step(model.text_model.layers[i], cfg.layer_types[i], h, T, block, cfg.gdn_chunk_size, cos, sin,
                       _no_fault())
        visits += 1
        if i in want:
            out[i] = np.ascontiguousarray(h[0, T:T + n].float().cpu().numpy())
    return out, visits


def _no_fault():
    from ..models.blockdiff import BreakMode

    return BreakMode()


class Session:
    def __init__(self, model, block: int = 32, threshold: float = 0.9, sub_block: int = 0, max_len: int = 8192):
        from ..infer import cached

        self.model, self.block, self.threshold = model, block, threshold
        self.sub_block = sub_block or None
        self.cached = cached
        self.cache = cached.BlockCache()
        self.passes = 0
        self.cur = None
        self.max_len = max_len

    def prefill(self, ids) -> int:
        dev = self.model.text_model.embed_tokens.weight.device
        self.cur = torch.tensor([list(ids)], dtype=torch.long, device=dev)
        if self.cur.shape[1] >= self.max_len:
            raise ValueError("prompt longer than max_len")
        n_full = (self.cur.shape[1] // self.block) * self.block
        before = self.passes
        for p0 in range(0, n_full, self.block):
            self.cached.block_pass(self.model, self.cache, self.cur[:, p0:p0 + self.block], p0, commit=True)
            self.passes += 1
        self._sync()
        return self.passes - before

    def begin_block(self) -> int:
        cfg = self.model.config
        n = self.cur.shape[1]
        self.p0 = (n // self.block) * self.block
        self.k = n - self.p0
        self.blk = torch.full((1, self.block), cfg.mask_id, dtype=torch.long, device=self.cur.device)
        self.blk[:, :self.k] = self.cur[:, self.p0:n]
        self.masked = torch.zeros(1, self.block, dtype=torch.bool, device=self.cur.device)
        self.masked[:, self.k:] = True
        return int(self.masked.sum())

    @torch.no_grad()
    def step(self) -> int:
        from .. import ops
        from ..infer.golden import select_commits

        cfg = self.model.config
        ids = torch.where(self.masked, torch.full_like(self.blk, cfg.mask_id), self.blk)
        hid = self.cached.block_pass(self.model, self.cache, ids, self.p0, commit=False)
        self.passes += 1
        logits = ops.linear(hid, self.model.lm_head.weight)
        commit, pick = select_commits(logits[0], self.masked[0], self.threshold, self.sub_block, 0.0)
        idx = torch.nonzero(commit)[:, 0]
        self.blk[0, idx] = pick[idx]
        self.masked[0, idx] = False
        left = int(self.masked.sum())
        self._sync()
        return left

    @torch.no_grad()
    def commit(self):
        self.cached.block_pass(self.model, self.cache, self.blk, self.p0, commit=True)
        self.passes += 1
        new = self.blk[:, self.k:]
        self.cur = torch.cat([self.cur, new], 1)
        self._sync()
        return [int(t) for t in new[0].tolist()]

    def _sync(self):
        if self.cur is not None and self.cur.is_cuda:
            torch.cuda.synchronize(self.cur.device)
