"""Golden block-wise confidence-threshold parallel decoder (no cache).

Behaviour of the reference's `decode.generate` (`decode.py:35-99`), kept exact because it is
the temperature-0 token stream every fast decoder must reproduce: per block start all-[MASK];
each step runs the full block-diffusion forward over prompt + generated tokens, takes argmax and
softmax confidence at the still-masked positions, commits every position with confidence >=
threshold and always at least the single most confident one, until the block is clean.
`sub_block` restricts each step to the leftmost sub-block that still holds a mask. The first
block resumes mid-block after the prompt tail.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ..models.blockdiff import block_diffusion_forward


@dataclass
class DecodeTrace:
    tokens: list
    forwards: int = 0
    generated: int = 0
    steps_per_block: list = field(default_factory=list)

    @property
    def tokens_per_forward(self) -> float:
        return self.generated / self.forwards if self.forwards else 0.0


def select_commits(logits, masked, threshold: float, sub_block: int | None, temperature: float, generator=None):
    """One denoise step's commit decision for one block.

    logits [block, V] (any float dtype), masked [block] bool. Returns (commit [block] bool,
    pick [block] long). Rule (`decode.py:69-91`): confidence = softmax max (or the sampled
    token's probability at temperature > 0); candidates = masked positions, restricted to the
    leftmost sub-block that still holds a mask; commit conf >= threshold, else the argmax one."""
    logits = logits.float()
    if temperature > 0:
        probs = torch.softmax(logits / temperature, -1)
        pick = torch.multinomial(probs, 1, generator=generator)[:, 0]
        conf = probs.gather(1, pick[:, None])[:, 0]
    else:
        probs = torch.softmax(logits, -1)
        conf, pick = probs.max(-1)
    cand = masked.clone()
    if sub_block:
        first = int(torch.nonzero(cand)[0])
        s0 = (first // sub_block) * sub_block
        window = torch.zeros_like(cand)
        window[s0 : s0 + sub_block] = True
        cand &= window
    conf = conf.masked_fill(~cand, -1.0)
    commit = cand & (conf >= threshold)
    if not bool(commit.any()):
        commit[int(conf.argmax())] = True
    return commit, pick


@torch.no_grad()
def generate(model, prompt_ids: list, *, n_blocks: int, block: int, mask_id: int, threshold: float = 0.9,
             sub_block: int | None = None, eos_id: int | None = None, temperature: float = 0.0,
             layers: int | None = None, generator=None) -> DecodeTrace:
    device = model.text_model.embed_tokens.weight.device
    cur = list(prompt_ids)
    trace = DecodeTrace(tokens=cur)
    for _ in range(n_blocks):
        n = len(cur)
        kb = n // block
        L = (kb + 1) * block
        known = torch.full((L,), mask_id, dtype=torch.long, device=device)
        if n:
            known[:n] = torch.tensor(cur, device=device)
        masked = torch.zeros(L, dtype=torch.bool, device=device)
        masked[n:] = True
        x0 = known.clone()  # block kb of x_0 is invisible to x_t block kb
        steps = 0
        while bool(masked.any()):
            xt = torch.where(masked, torch.full_like(known, mask_id), known)
            lt, _ = block_diffusion_forward(model, x0[None], xt[None], block, layers=layers)
            trace.forwards += 1
            steps += 1
            commit, pick = select_commits(lt[0, kb * block : L], masked[kb * block : L], threshold, sub_block,
                                          temperature, generator)
            idx = torch.nonzero(commit)[:, 0] + kb * block
            known[idx] = pick[idx - kb * block]
            masked[idx] = False
        trace.steps_per_block.append(steps)
        new = known[n:L].tolist()
        cur.extend(new)
        trace.generated += len(new)
        if eos_id is not None and eos_id in new:
            break
    trace.tokens = cur
    return trace
