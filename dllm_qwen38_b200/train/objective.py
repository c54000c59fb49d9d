"""Fast-dLLM v2 training objective: complementary masking + masked-token cross-entropy.

Same contract as the reference (`objective.py:1-84`): for every sequence draw one mask m with a
ratio t ~ U(0, 1) per (row, block) and train on both views m and (1 - m), so every scorable
token is a target exactly once per step. Prompt and padding positions are never noised and
never scored. [MASK] is one spare embedding row.
"""

from __future__ import annotations

import torch

from .. import ops


def mask_token_id(model, tokenizer) -> int:
    """First embedding row the tokenizer does not use (`objective.py:18-23`)."""
    rows = model.text_model.embed_tokens.weight.shape[0]
    n = len(tokenizer)
    if rows <= n:
        raise ValueError(f"no spare embedding row for [MASK]: rows={rows} tokenizer={n}; resize first")
    return n


def sample_complementary_masks(x0, prompt_len, block: int, generator=None, valid_len=None):
    """(m, m_complement) bool [B, L]; True = noised in that view (`objective.py:26-51`)."""
    B, L = x0.shape
    nb = L // block
    t = torch.rand(B, nb, 1, generator=generator, device=x0.device)
    u = torch.rand(B, nb, block, generator=generator, device=x0.device)
    m = (u < t).reshape(B, L)
    pos = torch.arange(L, device=x0.device)[None, :]
    scorable = pos >= prompt_len[:, None]
    if valid_len is not None:
        scorable &= pos < valid_len[:, None]
    m = m & scorable
    return m, (~m) & scorable


def apply_mask(x0, m, mask_id: int):
    return torch.where(m, torch.full_like(x0, mask_id), x0)


def complementary_step_inputs(x0, prompt_len, block: int, mask_id: int, generator=None, valid_len=None,
                              seed: int | None = None):
    """Both views stacked along batch: (x0_2B, xt_2B, m_2B) (`objective.py:72-76`). On CUDA with
    an integer `seed`, one kernel draws the masks (counter-based: a pure function of the seed and
    the element's (row, position)) and writes both views; otherwise torch's RNG with `generator`."""
    if seed is not None and x0.is_cuda:
        from ..ops import _native
        from ..ops import cuda as Cu

        out = tuple(_native.require().mask_sample(x0, prompt_len, valid_len, block, mask_id, seed))
        Cu.LAUNCHES[0] += 1  # one launch of this repository's kernels
        return out
    m, mc = sample_complementary_masks(x0, prompt_len, block, generator, valid_len)
    return torch.cat([x0, x0], 0), torch.cat([apply_mask(x0, m, mask_id), apply_mask(x0, mc, mask_id)], 0), torch.cat([m, mc], 0)


def masked_ce(logits_t, x0, m):
    """Mean CE over masked positions; (loss, n). n == 0 -> the caller must skip the step."""
    n = int(m.sum())
    if n == 0:
        return logits_t.new_zeros(()), 0
    return torch.nn.functional.cross_entropy(logits_t[m].float(), x0[m]), n


def masked_ce_sum_from_hidden(hidden_t, head_w, x0, m):
    """Sum of CE over masked rows, projecting only those rows (`objective.py:79-84`,
    `fsdp_train.py:618-623`). Returns (ce_sum fp32 scalar, n). With n == 0 the sum is a
    graph-connected zero so every parameter still receives a (zero) gradient."""
    idx = m.reshape(-1).nonzero().squeeze(1)
    n = int(idx.numel())
    if n == 0:
        return hidden_t.float().sum() * 0.0, 0
    rows = hidden_t.reshape(-1, hidden_t.shape[-1]).index_select(0, idx)
    tgt = x0.reshape(-1).index_select(0, idx)
    return ops.masked_ce_sum(rows, head_w, tgt), n


def masked_ce_from_hidden(hidden_t, head_w, x0, m):
    """Mean CE over masked rows; (loss, n)."""
    s, n = masked_ce_sum_from_hidden(hidden_t, head_w, x0, m)
    return (s / n if n else s), n
