"""Cached block-diffusion decoder: the golden decoder's token stream at a fraction of its cost.

The golden decoder (`decode.py:35-99` of the reference, `infer/golden.py` here) re-runs the full
two-stream forward over the whole prefix at every denoising step. Under the complementary mask,
noised block k sees exactly (a) its own block, bidirectionally, and (b) the clean prefix x_0
blocks < k: the attention keys/values of those clean tokens, and, for Gated DeltaNet layers, the
recurrent state and the short-conv tail at position k*block (the state fork). The clean prefix
never changes while block k is being decoded, so it is cached:

  * attention layers keep K/V of every committed clean token;
  * GDN layers keep the fp32 state after the committed tokens and the last (kernel-1) pre-conv
    projections (the conv tail).

A denoising step runs only the current block (B x block tokens) through the layers, attending to
[cache || block] with no mask and starting each GDN layer from the cached state and conv tail.
Committing a finished block runs the same block pass on its clean tokens -- the clean stream sees
exactly the same keys (block-causal = prefix + own block) -- and appends its K/V, advances the GDN
state and conv tail. The commit rule (threshold, at least one, sub-block window, temperature) is
the golden decoder's `select_commits`.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .. import ops
from ..config import FULL, LINEAR
from ..ops import reference as ref
from .golden import DecodeTrace, select_commits


@dataclass
class LayerCache:
    k: torch.Tensor | None = None  # [B, T, Hk, Dh]
    v: torch.Tensor | None = None
    S: torch.Tensor | None = None  # [B, Hv, Dk, Dv] fp32
    tail: torch.Tensor | None = None  # [B, K-1, conv_dim]


@dataclass
class BlockCache:
    layers: list = field(default_factory=list)
    length: int = 0  # committed clean tokens held


def _gdn_block(m, n, lc: LayerCache, commit: bool):
    """GDN over one block from the cached state/conv tail. n [B, T, D] -> [B, T, D]."""
    B, T, _ = n.shape
    w_in = torch.cat([m.in_proj_qkv.weight, m.in_proj_z.weight, m.in_proj_b.weight, m.in_proj_a.weight], 0)
    proj = ops.linear(n, w_in)
    raw, z, b, a = torch.split(proj, [m.conv_dim, m.value_dim, m.num_v_heads, m.num_v_heads], dim=-1)
    km1 = m.conv_kernel_size - 1
    tail = lc.tail if lc.tail is not None else raw.new_zeros(B, km1, m.conv_dim)
    seq = torch.cat([tail, raw], 1)
    mixed = ref.causal_conv_silu(seq, m.conv1d.weight[:, 0, :])[:, km1:]
    q, k, v = torch.split(mixed, [m.key_dim, m.key_dim, m.value_dim], dim=-1)
    q = q.reshape(B, T, m.num_k_heads, m.head_k_dim)
    k = k.reshape(B, T, m.num_k_heads, m.head_k_dim)
    v = v.reshape(B, T, m.num_v_heads, m.head_v_dim)
    g, beta = ref.gdn_gates(a, b, m.A_log, m.dt_bias)
    rep = m.num_v_heads // m.num_k_heads
    if rep > 1:
        q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
    core, states = ref.chunk_gated_delta_rule(q, k, v, g, beta, T, initial_state=lc.S, state_every=T)
    if commit:
        lc.S = states[:, -1].float()
        lc.tail = seq[:, -km1:].clone()
    y = ops.gated_rmsnorm(core, z.reshape(B, T, m.num_v_heads, m.head_v_dim), m.norm.weight, m.norm.eps)
    return ops.linear(y.reshape(B, T, m.value_dim), m.out_proj.weight)


def _attn_block(m, n, lc: LayerCache, cos, sin, commit: bool):
    """Attention of one block over [cached clean K/V || own block], no mask. n [B, T, D]."""
    B, T, _ = n.shape
    Hq, Hk, Dh = m.num_heads, m.num_kv_heads, m.head_dim
    proj = ops.linear(n, torch.cat([m.q_proj.weight, m.k_proj.weight, m.v_proj.weight], 0))
    qg, k, v = torch.split(proj, [2 * Hq * Dh, Hk * Dh, Hk * Dh], dim=-1)
    qg = qg.reshape(B, T, Hq, 2 * Dh)
    q, gate = qg[..., :Dh], qg[..., Dh:]
    k = k.reshape(B, T, Hk, Dh)
    v = v.reshape(B, T, Hk, Dh)
    q = ref.apply_rope(ref.rmsnorm(q, m.q_norm.weight, m.q_norm.eps), cos, sin)
    k = ref.apply_rope(ref.rmsnorm(k, m.k_norm.weight, m.k_norm.eps), cos, sin)
    kk = k if lc.k is None else torch.cat([lc.k, k], 1)
    vv = v if lc.v is None else torch.cat([lc.v, v], 1)
    allowed = torch.ones(T, kk.shape[1], dtype=torch.bool, device=n.device)
    if n.is_cuda:
        o = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2), scale=Dh ** -0.5, enable_gqa=True).transpose(1, 2)
    else:
        o = _attention_rect(q, kk, vv, Dh ** -0.5)
    del allowed
    if commit:
        lc.k, lc.v = kk, vv
    o = o * torch.sigmoid(gate)
    return ops.linear(o.reshape(B, T, Hq * Dh), m.o_proj.weight)


def _attention_rect(q, k, v, scale):
    """q [B, Tq, Hq, D] over k/v [B, Tk, Hk, D] with every key visible (fp32 softmax)."""
    rep = q.shape[2] // k.shape[2]
    qh = q.transpose(1, 2).float()
    kh = k.transpose(1, 2).float().repeat_interleave(rep, 1)
    vh = v.transpose(1, 2).float().repeat_interleave(rep, 1)
    p = torch.softmax((qh @ kh.transpose(-1, -2)) * scale, -1)
    return (p @ vh).transpose(1, 2).to(q.dtype)


@torch.no_grad()
def block_pass(model, cache: BlockCache, ids: torch.Tensor, p0: int, commit: bool) -> torch.Tensor:
    """Run one block of tokens at positions [p0, p0 + T) over the cache; returns final-normed hidden
    [B, T, D]. commit=True extends the cache with these tokens as clean tokens."""
    cfg = model.config
    tm = model.text_model
    B, T = ids.shape
    if not cache.layers:
        cache.layers = [LayerCache() for _ in range(cfg.num_hidden_layers)]
    h = ops.embedding(ids, tm.embed_tokens.weight)
    cos, sin = ref.rope_cos_sin(torch.arange(p0, p0 + T), cfg.rotary_dim, cfg.rope_theta, h.dtype, h.device)
    for i in range(cfg.num_hidden_layers):
        layer, kind, lc = tm.layers[i], cfg.layer_types[i], cache.layers[i]
        n = ops.rmsnorm(h, layer.input_layernorm.weight, layer.input_layernorm.eps)
        if kind == LINEAR:
            o = _gdn_block(layer.linear_attn, n, lc, commit)
        elif kind == FULL:
            o = _attn_block(layer.self_attn, n, lc, cos, sin, commit)
        else:
            raise ValueError(kind)
        h = h + o
        mm = layer.mlp
        x = ops.rmsnorm(h, layer.post_attention_layernorm.weight, layer.post_attention_layernorm.eps)
        h = h + ops.swiglu_mlp(x, mm.gate_proj.weight, mm.up_proj.weight, mm.down_proj.weight)
    if commit:
        cache.length = p0 + T
    return ops.rmsnorm(h, tm.norm.weight, tm.norm.eps)


@torch.no_grad()
def prefill(model, cache: BlockCache, ids: torch.Tensor, block: int) -> None:
    """Commit the prompt's whole blocks [0, (len // block) * block) as clean tokens, block by block."""
    n_full = (ids.shape[1] // block) * block
    for p0 in range(0, n_full, block):
        block_pass(model, cache, ids[:, p0 : p0 + block], p0, commit=True)


@torch.no_grad()
def generate(model, prompt_ids, *, n_blocks: int, block: int, mask_id: int, threshold: float = 0.9,
             sub_block: int | None = None, eos_id: int | None = None, temperature: float = 0.0,
             generator=None) -> DecodeTrace | list:
    """Same contract as `golden.generate`. `prompt_ids` is one list (returns a DecodeTrace) or a list
    of equal-length lists (batched; returns one DecodeTrace per row)."""
    batched = len(prompt_ids) > 0 and isinstance(prompt_ids[0], (list, tuple))
    rows = [list(p) for p in (prompt_ids if batched else [prompt_ids])]
    if len({len(r) for r in rows}) != 1:
        raise ValueError("batched decoding needs equal prompt lengths")
    device = model.text_model.embed_tokens.weight.device
    B = len(rows)
    traces = [DecodeTrace(tokens=list(r)) for r in rows]
    cur = torch.tensor(rows, dtype=torch.long, device=device)
    cache = BlockCache()
    prefill(model, cache, cur, block)
    head = model.lm_head.weight
    done = torch.zeros(B, dtype=torch.bool, device=device)
    for _ in range(n_blocks):
        n = cur.shape[1]
        kb = n // block
        p0 = kb * block
        blk = torch.full((B, block), mask_id, dtype=torch.long, device=device)
        blk[:, : n - p0] = cur[:, p0:n]
        masked = torch.zeros(B, block, dtype=torch.bool, device=device)
        masked[:, n - p0 :] = True
        masked &= ~done[:, None]
        steps = 0
        while bool(masked.any()):
            hid = block_pass(model, cache, torch.where(masked, torch.full_like(blk, mask_id), blk), p0, commit=False)
            logits = ops.linear(hid, head)
            steps += 1
            for r in range(B):
                if not bool(masked[r].any()):
                    continue
                traces[r].forwards += 1
                commit, pick = select_commits(logits[r], masked[r], threshold, sub_block, temperature, generator)
                idx = torch.nonzero(commit)[:, 0]
                blk[r, idx] = pick[idx]
                masked[r, idx] = False
        block_pass(model, cache, blk, p0, commit=True)
        new = blk[:, n - p0 :]
        cur = torch.cat([cur, new], 1)
        for r in range(B):
            if bool(done[r]):
                continue
            toks = new[r].tolist()
            traces[r].tokens.extend(toks)
            traces[r].generated += len(toks)
            traces[r].steps_per_block.append(steps)
            if eos_id is not None and eos_id in toks:
                done[r] = True
        if bool(done.all()):
            break
    return traces if batched else traces[0]
