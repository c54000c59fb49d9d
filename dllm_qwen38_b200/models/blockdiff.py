"""Fast-dLLM v2 block-diffusion forward with the state fork, over the two-stream layout.

Visibility contract (the reference's `blockdiff.py:3-8`, arXiv 2509.26328 §3), with
block(i) = i // block:

  M_BD  : x_t token i sees x_t token j  iff block(j) == block(i)
  M_OBC : x_t token i sees x_0 token j  iff block(j) <  block(i)
  M_BC  : x_0 token i sees x_0 token j  iff block(j) <= block(i)

Design. Both streams are one tensor ``h [B, 2L, D]`` (x_t at [0, L), x_0 at [L, 2L)). Every
token-wise op (norms, projections, MLP) therefore runs once over 2BL rows. The three places
where the streams interact resolve the contract by index arithmetic instead of reshapes:

* attention takes the complementary mask as a predicate on (query, key) positions;
* the short conv reads a noised token's taps that fall before its block from the clean stream
  (the conv-prefix half of the state fork);
* the delta rule runs x_0 once, keeps S_k at every block end, and starts noised block k from
  S_{k-1} (the recurrent half of the state fork, `blockdiff.py:159-177` of the reference).

``BreakMode`` carries the reference's three deliberate faults (`blockdiff.py:69-88`); each must
turn the equivalence check red.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import partial

import torch
from torch.utils.checkpoint import checkpoint as _grad_checkpoint

from .. import ops
from ..config import FULL, LINEAR
from ..ops import reference as ref


@dataclass
class BreakMode:
    """Deliberate faults (`blockdiff.py:69-88` of the reference)."""

    name: str = "none"

    @property
    def concat_causal_gdn(self) -> bool:
        # DeltaNet run over cat([x_t, x_0]) as one causal sequence
        return self.name == "concat-causal-gdn"

    @property
    def leak_xt_prefix(self) -> bool:
        # attention mask where x_t block k also sees x_t blocks < k
        return self.name == "mask-leak"

    @property
    def drop_conv_prefix(self) -> bool:
        # state forked, but the short conv of every noised block starts cold
        return self.name == "no-conv-prefix"


FAULTS = ("concat-causal-gdn", "mask-leak", "no-conv-prefix")


def rope_tables(cfg, L: int, dtype, device):
    """cos/sin [L, rotary_dim]; x_t and x_0 share positions 0..L-1 (`blockdiff.py:143-144`)."""
    return ref.rope_cos_sin(torch.arange(L), cfg.rotary_dim, cfg.rope_theta, dtype, device)


# ----------------------------------------------------------------------------- mixers


def gdn_mixer(m, n: torch.Tensor, L: int, block: int, chunk: int, fault: BreakMode) -> torch.Tensor:
    """Gated DeltaNet over both streams with the state fork. n [B, 2L, D] -> [B, 2L, D].

    Same math as the reference's two `gdn_mixer_forward` calls (`gdn.py:193-233`,
    `blockdiff.py:159-177`), done as one pass over the two-stream layout."""
    B, T2, _ = n.shape
    # one GEMM for the four input projections (qkv | z | b | a)
    w_in = getattr(m, "fused_in_weight", None)  # a sharding engine may supply the contiguous block
    if w_in is None:
        w_in = torch.cat([m.in_proj_qkv.weight, m.in_proj_z.weight, m.in_proj_b.weight, m.in_proj_a.weight], 0)
    proj = ops.linear(n, w_in)
    raw, z, b, a = torch.split(proj, [m.conv_dim, m.value_dim, m.num_v_heads, m.num_v_heads], dim=-1)
    if fault.concat_causal_gdn:
        conv_mode, core_mode = ref.CONV_CONCAT, ref.GDN_CONCAT
    else:
        conv_mode = ref.CONV_NOPREFIX if fault.drop_conv_prefix else ref.CONV_FORK
        core_mode = ref.GDN_FORK
    mixed = ops.conv_blockdiff(raw, m.conv1d.weight[:, 0, :], L, block, conv_mode)
    q, k, v = torch.split(mixed, [m.key_dim, m.key_dim, m.value_dim], dim=-1)
    q = q.reshape(B, T2, m.num_k_heads, m.head_k_dim)
    k = k.reshape(B, T2, m.num_k_heads, m.head_k_dim)
    v = v.reshape(B, T2, m.num_v_heads, m.head_v_dim)
    g, beta = ops.gdn_gates(a, b, m.A_log, m.dt_bias)
    core = ops.gdn_core_blockdiff(q, k, v, g, beta, L, block, chunk, core_mode)  # [B, 2L, Hv, Dv]
    y = ops.gated_rmsnorm(core, z.reshape(B, T2, m.num_v_heads, m.head_v_dim), m.norm.weight, m.norm.eps)
    return ops.linear(y.reshape(B, T2, m.value_dim), m.out_proj.weight)


def attn_mixer(m, n: torch.Tensor, L: int, block: int, cos, sin, fault: BreakMode) -> torch.Tensor:
    """Output-gated GQA attention under the complementary mask. n [B, 2L, D] -> [B, 2L, D]."""
    B, T2, _ = n.shape
    Hq, Hk, Dh = m.num_heads, m.num_kv_heads, m.head_dim
    # one GEMM for q|gate, k, v
    w_qkv = getattr(m, "fused_qkv_weight", None)
    if w_qkv is None:
        w_qkv = torch.cat([m.q_proj.weight, m.k_proj.weight, m.v_proj.weight], 0)
    proj = ops.linear(n, w_qkv)
    qg, k, v = torch.split(proj, [2 * Hq * Dh, Hk * Dh, Hk * Dh], dim=-1)
    qg = qg.reshape(B, T2, Hq, 2 * Dh)
    q, gate = torch.split(qg, Dh, dim=-1)  # one concatenation in backward, no zero-filled slice grads
    k = k.reshape(B, T2, Hk, Dh)
    v = v.reshape(B, T2, Hk, Dh)
    cos2, sin2 = torch.cat([cos, cos], 0), torch.cat([sin, sin], 0)
    q, k = ops.qk_norm_rope(q, k, m.q_norm.weight, m.k_norm.weight, m.q_norm.eps, cos2, sin2)
    o = ops.attention_blockdiff(q, k, v, L, block, Dh ** -0.5, fault.leak_xt_prefix)
    o = ops.output_gate(o, gate)
    return ops.linear(o.reshape(B, T2, Hq * Dh), m.o_proj.weight)


def mlp(m, x: torch.Tensor) -> torch.Tensor:
    w_gu = getattr(m, "fused_gate_up_weight", None)
    if w_gu is not None:
        return ops.swiglu_mlp_fused(x, w_gu, m.down_proj.weight)
    return ops.swiglu_mlp(x, m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight)


def layer_step(layer, kind: str, h: torch.Tensor, L: int, block: int, chunk: int, cos, sin, fault: BreakMode):
    """One decoder layer for both streams (the checkpointing unit). Pre-norm residual
    (HF:731-783); the MLP is shared by both streams and runs over all 2BL rows at once."""
    n = ops.rmsnorm(h, layer.input_layernorm.weight, layer.input_layernorm.eps)
    if kind == LINEAR:
        o = gdn_mixer(layer.linear_attn, n, L, block, chunk, fault)
    elif kind == FULL:
        o = attn_mixer(layer.self_attn, n, L, block, cos, sin, fault)
    else:
        raise ValueError(f"unknown layer type {kind}")
    h = h + o
    return h + mlp(layer.mlp, ops.rmsnorm(h, layer.post_attention_layernorm.weight, layer.post_attention_layernorm.eps))


def block_diffusion_forward(model, x0_ids: torch.Tensor, xt_ids: torch.Tensor, block: int, *,
                            fault: BreakMode | None = None, layers: int | None = None, output: str = "logits",
                            checkpointing: bool = False):
    """Training/inference forward over both streams (the reference's `block_diffusion_forward`,
    `blockdiff.py:96-203`).

    Returns (logits_t [B, L, V], logits_0 [B, L, V]), or with output="hidden" the final-normed
    hidden states (h_t, h_0) [B, L, D] so the caller projects only the rows it scores.
    checkpointing=True recomputes each layer in backward (non-reentrant, layer bound with
    functools.partial at call time: a closure over the loop variable re-ran the last layer for
    every checkpoint in the reference's history, `blockdiff.py:113-126`)."""
    fault = fault or BreakMode()
    cfg = model.config
    if x0_ids.shape != xt_ids.shape or x0_ids.ndim != 2:
        raise ValueError("x0_ids and xt_ids must both be [B, L]")
    B, L = x0_ids.shape
    if L % block:
        raise ValueError(f"L={L} is not a multiple of block={block}")
    tm = model.text_model
    h = ops.embedding(torch.cat([xt_ids, x0_ids], 1), tm.embed_tokens.weight)
    cos, sin = rope_tables(cfg, L, h.dtype, h.device)
    n_layers = cfg.num_hidden_layers if layers is None else layers
    chunk = cfg.gdn_chunk_size
    for i in range(n_layers):
        layer, kind = tm.layers[i], cfg.layer_types[i]
        if checkpointing and torch.is_grad_enabled():
            h = _grad_checkpoint(partial(layer_step, layer, kind), h, L, block, chunk, cos, sin, fault,
                                 use_reentrant=False)
        else:
            h = layer_step(layer, kind, h, L, block, chunk, cos, sin, fault)
    h = ops.rmsnorm(h, tm.norm.weight, tm.norm.eps)
    ht, h0 = h[:, :L], h[:, L:]
    if output == "hidden":
        return ht, h0
    w = model.lm_head.weight
    return ops.linear(ht, w), ops.linear(h0, w)
