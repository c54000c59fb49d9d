"""Independent oracles for the state-fork forward.

``reference_block_logits`` is the per-block recompute the reference uses as its oracle
(`blockdiff.py:206-228`): for each block k, an UNFORKED forward over
cat([x_0 blocks < k, x_t block k]) under a block-causal mask, keeping the last block's logits.
Here the unforked forward is `plain_forward`, written on the reference ops only (never the
dispatching op layer, never a CUDA kernel), with the Gated DeltaNet run either token by token
(the decode-form recurrence, HF:314-353 — the default, so the oracle shares no chunking code
with the candidate) or chunked.

``hf_text_model`` copies our weights into the installed HuggingFace `Qwen3_5TextModel`, which
pins our model definition to HF's math (tests compare the two on a plain causal forward).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ..config import FULL, LINEAR
from ..ops import reference as ref


def _gdn_plain(m, n: torch.Tensor, gdn: str, chunk: int) -> torch.Tensor:
    B, T, _ = n.shape
    raw = ref.linear(n, m.in_proj_qkv.weight)
    z = ref.linear(n, m.in_proj_z.weight)
    b = ref.linear(n, m.in_proj_b.weight)
    a = ref.linear(n, m.in_proj_a.weight)
    mixed = ref.causal_conv_silu(raw, m.conv1d.weight[:, 0, :])
    q, k, v = torch.split(mixed, [m.key_dim, m.key_dim, m.value_dim], dim=-1)
    q = q.reshape(B, T, m.num_k_heads, m.head_k_dim)
    k = k.reshape(B, T, m.num_k_heads, m.head_k_dim)
    v = v.reshape(B, T, m.num_v_heads, m.head_v_dim)
    g, beta = ref.gdn_gates(a, b, m.A_log, m.dt_bias)
    rep = m.num_v_heads // m.num_k_heads
    if rep > 1:
        q, k = q.repeat_interleave(rep, 2), k.repeat_interleave(rep, 2)
    if gdn == "recurrent":
        core, _ = ref.recurrent_gated_delta_rule(q, k, v, g, beta)
    else:
        import math

        core, _ = ref.chunk_gated_delta_rule(q, k, v, g, beta, math.gcd(chunk, T))
    y = ref.gated_rmsnorm(core, z.reshape(B, T, m.num_v_heads, m.head_v_dim), m.norm.weight, m.norm.eps)
    return ref.linear(y.reshape(B, T, -1), m.out_proj.weight)


def _attn_plain(m, n, allowed, cos, sin) -> torch.Tensor:
    B, T, _ = n.shape
    Hq, Hk, Dh = m.num_heads, m.num_kv_heads, m.head_dim
    qg = ref.linear(n, m.q_proj.weight).reshape(B, T, Hq, 2 * Dh)
    q, gate = qg[..., :Dh], qg[..., Dh:]
    k = ref.linear(n, m.k_proj.weight).reshape(B, T, Hk, Dh)
    v = ref.linear(n, m.v_proj.weight).reshape(B, T, Hk, Dh)
    q = ref.apply_rope(ref.rmsnorm(q, m.q_norm.weight, m.q_norm.eps), cos, sin)
    k = ref.apply_rope(ref.rmsnorm(k, m.k_norm.weight, m.k_norm.eps), cos, sin)
    o = ref.attention(q, k, v, allowed, Dh ** -0.5) * torch.sigmoid(gate)
    return ref.linear(o.reshape(B, T, -1), m.o_proj.weight)


@torch.no_grad()
def plain_forward(model, ids: torch.Tensor, allowed: torch.Tensor, *, layers: int | None = None,
                  gdn: str = "recurrent", output: str = "logits") -> torch.Tensor:
    """Unforked single-stream forward: attention under `allowed` [T, T], causal DeltaNet."""
    cfg = model.config
    tm = model.text_model
    B, T = ids.shape
    h = F.embedding(ids, tm.embed_tokens.weight)
    cos, sin = ref.rope_cos_sin(torch.arange(T), cfg.rotary_dim, cfg.rope_theta, h.dtype, h.device)
    for i in range(cfg.num_hidden_layers if layers is None else layers):
        layer, kind = tm.layers[i], cfg.layer_types[i]
        n = ref.rmsnorm(h, layer.input_layernorm.weight, layer.input_layernorm.eps)
        if kind == LINEAR:
            h = h + _gdn_plain(layer.linear_attn, n, gdn, cfg.gdn_chunk_size)
        elif kind == FULL:
            h = h + _attn_plain(layer.self_attn, n, allowed, cos, sin)
        mm = layer.mlp
        x = ref.rmsnorm(h, layer.post_attention_layernorm.weight, layer.post_attention_layernorm.eps)
        h = h + ref.linear(ref.swiglu(ref.linear(x, mm.gate_proj.weight), ref.linear(x, mm.up_proj.weight)), mm.down_proj.weight)
    h = ref.rmsnorm(h, tm.norm.weight, tm.norm.eps)
    return h if output == "hidden" else ref.linear(h, model.lm_head.weight)


@torch.no_grad()
def reference_block_logits(model, x0_ids, xt_ids, block: int, *, layers: int | None = None, gdn: str = "recurrent"):
    """Per block k: unforked forward over cat([x_0[:k*block], x_t block k]) under a block-causal
    mask; returns the last block's logits concatenated over k -> [B, L, V]."""
    L = x0_ids.shape[1]
    outs = []
    for k in range(L // block):
        seq = torch.cat([x0_ids[:, : k * block], xt_ids[:, k * block : (k + 1) * block]], 1)
        allowed = ref.block_causal_allowed(seq.shape[1], block, seq.device)
        outs.append(plain_forward(model, seq, allowed, layers=layers, gdn=gdn)[:, -block:])
    return torch.cat(outs, 1)


@torch.no_grad()
def reference_clean_logits(model, x0_ids, block: int, *, layers: int | None = None, gdn: str = "recurrent"):
    """Unforked forward over x_0 under the block-causal mask (`blockdiff.py:231-243`)."""
    allowed = ref.block_causal_allowed(x0_ids.shape[1], block, x0_ids.device)
    return plain_forward(model, x0_ids, allowed, layers=layers, gdn=gdn)


def hf_text_model(model):
    """Our weights inside the installed HF `Qwen3_5TextModel` (eager attention, fp32 as ours).
    Raises ImportError if this transformers has no qwen3_5."""
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

    c = model.config
    half = c.rotary_dim // 2
    sec = [half - 2 * (half // 4), half // 4, half // 4]  # text positions: any split is plain RoPE
    hc = Qwen3_5TextConfig(
        vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
        num_hidden_layers=c.num_hidden_layers, layer_types=list(c.layer_types),
        num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim,
        linear_num_key_heads=c.linear_num_key_heads, linear_num_value_heads=c.linear_num_value_heads,
        linear_key_head_dim=c.linear_key_head_dim, linear_value_head_dim=c.linear_value_head_dim,
        linear_conv_kernel_dim=c.linear_conv_kernel_dim, rms_norm_eps=c.rms_norm_eps,
        max_position_embeddings=8192,
        rope_parameters={"rope_type": "default", "rope_theta": c.rope_theta, "mrope_section": sec,
                         "partial_rotary_factor": c.partial_rotary_factor},
        attn_implementation="eager",
    )
    hm = Qwen3_5TextModel(hc).eval().to(next(model.parameters()).dtype)
    missing, unexpected = hm.load_state_dict(model.text_model.state_dict(), strict=False)
    bad = [k for k in missing if "rotary" not in k] + list(unexpected)
    if bad:
        raise ValueError(f"HF key mismatch: {bad[:10]}")
    return hm
