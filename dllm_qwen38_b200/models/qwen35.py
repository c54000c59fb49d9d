"""Hybrid Gated DeltaNet / gated-attention text model: the parameter container.

The module tree mirrors HF `Qwen3_5TextModel` attribute names one for one (HF
modeling_qwen3_5.py:356-414 GDN, :620-692 attention, :695-708 MLP, :711-728 norm, :731-783
layer) so that `state_dict()` keys are the HF text-model keys and checkpoints load in both
directions. Modules here hold parameters only; the math lives in `models/blockdiff.py` over the
ops layer, which never calls a submodule's forward. That is deliberate: the reference's FSDP
trainer had to wrap whole layer steps because its forward reached into submodules around FSDP
hooks (`fsdp_train.py:3-10`); our sharding engine gathers flat per-layer buffers explicitly, so
the trap cannot arise.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from ..config import FULL, LINEAR, ModelConfig


class RMSNorm(nn.Module):
    """(1 + w) RMSNorm; w zero-initialised (HF:711-728)."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(dim))
        self.eps = eps


class GatedRMSNorm(nn.Module):
    """w * rmsnorm(x) * silu(z); w one-initialised (HF:175-190)."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps


class Conv1dWeight(nn.Module):
    """Holds a depthwise conv weight with HF's nn.Conv1d shape [C, 1, K] (no bias)."""

    def __init__(self, channels: int, kernel: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(channels, 1, kernel))


def _lin(i: int, o: int) -> nn.Linear:
    return nn.Linear(i, o, bias=False)


class GatedDeltaNet(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        D = cfg.hidden_size
        self.num_k_heads = cfg.linear_num_key_heads
        self.num_v_heads = cfg.linear_num_value_heads
        self.head_k_dim = cfg.linear_key_head_dim
        self.head_v_dim = cfg.linear_value_head_dim
        self.key_dim = cfg.key_dim
        self.value_dim = cfg.value_dim
        self.conv_dim = cfg.conv_dim
        self.conv_kernel_size = cfg.linear_conv_kernel_dim
        self.in_proj_qkv = _lin(D, cfg.conv_dim)
        self.in_proj_z = _lin(D, cfg.value_dim)
        self.in_proj_b = _lin(D, cfg.linear_num_value_heads)
        self.in_proj_a = _lin(D, cfg.linear_num_value_heads)
        self.conv1d = Conv1dWeight(cfg.conv_dim, cfg.linear_conv_kernel_dim)
        self.dt_bias = nn.Parameter(torch.ones(cfg.linear_num_value_heads))
        self.A_log = nn.Parameter(torch.zeros(cfg.linear_num_value_heads))
        self.norm = GatedRMSNorm(cfg.linear_value_head_dim, cfg.rms_norm_eps)
        self.out_proj = _lin(cfg.value_dim, D)


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        D, Hq, Hk, Dh = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        self.num_heads, self.num_kv_heads, self.head_dim = Hq, Hk, Dh
        # q_proj emits [q_h | gate_h] per head (HF:652-656): row block h*2Dh..(h+1)*2Dh
        self.q_proj = _lin(D, Hq * Dh * 2)
        self.k_proj = _lin(D, Hk * Dh)
        self.v_proj = _lin(D, Hk * Dh)
        self.o_proj = _lin(Hq * Dh, D)
        self.q_norm = RMSNorm(Dh, cfg.rms_norm_eps)
        self.k_norm = RMSNorm(Dh, cfg.rms_norm_eps)


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.gate_proj = _lin(cfg.hidden_size, cfg.intermediate_size)
        self.up_proj = _lin(cfg.hidden_size, cfg.intermediate_size)
        self.down_proj = _lin(cfg.intermediate_size, cfg.hidden_size)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, idx: int):
        super().__init__()
        self.layer_type = cfg.layer_types[idx]
        if self.layer_type == LINEAR:
            self.linear_attn = GatedDeltaNet(cfg)
        elif self.layer_type == FULL:
            self.self_attn = Attention(cfg)
        else:  # pragma: no cover - ModelConfig validates
            raise ValueError(self.layer_type)
        self.mlp = MLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class TextModel(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.config = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(cfg, i) for i in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class BlockDiffusionLM(nn.Module):
    """Text tower + lm_head. State-dict keys: ``text_model.<HF text key>`` and ``lm_head.weight``
    (the reference's single-device safetensors layout, `train.py:270-276`)."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.config = cfg
        self.text_model = TextModel(cfg)
        self.lm_head = _lin(cfg.hidden_size, cfg.vocab_size)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.text_model.embed_tokens.weight

    @property
    def head_weight(self) -> torch.Tensor:
        return self.lm_head.weight

    def unique_parameters(self) -> list[nn.Parameter]:
        """Parameters deduplicated by identity (a tied head is stepped once, `train.py:134-139`)."""
        seen, out = set(), []
        for p in self.parameters():
            if id(p) not in seen:
                seen.add(id(p))
                out.append(p)
        return out


@torch.no_grad()
def init_weights(model: BlockDiffusionLM, seed: int = 0) -> BlockDiffusionLM:
    """Random init as HF's `_init_weights` (HF:802-812): Linear/Embedding/Conv ~ N(0,
    initializer_range); RMSNorm w = 0 (the (1+w) form); gated norm w = 1; dt_bias = 1; A_log = log(U(0, 16)) (HF GDN __init__,
    HF:389-393). Deterministic in (`seed`, device type) and independent of the global RNG; values
    are drawn on the parameters' own device so a large model never round-trips through the host."""
    cfg = model.config
    dev = next(model.parameters()).device
    g = torch.Generator(device=dev).manual_seed(seed)
    std = cfg.initializer_range

    def fill(p: torch.Tensor, t: torch.Tensor):
        p.copy_(t.to(dtype=p.dtype))

    def rand(shape):
        return torch.rand(shape, generator=g, device=dev)

    def randn(shape):
        return torch.randn(shape, generator=g, device=dev)

    done = set()
    for name, p in model.named_parameters(remove_duplicate=True):
        if id(p) in done:
            continue
        done.add(id(p))
        if name == "lm_head.weight" and cfg.head_init == "linear_default":
            # nn.Linear's own default (kaiming-uniform, bound 1/sqrt(fan_in)): the reference's
            # tiny model uses a bare nn.Linear head (`blockdiff.py:276`)
            fill(p, (rand(p.shape) * 2 - 1) / math.sqrt(p.shape[1]))
        elif name.endswith("dt_bias"):
            p.fill_(1.0)
        elif name.endswith("A_log"):
            fill(p, torch.log(rand(p.shape) * 16 + 1e-3))
        elif name.endswith("linear_attn.norm.weight"):
            p.fill_(1.0)
        elif p.ndim == 1:  # (1+w) RMSNorm weights
            p.zero_()
        else:
            # draw in row slabs so a [248320, 5120] table never needs an fp32 copy of itself
            rows = max(1, (1 << 26) // max(1, p[0].numel()))
            for r0 in range(0, p.shape[0], rows):
                sl = p[r0 : r0 + rows]
                fill(sl, randn(sl.shape) * std)
    return model


def build_model(cfg: ModelConfig, seed: int = 0, device="cpu", dtype=torch.float32) -> BlockDiffusionLM:
    with torch.device("meta"):
        m = BlockDiffusionLM(cfg).to(dtype)
    m = m.to_empty(device=device)
    if cfg.tie_word_embeddings:  # to_empty breaks the tie; restore it
        m.lm_head.weight = m.text_model.embed_tokens.weight
    init_weights(m, seed)
    return m
