"""Model configuration for the hybrid Gated DeltaNet / gated-attention Qwen family.

One dataclass covers every size. Field names follow the HF `Qwen3_5TextConfig` spelling so an
HF `config.json` maps onto it key for key (reference: `equivalence.py:49` reads the HF config;
`blockdiff.py:257-273` builds the tiny one inline).

Presets:
  * ``tiny_ref``  -- the reference's own CPU test model (`blockdiff.py:246-278`): vocab 256,
    hidden 64, 8 layers, untied head.
  * ``tiny``      -- the CPU fp32 equivalence config: vocab 1024 with [MASK]=1023, hidden 128,
    8 layers [GDN,GDN,GDN,Attn]x2, GDN 4/4 heads of dim 32, attention 4q/2kv dim 32,
    RoPE theta 1e7, FFN 384, tied embeddings.
  * ``0.8b``      -- 24 layers (18 GDN + 6 attention), hidden 1024, FFN 3584, GDN 16/16 heads of
    dim 128, attention 8q/2kv of dim 256, vocab 248320, tied.
  * ``27b``       -- 64 layers (48 GDN + 16 attention), hidden 5120, FFN 17408, GDN 16 qk / 48 v
    heads of dim 128, attention 24q/4kv of dim 256, vocab 248320.
"""

from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field

LINEAR = "linear_attention"
FULL = "full_attention"


def hybrid_layer_types(n_layers: int, interval: int = 4) -> list[str]:
    """3:1 interleave: every `interval`-th layer is full attention, the rest Gated DeltaNet."""
    return [FULL if (i + 1) % interval == 0 else LINEAR for i in range(n_layers)]


@dataclass
class ModelConfig:
    vocab_size: int = 1024
    hidden_size: int = 128
    intermediate_size: int = 384
    num_hidden_layers: int = 8
    layer_types: list = field(default_factory=lambda: hybrid_layer_types(8))
    # gated softmax attention
    num_attention_heads: int = 4
    num_key_value_heads: int = 2
    head_dim: int = 32
    rope_theta: float = 1e7
    partial_rotary_factor: float = 0.25
    # Gated DeltaNet
    linear_num_key_heads: int = 4
    linear_num_value_heads: int = 4
    linear_key_head_dim: int = 32
    linear_value_head_dim: int = 32
    linear_conv_kernel_dim: int = 4
    gdn_chunk_size: int = 64
    # misc
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    initializer_range: float = 0.02
    head_init: str = "normal"  # untied head: "normal" (N(0, initializer_range)) or "linear_default"
    mask_token_id: int | None = None  # None -> vocab_size - 1
    name: str = "custom"

    def __post_init__(self):
        if len(self.layer_types) != self.num_hidden_layers:
            raise ValueError(f"layer_types has {len(self.layer_types)} entries for {self.num_hidden_layers} layers")
        for t in self.layer_types:
            if t not in (LINEAR, FULL):
                raise ValueError(f"unknown layer type {t!r}")

    # ---- derived sizes
    @property
    def key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def mask_id(self) -> int:
        return self.vocab_size - 1 if self.mask_token_id is None else self.mask_token_id

    def truncated(self, layers: int | None) -> "ModelConfig":
        """Copy keeping only the first `layers` layers (the reference's first-N-layers runs)."""
        if layers is None or layers == self.num_hidden_layers:
            return self
        if not 1 <= layers <= self.num_hidden_layers:
            raise ValueError(f"layers={layers} outside 1..{self.num_hidden_layers}")
        return dataclasses.replace(self, num_hidden_layers=layers, layer_types=list(self.layer_types[:layers]))

    def param_count(self, embeddings: bool = True) -> int:
        D, F = self.hidden_size, self.intermediate_size
        n = 0
        for t in self.layer_types:
            n += 2 * D + 3 * D * F  # two norms + SwiGLU
            if t == LINEAR:
                Hv = self.linear_num_value_heads
                n += D * self.conv_dim + D * self.value_dim + 2 * D * Hv + self.value_dim * D
                n += self.conv_dim * self.linear_conv_kernel_dim + 2 * Hv + self.linear_value_head_dim
            else:
                Hq, Hk, Dh = self.num_attention_heads, self.num_key_value_heads, self.head_dim
                n += D * Hq * Dh * 2 + 2 * D * Hk * Dh + Hq * Dh * D + 2 * Dh
        n += D  # final norm
        if embeddings:
            n += self.vocab_size * D * (1 if self.tie_word_embeddings else 2)
        return n

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    # ---- HF interop
    @classmethod
    def from_hf_dict(cls, d: dict, name: str = "hf") -> "ModelConfig":
        """Map an HF Qwen3.5 `config.json` (text config, or the VLM wrapper's text_config)."""
        if "text_config" in d and isinstance(d["text_config"], dict):
            tie = d.get("tie_word_embeddings", d["text_config"].get("tie_word_embeddings", False))
            d = dict(d["text_config"], tie_word_embeddings=tie)
        rope = d.get("rope_parameters") or d.get("rope_scaling") or {}
        n = d["num_hidden_layers"]
        return cls(
            vocab_size=d["vocab_size"],
            hidden_size=d["hidden_size"],
            intermediate_size=d["intermediate_size"],
            num_hidden_layers=n,
            layer_types=list(d.get("layer_types") or hybrid_layer_types(n, d.get("full_attention_interval", 4))),
            num_attention_heads=d["num_attention_heads"],
            num_key_value_heads=d["num_key_value_heads"],
            head_dim=d.get("head_dim", d["hidden_size"] // d["num_attention_heads"]),
            rope_theta=float(rope.get("rope_theta", d.get("rope_theta", 1e7))),
            partial_rotary_factor=float(rope.get("partial_rotary_factor", d.get("partial_rotary_factor", 0.25))),
            linear_num_key_heads=d["linear_num_key_heads"],
            linear_num_value_heads=d["linear_num_value_heads"],
            linear_key_head_dim=d["linear_key_head_dim"],
            linear_value_head_dim=d["linear_value_head_dim"],
            linear_conv_kernel_dim=d.get("linear_conv_kernel_dim", 4),
            rms_norm_eps=d.get("rms_norm_eps", 1e-6),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            initializer_range=d.get("initializer_range", 0.02),
            name=name,
        )

    def to_hf_dict(self) -> dict:
        """HF Qwen3.5 text `config.json` for this config (the inverse of `from_hf_dict`)."""
        return {"model_type": "qwen3_5_text", "architectures": ["Qwen3_5ForCausalLM"],
                "vocab_size": self.vocab_size, "hidden_size": self.hidden_size,
                "intermediate_size": self.intermediate_size, "num_hidden_layers": self.num_hidden_layers,
                "layer_types": list(self.layer_types), "num_attention_heads": self.num_attention_heads,
                "num_key_value_heads": self.num_key_value_heads, "head_dim": self.head_dim,
                "rope_parameters": {"rope_type": "default", "rope_theta": self.rope_theta,
                                    "partial_rotary_factor": self.partial_rotary_factor},
                "linear_num_key_heads": self.linear_num_key_heads,
                "linear_num_value_heads": self.linear_num_value_heads,
                "linear_key_head_dim": self.linear_key_head_dim, "linear_value_head_dim": self.linear_value_head_dim,
                "linear_conv_kernel_dim": self.linear_conv_kernel_dim, "rms_norm_eps": self.rms_norm_eps,
                "tie_word_embeddings": self.tie_word_embeddings, "initializer_range": self.initializer_range,
                "torch_dtype": "bfloat16"}

    @classmethod
    def from_pretrained_dir(cls, path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_hf_dict(json.load(f), name=os.path.basename(path.rstrip("/")))


def _tiny_ref() -> ModelConfig:
    return ModelConfig(
        vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=8,
        layer_types=hybrid_layer_types(8), num_attention_heads=4, num_key_value_heads=2, head_dim=16,
        rope_theta=1e4, partial_rotary_factor=0.25, linear_num_key_heads=2, linear_num_value_heads=4,
        linear_key_head_dim=16, linear_value_head_dim=16, linear_conv_kernel_dim=4,
        tie_word_embeddings=False, head_init="linear_default", name="tiny_ref",
    )


def _tiny() -> ModelConfig:
    return ModelConfig(name="tiny")


def _p8b() -> ModelConfig:
    return ModelConfig(
        vocab_size=248320, hidden_size=1024, intermediate_size=3584, num_hidden_layers=24,
        layer_types=hybrid_layer_types(24), num_attention_heads=8, num_key_value_heads=2, head_dim=256,
        rope_theta=1e7, partial_rotary_factor=0.25, linear_num_key_heads=16, linear_num_value_heads=16,
        linear_key_head_dim=128, linear_value_head_dim=128, tie_word_embeddings=True, name="0.8b",
    )


def _p27b() -> ModelConfig:
    return ModelConfig(
        vocab_size=248320, hidden_size=5120, intermediate_size=17408, num_hidden_layers=64,
        layer_types=hybrid_layer_types(64), num_attention_heads=24, num_key_value_heads=4, head_dim=256,
        rope_theta=1e7, partial_rotary_factor=0.25, linear_num_key_heads=16, linear_num_value_heads=48,
        linear_key_head_dim=128, linear_value_head_dim=128, tie_word_embeddings=False, name="27b",
    )


PRESETS = {"tiny_ref": _tiny_ref, "tiny": _tiny, "0.8b": _p8b, "27b": _p27b}


def preset(name: str, layers: int | None = None, **overrides) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}")
    cfg = PRESETS[name]()
    if overrides:
        cfg = dataclasses.replace(cfg, **overrides)
    return cfg.truncated(layers)
