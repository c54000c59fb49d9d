"""Build a model from a preset name or load one from an HF Qwen3.5 checkpoint directory.

HF checkpoints (the reference's load source, `equivalence.py:39-72`) store the text tower under
``model.language_model.*`` (image-text-to-text wrapper) or ``model.*`` (causal LM), plus
``lm_head.weight``. Our own single-device checkpoints use ``text_model.*`` / ``lm_head.*``
(`train.py:270-276`). Both are read here; tensors for layers beyond ``layers`` are never loaded
(the reference loads all 64 layers in bf16, then drops the tail; we skip it at read time).
"""

from __future__ import annotations

import glob
import json
import os
import re

import torch

from ..config import PRESETS, ModelConfig, preset
from ..models.qwen35 import BlockDiffusionLM, build_model

_PREFIXES = ("model.language_model.", "model.", "text_model.", "language_model.")


def text_key(k: str) -> str | None:
    """Checkpoint key -> our key (``text_model.<x>`` / ``lm_head.weight``), or None to skip."""
    if k.startswith("lm_head."):
        return k
    for pre in _PREFIXES:
        if k.startswith(pre):
            rest = k[len(pre):]
            if rest.startswith(("visual.", "mtp.")):
                return None
            return "text_model." + rest
    return None


def _layer_of(k: str) -> int | None:
    m = re.match(r"^text_model\.layers\.(\d+)\.", k)
    return int(m.group(1)) if m else None


def load_state_into(model: BlockDiffusionLM, files: list, layers: int | None = None, strict: bool = True) -> dict:
    """Stream safetensors files into `model` (already materialised). Returns counts."""
    from safetensors import safe_open

    own = dict(model.named_parameters(remove_duplicate=False))
    seen, skipped = set(), 0
    for f in files:
        with safe_open(f, framework="pt") as sf:
            for k in sf.keys():
                ok = text_key(k)
                if ok is None:
                    skipped += 1
                    continue
                li = _layer_of(ok)
                if li is not None and layers is not None and li >= layers:
                    skipped += 1
                    continue
                if ok not in own:
                    if strict:
                        raise KeyError(f"checkpoint key {k} -> {ok} has no parameter")
                    skipped += 1
                    continue
                with torch.no_grad():
                    own[ok].copy_(sf.get_tensor(k).to(own[ok].dtype))
                seen.add(ok)
    missing = [k for k in own if k not in seen and not (k == "lm_head.weight" and model.config.tie_word_embeddings)]
    if strict and missing:
        raise KeyError(f"parameters missing from checkpoint: {missing[:10]}")
    return {"loaded": len(seen), "skipped": skipped, "missing": missing}


def load_model(name_or_dir: str, *, dtype=torch.float32, device="cpu", layers: int | None = None, seed: int = 0):
    """(model, tokenizer-or-None). A preset name gives a random-init model and no tokenizer."""
    if name_or_dir in PRESETS:
        return build_model(preset(name_or_dir, layers=layers), seed=seed, device=device, dtype=dtype), None
    if not os.path.isdir(name_or_dir):
        raise FileNotFoundError(f"{name_or_dir}: neither a preset ({sorted(PRESETS)}) nor a checkpoint directory")
    with open(os.path.join(name_or_dir, "config.json")) as f:
        hf = json.load(f)
    cfg = ModelConfig.from_hf_dict(hf).truncated(layers)
    model = build_model(cfg, seed=seed, device=device, dtype=dtype)
    files = sorted(glob.glob(os.path.join(name_or_dir, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"{name_or_dir}: no *.safetensors")
    load_state_into(model, files, layers=layers)
    tok = None
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(name_or_dir)
    except Exception:  # noqa: BLE001 - a weights-only dir has no tokenizer
        tok = None
    return model, tok


def spare_rows(model, tok) -> dict:
    rows = model.text_model.embed_tokens.weight.shape[0]
    return {"embedding_rows": rows, "tokenizer_len": len(tok), "spare_rows": rows - len(tok)}
