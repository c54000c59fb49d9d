"""Write a model as an HF-layout checkpoint directory (`config.json` + `model.safetensors`, text
tower under ``model.language_model.*``), readable by `io.hf_load.load_model` and by the
weight-space tools. The inverse of `hf_load`; used to freeze a trained or edited model for the
completion server and the weight-space bench (the reference exports a trained model as one
`model.safetensors` at `src/dllm_qwen38/train.py:270-276`)."""

from __future__ import annotations

import json
import os

import torch


def save_model_dir(model, out_dir: str, dtype=torch.bfloat16) -> str:
    from safetensors.torch import save_file

    os.makedirs(out_dir, exist_ok=False)
    cfg = model.config
    state = {f"model.language_model.{k}": v for k, v in model.text_model.state_dict().items()}
    if not cfg.tie_word_embeddings:
        state["lm_head.weight"] = model.lm_head.weight
    save_file({k: v.detach().to("cpu", dtype).contiguous().clone() for k, v in state.items()},
              os.path.join(out_dir, "model.safetensors"))
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg.to_hf_dict(), f, indent=2)
        f.write("\n")
    return out_dir
