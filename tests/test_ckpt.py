"""Checkpoint save/resume of the sharded engine (CPU): bit-exact resume, fingerprints that fail
closed, atomic commit, keep-last-2; reference-layout import with loud failures."""

import copy
import os

import pytest
import torch

from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.io import ckpt
from dllm_qwen38_b200.models.qwen35 import build_model


def _batches(n, seed=5):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randint(0, 255, (2, 32), generator=g), torch.zeros(2, dtype=torch.long),
             torch.full((2,), 32, dtype=torch.long)) for _ in range(n)]


def _trainer(seed=0):
    from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

    cfg = preset("tiny_ref")
    return FSDPTrainer(build_model(cfg, seed=seed), block=8, mask_id=cfg.mask_id, lr=1e-3)


def test_resume_is_bit_exact_and_fingerprints_verify(tmp_path):
    data = _batches(4)
    a = _trainer()
    losses_a = []
    for i, (x, p, v) in enumerate(data):
        losses_a.append(float(a.step(x, p, v)))
        if i == 1:
            ckpt.save_engine(a.engine, str(tmp_path), gstep=2, seq_tokens=128)
    b = _trainer(seed=123)  # different init: everything must come from the checkpoint
    info = ckpt.load_engine(b.engine, str(tmp_path), 2)
    assert info["fp_ok"] and info["seq_tokens"] == 128 and info["step"] == 2
    b.gstep = 2
    losses_b = [float(b.step(x, p, v)) for x, p, v in data[2:]]
    assert losses_b == losses_a[2:]


def test_fingerprint_mismatch_and_missing_file_fail_closed(tmp_path):
    a = _trainer()
    x, p, v = _batches(1)[0]
    a.step(x, p, v)
    ckpt.save_engine(a.engine, str(tmp_path), gstep=1, seq_tokens=64)
    fp = tmp_path / "fingerprints" / "step-1.tsv"
    line = fp.read_text().split("\t")
    fp.write_text("\t".join([line[0], "0" * 16, line[2]]))
    assert not ckpt.load_engine(_trainer().engine, str(tmp_path), 1)["fp_ok"]
    os.remove(fp)
    assert not ckpt.load_engine(_trainer().engine, str(tmp_path), 1)["fp_ok"]


def test_commit_by_rename_and_keep_last_two(tmp_path):
    a = _trainer()
    os.makedirs(tmp_path / "step-00000009.tmp")  # an interrupted save never counts
    for s in (1, 2, 3):
        ckpt.save_engine(a.engine, str(tmp_path), gstep=s, seq_tokens=s, fingerprint_save=False)
    names = sorted(e for e in os.listdir(tmp_path) if e.startswith("step-") and not e.endswith(".tmp"))
    assert names == ["step-00000002", "step-00000003"]
    assert ckpt.latest_checkpoint(str(tmp_path)) == 3


def test_plain_fqn_and_restore_into_fail_loudly():
    assert ckpt.plain_fqn("text_model.layers.7.layer.mlp.up_proj.weight") == "text_model.layers.7.mlp.up_proj.weight"
    assert ckpt.plain_fqn("text_model.norm.weight") == "text_model.norm.weight"
    assert ckpt.plain_fqn("lm_head.weight") == "lm_head.weight"
    assert ckpt.plain_fqn("optim.x") is None
    m = build_model(preset("tiny_ref"), seed=0)
    full = {f"text_model.{k}": v.clone() for k, v in m.text_model.state_dict().items()}
    full["lm_head.weight"] = m.lm_head.weight.detach().clone()
    m2 = build_model(preset("tiny_ref"), seed=9)
    ckpt.restore_into(m2, full)
    assert torch.equal(m2.lm_head.weight, m.lm_head.weight)
    for broken in ({k: v for k, v in full.items() if k != "lm_head.weight"},
                   {**full, "text_model.bogus.weight": torch.zeros(1)},
                   {**full, "foreign.thing": torch.zeros(1)}):
        with pytest.raises(ValueError):
            ckpt.restore_into(copy.deepcopy(m2), broken)


def test_export_safetensors_roundtrip(tmp_path):
    from dllm_qwen38_b200.io.hf_load import load_state_into

    a = _trainer()
    x, p, v = _batches(1)[0]
    a.step(x, p, v)
    path = str(tmp_path / "model.safetensors")
    ckpt.export_safetensors(a.engine, path)
    m = build_model(preset("tiny_ref"), seed=77)
    load_state_into(m, [path])
    full = a.engine.full_state()
    assert torch.equal(m.text_model.norm.weight.detach(), full["text_model.norm.weight"])
