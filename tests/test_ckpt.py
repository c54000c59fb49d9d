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


def _reference_pkg():
    """The reference package installed offline under baseline/_ref (skipped when absent)."""
    import sys

    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(os.path.join(root, "dllm_qwen38")):
        pytest.skip("reference package not installed under baseline/_ref")
    if root not in sys.path:
        sys.path.insert(0, root)
    import dllm_qwen38.blockdiff as rbd
    import dllm_qwen38.gsm8k_eval as rge

    return rbd, rge


def test_convert_to_reference_layout_reads_back_through_the_reference_tools(tmp_path):
    """An engine checkpoint rewritten in the reference's DCP layout: per-parameter entries named
    `text_model.layers.N.layer.*`, bf16 model and moments, step / seq_tokens. The reference's own
    eval reader (`gsm8k_eval.dcp_model_tensors` + `restore_into`) loads it into its HF model with
    no missing or unexpected key, and the weights are our master weights rounded to bf16."""
    a = _trainer()
    for x, p, v in _batches(2):
        a.step(x, p, v)
    ckpt.save_engine(a.engine, str(tmp_path / "ours"), gstep=2, seq_tokens=256)
    cfg = preset("tiny_ref")
    rep = ckpt.convert_to_reference(ckpt.ckpt_path(str(tmp_path / "ours"), 2), str(tmp_path / "ref"), cfg)
    assert rep["step"] == 2 and rep["seq_tokens"] == 256
    tensors, step, seq = ckpt.reference_dcp_tensors(str(tmp_path / "ref"))
    assert step == 2 and seq == 256
    assert any(k.startswith("text_model.layers.3.layer.") for k in tensors)
    assert all(t.dtype == torch.bfloat16 for t in tensors.values())
    full = a.engine.full_state()
    for k, t in tensors.items():
        ours = ckpt.plain_fqn(k)
        assert torch.equal(t, full[ours].to(torch.bfloat16)), k

    rbd, rge = _reference_pkg()
    model, lm_head = rbd.tiny_text_model(seed=1)
    got, rstep, rseq = rge.dcp_model_tensors(str(tmp_path / "ref"))
    assert (rstep, rseq) == (2, 256)
    model, lm_head = model.to(torch.bfloat16), lm_head.to(torch.bfloat16)
    rge.restore_into(model, lm_head, got, ctx="converted")  # raises on any missing/unexpected key
    sd = model.state_dict()
    for k, t in full.items():
        if k == "lm_head.weight":
            assert torch.equal(lm_head.weight, t.to(torch.bfloat16))
        else:
            assert torch.equal(sd[k[len("text_model."):]], t.to(torch.bfloat16)), k


def test_convert_cli_round_trip_into_our_loader(tmp_path):
    a = _trainer()
    x, p, v = _batches(1)[0]
    a.step(x, p, v)
    ckpt.save_engine(a.engine, str(tmp_path / "ours"), gstep=1, seq_tokens=64)
    rc = ckpt.main(["to-reference", ckpt.ckpt_path(str(tmp_path / "ours"), 1), str(tmp_path / "ref"),
                    "--model", "tiny_ref"])
    assert rc == 0
    m = build_model(preset("tiny_ref"), seed=9)
    tensors, _, _ = ckpt.any_dcp_tensors(str(tmp_path / "ref"), m.config)
    ckpt.restore_into(m, tensors)
    full = a.engine.full_state()
    for k, t in m.state_dict().items():
        key = "text_model." + k if not k.startswith("lm_head") else k
        if key in full:
            assert torch.equal(t, full[key].to(torch.bfloat16).float()), k
