"""Weight-space bench (dllm_qwen38_b200/weight_space) on CPU: statistics against scipy, audit and
scorer contracts, exclusive writers, and the full loop — model dir -> loopback server -> resumable
runs -> surgery -> launched runs -> paired compare -> collected bundle -> uncertainty."""

import argparse
import json
import math
import os
import pathlib
import socket
import threading

import numpy as np
import pytest
import torch

from dllm_qwen38_b200.weight_space import bench, collect, controller_claim, split_audit, surgery, uncertainty
from dllm_qwen38_b200.weight_space import symbolic_score
from dllm_qwen38_b200.weight_space.common import digest, digest_tree


def test_binomial_intervals_match_clopper_pearson():
    from scipy.stats import beta

    for k, n in ((0, 10), (3, 10), (10, 10), (17, 40), (1, 1)):
        lo, hi = uncertainty.binomial_interval(k, n, 0.95)
        want_lo = 0.0 if k == 0 else beta.ppf(0.025, k, n - k + 1)
        want_hi = 1.0 if k == n else beta.ppf(0.975, k + 1, n - k)
        assert abs(lo - want_lo) < 1e-9 and abs(hi - want_hi) < 1e-9, (k, n, lo, hi, want_lo, want_hi)
    r = uncertainty.paired_interval(40, 7, 2)
    assert r["interval"][0] <= r["observed_delta"] <= r["interval"][1]
    with pytest.raises(ValueError):
        uncertainty.paired_interval(5, 4, 3)


def test_mcnemar_and_bootstrap():
    from scipy.stats import binomtest

    assert bench.mcnemar_exact(0, 0) == 1.0
    for w, l in ((5, 0), (7, 2), (3, 3), (12, 4)):
        assert math.isclose(bench.mcnemar_exact(w, l), binomtest(w, w + l, 0.5).pvalue, rel_tol=1e-12)


def test_final_number_contract():
    assert bench.final_number("work\nFINAL: 1,234\n") == "1234"
    assert bench.final_number("FINAL: 3.50.") == "3.5"
    assert bench.final_number("<think>FINAL: 3") is None  # unfinished reasoning
    assert bench.final_number("<think>FINAL: 3</think>\nFINAL: 4") == "4"
    assert bench.final_number("FINAL: 1\nFINAL: 2") is None


def test_split_audit_flags(tmp_path):
    def split(name, qs):
        p = tmp_path / f"{name}.json"
        p.write_text(json.dumps({"split": name, "cases": [{"id": f"{name}{i}", "question": q} for i, q in enumerate(qs)]}))
        return p

    dev = split("dev", ["Tom has 3 apples and buys 4 more. How many?", "A train leaves at noon."])
    val = split("validation", ["tom has  3 apples and buys 4 more. how many?", "Tom has 9 apples and buys 2 more. How many?",
                               "Completely unrelated text about geometry of circles."])
    rep = split_audit.audit([dev], [val])
    assert rep["cross_split_pair_count"] == 6
    reasons = {(f["dev_id"], f["validation_id"]): f["reasons"] for f in rep["flagged_pairs"]}
    assert "normalised_exact" in reasons[("dev0", "validation0")]
    assert "number_masked_exact" in reasons[("dev0", "validation1")]
    assert ("dev1", "validation2") not in reasons


def test_controller_claim_is_exclusive(tmp_path):
    h = "a" * 64
    controller_claim.claim(tmp_path, h)
    with pytest.raises(FileExistsError):
        controller_claim.claim(tmp_path, h)
    with pytest.raises(ValueError):
        controller_claim.claim(tmp_path, "nothex")


def test_boxed_scorer():
    s = symbolic_score.score
    assert s("1/2", r"so \boxed{\frac{1}{2}}")["correct"] is True
    assert s("12", r"<think>\boxed{3}</think> the answer is \boxed{12}")["correct"] is True
    assert s("12", r"\boxed{13}")["correct"] is False
    assert s("12", "<think> never closed")["status"] == "unfinished_thinking"
    assert s("12", "no box here")["status"] == "missing_box"
    from dllm_qwen38_b200.weight_space.symbolic_process import score_isolated

    r = score_isolated("7", r"\boxed{7}", timeout_seconds=60)
    assert r["correct"] is True and r["profile"] == symbolic_score.PROFILE


def test_prepare_splits(tmp_path):
    src = tmp_path / "train.jsonl"
    src.write_text("".join(json.dumps({"question": f"What is {i} + {i}?", "answer": f"steps #### {2 * i}"}) + "\n"
                           for i in range(7)))
    bench.prepare(argparse.Namespace(source=str(src), output=str(tmp_path / "d"), size=3))
    dev = json.loads((tmp_path / "d" / "dev.json").read_text())
    val = json.loads((tmp_path / "d" / "validation.json").read_text())
    assert len(dev["cases"]) == 3 and len(val["cases"]) == 3
    assert not {c["id"] for c in dev["cases"]} & {c["id"] for c in val["cases"]}
    with pytest.raises(FileExistsError):  # writers never overwrite
        bench.prepare(argparse.Namespace(source=str(src), output=str(tmp_path / "d"), size=3))


def _synthetic_capture(d: pathlib.Path, prompts: int, layer: int, width: int, direction: np.ndarray):
    d.mkdir()
    rng = np.random.default_rng(0)
    rows = []
    base = rng.normal(size=width).astype(np.float32)
    for p in range(prompts):
        v = base.copy()
        if p in (1, 3, 5):  # the "late" member of each pair moves along the direction
            v += 2.0 * direction + 0.05 * rng.normal(size=width).astype(np.float32)
        x = np.stack([rng.normal(size=width).astype(np.float32), v])  # [T=2, D]
        f = f"p{p}-l{layer}.f32"
        x.astype("<f4").tofile(d / f)
        rows.append({"prompt": p, "layer": layer, "file": f, "rows": 2, "cols": width, "bytes": x.nbytes})
    (d / "index.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    (d / "status.json").write_text(json.dumps({"ok": True, "prompts": prompts, "tensors": prompts,
                                               "layer_visits": prompts * (layer + 1), "error": ""}))


def test_capture_to_direction(tmp_path):
    from dllm_qwen38_b200.weight_space.derive_direction import derive

    width = 16
    d = np.zeros(width, np.float32)
    d[3] = 1.0
    _synthetic_capture(tmp_path / "cap", 8, 1, width, d)
    rep = derive(tmp_path / "cap", tmp_path / "dir", 1, 8, [(0, 1), (2, 3), (4, 5)], (6, 7), 0.5)
    assert rep["gate_passed"] and rep["reset_control_max_abs"] == 0.0
    got = np.load(tmp_path / "dir" / "direction-1.npy")
    assert float(got @ d) > 0.99
    with pytest.raises(ValueError):  # prompts not covered exactly once
        derive(tmp_path / "cap", tmp_path / "dir2", 1, 8, [(0, 1), (2, 3)], (6, 7), 0.5)


def _model_dir(tmp_path) -> pathlib.Path:
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.io.hf_save import save_model_dir
    from dllm_qwen38_b200.models.qwen35 import build_model

    m = build_model(preset("tiny", layers=2), seed=0, device="cpu", dtype=torch.float32)
    return pathlib.Path(save_model_dir(m, str(tmp_path / "model"), dtype=torch.bfloat16))


def test_surgery_projects_out_and_preserves_other_bytes(tmp_path):
    md = _model_dir(tmp_path)
    src = md / "model.safetensors"
    table, _ = surgery.read_header(src)
    name = "model.language_model.layers.0.mlp.down_proj.weight"
    hidden = table[name]["shape"][0]
    d = np.random.default_rng(1).normal(size=hidden)
    np.save(tmp_path / "dir.npy", d)
    spec = tmp_path / "spec.json"
    spec.write_text(json.dumps({"hypothesis": "test", "edits": [{"tensor": name, "direction": "dir.npy",
                                                                  "strength": 1.0}]}))
    j = surgery.apply(src, digest(src), tmp_path / "edited.safetensors", spec)
    e = j["edits"][0]
    assert j["state"] == "complete" and j["bytes_outside_edited_tensors_equal"]
    assert e["projection_norm_after"] < 0.02 * e["projection_norm_before"]
    assert e["values_changed"] > 0
    spec0 = tmp_path / "spec0.json"
    spec0.write_text(json.dumps({"hypothesis": "no-op", "edits": [{"tensor": name, "direction": "dir.npy",
                                                                    "strength": 0.0}]}))
    surgery.apply(src, digest(src), tmp_path / "same.safetensors", spec0)
    assert digest(tmp_path / "same.safetensors") == digest(src)
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps({"hypothesis": "x", "edits": [{"tensor": "model.language_model.embed_tokens.weight",
                                                              "direction": "dir.npy", "strength": 0.5}]}))
    with pytest.raises(ValueError):
        surgery.apply(src, digest(src), tmp_path / "bad.safetensors", bad)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_server_runs_compare_collect_uncertainty(tmp_path):
    from dllm_qwen38_b200.weight_space import launch
    from dllm_qwen38_b200.weight_space.server import Engine, serve

    md = _model_dir(tmp_path)
    data = tmp_path / "data"
    src = tmp_path / "train.jsonl"
    src.write_text("".join(json.dumps({"question": f"Add {i} and {i}.", "answer": f"#### {2 * i}"}) + "\n"
                           for i in range(4)))
    bench.prepare(argparse.Namespace(source=str(src), output=str(data), size=2))
    sha = digest_tree(md)
    # in-process server: run, interrupt, resume
    eng = Engine(str(md), "bytes", block=8, threshold=0.9, sub_block=0, n_ctx=2048)
    srv = serve(eng, 0)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{srv.server_address[1]}"
    try:
        args = dict(server=url, model=str(md), model_sha256=sha, backend_commit="test", data=str(data / "dev.json"),
                    max_tokens=8, thinking="off", seed=42, timeout=120)
        bench.run(argparse.Namespace(condition="a", output=str(tmp_path / "runA"), limit=1, **args))
        with pytest.raises(ValueError):  # the manifest pins the case list
            bench.run(argparse.Namespace(condition="a", output=str(tmp_path / "runA"), limit=0, **args))
        summ = bench.run(argparse.Namespace(condition="b", output=str(tmp_path / "runB"), limit=1, **args))
        assert summ["n"] == 1 and summ["generated_tokens"] <= 8
        res = bench.compare(argparse.Namespace(baseline=str(tmp_path / "runA"), candidate=str(tmp_path / "runB"),
                                               output=None))
        assert res["wins"] == res["losses"] == 0 and res["mcnemar_exact_two_sided_p"] == 1.0
    finally:
        srv.shutdown()
        srv.server_close()
    # launched runs: baseline and an edited candidate, collected and analysed
    name = "model.language_model.layers.1.mlp.down_proj.weight"
    table, _ = surgery.read_header(md / "model.safetensors")
    np.save(tmp_path / "dir.npy", np.random.default_rng(2).normal(size=table[name]["shape"][0]))
    spec = tmp_path / "spec.json"
    spec.write_text(json.dumps({"hypothesis": "h", "edits": [{"tensor": name, "direction": "dir.npy",
                                                               "strength": 0.5}]}))
    cand = tmp_path / "cand_model"
    cand.mkdir()
    (cand / "config.json").write_bytes((md / "config.json").read_bytes())
    surgery.apply(md / "model.safetensors", digest(md / "model.safetensors"), cand / "model.safetensors", spec)
    os.remove(str(cand / "model.safetensors") + ".edit.json")  # the journal is kept outside the model dir
    conds = []
    for cname, mdir in (("base", md), ("cand", cand)):
        cfgp = tmp_path / f"{cname}.launch.json"
        cfgp.write_text(json.dumps({"model": str(mdir), "model_sha256": digest_tree(mdir), "output": str(tmp_path / f"run_{cname}"),
                                    "data": str((data / "dev.json").resolve()), "condition": cname,
                                    "backend_commit": "test", "port": _free_port(), "tokenizer": "bytes", "block": 8,
                                    "n_ctx": 2048, "limit": 2, "max_tokens": 8, "startup_timeout": 240}))
        assert launch.main([str(cfgp)]) == 0
        st = json.loads((tmp_path / f"run_{cname}" / "process-status.json").read_text())
        assert st["state"] == "completed" and st["engine_stopped"]
        conds.append({"name": cname, "run": f"run_{cname}"})
    plan = tmp_path / "plan.json"
    plan.write_text(json.dumps({"qualification": "test", "conditions": conds, "paired": [["base", "cand"]]}))
    bundle = collect.collect(plan)
    assert bundle["paired"][0]["result"]["baseline"]["n"] == 2
    (tmp_path / "bundle.json").write_text(json.dumps(bundle))
    u = uncertainty.analyze(tmp_path / "bundle.json")
    lo, hi = u["comparisons"][0]["interval"]
    assert -1.0 <= lo <= u["comparisons"][0]["observed_delta"] <= hi <= 1.0


def test_capture_reader_checks_accounting(tmp_path):
    from dllm_qwen38_b200.weight_space.capture_data import load_vectors

    d = np.zeros(8, np.float32)
    _synthetic_capture(tmp_path / "cap", 4, 2, 8, d)
    vecs, acct = load_vectors(tmp_path / "cap", 4, [2], width=8)
    assert acct["vectors"] == 4 and vecs[(0, 2)].shape == (8,)
    with pytest.raises(ValueError, match="width"):
        load_vectors(tmp_path / "cap", 4, [2], width=16)
    with pytest.raises(ValueError, match="accounting"):  # a layer that was never captured
        load_vectors(tmp_path / "cap", 4, [1, 2])
    st = json.loads((tmp_path / "cap" / "status.json").read_text())
    (tmp_path / "cap" / "status.json").write_text(json.dumps(dict(st, ok=False)))
    with pytest.raises(ValueError, match="did not complete"):
        load_vectors(tmp_path / "cap", 4, [2])
    (tmp_path / "cap" / "status.json").write_text(json.dumps(st))
    np.full(16, np.nan, "<f4").tofile(tmp_path / "cap" / "p3-l2.f32")  # same size, not finite
    with pytest.raises(ValueError, match="non-finite"):
        load_vectors(tmp_path / "cap", 4, [2])
    np.zeros(15, "<f4").tofile(tmp_path / "cap" / "p3-l2.f32")  # one value short
    with pytest.raises(ValueError, match="byte count"):
        load_vectors(tmp_path / "cap", 4, [2])


def test_prepare_math_selects_hard_single_integer_problems(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq

    from dllm_qwen38_b200.weight_space import prepare_math

    rows = []
    for i in range(10):  # eligible: level 4/5, exactly one boxed plain integer
        rows.append({"problem": f"problem {i}", "level": "Level 5" if i % 2 else "Level 4",
                     "solution": f"so \\boxed{{{1000 + i:,}}}", "type": "Algebra"})
    rows += [
        {"problem": "easy", "level": "Level 2", "solution": "\\boxed{3}", "type": "Algebra"},
        {"problem": "two boxes", "level": "Level 5", "solution": "\\boxed{3} or \\boxed{4}", "type": "Algebra"},
        {"problem": "fraction", "level": "Level 5", "solution": "\\boxed{\\frac{1}{2}}", "type": "Algebra"},
        {"problem": "problem 3", "level": "Level 5", "solution": "\\boxed{7}", "type": "Algebra"},  # duplicate
    ]
    src = tmp_path / "src" / "algebra"
    src.mkdir(parents=True)
    pq.write_table(pa.Table.from_pylist(rows), src / "train.parquet")
    out = tmp_path / "out"
    assert prepare_math.main(["--source", str(tmp_path / "src"), "--output", str(out), "--size", "4"]) == 0
    dev = json.loads((out / "dev.json").read_text())
    val = json.loads((out / "validation.json").read_text())
    cases = dev["cases"] + val["cases"]
    assert len(dev["cases"]) == 4 and len(val["cases"]) == 4
    assert [c["id"] for c in cases] == sorted(c["id"] for c in cases)  # hash order, dev first
    assert {c["question"] for c in cases} <= {f"problem {i}" for i in range(10)}
    assert all(c["answer"].isdigit() and "," not in c["answer"] for c in cases)
    assert dev["sources"][0]["file"] == "algebra/train.parquet"
    with pytest.raises(FileExistsError):  # outputs are never overwritten
        prepare_math.main(["--source", str(tmp_path / "src"), "--output", str(out), "--size", "4"])
    with pytest.raises(ValueError, match="not enough"):
        prepare_math.main(["--source", str(tmp_path / "src"), "--output", str(tmp_path / "o2"), "--size", "6"])
    pq.write_table(pa.Table.from_pylist(rows), src / "test.parquet")
    with pytest.raises(ValueError, match="test split"):
        prepare_math.main(["--source", str(tmp_path / "src"), "--output", str(tmp_path / "o3"), "--size", "2"])
