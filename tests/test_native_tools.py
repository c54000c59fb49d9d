"""Native capture/meter tools (C++ driving the engine through an embedded interpreter), CPU."""

import json
import os
import subprocess

import numpy as np
import pytest
import torch

from dllm_qwen38_b200 import native_tools

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def tools():
    try:
        return native_tools.build()
    except (OSError, subprocess.CalledProcessError) as e:  # no compiler / libpython on this host
        pytest.skip(f"cannot build the native tools: {e}")


def _run(tool, args, cwd):
    env = dict(os.environ, BDLLM_ROOT=ROOT, CUDA_VISIBLE_DEVICES="")
    return subprocess.run([native_tools.tool_path(tool)] + args, cwd=cwd, env=env, capture_output=True, text=True,
                          timeout=600)


def test_capture_matches_api_and_writes_contract(tools, tmp_path):
    from dllm_qwen38_b200.native_tools import api

    (tmp_path / "p.jsonl").write_text('{"ids": [1, 2, 3, 4, 5, 6, 7, 8, 9, 10]}\n{"ids": [11, 12, 13]}\n')
    r = _run("capture", ["--model", "tiny_ref", "--prompts", "p.jsonl", "--layers", "1,3", "--out", "cap",
                         "--block", "8"], tmp_path)
    assert r.returncode == 0, r.stderr
    st = json.loads((tmp_path / "cap" / "status.json").read_text())
    assert st == {"ok": True, "prompts": 2, "tensors": 4, "layer_visits": 8, "error": ""}
    idx = [json.loads(x) for x in (tmp_path / "cap" / "index.jsonl").read_text().splitlines()]
    assert [(e["prompt"], e["layer"], e["rows"]) for e in idx] == [(0, 1, 10), (0, 3, 10), (1, 1, 3), (1, 3, 3)]
    torch.set_num_threads(1)
    model = api.load("tiny_ref")
    want, _ = api.capture(model, list(range(1, 11)), [3], block=8)
    got = np.fromfile(tmp_path / "cap" / "p0-l3.f32", dtype=np.float32).reshape(10, -1)
    assert np.allclose(got, want[3], atol=1e-5)


def test_capture_rejects_too_many_prompts(tools, tmp_path):
    (tmp_path / "p.jsonl").write_text("".join('{"ids": [1, 2]}\n' for _ in range(9)))
    r = _run("capture", ["--model", "tiny_ref", "--prompts", "p.jsonl", "--layers", "0", "--out", "cap"], tmp_path)
    assert r.returncode != 0
    st = json.loads((tmp_path / "cap" / "status.json").read_text())
    assert st["ok"] is False and "8 prompts" in st["error"]


def test_meter_accounting_and_tokens_match_the_decoder(tools, tmp_path):
    from dllm_qwen38_b200.infer import cached
    from dllm_qwen38_b200.native_tools import api

    (tmp_path / "p.json").write_text('{"ids": [5, 6, 7, 8, 9, 10, 11, 12, 13]}')
    r = _run("meter", ["--model", "tiny_ref", "--prompt", "p.json", "--blocks", "3", "--block", "8", "--out", "m"],
             tmp_path)
    assert r.returncode == 0, r.stderr
    rep = json.loads((tmp_path / "m" / "meter.json").read_text())
    calls = [json.loads(x) for x in (tmp_path / "m" / "calls.jsonl").read_text().splitlines()]
    steps = sum(1 for c in calls if c["call"] == "step")
    assert rep["prefill"]["passes"] == 1  # one whole prompt block
    assert rep["decode"]["passes"] == steps + 3  # one per step + one commit per block
    assert rep["generated"] == (8 - 9 % 8) + 2 * 8
    toks = [int(x) for x in (tmp_path / "m" / "tokens.txt").read_text().split()]
    torch.set_num_threads(1)
    tr = cached.generate(api.load("tiny_ref"), list(range(5, 14)), n_blocks=3, block=8,
                         mask_id=api.load("tiny_ref").config.mask_id, threshold=0.9)
    assert toks == tr.tokens[9:]
