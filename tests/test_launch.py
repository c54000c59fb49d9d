"""Launcher: command construction and report extraction (CPU)."""

import json

from dllm_qwen38_b200 import launch


def test_commands_single_and_torchrun():
    c = launch.command("equivalence", 1, 29541, 100, ["--tiny"])
    assert c[:4] == ["timeout", "-k", "60", "100"] and c[-3:] == ["-m", "dllm_qwen38_b200.equivalence", "--tiny"]
    c = launch.command("fsdp", 8, 29600, 100, ["--steps", "2"])
    assert "torch.distributed.run" in c and "--nproc-per-node=8" in c and "127.0.0.1" in c
    assert c[-4:] == ["dllm_qwen38_b200.train.fsdp_train", "--steps", "2"][-4:] or c[-3:] == ["dllm_qwen38_b200.train.fsdp_train", "--steps", "2"]
    c = launch.command("bench", 2, 29600, 100, [])
    assert c[-3:-2][0].endswith("bench.py") and c[-2:] == ["--gpus", "2"]


def test_report_extraction_prefers_report_line():
    lines = ["noise", 'REPORT\t{"a": 1}', '{"b": 2}']
    assert launch.extract_report(lines) == {"a": 1}
    assert launch.extract_report(["x", json.dumps({"metric": "m", "value": 3})]) == {"metric": "m", "value": 3}
    assert launch.extract_report(["nothing here"]) is None


def test_dry_run_prints_command(capsys):
    assert launch.main(["decode", "--gpus", "2", "--dry-run", "--", "--batch", "32"]) == 0
    out = capsys.readouterr().out
    assert "torch.distributed.run" in out and "dllm_qwen38_b200.bench.decode --batch 32" in out


def test_package_command_list_names_importable_modules(capsys):
    import importlib

    from dllm_qwen38_b200.__main__ import COMMANDS, main

    assert main([]) == 0
    out = capsys.readouterr().out
    for cmd, _ in COMMANDS:
        assert cmd in out
        importlib.import_module("dllm_qwen38_b200." + cmd)  # every listed command exists
