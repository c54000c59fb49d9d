"""State-fork equivalence on the tiny models (CPU, fp32). Counts are asserted, not booleans:
every check must pass and every fault must be detected (mirrors the reference's
tests/test_equivalence.py:11-47)."""

import torch

from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.equivalence import run
from dllm_qwen38_b200.models.blockdiff import FAULTS, block_diffusion_forward
from dllm_qwen38_b200.models.oracle import reference_block_logits
from dllm_qwen38_b200.models.qwen35 import build_model


def _assert_all_green(rep):
    failed = [c["name"] for c in rep["checks"] if not c["pass"]]
    assert failed == [], rep["checks"]
    undetected = [f["fault"] for f in rep["faults"] if not f["detected"]]
    assert undetected == [], rep["faults"]
    assert rep["faults_total"] == len(FAULTS) == 3


def test_state_fork_matches_oracle_and_faults_are_caught_tiny_ref():
    m = build_model(preset("tiny_ref"), seed=0)
    rep = run(m, block=8, nblocks=4, layers=None, tol=1e-3, change_floor=0.1, seed=0, device="cpu")
    _assert_all_green(rep)
    assert rep["checks_total"] == 5


def test_state_fork_config1_block32_batch2():
    """The CPU fp32 config: vocab 1024, hidden 128, batch 2, L=128, block 32 (4 blocks)."""
    m = build_model(preset("tiny"), seed=0)
    rep = run(m, block=32, nblocks=4, layers=None, tol=1e-3, change_floor=1e-2, seed=0, device="cpu", batch=2)
    _assert_all_green(rep)
    assert rep["checks"][0]["max_abs_diff"] < 1e-4


def test_layer_truncation_runs_the_first_n_layers_only():
    m = build_model(preset("tiny_ref"), seed=1)
    rep = run(m, block=8, nblocks=2, layers=3, tol=1e-3, change_floor=0.05, seed=1, device="cpu")
    assert rep["layers"] == 3
    assert rep["layer_types"] == ["linear_attention"] * 3
    assert rep["checks_passed"] == rep["checks_total"]


def test_batched_forward_equals_per_row_and_oracle():
    m = build_model(preset("tiny_ref"), seed=2)
    block, nb, B = 8, 3, 3
    torch.manual_seed(2)
    x0 = torch.randint(0, 256, (B, block * nb))
    xt = x0.clone()
    xt[torch.rand(B, block * nb) < 0.5] = 255
    with torch.no_grad():
        lt, _ = block_diffusion_forward(m, x0, xt, block)
        rows = [block_diffusion_forward(m, x0[i : i + 1], xt[i : i + 1], block)[0] for i in range(B)]
        oracle = reference_block_logits(m, x0, xt, block)
    assert lt.shape == (B, block * nb, 256)
    assert float((lt - torch.cat(rows, 0)).abs().max()) < 1e-5
    assert float((lt - oracle).abs().max()) < 1e-3


def test_block_larger_than_chunk_and_chunk_not_multiple_of_block():
    """block 16 with chunk 8 (states every 2 chunks) and block 8 with chunk 64 (mid-chunk states)."""
    for chunk, block in [(8, 16), (64, 8), (24, 8)]:
        cfg = preset("tiny_ref", gdn_chunk_size=chunk)
        m = build_model(cfg, seed=3)
        rep = run(m, block=block, nblocks=3, layers=None, tol=1e-3, change_floor=0.05, seed=3, device="cpu")
        assert rep["checks_passed"] == rep["checks_total"], (chunk, block, rep["checks"])


def test_model_matches_huggingface_qwen3_5():
    """Our parameter tree loads into HF's Qwen3_5TextModel and both compute the same hidden
    states on a plain block-causal forward: the model definition is HF's math."""
    import pytest

    if torch.cuda.is_available():  # HF then routes CPU tensors to its Triton fast path
        pytest.skip("host-only parity check")

    from dllm_qwen38_b200.models.oracle import hf_text_model, plain_forward
    from dllm_qwen38_b200.ops import reference as ref

    m = build_model(preset("tiny_ref"), seed=4)
    try:
        hm = hf_text_model(m)
    except ImportError:
        pytest.skip("transformers without qwen3_5")
    ids = torch.randint(0, 256, (1, 24))
    allowed = ref.block_causal_allowed(24, 8, "cpu")
    with torch.no_grad():
        hs = hm(input_ids=ids, attention_mask=ref.additive_mask(allowed, torch.float32)[None, None], use_cache=False).last_hidden_state
        mine = plain_forward(m, ids, allowed, output="hidden")
    assert float((hs - mine).abs().max()) < 1e-4
