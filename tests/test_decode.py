"""Golden decoder contract (the reference's decode.py:35-99)."""

import torch

from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.infer.golden import generate, select_commits
from dllm_qwen38_b200.models.qwen35 import build_model


def test_commit_rule_threshold_argmax_and_subblock_window():
    V = 5
    logits = torch.zeros(8, V)  # confidence 1/V everywhere
    logits[2, 3] = 10.0  # confident
    logits[6, 1] = 10.0  # confident but outside the first sub-block window
    masked = torch.ones(8, dtype=torch.bool)
    commit, pick = select_commits(logits, masked, 0.9, None, 0.0)
    assert commit.tolist() == [False, False, True, False, False, False, True, False]
    assert int(pick[2]) == 3 and int(pick[6]) == 1
    commit, _ = select_commits(logits, masked, 0.9, 4, 0.0)
    assert commit.tolist() == [False, False, True, False, False, False, False, False]
    # nothing clears the threshold -> exactly the single most confident candidate
    commit, _ = select_commits(torch.zeros(8, V), masked, 0.9, None, 0.0)
    assert int(commit.sum()) == 1


def test_generate_is_deterministic_and_counts_forwards():
    m = build_model(preset("tiny_ref"), seed=0)
    a = generate(m, [1, 2, 3], n_blocks=2, block=8, mask_id=255, threshold=0.9)
    b = generate(m, [1, 2, 3], n_blocks=2, block=8, mask_id=255, threshold=0.9)
    assert a.tokens == b.tokens
    assert a.generated == (8 - 3) + 8  # resumes mid-block after the prompt tail
    assert len(a.tokens) == 3 + a.generated
    assert a.forwards == sum(a.steps_per_block) and a.forwards <= a.generated
    assert 255 not in a.tokens[3:]
