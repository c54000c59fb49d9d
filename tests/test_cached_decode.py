"""The cached block decoder reproduces the golden (no-cache) decoder's temperature-0 token stream
and trace, including a prompt that ends mid-block, the sub-block window and batching."""

import pytest
import torch

from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.infer import cached, golden
from dllm_qwen38_b200.models.qwen35 import build_model


@pytest.mark.parametrize("name,prompt_len,sub_block,threshold", [
    ("tiny_ref", 8, None, 0.9), ("tiny_ref", 11, None, 0.5), ("tiny_ref", 13, 4, 0.9), ("tiny", 16, None, 0.3)])
def test_cached_equals_golden(name, prompt_len, sub_block, threshold):
    torch.manual_seed(0)
    m = build_model(preset(name), seed=1)
    V = m.config.vocab_size
    prompt = torch.randint(0, V - 1, (prompt_len,)).tolist()
    kw = dict(n_blocks=3, block=8, mask_id=V - 1, threshold=threshold, sub_block=sub_block)
    g = golden.generate(m, prompt, **kw)
    c = cached.generate(m, prompt, **kw)
    assert c.tokens == g.tokens
    assert c.forwards == g.forwards and c.steps_per_block == g.steps_per_block
    assert c.generated == g.generated


def test_batched_cached_decode_equals_per_row_golden():
    m = build_model(preset("tiny_ref"), seed=2)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 255, (10,), generator=g).tolist() for _ in range(3)]
    kw = dict(n_blocks=2, block=8, mask_id=255, threshold=0.7)
    rows = cached.generate(m, prompts, **kw)
    for p, r in zip(prompts, rows):
        assert r.tokens == golden.generate(m, p, **kw).tokens


def test_eos_stops_after_the_block_containing_it():
    m = build_model(preset("tiny_ref"), seed=4)
    prompt = list(range(8))
    first = cached.generate(m, prompt, n_blocks=1, block=8, mask_id=255, threshold=0.9)
    eos = first.tokens[8 + 3]
    tr = cached.generate(m, prompt, n_blocks=4, block=8, mask_id=255, threshold=0.9, eos_id=eos)
    gt = golden.generate(m, prompt, n_blocks=4, block=8, mask_id=255, threshold=0.9, eos_id=eos)
    assert tr.tokens == gt.tokens and len(tr.steps_per_block) == len(gt.steps_per_block)
