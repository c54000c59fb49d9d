"""Parity with the reference's own code (CPU, fp32), where the reference package is installed under
baseline/_ref (skipped otherwise).

The reference runs its stock functions on the same weights through the installed HuggingFace
`Qwen3_5TextModel` (our weights copied in by `models.oracle.hf_text_model`): its state-fork
training forward (`blockdiff.block_diffusion_forward`, with and without each deliberate fault) and
its golden block decoder (`decode.generate`). Ours must give the same logits and the same token
stream. One adapter is installed, because transformers 5.5 here ships `causal_conv1d_fn = None`
where the reference's pinned transformers provides a callable: a depthwise causal conv + SiLU in
torch, the function's documented contract.
"""

import os
import sys

import pytest
import torch

from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.models.blockdiff import FAULTS, BreakMode, block_diffusion_forward
from dllm_qwen38_b200.models.qwen35 import build_model

ROOT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _reference():
    if not os.path.isdir(os.path.join(ROOT, "dllm_qwen38")):
        pytest.skip("reference package not installed under baseline/_ref")
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import torch.nn.functional as F

    import dllm_qwen38.blockdiff as rbd
    import dllm_qwen38.decode as rdec
    import dllm_qwen38.gdn as rgdn

    def causal_conv1d_fn(x, weight, bias=None, activation=None, **_):
        K = weight.shape[-1]
        y = F.conv1d(F.pad(x, (K - 1, 0)), weight[:, None, :].to(x.dtype), bias, groups=x.shape[1])
        return F.silu(y) if activation in ("silu", "swish") else y

    rgdn.causal_conv1d_fn = causal_conv1d_fn
    rgdn.set_impl("torch")
    return rbd, rdec


def _pair(seed=0):
    from dllm_qwen38_b200.models.oracle import hf_text_model

    m = build_model(preset("tiny_ref"), seed=seed)
    hm = hf_text_model(m)
    head = torch.nn.Linear(m.config.hidden_size, m.config.vocab_size, bias=False)
    with torch.no_grad():
        head.weight.copy_(m.lm_head.weight)
    return m, hm, head


@pytest.mark.parametrize("fault", ["none", *FAULTS])
def test_state_fork_forward_matches_the_reference_implementation(fault):
    rbd, _ = _reference()
    m, hm, head = _pair(seed=3)
    g = torch.Generator().manual_seed(7)
    B, block, nb = 2, 8, 4
    x0 = torch.randint(0, 255, (B, block * nb), generator=g)
    xt = x0.clone()
    xt[torch.rand(B, block * nb, generator=g) < 0.5] = 255
    with torch.no_grad():
        ours_t, ours_0 = block_diffusion_forward(m, x0, xt, block, fault=BreakMode(fault))
        ref_t, ref_0 = rbd.block_diffusion_forward(hm, head, x0, xt, block, fault=rbd.BreakMode(fault))
    assert float((ours_t - ref_t).abs().max()) < 1e-4
    assert float((ours_0 - ref_0).abs().max()) < 1e-4


def test_golden_decoder_token_stream_matches_the_reference_decoder():
    from dllm_qwen38_b200.infer.golden import generate

    _, rdec = _reference()
    m, hm, head = _pair(seed=5)
    prompt = [3, 17, 42, 99, 7, 1, 250, 13, 8, 64]
    kw = dict(n_blocks=3, block=8, mask_id=255, threshold=0.2, sub_block=4)
    with torch.no_grad():
        ours = generate(m, prompt, **kw)
        ref = rdec.generate(hm, head, prompt, **kw)
    assert ours.tokens == ref.tokens
    assert ours.forwards == ref.forwards
    assert list(ours.steps_per_block) == list(ref.steps_per_block)
