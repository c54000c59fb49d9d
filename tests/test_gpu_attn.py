"""Complementary-mask flash attention (forward and backward) against the fp32 reference."""

import pytest
import torch

from dllm_qwen38_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("leak", [False, True])
@pytest.mark.parametrize("B,L,block,Hq,Hk,D", [(2, 64, 16, 4, 2, 32), (1, 96, 32, 6, 2, 128), (1, 128, 32, 4, 1, 256),
                                               (2, 24, 8, 4, 2, 16), (1, 100, 20, 4, 2, 128), (2, 192, 32, 6, 1, 256)])
def test_attention_fwd_bwd(leak, B, L, block, Hq, Hk, D):
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(0)
    T2 = 2 * L
    q = torch.randn(B, T2, Hq, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    kv = torch.randn(B, T2, 2 * Hk * D + 8, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = kv[..., : Hk * D].reshape(B, T2, Hk, D)
    v = kv[..., Hk * D : 2 * Hk * D].reshape(B, T2, Hk, D)
    o = Cu.attention_blockdiff(q, k, v, L, block, D ** -0.5, leak)
    do = torch.randn_like(o)
    o.backward(do)
    qf = q.detach().float().requires_grad_(True)
    kvf = kv.detach().float().requires_grad_(True)
    kf = kvf[..., : Hk * D].reshape(B, T2, Hk, D)
    vf = kvf[..., Hk * D : 2 * Hk * D].reshape(B, T2, Hk, D)
    allowed = ref.complementary_allowed(L, block, "cuda", leak)
    orf = ref.attention(qf, kf, vf, allowed, D ** -0.5)
    orf.backward(do.float())
    assert _rel(o, orf) < 1e-2, _rel(o, orf)
    assert _rel(q.grad, qf.grad) < 2e-2, _rel(q.grad, qf.grad)
    assert _rel(kv.grad, kvf.grad) < 2e-2, _rel(kv.grad, kvf.grad)


@pytest.mark.parametrize("leak", [False, True])
@pytest.mark.parametrize("B,L,block,Hq,Hk,D,qscale", [(2, 320, 32, 6, 1, 256, 1.0), (1, 200, 8, 4, 2, 128, 6.0),
                                                      (1, 256, 32, 2, 1, 256, 12.0), (1, 100, 20, 2, 1, 128, 3.0)])
def test_attention_forward_many_tiles(leak, B, L, block, Hq, Hk, D, qscale):
    """Many key tiles per query tile (the tcgen05 forward's pipeline, tile skipping, masks inside
    partial tiles, row tails) and large score ranges (the running max moves by more than 2^8, so
    the TMEM output is rescaled), against fp32; the row log2-sum-exp too."""
    from dllm_qwen38_b200 import _C

    torch.manual_seed(1)
    T2 = 2 * L
    q = (torch.randn(B, T2, Hq, D, device="cuda") * qscale).to(torch.bfloat16)
    k = torch.randn(B, T2, Hk, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, T2, Hk, D, device="cuda", dtype=torch.bfloat16)
    o, lse2 = _C.attn_fwd(q, k, v, L, block, D ** -0.5, leak)
    torch.cuda.synchronize()
    allowed = ref.complementary_allowed(L, block, "cuda", leak)
    orf = ref.attention(q.float(), k.float(), v.float(), allowed, D ** -0.5)
    assert _rel(o, orf) < 1e-2, _rel(o, orf)
    rep = Hq // Hk
    s = torch.einsum("bihd,bjhd->bhij", q.float(), k.float().repeat_interleave(rep, 2)) * D ** -0.5
    s = s.masked_fill(~allowed, float("-inf"))
    want = torch.logsumexp(s, -1) / torch.log(torch.tensor(2.0))
    assert float((lse2 - want).abs().max()) < 2e-2 * max(1.0, float(want.abs().max()))
    from dllm_qwen38_b200.ops import cuda as Cu

    Cu.check_errors()
