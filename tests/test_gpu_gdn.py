"""State-fork GDN kernels (forward and backward) against the fp32 PyTorch reference."""

import pytest
import torch

from dllm_qwen38_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("mode", ["fork", "concat"])
@pytest.mark.parametrize("B,L,block,Hk,Hv,D", [(2, 64, 16, 2, 4, 32), (1, 96, 32, 2, 6, 128), (2, 32, 8, 4, 4, 16),
                                               (1, 256, 64, 2, 4, 64), (2, 256, 128, 2, 2, 32), (1, 192, 64, 1, 3, 128)])
def test_gdn_core_fwd_bwd(mode, B, L, block, Hk, Hv, D):
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(0)
    T2 = 2 * L
    mixed = torch.randn(B, T2, 2 * Hk * D + Hv * D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    q = mixed[..., : Hk * D].reshape(B, T2, Hk, D)
    k = mixed[..., Hk * D : 2 * Hk * D].reshape(B, T2, Hk, D)
    v = mixed[..., 2 * Hk * D :].reshape(B, T2, Hv, D)
    g = (-torch.rand(B, T2, Hv, device="cuda") * 0.5).requires_grad_(True)
    beta = torch.rand(B, T2, Hv, device="cuda").requires_grad_(True)
    o = Cu.gdn_core_blockdiff(q, k, v, g, beta, L, block, 64, mode)
    do = torch.randn_like(o)
    o.backward(do)
    mf = mixed.detach().float().requires_grad_(True)
    gf, bf = g.detach().clone().requires_grad_(True), beta.detach().clone().requires_grad_(True)
    qf = mf[..., : Hk * D].reshape(B, T2, Hk, D)
    kf = mf[..., Hk * D : 2 * Hk * D].reshape(B, T2, Hk, D)
    vf = mf[..., 2 * Hk * D :].reshape(B, T2, Hv, D)
    orf = ref.gdn_core_blockdiff(qf, kf, vf, gf, bf, L, block, block, mode)
    orf.backward(do.float())
    assert _rel(o, orf) < 1e-2, _rel(o, orf)
    assert _rel(mixed.grad, mf.grad) < 2e-2, _rel(mixed.grad, mf.grad)
    assert _rel(g.grad, gf.grad) < 2e-2, _rel(g.grad, gf.grad)
    assert _rel(beta.grad, bf.grad) < 2e-2, _rel(beta.grad, bf.grad)
    Cu.check_errors()


def test_kernel_diff_probe_on_a_real_mixer():
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model
    from dllm_qwen38_b200.ops import kernel_diff
    from dllm_qwen38_b200.ops import reference as ref

    cfg = preset("tiny", hidden_size=256, linear_key_head_dim=64, linear_value_head_dim=64, linear_num_key_heads=2,
                 linear_num_value_heads=4, layers=1)
    model = build_model(cfg, seed=0, device="cuda", dtype=torch.bfloat16)
    ids = torch.randint(0, cfg.mask_id, (1, 512), device="cuda", generator=torch.Generator(device="cuda").manual_seed(0))
    layer = model.text_model.layers[0]
    n = ref.rmsnorm(model.text_model.embed_tokens(ids), layer.input_layernorm.weight, layer.input_layernorm.eps)
    res = kernel_diff.mixer_diff(layer.linear_attn, n, 256, 32)
    assert res["impl"] == "native"
    assert res["out_max_abs_diff"] < 2e-2 * max(1.0, res["out_max_abs"]), res
    assert res["states_max_abs_diff"] < 2e-2 * max(1.0, res["states_max_abs"]), res
