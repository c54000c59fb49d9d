"""Norm kernels (forward and backward) against fp32 PyTorch references."""

import pytest
import torch

from dllm_qwen38_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _fp32_grads(fn, *tensors, dy):
    ts = [t.detach().float().requires_grad_(True) for t in tensors]
    out = fn(*ts)
    out.backward(dy.float())
    return out, [t.grad for t in ts]


@pytest.mark.parametrize("D", [128, 1024, 5120])
def test_rmsnorm_fwd_bwd(D):
    from dllm_qwen38_b200.ops import cuda as C

    torch.manual_seed(0)
    x = torch.randn(3, 333, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(D, device="cuda") * 0.1).to(torch.bfloat16).requires_grad_(True)
    y = C.rmsnorm(x, w, 1e-6)
    dy = torch.randn_like(y)
    y.backward(dy)
    yr, (dxr, dwr) = _fp32_grads(lambda a, b: ref.rmsnorm(a, b, 1e-6), x, w, dy=dy)
    assert _rel(y, yr) < 1e-2 and _rel(x.grad, dxr) < 1e-2 and _rel(w.grad, dwr) < 1e-2


@pytest.mark.parametrize("D,pad", [(32, 8), (64, 8), (96, 8), (128, 8), (128, 1), (256, 8)])
def test_gated_rmsnorm_fwd_bwd(D, pad):
    """z is read in place from a wider projection row (token stride 6 D + pad): pad 8 keeps the
    per-lane vectors aligned, pad 1 takes the element-wise path."""
    from dllm_qwen38_b200.ops import cuda as C

    torch.manual_seed(1)
    x = torch.randn(2, 100, 6, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    zfull = torch.randn(2, 100, 6 * D + pad, device="cuda", dtype=torch.bfloat16)
    z = zfull[..., : 6 * D].reshape(2, 100, 6, D).detach().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    y = C.gated_rmsnorm(x, z, w, 1e-6)
    dy = torch.randn_like(y)
    y.backward(dy)
    yr, (dxr, dzr, dwr) = _fp32_grads(lambda a, b, c: ref.gated_rmsnorm(a, b, c, 1e-6), x, z, w, dy=dy)
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, dxr) < 2e-2 and _rel(z.grad, dzr) < 2e-2 and _rel(w.grad, dwr) < 2e-2


@pytest.mark.parametrize("Dh,R", [(32, 8), (256, 64)])
def test_qk_norm_rope_strided_fwd_bwd(Dh, R):
    from dllm_qwen38_b200.ops import cuda as C

    torch.manual_seed(2)
    B, L, Hq, Hk = 2, 48, 4, 2
    qg = torch.randn(B, 2 * L, Hq, 2 * Dh, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, 2 * L, Hk, Dh, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    q = qg[..., :Dh]
    wq = (0.1 * torch.randn(Dh, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    wk = (0.1 * torch.randn(Dh, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    cos, sin = ref.rope_cos_sin(torch.arange(L), R, 1e7, torch.bfloat16, "cuda")
    cos2, sin2 = torch.cat([cos, cos]), torch.cat([sin, sin])
    qo, ko = C.qk_norm_rope(q, k, wq, wk, 1e-6, cos2, sin2)
    dq, dk = torch.randn_like(qo), torch.randn_like(ko)
    (qo.float() * dq.float()).sum().add((ko.float() * dk.float()).sum()).backward()

    def f(qq, kk, a, b):
        return torch.cat([ref.apply_rope(ref.rmsnorm(qq, a, 1e-6), cos2.float(), sin2.float()).flatten(),
                          ref.apply_rope(ref.rmsnorm(kk, b, 1e-6), cos2.float(), sin2.float()).flatten()])

    qf = q.detach().float().requires_grad_(True)
    kf, wqf, wkf = (t.detach().float().requires_grad_(True) for t in (k, wq, wk))
    out = f(qf, kf, wqf, wkf)
    out.backward(torch.cat([dq.float().flatten(), dk.float().flatten()]))
    assert _rel(torch.cat([qo.flatten(), ko.flatten()]), out) < 1e-2
    assert _rel(qg.grad[..., :Dh], qf.grad) < 2e-2 and float(qg.grad[..., Dh:].abs().max()) == 0
    assert _rel(k.grad, kf.grad) < 2e-2
    assert _rel(wq.grad, wqf.grad) < 2e-2 and _rel(wk.grad, wkf.grad) < 2e-2
