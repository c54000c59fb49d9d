"""The tcgen05 / TMEM / TMA state-fork GDN forward (`csrc/gdn_tc.cu`) against fp32 references.

Checks the output of both streams against the fp32 state-fork reference, the chunk-entry states
against the fp32 chunked specification of the clean stream, the gradients of the whole op (the
backward consumes the states this forward saves) against autograd of the fp32 reference, and the
27B head shape (48 v-heads over 16 qk-heads, head dim 128) at L 2048. Tolerances: relative
Frobenius error 1e-2 and max-abs error within 3 % of the reference's largest magnitude.
"""

import pytest
import torch

from dllm_qwen38_b200.ops import gdn_chunked
from dllm_qwen38_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _close(a, b, rel=1e-2, mabs=3e-2):
    r = _rel(a, b)
    m = float((a.float() - b.float()).abs().max()) / (float(b.float().abs().max()) + 1e-12)
    assert r < rel and m < mabs, (r, m)


def _inputs(B, L, Hk, Hv, D=128, seed=0, grad=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T2 = 2 * L
    mixed = torch.randn(B, T2, 2 * Hk * D + Hv * D, device="cuda", dtype=torch.bfloat16, generator=g)
    gate = -torch.nn.functional.softplus(torch.randn(B, T2, Hv, device="cuda", generator=g))
    beta = torch.sigmoid(torch.randn(B, T2, Hv, device="cuda", generator=g))
    if grad:
        mixed.requires_grad_(True)
        gate.requires_grad_(True)
        beta.requires_grad_(True)
    q = mixed[..., : Hk * D].reshape(B, T2, Hk, D)
    k = mixed[..., Hk * D : 2 * Hk * D].reshape(B, T2, Hk, D)
    v = mixed[..., 2 * Hk * D :].reshape(B, T2, Hv, D)
    return mixed, q, k, v, gate, beta


@pytest.mark.parametrize("B,L,Hk,Hv", [(1, 128, 1, 1), (2, 256, 2, 6), (1, 512, 1, 3), (1, 2048, 16, 48)])
def test_gdn_tc_forward_matches_fp32(B, L, Hk, Hv):
    from dllm_qwen38_b200 import _C

    _, q, k, v, gate, beta = _inputs(B, L, Hk, Hv, seed=B * 7 + L)
    assert _C.gdn_tc_eligible(q, k, v, L, 32, False)
    o, S_in = _C.gdn_fwd_tc(q, k, v, gate.contiguous(), beta.contiguous(), L)
    torch.cuda.synchronize()
    with torch.no_grad():
        orf = ref.gdn_core_blockdiff(q.float(), k.float(), v.float(), gate, beta, L, 32, 32, "fork")
        rep = Hv // Hk
        qc, kc = q[:, L:].float().repeat_interleave(rep, 2), k[:, L:].float().repeat_interleave(rep, 2)
        _, S_ref, _, _ = gdn_chunked.forward(qc, kc, v[:, L:].float(), gate[:, L:], beta[:, L:], 32)
    _close(o[:, :L], orf[:, :L])  # noised blocks (forked from the clean states)
    _close(o[:, L:], orf[:, L:])  # clean stream
    # S_in: bf16 S^T rows [B, nb, Hv, Dv, Dk]; the spec's states are [B, Hv, nb, Dk, Dv]
    assert S_in.dtype == torch.bfloat16
    _close(S_in.transpose(-1, -2), S_ref.transpose(1, 2))


def test_gdn_tc_forward_matches_the_mma_sync_kernels():
    from dllm_qwen38_b200 import _C

    B, L, Hk, Hv = 2, 384, 2, 4
    _, q, k, v, gate, beta = _inputs(B, L, Hk, Hv, seed=3)
    o, S_in = _C.gdn_fwd_tc(q, k, v, gate.contiguous(), beta.contiguous(), L)
    o2, S2, _ = _C.gdn_fwd(q, k, v, gate.contiguous(), beta.contiguous(), L, 32, False)
    _close(o, o2)
    _close(S_in.transpose(-1, -2), S2)


def test_gdn_tc_op_forward_backward_against_autograd():
    """Through the op (the tensor-core forward is taken), gradients of the fp32 reference."""
    from dllm_qwen38_b200.ops import cuda as Cu

    B, L, Hk, Hv = 1, 256, 2, 6
    mixed, q, k, v, gate, beta = _inputs(B, L, Hk, Hv, seed=5, grad=True)
    o = Cu.gdn_core_blockdiff(q, k, v, gate, beta, L, 32, 64, "fork")
    do = torch.randn_like(o)
    o.backward(do)
    mf = mixed.detach().float().requires_grad_(True)
    gf, bf = gate.detach().clone().requires_grad_(True), beta.detach().clone().requires_grad_(True)
    D = 128
    qf = mf[..., : Hk * D].reshape(B, 2 * L, Hk, D)
    kf = mf[..., Hk * D : 2 * Hk * D].reshape(B, 2 * L, Hk, D)
    vf = mf[..., 2 * Hk * D :].reshape(B, 2 * L, Hv, D)
    orf = ref.gdn_core_blockdiff(qf, kf, vf, gf, bf, L, 32, 32, "fork")
    orf.backward(do.float())
    _close(o, orf)
    assert _rel(mixed.grad, mf.grad) < 2e-2, _rel(mixed.grad, mf.grad)
    assert _rel(gate.grad, gf.grad) < 2e-2, _rel(gate.grad, gf.grad)
    assert _rel(beta.grad, bf.grad) < 2e-2, _rel(beta.grad, bf.grad)
    Cu.check_errors()


@pytest.mark.parametrize("B,L,Hk,Hv", [(2, 128, 1, 2), (1, 1024, 16, 48)])
def test_gdn_tc_backward_matches_fp32_autograd(B, L, Hk, Hv):
    """The tensor-core backward chunk kernels (noised blocks and clean chunks) through the op, on
    the 27B head shape at L 1024 and a small batched case, against autograd of the fp32 reference."""
    from dllm_qwen38_b200.ops import cuda as Cu

    mixed, q, k, v, gate, beta = _inputs(B, L, Hk, Hv, seed=L + Hv, grad=True)
    o = Cu.gdn_core_blockdiff(q, k, v, gate, beta, L, 32, 64, "fork")
    do = torch.randn_like(o)
    o.backward(do)
    Cu.check_errors()
    mf = mixed.detach().float().requires_grad_(True)
    gf, bf = gate.detach().clone().requires_grad_(True), beta.detach().clone().requires_grad_(True)
    D = 128
    qf = mf[..., : Hk * D].reshape(B, 2 * L, Hk, D)
    kf = mf[..., Hk * D : 2 * Hk * D].reshape(B, 2 * L, Hk, D)
    vf = mf[..., 2 * Hk * D :].reshape(B, 2 * L, Hv, D)
    orf = ref.gdn_core_blockdiff(qf, kf, vf, gf, bf, L, 32, 32, "fork")
    orf.backward(do.float())
    for name, got, want in (("q", mixed.grad[..., : Hk * D], mf.grad[..., : Hk * D]),
                            ("k", mixed.grad[..., Hk * D : 2 * Hk * D], mf.grad[..., Hk * D : 2 * Hk * D]),
                            ("v", mixed.grad[..., 2 * Hk * D :], mf.grad[..., 2 * Hk * D :]),
                            ("g", gate.grad, gf.grad), ("beta", beta.grad, bf.grad)):
        r = _rel(got, want)
        assert r < 2e-2, (name, r)
