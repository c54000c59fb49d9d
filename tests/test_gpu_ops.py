"""Conv, SwiGLU MLP, masked CE and AdamW kernels against fp32 PyTorch references."""

import pytest
import torch

from dllm_qwen38_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("mode", ["fork", "no-prefix", "concat"])
@pytest.mark.parametrize("L,block,C", [(64, 16, 64), (96, 32, 40 * 8), (100, 20, 64)])
def test_conv_fwd_bwd(mode, L, block, C):
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(0)
    raw = torch.randn(2, 2 * L, C, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(C, 4, device="cuda") * 0.5).requires_grad_(True)
    y = Cu.conv_blockdiff(raw, w, L, block, mode)
    dy = torch.randn_like(y)
    y.backward(dy)
    rf, wf = raw.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    yr = ref.conv_blockdiff(rf, wf, L, block, mode)
    yr.backward(dy.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(raw.grad, rf.grad) < 1e-2
    assert _rel(w.grad, wf.grad) < 1e-2


def test_swiglu_mlp_fwd_bwd():
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(1)
    D, F = 256, 512
    x = torch.randn(3, 100, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    ws = [(torch.randn(*s, device="cuda") * s[1] ** -0.5).to(torch.bfloat16).requires_grad_(True)
          for s in ((F, D), (F, D), (D, F))]
    y = Cu.swiglu_mlp(x, *ws)
    dy = torch.randn_like(y)
    y.backward(dy)
    xf = x.detach().float().requires_grad_(True)
    wf = [w.detach().float().requires_grad_(True) for w in ws]
    yr = ref.linear(ref.swiglu(ref.linear(xf, wf[0]), ref.linear(xf, wf[1])), wf[2])
    yr.backward(dy.float())
    assert _rel(y, yr) < 2e-2
    assert _rel(x.grad, xf.grad) < 2e-2
    for w, r in zip(ws, wf):
        assert _rel(w.grad, r.grad) < 2e-2


def test_masked_ce_fwd_bwd():
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(2)
    n, D, V = 300, 256, 5000 - 8
    h = torch.randn(n, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(V, D, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    t = torch.randint(0, V, (n,), device="cuda")
    loss = Cu.masked_ce_sum(h, w, t) / n
    loss.backward()
    hf, wf = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lr = ref.masked_ce_sum(hf, wf, t) / n
    lr.backward()
    assert abs(float(loss) - float(lr)) < 1e-2 * float(lr)
    assert _rel(h.grad, hf.grad) < 2e-2 and _rel(w.grad, wf.grad) < 2e-2


def test_masked_ce_full_vocab_preset_grad_and_device_scale():
    """4096 target rows over the full 248,320-row vocabulary against fp32, with the upstream
    gradient scale kept on the device and dW added in place into a preset bf16 gradient (the
    sharded engine's layout: no fp32 [V, D] temporary, no host synchronisation in the backward)."""
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(4)
    n, D, V = 4096, 256, 248320
    h = torch.randn(n, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(V, D, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    w.grad = torch.zeros_like(w)  # preset gradient buffer: the CE backward accumulates into it
    t = torch.randint(0, V, (n,), device="cuda")
    scale = torch.tensor(1.0 / n, device="cuda")
    loss = Cu.masked_ce_sum(h, w, t) * scale
    loss.backward()
    hf, wf = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lr = ref.masked_ce_sum(hf, wf, t) / n
    lr.backward()
    assert abs(float(loss) - float(lr)) < 1e-2 * float(lr)
    assert _rel(h.grad, hf.grad) < 2e-2 and _rel(w.grad, wf.grad) < 2e-2
    m = float((w.grad.float() - wf.grad).abs().max()) / float(wf.grad.abs().max())
    assert m < 3e-2, m


def test_adamw_matches_reference_update():
    from dllm_qwen38_b200.train.optim import MasterAdamW

    torch.manual_seed(3)
    p_gpu = torch.nn.Parameter(torch.randn(1000, device="cuda").to(torch.bfloat16))
    p_cpu = torch.nn.Parameter(p_gpu.detach().float().cpu())
    og, oc = MasterAdamW([p_gpu], lr=1e-2), MasterAdamW([p_cpu], lr=1e-2)
    for _ in range(3):
        g = torch.randn(1000)
        p_gpu.grad = g.to("cuda", torch.bfloat16)
        p_cpu.grad = g.to(torch.bfloat16).float()
        og.step(clip=1.0)
        oc.step(clip=1.0)
    assert _rel(og.master[0].cpu(), p_cpu.detach()) < 1e-5


@pytest.mark.parametrize("n,gdt", [(1003, torch.bfloat16), (4096 * 37 + 2, torch.bfloat16), (999, torch.float32)])
def test_adamw_flat_vector_kernel_against_fp32(n, gdt):
    """The flat AdamW (4 elements per thread, n % 4 tail) against the fp32 update with a device
    clip coefficient."""
    from dllm_qwen38_b200.ops import cuda as C

    torch.manual_seed(4)
    w = torch.randn(n, device="cuda")
    m = torch.randn(n, device="cuda").abs() * 0.1
    v = torch.randn(n, device="cuda").abs() * 0.01
    g = torch.randn(n, device="cuda").to(gdt)
    p = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    coef = torch.tensor(0.7, device="cuda")
    lr, b1, b2, eps, wd, bc1, bc2 = 1e-2, 0.9, 0.95, 1e-8, 0.1, 0.5, 0.3
    gf = g.float() * 0.7
    m_ref = b1 * m + (1 - b1) * gf
    v_ref = b2 * v + (1 - b2) * gf * gf
    w_ref = w * (1 - lr * wd) - lr * (m_ref / bc1) / ((v_ref / bc2).sqrt() + eps)
    C.adamw_flat(w, p, g, m, v, lr, b1, b2, eps, wd, coef, bc1, bc2)
    torch.cuda.synchronize()
    assert _rel(m, m_ref) < 1e-6 and _rel(v, v_ref) < 1e-6 and _rel(w, w_ref) < 1e-6
    assert torch.equal(p, w.to(torch.bfloat16))


def test_gdn_gates_fwd_bwd_against_reference():
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(0)
    B, T, H = 2, 64, 12
    proj = torch.randn(B, T, 40 + 2 * H, device="cuda").bfloat16()
    a, b = proj[..., 40:40 + H], proj[..., 40 + H:]
    A_log = torch.randn(H, device="cuda") * 0.5
    dt = torch.randn(H, device="cuda") * 0.5
    ar, br = a.float().clone().requires_grad_(True), b.float().clone().requires_grad_(True)
    Ar, dr = A_log.clone().requires_grad_(True), dt.clone().requires_grad_(True)
    g_ref, beta_ref = ref.gdn_gates(ar, br, Ar, dr)
    An, dn = A_log.clone().requires_grad_(True), dt.clone().requires_grad_(True)
    an, bn = a.clone().requires_grad_(True), b.clone().requires_grad_(True)
    g, beta = Cu.gdn_gates(an, bn, An, dn)
    assert torch.allclose(g, g_ref, rtol=1e-4, atol=1e-5) and torch.allclose(beta, beta_ref, rtol=1e-4, atol=1e-5)
    wg, wb = torch.randn_like(g), torch.randn_like(beta)
    ((g_ref * wg).sum() + (beta_ref * wb).sum()).backward()
    ((g * wg).sum() + (beta * wb).sum()).backward()
    assert torch.allclose(an.grad.float(), ar.grad, rtol=2e-2, atol=2e-2)
    assert torch.allclose(bn.grad.float(), br.grad, rtol=2e-2, atol=2e-2)
    assert torch.allclose(An.grad, Ar.grad, rtol=1e-3, atol=1e-3)
    assert torch.allclose(dn.grad, dr.grad, rtol=1e-3, atol=1e-3)


def test_embedding_fwd_bwd_against_torch():
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(0)
    table = torch.randn(300, 64, device="cuda").bfloat16().requires_grad_(True)
    ids = torch.randint(0, 300, (3, 50), device="cuda")
    ids[0, :5] = 7  # repeated rows accumulate
    h = Cu.embedding(ids, table)
    assert torch.equal(h, torch.nn.functional.embedding(ids, table.detach()))
    dh = torch.randn_like(h)
    h.backward(dh)
    want = torch.zeros(300, 64, device="cuda").index_add_(0, ids.reshape(-1), dh.reshape(-1, 64).float())
    assert torch.allclose(table.grad.float(), want, rtol=1e-2, atol=1e-2)


def test_embedding_sorted_gradient_into_bf16():
    """Per-id sums of the sorted rows written as bf16 rows (the one-rank engine's embedding
    gradient), against fp32 index_add; ids absent from the batch keep the zeros."""
    from dllm_qwen38_b200 import _C

    torch.manual_seed(1)
    V, D = 1000, 5120
    ids = torch.randint(0, V, (2 * 7000,), device="cuda")
    ids[:6000] = 3  # one long run, as the mask token makes in the noised stream
    dh = torch.randn(ids.numel(), D, device="cuda").bfloat16()
    g = torch.zeros(V, D, device="cuda", dtype=torch.bfloat16)
    sid, perm = torch.sort(ids)
    _C.embed_bwd_sorted(g, sid, perm, dh)
    want = torch.zeros(V, D, device="cuda").index_add_(0, ids, dh.float())
    assert _rel(g, want) < 5e-3
    absent = torch.ones(V, dtype=torch.bool, device="cuda")
    absent[ids] = False
    assert bool((g[absent] == 0).all())


def test_output_gate_fwd_bwd_with_the_gate_read_in_place():
    """o * sigmoid(gate) with the gate a strided half of a q|gate projection, forward and
    backward against fp32 autograd."""
    from dllm_qwen38_b200 import ops

    torch.manual_seed(3)
    B, T, H, D = 2, 96, 6, 256
    qg = torch.randn(B, T, H, 2 * D, device="cuda").bfloat16().requires_grad_(True)
    _, gate = torch.split(qg, D, dim=-1)
    o = torch.randn(B, T, H, D, device="cuda").bfloat16().requires_grad_(True)
    y = ops.output_gate(o, gate)
    assert ops.last_impl("output_gate") == "native"
    dy = torch.randn_like(y)
    y.backward(dy)
    of, qf = o.detach().float().requires_grad_(True), qg.detach().float().requires_grad_(True)
    yf = of * torch.sigmoid(qf[..., D:])
    yf.backward(dy.float())
    assert _rel(y, yf) < 1e-2
    assert _rel(o.grad, of.grad) < 1e-2 and _rel(qg.grad, qf.grad) < 1e-2
    assert float(qg.grad[..., :D].abs().max()) == 0.0  # the q half gets nothing from the gate


def test_swiglu_act_matches_the_gemm_epilogue():
    """The activation rebuilt from the stored bf16 gate|up equals the one the SwiGLU GEMM wrote."""
    from dllm_qwen38_b200 import _C
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(2)
    x = torch.randn(4096, 1024, device="cuda").bfloat16()
    w = (torch.randn(2 * 3584, 1024, device="cuda") * 0.03).bfloat16()
    act, gu = Cu.gemm_swiglu(x, w, 3584, store_gu=True)
    assert torch.equal(_C.swiglu_act(gu), act)


@pytest.mark.parametrize("xdt,ddt", [(torch.float32, None), (torch.bfloat16, None), (torch.bfloat16, torch.float32),
                                     (torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32)])
@pytest.mark.parametrize("n", [8, 1000003, 4096 * 33])
def test_sumsq_with_copy(xdt, ddt, n):
    """sq += ||x||^2 (fp32 accumulate) with the optional fused copy into dst, vector tails included."""
    from dllm_qwen38_b200 import _C

    torch.manual_seed(4)
    x = torch.randn(n, device="cuda").to(xdt)
    sq = torch.full((1,), 2.5, device="cuda")
    dst = torch.empty(n, device="cuda", dtype=ddt) if ddt is not None else None
    _C.sumsq_(x, sq, dst)
    torch.cuda.synchronize()
    want = 2.5 + float(x.double().pow(2).sum())
    assert abs(float(sq[0]) - want) < 1e-4 * want
    if dst is not None:
        assert torch.equal(dst, x.to(ddt))


def test_mask_sample_kernel_complementary_views():
    """The fused mask kernel: both views partition the scorable positions, prompt and padding are
    never noised, [MASK] sits exactly where a view masks, a seed reproduces its masks, and the
    per-block ratios spread over (0, 1) with mean 1/2 (t ~ U(0, 1) per block)."""
    from dllm_qwen38_b200.train.objective import complementary_step_inputs

    B, L, block, mask_id = 4, 4096, 32, 999
    g = torch.Generator(device="cuda").manual_seed(0)
    x0 = torch.randint(0, 900, (B, L), device="cuda", generator=g)
    pl = torch.tensor([0, 17, 100, 0], device="cuda")
    vl = torch.tensor([L, L, L - 50, L - 1], device="cuda")
    x0_2, xt_2, m_2 = complementary_step_inputs(x0, pl, block, mask_id, None, vl, seed=1234)
    pos = torch.arange(L, device="cuda")[None]
    scor = (pos >= pl[:, None]) & (pos < vl[:, None])
    m, mc = m_2[:B], m_2[B:]
    assert torch.equal(x0_2[:B], x0) and torch.equal(x0_2[B:], x0)
    assert not bool((m & mc).any()) and torch.equal(m | mc, scor)
    assert torch.equal(xt_2, torch.where(m_2, torch.full_like(x0_2, mask_id), x0_2))
    again = complementary_step_inputs(x0, pl, block, mask_id, None, vl, seed=1234)
    assert torch.equal(again[2], m_2)
    other = complementary_step_inputs(x0, pl, block, mask_id, None, vl, seed=1235)
    assert not torch.equal(other[2], m_2)
    ratio = m[0].float().view(-1, block).mean(1)  # row 0: every position scorable
    assert 0.4 < float(ratio.mean()) < 0.6
    assert float(ratio.min()) < 0.15 and float(ratio.max()) > 0.85
