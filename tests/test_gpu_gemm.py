"""tcgen05 GEMM numerics against an fp32 PyTorch reference of the same contraction."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from dllm_qwen38_b200.ops import cuda as C

    return C


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


SHAPES = [(128, 256, 64), (256, 512, 128), (300, 200, 72), (1000, 1040, 520), (2048, 4096, 1024), (64, 48, 5120)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_nt_bf16_and_f32(M, N, K):
    C = _ops()
    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    ref = a.float() @ b.float().t()
    assert _rel(C.gemm_nt(a, b), ref) < 1e-2
    assert _rel(C.gemm_nt(a, b, out_dtype=torch.float32), ref) < 1e-5
    r = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    assert _rel(C.gemm_nt(a, b, residual=r), ref + r.float()) < 1e-2
    C.check_errors()


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_nn_and_tn(M, N, K):
    C = _ops()
    torch.manual_seed(1)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    bkn = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    assert N % 8 == 0
    assert _rel(C.gemm_nn(a, bkn, out_dtype=torch.float32), a.float() @ bkn.float()) < 1e-5
    if M % 8:
        return  # an MN-major operand's inner (M) extent must keep 16-byte rows for TMA
    akm = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)
    assert _rel(C.gemm_tn(akm, bkn), akm.float().t() @ bkn.float()) < 1e-5
    acc = torch.ones(M, N, device="cuda")
    C.gemm_tn(akm, bkn, out=acc, accumulate=True)
    assert _rel(acc, akm.float().t() @ bkn.float() + 1) < 1e-5
    C.check_errors()


@pytest.fixture(params=["1", "0"], ids=["256x512", "256x256"])
def pair_width(request, monkeypatch):
    """Both tile widths of the two-CTA kernel (the variable is read at every GEMM call)."""
    monkeypatch.setenv("BDLLM_GEMM_WIDE", request.param)
    return request.param


@pytest.mark.parametrize("M,N,K", [(4096, 2560, 1024), (4104, 2568, 520), (8192, 5200, 256)])
def test_cta_pair_all_majors(M, N, K, pair_width):
    """Shapes with >= 148 256x256 tiles take the two-CTA (cta_group::2) kernel: K-major and
    MN-major operands, bf16 / fp32 / in-place accumulate epilogues, M, N and K tails. In the
    256 x 512 variant, 4096 x 2560 leaves a partial last wave (split into half-tiles), 2568 and
    5200 leave a last tile column whose second half lies beyond N."""
    from dllm_qwen38_b200 import _C

    torch.manual_seed(5)
    a_mk = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    a_km = a_mk.t().contiguous()
    b_nk = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    b_kn = b_nk.t().contiguous()
    ref = a_mk.float() @ b_nk.float().t()
    for a_mn in (False, True):
        for b_mn in (False, True):
            if a_mn and not b_mn:
                continue
            a, lda = (a_km, M) if a_mn else (a_mk, K)
            b, ldb = (b_kn, N) if b_mn else (b_nk, K)
            c32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
            _C.gemm(a, a_mn, lda, b, b_mn, ldb, M, N, K, c32, N, 1)
            assert _rel(c32, ref) < 1e-5, (a_mn, b_mn)
            c16 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            _C.gemm(a, a_mn, lda, b, b_mn, ldb, M, N, K, c16, N, 0)
            assert _rel(c16, ref) < 1e-2, (a_mn, b_mn)
            acc = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
            want = acc.float() + ref
            _C.gemm(a, a_mn, lda, b, b_mn, ldb, M, N, K, acc, N, 2, acc, N)  # in place, as wgrad runs it
            assert _rel(acc, want) < 1e-2, (a_mn, b_mn)
    _ops().check_errors()


def test_bn128_variant():
    from dllm_qwen38_b200 import _C

    torch.manual_seed(2)
    a = torch.randn(512, 256, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(384, 256, device="cuda", dtype=torch.bfloat16)
    c = torch.empty(512, 384, device="cuda", dtype=torch.float32)
    _C.gemm(a, False, 256, b, False, 256, 512, 384, 256, c, 384, 1, None, 0, None, 128)
    assert _rel(c, a.float() @ b.float().t()) < 1e-5


@pytest.mark.parametrize("M,F,K", [(256, 384, 128), (1000, 1000, 520), (4096, 3584, 1024), (4096, 3600, 512)])
def test_swiglu_epilogue(M, F, K, pair_width):
    C = _ops()
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2 * F, K, device="cuda", dtype=torch.bfloat16) * K ** -0.5
    act, gu = C.gemm_swiglu(x, w, F, store_gu=True)
    g = (x.float() @ w[:F].float().t())
    u = (x.float() @ w[F:].float().t())
    assert _rel(gu[:, :F], g) < 1e-2 and _rel(gu[:, F:], u) < 1e-2
    ref = torch.nn.functional.silu(gu[:, :F].float()) * gu[:, F:].float()
    assert _rel(act, ref) < 1e-2


def test_linear_autograd_matches_fp32():
    C = _ops()
    torch.manual_seed(4)
    x = torch.randn(3, 100, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(384, 256, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    y = C.linear(x, w)
    dy = torch.randn_like(y)
    y.backward(dy)
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    (xf @ wf.t()).backward(dy.float())
    assert _rel(y, xf @ wf.t()) < 1e-2
    assert _rel(x.grad, xf.grad) < 1e-2
    assert _rel(w.grad, wf.grad) < 1e-2


@pytest.mark.parametrize("M,N,K", [(32, 5120, 8192), (64, 1024, 4096), (16, 2048, 17408)])
def test_splitk_skinny_gemm(M, N, K):
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    r = torch.randn(M, N, device="cuda").bfloat16()
    assert Cu._splits(M, N, K) > 1
    want = a.float() @ b.float().t()
    got = Cu.gemm_nt(a, b)
    assert float((got.float() - want).abs().max()) < 2e-2 * float(want.abs().max())
    got_r = Cu.gemm_nt(a, b, residual=r)
    assert float((got_r.float() - (want + r.float())).abs().max()) < 2e-2 * float(want.abs().max())
