"""Per-kernel benchmarks with roofline fractions (one op, one shape, one JSON line).

    python -m dllm_qwen38_b200.bench.kernels gemm --M 8192 --N 5120 --K 5120
    python -m dllm_qwen38_b200.bench.kernels gdn --L 8192 --block 32 [--impl reference]
    python -m dllm_qwen38_b200.bench.kernels attn --L 4096 --block 32
    python -m dllm_qwen38_b200.bench.kernels ce --rows 8192 --vocab 248320
    python -m dllm_qwen38_b200.bench.kernels conv|rmsnorm|adamw ...

Timing: CUDA events on the launching stream around each iteration, after warm-up, with a write of
a buffer larger than L2 (256 MiB) before every timed iteration; the median is reported.
Denominators are the measured copy bandwidth and cuBLAS bf16 rate in MEASURED_PEAKS.json at the
repository root (fallback 6.65 TB/s and 1.59 PFLOP/s when absent). The GDN op is the state-fork
sweep of the inference/training shapes (48 v heads / 16 qk heads, dk = dv = 128, rows =
batch x (blocks + 1)); `--impl reference` runs the reference's own chunked torch function
(`gdn.py:48-123`) the way its block-diffusion forward uses it (`blockdiff.py:159-177`).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]) * 1e9, float(p["bf16_tflops"]) * 1e12, "measured"
    except Exception:  # noqa: BLE001
        return 6.65e12, 1.59e15, "fallback"


def timeit(fn, iters: int, warmup: int) -> float:
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for i in range(iters):
        flush.fill_(i & 0xFF)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def sustained(fn, seconds: float):
    """Mean ms of `fn` run back to back for about `seconds` (CUDA events around the whole loop),
    with the SM clocks sampled during it."""
    from ..utils.clocks import ClockSampler

    for _ in range(5):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        fn()
    e1.record()
    torch.cuda.synchronize()
    n = max(10, int(seconds * 1000.0 / max(e0.elapsed_time(e1) / 10, 1e-3)))
    sampler = ClockSampler(gpu=torch.cuda.current_device()).start()
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n, sampler.stop()


def op_gemm(a):
    """--layout nt: y[M,N] = x[M,K] w[N,K]^T (forward); nn: x[M,K] w[K,N] (input gradient, w read
    N-contiguous); tn: g[M,N] += a[K,M]^T b[K,N] into bf16 (weight gradient, both operands
    MN-major, accumulated in place as the training step runs it)."""
    from ..ops import cuda as Cu

    if a.layout == "nt":
        x = torch.randn(a.M, a.K, device="cuda").bfloat16()
        w = torch.randn(a.N, a.K, device="cuda").bfloat16()
        fn = (lambda: torch.matmul(x, w.t())) if a.impl == "cublas" else (lambda: Cu.gemm_nt(x, w))
    elif a.layout == "nn":
        x = torch.randn(a.M, a.K, device="cuda").bfloat16()
        w = torch.randn(a.K, a.N, device="cuda").bfloat16()
        fn = (lambda: torch.matmul(x, w)) if a.impl == "cublas" else (lambda: Cu.gemm_nn(x, w))
    else:
        at = torch.randn(a.K, a.M, device="cuda").bfloat16()
        bt = torch.randn(a.K, a.N, device="cuda").bfloat16()
        g = torch.zeros(a.M, a.N, device="cuda").bfloat16()
        if a.impl == "cublas":
            fn = lambda: g.addmm_(at.t(), bt)  # noqa: E731
        else:
            fn = lambda: Cu._C.gemm(at, True, a.M, bt, True, a.N, a.M, a.N, a.K, g, a.N, Cu.EPI_ADD_BF16, g, a.N)  # noqa: E731
    return fn, 2.0 * a.M * a.N * a.K, 2.0 * (a.M * a.K + a.N * a.K + a.M * a.N)


def op_swiglu(a):
    """act[M, N] = silu(x Wg^T) * (x Wu^T), x [M, K], [Wg; Wu] [2N, K] (the MLP's gate/up GEMM with
    its SwiGLU epilogue); --layout tn also stores the bf16 (gate | up) [M, 2N], as the backward's
    recomputation does. cublas: the [M, 2N] product, then torch's silu * up."""
    from ..ops import cuda as Cu

    x = torch.randn(a.M, a.K, device="cuda").bfloat16()
    w = (torch.randn(2 * a.N, a.K, device="cuda") * a.K ** -0.5).bfloat16()
    gu = a.layout == "tn"
    if a.impl == "cublas":
        def fn():
            y = torch.matmul(x, w.t())
            return torch.nn.functional.silu(y[:, : a.N]) * y[:, a.N :]
    else:
        def fn():
            return Cu.gemm_swiglu(x, w, a.N, gu)
    return fn, 4.0 * a.M * a.N * a.K, 2.0 * (a.M * a.K + 2 * a.N * a.K + a.M * a.N * (3 if gu else 1))


def _gdn_inputs(a):
    B, L, Hk, Hv, D = a.B, a.L, 16, 48, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, 2 * L, Hk, D, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, 2 * L, Hk, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, 2 * L, Hv, D, device="cuda", generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(B, 2 * L, Hv, device="cuda", generator=g))
    lg = -torch.nn.functional.softplus(torch.randn(B, 2 * L, Hv, device="cuda", generator=g))
    return q, k, v, lg, beta


def op_gdn(a):
    """forward + backward of the state-fork delta rule over [x_t || x_0] of length 2L."""
    q, k, v, lg, beta = _gdn_inputs(a)
    B, L, Hv, D = a.B, a.L, 48, 128
    nb = L // a.block
    if a.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        from dllm_qwen38.gdn import chunk_gated_delta_rule_with_states as rf

        def fn():
            qq, kk, vv, gg, bb = (t.detach().requires_grad_(True) for t in (q, k, v, lg, beta))
            rep = Hv // qq.shape[2]
            qr, kr = qq.repeat_interleave(rep, 2), kk.repeat_interleave(rep, 2)
            sl = slice(L, 2 * L)
            o0, st = rf(qr[:, sl], kr[:, sl], vv[:, sl], gg[:, sl], bb[:, sl], a.block)
            init = torch.cat([torch.zeros_like(st[:, :1]), st[:, :-1]], 1).reshape(B * nb, Hv, D, D)
            rs = lambda x: x[:, :L].reshape(B * nb, a.block, *x.shape[2:])  # noqa: E731
            ot, _ = rf(rs(qr), rs(kr), rs(vv), rs(gg), rs(bb), a.block, initial_state=init, need_states=False)
            (o0.float().sum() + ot.float().sum()).backward()
    else:
        from ..ops import cuda as Cu

        def fn():
            qq, kk, vv, gg, bb = (t.detach().requires_grad_(True) for t in (q, k, v, lg, beta))
            o = Cu.gdn_core_blockdiff(qq, kk, vv, gg, bb, L, a.block, 64, "fork")
            o.float().sum().backward()
    # model FLOPs of the chunked algebra per (chunk, head): forward 6 C D^2 (W S, q S, K~^T V') +
    # 10 C^2 D (k k^T, q k^T, T X, T Y, P V'); backward about twice that
    C = a.block
    chunks = B * (2 * L // C)
    flops = chunks * Hv * (18.0 * C * D * D + 30.0 * C * C * D)
    byts = 2 * (q.numel() + k.numel() + 2 * v.numel()) * 2 + B * nb * Hv * D * D * 4 * 2
    return fn, flops, byts


def op_gdn_fwd(a):
    """forward only of the state-fork delta rule (the tcgen05 kernels when eligible; BDLLM_GDN_TC=0
    selects the mma.sync kernels)."""
    q, k, v, lg, beta = _gdn_inputs(a)
    from ..ops import cuda as Cu

    def fn():
        with torch.no_grad():
            Cu.gdn_core_blockdiff(q, k, v, lg, beta, a.L, a.block, 64, "fork")

    B, L, Hv, D, C = a.B, a.L, 48, 128, a.block
    chunks = B * (2 * L // C)
    flops = chunks * Hv * (6.0 * C * D * D + 10.0 * C * C * D)
    byts = (q.numel() + k.numel() + v.numel()) * 2 + v.numel() * 2 + B * (L // C) * Hv * D * D * 4
    return fn, flops, byts


def op_attn(a):
    from ..ops import cuda as Cu

    B, L, Hq, Hk, D = a.B, a.L, 24, 4, 256
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, 2 * L, Hq, D, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, 2 * L, Hk, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, 2 * L, Hk, D, device="cuda", generator=g).bfloat16()

    if a.impl == "reference":
        # the reference's additive [1, 1, 2L, 2L] mask (`blockdiff.py:50-66`) through torch SDPA with
        # the kv heads repeated, as its HF sdpa attention layers run it
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        from dllm_qwen38.blockdiff import complementary_mask

        mask = complementary_mask(L, a.block, torch.bfloat16, q.device)

        def fn():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            rep = Hq // Hk
            qt, kt, vt = (x.transpose(1, 2) for x in (qq, kk.repeat_interleave(rep, 2), vv.repeat_interleave(rep, 2)))
            o = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, scale=D ** -0.5)
            o.float().sum().backward()
    else:
        def fn():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            o = Cu.attention_blockdiff(qq, kk, vv, L, a.block, D ** -0.5)
            o.float().sum().backward()
    # allowed pairs of the complementary mask: x_t rows see their block + earlier clean blocks
    # (~L^2/2 + L*block), x_0 rows the clean prefix (~L^2/2): ~L^2 pairs; fwd 4 D + bwd 10 D flops/pair
    pairs = float(L) * L + L * a.block
    flops = B * Hq * pairs * D * 14.0
    byts = 2 * (q.numel() * 3 + k.numel() * 3 + v.numel() * 3)
    return fn, flops, byts


def op_attn_fwd(a):
    """forward only (O and the row log2-sum-exp), same operands and pair count as `attn`"""
    from ..ops import cuda as Cu

    B, L, Hq, Hk, D = a.B, a.L, 24, 4, 256
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, 2 * L, Hq, D, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, 2 * L, Hk, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, 2 * L, Hk, D, device="cuda", generator=g).bfloat16()
    fn = lambda: Cu._C.attn_fwd(q, k, v, L, a.block, D ** -0.5, False)  # noqa: E731
    pairs = float(L) * L + L * a.block
    return fn, B * Hq * pairs * D * 4.0, 2 * (q.numel() * 2 + k.numel() + v.numel())


def op_ce(a):
    from ..ops import cuda as Cu

    h = torch.randn(a.rows, a.D, device="cuda").bfloat16()
    w = (torch.randn(a.vocab, a.D, device="cuda") * 0.02).bfloat16()
    t = torch.randint(0, a.vocab, (a.rows,), device="cuda")

    def fn():
        hh, ww = h.detach().requires_grad_(True), w.detach().requires_grad_(True)
        Cu.masked_ce_sum(hh, ww, t).backward()
    return fn, 6.0 * a.rows * a.vocab * a.D, 2.0 * (a.rows * a.vocab * 2 + a.vocab * a.D * 2)


def op_conv(a):
    from ..ops import cuda as Cu

    C = 10240
    raw = torch.randn(a.B, 2 * a.L, C, device="cuda").bfloat16()
    w = torch.randn(C, 4, device="cuda") * 0.3

    def fn():
        rr, ww = raw.detach().requires_grad_(True), w.detach().requires_grad_(True)
        Cu.conv_blockdiff(rr, ww, a.L, a.block, "fork").float().sum().backward()
    n = raw.numel()
    return fn, 16.0 * n, 2.0 * n * 5


def op_rmsnorm(a):
    from ..ops import cuda as Cu

    x = torch.randn(a.rows, a.D, device="cuda").bfloat16()
    w = torch.zeros(a.D, device="cuda").bfloat16()
    return (lambda: Cu.rmsnorm(x, w, 1e-6)), 4.0 * x.numel(), 4.0 * x.numel()


def op_rmsnorm_bwd(a):
    """RMSNorm(1+w) backward (`_C.rmsnorm_bwd`): dx and the weight-gradient partial rows, then
    their column sum; algorithmic bytes = read x and dy, write dx."""
    from ..ops import cuda as Cu

    x = torch.randn(a.rows, a.D, device="cuda").bfloat16()
    dy = torch.randn_like(x)
    w1 = torch.ones(a.D, device="cuda")
    return (lambda: Cu._C.rmsnorm_bwd(dy, x, w1, 1e-6)), 8.0 * x.numel(), 6.0 * x.numel()


def op_adamw(a):
    from ..ops import cuda as Cu

    n = a.n
    w = torch.randn(n, device="cuda")
    p = w.bfloat16()
    gr = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    return (lambda: Cu.adamw_flat(w, p, gr, m, v, 1e-5, 0.9, 0.95, 1e-8, 0.0, 1.0, 0.1, 0.05)), 12.0 * n, 30.0 * n


def op_qknorm(a):
    """q and k RMSNorm(1+w) + partial RoPE, forward + backward (`_C.qk_norm_rope_fwd/bwd`), 27B
    attention shapes: q [B, 2L, 24, 256], k [B, 2L, 4, 256], rotary dim 64"""
    from ..config import preset
    from ..models.blockdiff import rope_tables
    from ..ops import cuda as Cu

    cfg = preset("27b")
    B, T2, D = a.B, 2 * a.L, 256
    q = torch.randn(B, T2, 24, D, device="cuda").bfloat16()
    k = torch.randn(B, T2, 4, D, device="cuda").bfloat16()
    w1 = torch.ones(D, device="cuda")
    cos, sin = rope_tables(cfg, a.L, torch.bfloat16, "cuda")
    cos, sin = torch.cat([cos, cos]), torch.cat([sin, sin])  # both streams share positions 0..L-1
    dq, dk = torch.randn_like(q), torch.randn_like(k)

    def fn():
        Cu._C.qk_norm_rope_fwd(q, w1, cos, sin, 1e-6)
        Cu._C.qk_norm_rope_fwd(k, w1, cos, sin, 1e-6)
        Cu._C.qk_norm_rope_bwd(dq, q, w1, cos, sin, 1e-6)
        Cu._C.qk_norm_rope_bwd(dk, k, w1, cos, sin, 1e-6)
    n = q.numel() + k.numel()
    return fn, 20.0 * n, 2.0 * n * 5  # fwd: read x, write y; bwd: read dy, x, write dx


def op_gnorm(a):
    """gated RMSNorm of the GDN output, forward + backward (`_C.gated_rmsnorm_fwd/bwd`): rows =
    B x 2L x 48 heads of 128"""
    from ..ops import cuda as Cu

    rows = a.B * 2 * a.L * 48
    x = torch.randn(rows, 128, device="cuda").bfloat16()
    z = torch.randn(rows, 128, device="cuda").bfloat16()
    w = torch.ones(128, device="cuda").bfloat16()
    dy = torch.randn_like(x)

    def fn():
        Cu._C.gated_rmsnorm_fwd(x, z, w, 1e-6)
        Cu._C.gated_rmsnorm_bwd(dy, x, z, w, 1e-6)
    n = x.numel()
    return fn, 24.0 * n, 2.0 * n * 8  # fwd: x, z -> y; bwd: dy, x, z -> dx, dz


def op_dswiglu(a):
    """SwiGLU backward elementwise (`_C.dswiglu`): d(gate|up) from d(act) and the stored gate|up,
    rows = B x 2L, F = 17408"""
    from ..ops import cuda as Cu

    rows, F = a.B * 2 * a.L, 17408
    dact = torch.randn(rows, F, device="cuda").bfloat16()
    gu = torch.randn(rows, 2 * F, device="cuda").bfloat16()
    return (lambda: Cu._C.dswiglu(dact, gu)), 10.0 * rows * F, 2.0 * rows * F * 5


def op_gates(a):
    """GDN gates forward + backward (`_C.gdn_gates_fwd/bwd`): beta = sigmoid(b), g = -exp(A_log)
    softplus(a + dt_bias), rows = B x 2L, 48 heads"""
    from ..ops import cuda as Cu

    rows, H = a.B * 2 * a.L, 48
    av = torch.randn(rows, H, device="cuda").bfloat16()
    bv = torch.randn(rows, H, device="cuda").bfloat16()
    A_log = torch.randn(H, device="cuda")
    dt = torch.randn(H, device="cuda")
    dg, db = torch.randn(rows, H, device="cuda"), torch.randn(rows, H, device="cuda")

    def fn():
        Cu._C.gdn_gates_fwd(av, bv, A_log, dt)
        Cu._C.gdn_gates_bwd(dg, db, av, bv, A_log, dt)
    return fn, 30.0 * rows * H, rows * H * (2 * 2 + 4 * 2 + 4 * 2 + 2 * 2 * 2)


def op_decode(a):
    """decode confidence (softmax max probability + argmax over the vocab per row) and the
    threshold commit rule (`_C.confidence`, `_C.commit`): batch 32 x block 32 rows"""
    from ..ops import cuda as Cu

    Bd, T = 32, 32
    logits = torch.randn(Bd * T, a.vocab, device="cuda").bfloat16()
    conf = torch.zeros(Bd * T, device="cuda")
    pick = torch.zeros(Bd * T, dtype=torch.long, device="cuda")
    ids = torch.zeros(Bd, T, dtype=torch.long, device="cuda")
    masked = torch.ones(Bd, T, dtype=torch.bool, device="cuda")
    fw = torch.zeros(Bd, dtype=torch.int32, device="cuda")
    left = torch.zeros(Bd, dtype=torch.int32, device="cuda")

    def fn():
        masked.fill_(True)
        Cu._C.confidence(logits, conf, pick)
        Cu._C.commit(conf, pick, masked, ids, 0.9, 8, fw, left)
    return fn, 4.0 * logits.numel(), 2.0 * logits.numel()


def op_embed(a):
    """embedding rows forward + gradient scatter-add (`_C.embed_fwd`, `_C.embed_bwd_`): B x 2L ids
    into a [vocab, 5120] table"""
    from ..ops import cuda as Cu

    D = 5120
    table = torch.randn(a.vocab, D, device="cuda").bfloat16()
    ids = torch.randint(0, a.vocab, (a.B * 2 * a.L,), device="cuda")
    dh = torch.randn(ids.numel(), D, device="cuda").bfloat16()
    grad = torch.zeros(a.vocab, D, device="cuda")

    def fn():
        Cu._C.embed_fwd(ids, table)
        Cu._C.embed_bwd_(grad, ids, dh)
    return fn, 1.0 * ids.numel() * D, ids.numel() * D * (2 + 2 + 2 + 8)


def op_embed_sorted(a):
    """embedding-table gradient as sorted per-id sums straight into a bf16 [vocab, 5120] gradient
    (`_C.embed_bwd_sorted`, the one-rank untied path): --rows token rows (default B x 2L x 2, the
    two views of both streams), of which --run carry one id (the mask token fills about half of
    the noised rows, so its run is the longest one)"""
    from ..ops import cuda as Cu

    D, N = 5120, a.B * 4 * a.L if a.rows == 8192 else a.rows
    g = torch.Generator(device="cuda").manual_seed(0)
    ids = torch.randint(0, a.vocab - 1, (N,), device="cuda", generator=g)
    ids[: min(a.run, N)] = a.vocab - 1
    dh = torch.randn(N, D, device="cuda", generator=g).bfloat16()
    grad = torch.zeros(a.vocab, D, device="cuda", dtype=torch.bfloat16)
    sid, perm = torch.sort(ids, stable=True)

    def fn():
        Cu._C.embed_bwd_sorted(grad, sid, perm, dh)
    return fn, 1.0 * N * D, N * D * 2 + N * 16 + torch.unique(ids).numel() * D * 2


OPS = {"gemm": op_gemm, "swiglu": op_swiglu, "rmsnorm_bwd": op_rmsnorm_bwd, "gdn": op_gdn, "gdn_fwd": op_gdn_fwd, "attn": op_attn, "attn_fwd": op_attn_fwd, "ce": op_ce, "conv": op_conv, "rmsnorm": op_rmsnorm, "qknorm": op_qknorm, "gnorm": op_gnorm,
       "dswiglu": op_dswiglu, "gates": op_gates, "decode": op_decode, "embed": op_embed, "embed_sorted": op_embed_sorted,
       "adamw": op_adamw}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("op", choices=sorted(OPS))
    p.add_argument("--impl", default="native", choices=["native", "reference", "cublas"])
    p.add_argument("--M", type=int, default=8192)
    p.add_argument("--N", type=int, default=5120)
    p.add_argument("--K", type=int, default=5120)
    p.add_argument("--layout", default="nt", choices=["nt", "nn", "tn"], help="gemm operand majors")
    p.add_argument("--B", type=int, default=1)
    p.add_argument("--L", type=int, default=4096)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--rows", type=int, default=8192)
    p.add_argument("--D", type=int, default=5120)
    p.add_argument("--vocab", type=int, default=248320)
    p.add_argument("--run", type=int, default=8000, help="embed_sorted: rows that carry one id")
    p.add_argument("--n", type=int, default=400_000_000)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--sustain", type=float, default=0.0,
                   help="seconds: run the op back to back (no L2 flush) with the SM clocks sampled, "
                        "the rate under the power cap rather than a burst")
    a = p.parse_args(argv)
    sys.path.insert(0, ROOT)
    fn, flops, byts = OPS[a.op](a)
    clocks = None
    if a.sustain > 0:
        ms, clocks = sustained(fn, a.sustain)
    else:
        ms = timeit(fn, a.iters, a.warmup)
    bw, tf, src = peaks()
    s = ms / 1e3
    out = {"op": a.op, "impl": a.impl, "ms": round(ms, 4), "tflops": round(flops / s / 1e12, 2),
           "gbs": round(byts / s / 1e9, 1), "frac_bf16_peak": round(flops / s / tf, 3),
           "frac_hbm_peak": round(byts / s / bw, 3), "peaks": src,
           "shape": {k: getattr(a, k) for k in ("M", "N", "K", "layout", "B", "L", "block", "rows", "D", "vocab", "n")}}
    if clocks is not None:
        out["sustained_s"] = a.sustain
        out["clocks"] = clocks
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
