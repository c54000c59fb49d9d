"""Autograd-aware wrappers around the sm_100a kernels (``dllm_qwen38_b200._C``).

Each wrapper replaces one library path of the reference: the chunked delta rule
(`src/dllm_qwen38/gdn.py:48-123`) and its autograd backward, the GDN mixer's conv, gates and
gated norm (`gdn.py:212-233`), the masked attention (`blockdiff.py:178-182`, HF eager or SDPA over
a dense mask), the masked-row lm_head + CE (`objective.py:79-84`, `fsdp_train.py:618-623`) and
single-tensor AdamW (`fsdp_train.py:779`).

Conventions of the GEMM entry (``_C.gemm``): C[m, n] = sum_k A(m, k) B(n, k); A is K-major
([M, K]) or MN-major ([K, M]); B is K-major ([N, K]) or MN-major ([K, N]). With those two bits
the three GEMMs of a linear layer need no transposes:

    forward  y  = x  W^T : A = x  (K-major), B = W (K-major)
    dgrad    dx = dy W   : A = dy (K-major), B = W (MN-major, rows = out features)
    wgrad    dW = dy^T x : A = dy (MN-major), B = x (MN-major)
"""

from __future__ import annotations

import torch

from ._native import require as _require

_C = _require()  # `_C`, or the debug-bounds build `_C_dbg` under BDLLM_DEBUG_BOUNDS=1

EPI_BF16, EPI_F32, EPI_ADD_BF16, EPI_ACC_F32, EPI_SWIGLU = 0, 1, 2, 3, 4

# ops that have no sm_100a kernel yet; on CUDA tensors they run the torch reference and are
# recorded as 'torch-cuda' by ops.last_impl()
TORCH_ON_CUDA: set = set()


# native kernel launches issued through this module (benchmarks report the count of a region)
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def _c2(t: torch.Tensor) -> torch.Tensor:
    """Flatten to 2-D with a unit inner stride (no copy when already so)."""
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1 or (t2.stride(0) % 8) or (t2.data_ptr() % 16):
        t2 = t2.contiguous()
    return t2


_NUM_SMS = [0]

# set by the sharded engine while a layer's weights are being gathered: a callable
# (a, w, out, epi, gu) -> bool that runs the fused all-gather -> GEMM when w is one of the layer's
# weights not gathered yet
AG_HOOK = [None]


def _splits(M: int, N: int, K: int) -> int:
    """k-splits for a skinny bf16 GEMM whose output tiles cannot fill the GPU (1 = no split)."""
    if M > 256 or K < 2048 or N % 4:
        return 1
    if not _NUM_SMS[0]:
        _NUM_SMS[0] = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    tiles = ((M + 127) // 128) * ((N + 255) // 256)
    if 2 * tiles > _NUM_SMS[0]:
        return 1
    return max(1, min((K + 63) // 64 // 4, _NUM_SMS[0] // tiles))  # one wave of (tile, split) items


def gemm_nt(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, out_dtype=torch.bfloat16,
            residual: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """out[M, N] = a[M, K] @ b[N, K]^T (both K-major). residual: out = a b^T + residual (bf16).
    accumulate: fp32 out += a b^T. Skinny bf16 problems (decode) run split-K."""
    a2, b2 = _c2(a), _c2(b)
    M, K = a2.shape
    N = b2.shape[0]
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=out_dtype)
    if AG_HOOK[0] is not None and residual is None and not accumulate and out.dtype == torch.bfloat16:
        if AG_HOOK[0](a2, b2, out, EPI_BF16, None):  # this weight is gathered by this GEMM (fused)
            _count()
            return out
    S = _splits(M, N, K) if (out.dtype == torch.bfloat16 and not accumulate) else 1
    if S > 1:
        ws = torch.empty(S * M * N, device=a.device, dtype=torch.float32)
        _C.gemm_splitk(a2, b2, out, ws, S, _c2(residual) if residual is not None else None)
        _count(2)
        return out
    if accumulate:
        epi = EPI_ACC_F32
    elif residual is not None:
        epi = EPI_ADD_BF16
    else:
        epi = EPI_F32 if out.dtype == torch.float32 else EPI_BF16
    r = _c2(residual) if residual is not None else None
    _C.gemm(a2, False, a2.stride(0), b2, False, b2.stride(0), M, N, K, out, out.stride(0), epi,
            r, r.stride(0) if r is not None else 0)
    _count()
    return out


def gemm_nn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, out_dtype=torch.bfloat16,
            residual: torch.Tensor | None = None, alpha: float = 1.0,
            alpha_t: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = a[M, K] @ b[K, N] (b MN-major: row-major [K, N]). alpha_t: a one-element fp32
    device tensor that also scales the product (read by the epilogue: no host synchronisation)."""
    a2, b2 = _c2(a), _c2(b)
    M, K = a2.shape
    N = b2.shape[1]
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=out_dtype)
    epi = EPI_ADD_BF16 if residual is not None else (EPI_F32 if out.dtype == torch.float32 else EPI_BF16)
    r = _c2(residual) if residual is not None else None
    _C.gemm(a2, False, a2.stride(0), b2, True, b2.stride(0), M, N, K, out, out.stride(0), epi,
            r, r.stride(0) if r is not None else 0, None, 256, alpha, alpha_t)
    _count()
    return out


def gemm_tn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, out_dtype=torch.float32,
            accumulate: bool = False, alpha: float = 1.0, alpha_t: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = a[K, M]^T @ b[K, N] (both MN-major) -- the weight-gradient GEMM."""
    a2, b2 = _c2(a), _c2(b)
    K, M = a2.shape
    N = b2.shape[1]
    if out is None:
        out = torch.zeros(M, N, device=a.device, dtype=out_dtype) if accumulate else torch.empty(
            M, N, device=a.device, dtype=out_dtype)
    epi = EPI_ACC_F32 if accumulate else (EPI_F32 if out.dtype == torch.float32 else EPI_BF16)
    _C.gemm(a2, True, a2.stride(0), b2, True, b2.stride(0), M, N, K, out, out.stride(0), epi, None, 0, None, 256,
            alpha, alpha_t)
    _count()
    return out


def wgrad(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor, alpha_t: torch.Tensor | None = None):
    """Weight gradient (alpha_t *) dy^T x for leaf weight `w`. When `w.grad` is a preset bf16
    buffer (the sharded engine's flat gradient views) the GEMM epilogue adds into it in place (one
    rounding, no fp32 temporary) and None is returned; otherwise the gradient tensor."""
    g = w.grad if (w.is_leaf and w.requires_grad) else None
    if g is not None and g.dtype == torch.bfloat16 and g.shape == w.shape and g.stride(-1) == 1 \
            and g.dim() == 2 and g.stride(0) % 8 == 0 and g.data_ptr() % 16 == 0:
        K, M = dy2.shape
        N = x2.shape[1]
        _C.gemm(dy2, True, dy2.stride(0), x2, True, x2.stride(0), M, N, K, g, g.stride(0), EPI_ADD_BF16, g,
                g.stride(0), None, 256, 1.0, alpha_t)
        _count()
        return None
    if w.dtype == torch.bfloat16:  # bf16 result straight from the epilogue
        return gemm_tn(dy2, x2, out_dtype=torch.bfloat16, alpha_t=alpha_t)
    return gemm_tn(dy2, x2, out_dtype=torch.float32, alpha_t=alpha_t).to(w.dtype)


def gemm_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, F: int, store_gu: bool):
    """act[M, F] = silu(x Wg^T) * (x Wu^T) with w_gate_up = [Wg; Wu] ([2F, K], contiguous rows).
    Returns (act, gu) where gu [M, 2F] holds the bf16 (gate | up) when store_gu."""
    x2 = _c2(x)
    M, K = x2.shape
    act = torch.empty(M, F, device=x.device, dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * F, device=x.device, dtype=torch.bfloat16) if store_gu else None
    if AG_HOOK[0] is not None and AG_HOOK[0](x2, w_gate_up, act, EPI_SWIGLU, gu):
        _count()
        return act, gu
    _C.gemm(x2, False, x2.stride(0), w_gate_up, False, w_gate_up.stride(0), M, F, K, act, act.stride(0), EPI_SWIGLU,
            None, 0, gu)
    _count()
    return act, gu


# ----------------------------------------------------------------------------- linear


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        saved = ActStore.take() if ActStore.gemms else None
        if saved is not None:
            return saved[0]
        y = gemm_nt(x, w).reshape(*x.shape[:-1], w.shape[0])
        if ActStore.gemms:
            ActStore.put(y)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy2 = _c2(dy.to(torch.bfloat16))
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm_nn(dy2, w).reshape(x.shape)
        if ctx.needs_input_grad[1]:
            dw = wgrad(dy2, _c2(x), w)
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise TypeError(f"native linear runs bf16 operands (got {x.dtype}, {w.dtype})")
    return _Linear.apply(x, w)


# ----------------------------------------------------------------------------- norms


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        w1 = 1.0 + w.float()
        ctx.save_for_backward(x, w1)
        ctx.eps, ctx.wdtype = eps, w.dtype
        _count()
        return _C.rmsnorm_fwd(x, w1, eps)

    @staticmethod
    def backward(ctx, dy):
        x, w1 = ctx.saved_tensors
        dx, dw = _C.rmsnorm_bwd(dy, x, w1, ctx.eps)
        _count(2)
        return dx, dw.to(ctx.wdtype), None


def rmsnorm(x, w, eps):
    return _RMSNorm.apply(x, w, eps)


class _GatedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, z, w, eps):
        ctx.save_for_backward(x, z, w)
        ctx.eps = eps
        _count()
        return _C.gated_rmsnorm_fwd(x, z, w, eps)

    @staticmethod
    def backward(ctx, dy):
        x, z, w = ctx.saved_tensors
        dx, dz, dw = _C.gated_rmsnorm_bwd(dy, x, z, w, ctx.eps)
        _count(2)
        return dx, dz, dw.to(w.dtype), None


def gated_rmsnorm(x, z, w, eps):
    return _GatedRMSNorm.apply(x, z, w, eps)


class _OutputGate(torch.autograd.Function):
    """o * sigmoid(gate), the gate read in place from the q|gate projection (one kernel each way,
    sigmoid recomputed in the backward)."""

    @staticmethod
    def forward(ctx, o, gate):
        ctx.save_for_backward(o, gate)
        _count()
        return _C.out_gate_fwd(o, gate)

    @staticmethod
    def backward(ctx, dy):
        o, gate = ctx.saved_tensors
        do, dg = _C.out_gate_bwd(dy, o, gate)
        _count()
        return do.view(o.shape), dg.view(gate.shape)


def output_gate(o, gate):
    return _OutputGate.apply(o, gate)


class _QKNormRope(torch.autograd.Function):
    """q/k [B, T2, H, Dh] strided views (q is a slice of the q|gate projection)."""

    @staticmethod
    def forward(ctx, q, k, wq, wk, eps, cos, sin):
        wq1, wk1 = 1.0 + wq.float(), 1.0 + wk.float()
        ctx.save_for_backward(q, k, wq1, wk1, cos, sin)
        ctx.eps, ctx.dt = eps, wq.dtype
        _count(2)
        return _C.qk_norm_rope_fwd(q, wq1, cos, sin, eps), _C.qk_norm_rope_fwd(k, wk1, cos, sin, eps)

    @staticmethod
    def backward(ctx, dq, dk):
        q, k, wq1, wk1, cos, sin = ctx.saved_tensors
        dqs, dwq = _C.qk_norm_rope_bwd(dq, q, wq1, cos, sin, ctx.eps)
        dks, dwk = _C.qk_norm_rope_bwd(dk, k, wk1, cos, sin, ctx.eps)
        _count(4)
        return dqs, dks, dwq.to(ctx.dt), dwk.to(ctx.dt), None, None, None


def qk_norm_rope(q, k, wq, wk, eps, cos, sin):
    return _QKNormRope.apply(q, k, wq, wk, eps, cos, sin)


# ----------------------------------------------------------------------------- MLP


class _SwiGLUMLP(torch.autograd.Function):
    """down(silu(x Wg^T) * (x Wu^T)) with w_gu = [Wg; Wu]: one GEMM for gate|up with the SwiGLU
    epilogue (keeping the bf16 gate|up for backward), one for down. Backward: d(act) = dy Wd,
    the SwiGLU derivative kernel, then dx = dgu [Wg; Wu] and the two weight-gradient GEMMs."""

    @staticmethod
    def forward(ctx, x, w_gu, w_down):
        F = w_gu.shape[0] // 2
        saved = ActStore.take() if ActStore.gemms else None
        if saved is not None:
            y, act, gu = saved
            if act is None:  # kept without the activation: rebuilt from the kept bf16 gate|up
                act = _C.swiglu_act(gu)
                _count()
        else:
            # the saving forward (no grad) keeps gate|up for the backward it will serve, and, when
            # memory is short, not the activation, which one element-wise pass rebuilds from it
            need = any(ctx.needs_input_grad) or (ActStore.gemms and ActStore.mode == "save")
            act, gu = gemm_swiglu(x, w_gu, F, store_gu=need)
            y = gemm_nt(act, w_down).reshape(*x.shape[:-1], w_down.shape[0])
            if ActStore.gemms:
                ActStore.put(y, act if (ActStore.keep_act or gu is None) else None, gu)
        ctx.save_for_backward(x, w_gu, w_down, act, gu)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w_gu, w_down, act, gu = ctx.saved_tensors
        dy2 = _c2(dy.to(torch.bfloat16))
        x2 = _c2(x)
        dact = gemm_nn(dy2, w_down)
        dgu = _C.dswiglu(dact, gu)
        _count()
        dx = gemm_nn(dgu, w_gu).reshape(x.shape)
        dw_gu = wgrad(dgu, x2, w_gu) if ctx.needs_input_grad[1] else None
        dw_down = wgrad(dy2, act, w_down) if ctx.needs_input_grad[2] else None
        return dx, dw_gu, dw_down


def swiglu_mlp(x, w_gate, w_up, w_down):
    return _SwiGLUMLP.apply(x, torch.cat([w_gate, w_up], 0), w_down)


def swiglu_mlp_fused(x, w_gu, w_down):
    return _SwiGLUMLP.apply(x, w_gu, w_down)


# ----------------------------------------------------------------------------- conv

_CONV_MODE = {"fork": 0, "no-prefix": 1, "concat": 2}


class _Conv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, raw, w, L, block, mode):
        ctx.save_for_backward(raw, w)
        ctx.cfg = (L, block, _CONV_MODE[mode])
        _count()
        return _C.conv_fwd(raw, w, L, block, _CONV_MODE[mode])

    @staticmethod
    def backward(ctx, dy):
        raw, w = ctx.saved_tensors
        draw, dw = _C.conv_bwd(dy, raw, w, *ctx.cfg)
        _count(4)
        return draw, dw.to(w.dtype), None, None, None


def conv_blockdiff(raw, w, L, block, mode):
    if raw.stride(-1) != 1 or raw.stride(1) % 8:
        raw = raw.contiguous()
    return _Conv.apply(raw, w, L, block, mode)


# ----------------------------------------------------------------------------- loss


class _MaskedCE(torch.autograd.Function):
    """sum_rows CE(h W^T, t). Forward: logits by GEMM (bf16, [n, V]), one row kernel writes the
    per-row loss and overwrites the logits with (softmax - onehot), which the backward keeps as
    dlogits (n x V bf16: 2 GiB at n = 4096, V = 248,320; the cost of not recomputing the logits
    GEMM). Backward: dh = g * dlogits W, dW = g * dlogits^T h; g stays a device scalar that the
    GEMM epilogues read, and dW is added in place into a preset bf16 gradient when there is one."""

    @staticmethod
    def forward(ctx, h, w, tgt):
        h2 = _c2(h)
        logits = gemm_nt(h2, w)
        loss = _C.ce_rows_(logits, tgt)
        _count()
        ctx.save_for_backward(h2, w, logits)
        return loss.sum()

    @staticmethod
    def backward(ctx, g):
        h2, w, dlogits = ctx.saved_tensors
        # the upstream scale stays on the device: both GEMM epilogues read it (no host sync)
        gt = g.detach().float().reshape(1).contiguous()
        dh = gemm_nn(dlogits, w, alpha_t=gt) if ctx.needs_input_grad[0] else None
        # dW accumulates into a preset bf16 gradient buffer in place when the engine set one
        dw = wgrad(dlogits, h2, w, alpha_t=gt) if ctx.needs_input_grad[1] else None
        return dh, dw, None


def masked_ce_sum(hidden, w, targets):
    return _MaskedCE.apply(hidden, w, targets)


# ----------------------------------------------------------------------------- GDN


class ActStore:
    """Selective activation saving across activation checkpointing: in "save" mode the GDN core
    and attention forwards keep their outputs (and the state snapshots / log-sum-exps their
    backward needs) per layer; in "reuse" mode the recomputation inside the backward returns them
    instead of running those kernels again. Keyed by layer, consumed in call order. With `gemms`
    set, the projection GEMMs and the SwiGLU MLP keep their outputs too (the MLP also its gate|up
    and activation), so the recomputation runs only the cheap elementwise / norm kernels."""

    mode = None
    gemms = False
    keep_act = False  # the MLP keeps its activation too (else the backward rebuilds it from gate|up)
    key = None
    data: dict = {}
    pos = 0

    @classmethod
    def begin(cls, mode: str, key) -> None:
        cls.mode, cls.key, cls.pos = mode, key, 0
        if mode == "save":
            cls.data[key] = []

    @classmethod
    def end(cls) -> None:
        if cls.mode == "reuse":
            cls.data.pop(cls.key, None)
        cls.mode = cls.key = None

    @classmethod
    def take(cls):
        if cls.mode != "reuse":
            return None
        saved = cls.data.get(cls.key)
        if saved is None or cls.pos >= len(saved):
            return None
        cls.pos += 1
        return saved[cls.pos - 1]

    @classmethod
    def put(cls, *ts) -> None:
        if cls.mode == "save":
            cls.data[cls.key].append(ts)

    @classmethod
    def clear(cls) -> None:
        cls.data.clear()
        cls.mode = cls.key = None


class _GDNCore(torch.autograd.Function):
    """State-fork chunked gated delta rule over the [B, 2L] layout (chunk = block). q, k
    [B, 2L, Hk, Dk] and v [B, 2L, Hv, Dv] may be strided views of the conv output; g, beta
    [B, 2L, Hv]. Saves the fp32 chunk-entry states for backward."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, L, block, concat):
        gf = g.float().contiguous()
        bf = beta.float().contiguous()
        saved = ActStore.take()
        if saved is not None:
            o, S_in = saved
        else:
            if _C.gdn_tc_eligible(q, k, v, L, block, concat):  # tcgen05 / TMEM / TMA forward
                o, S_in = _C.gdn_fwd_tc(q, k, v, gf, bf, L)
                _count(2)
            else:
                o, S_in, _ = _C.gdn_fwd(q, k, v, gf, bf, L, block, concat)
                _count(3)
            ActStore.put(o, S_in)
        ctx.save_for_backward(q, k, v, gf, bf, S_in)
        ctx.cfg = (L, block, concat)
        ctx.dtypes = (g.dtype, beta.dtype)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, gf, bf, S_in = ctx.saved_tensors
        L, block, concat = ctx.cfg
        dq, dk, dv, dg, db = _C.gdn_bwd(do, q, k, v, gf, bf, S_in, L, block, concat)
        _count(3 if concat else 4)
        Hk, Hv = q.shape[2], v.shape[2]
        if Hv != Hk:  # the kernel returns per-v-head gradients; sum each repeat group (one pass each)
            dq = _C.group_sum(dq, Hk)
            dk = _C.group_sum(dk, Hk)
            _count(2)
        return dq, dk, dv, dg.to(ctx.dtypes[0]), db.to(ctx.dtypes[1]), None, None, None


class _Gates(torch.autograd.Function):
    """beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias), both fp32 (a, b bf16 views)."""

    @staticmethod
    def forward(ctx, a, b, A_log, dt_bias):
        g, beta = _C.gdn_gates_fwd(a, b, A_log, dt_bias)
        ctx.save_for_backward(a, b, A_log, dt_bias)
        _count()
        return g, beta

    @staticmethod
    def backward(ctx, dg, dbeta):
        a, b, A_log, dt_bias = ctx.saved_tensors
        if dg is None:
            dg = torch.zeros(a.shape, device=a.device, dtype=torch.float32)
        if dbeta is None:
            dbeta = torch.zeros(a.shape, device=a.device, dtype=torch.float32)
        da, db, dA, ddt = _C.gdn_gates_bwd(dg, dbeta, a, b, A_log, dt_bias)
        _count()
        return da, db, dA.to(A_log.dtype), ddt.to(dt_bias.dtype)


def gdn_gates(a, b, A_log, dt_bias):
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        a, b = a.to(torch.bfloat16), b.to(torch.bfloat16)
    return _Gates.apply(a, b, A_log, dt_bias)


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, table):
        ids_c = ids.contiguous()
        ctx.save_for_backward(ids_c)
        ctx.shape, ctx.dt = table.shape, table.dtype
        _count()
        return _C.embed_fwd(ids_c, table.contiguous())

    @staticmethod
    def backward(ctx, dh):
        (ids,) = ctx.saved_tensors
        grad = torch.zeros(ctx.shape, device=dh.device, dtype=torch.float32)
        _C.embed_bwd_(grad, ids, dh)
        _count()
        return None, grad.to(ctx.dt)


def embedding(ids, table):
    if table.dtype != torch.bfloat16:
        raise TypeError("native embedding: bf16 table")
    return _Embedding.apply(ids, table)


class _GDNCoreBlocks(torch.autograd.Function):
    """The state fork for blocks of more than 32 tokens (the kernels chunk at 32): the clean stream
    x_0 is one causal run chunked at 32; every noised block of x_t is an independent run that
    starts from the clean state at its block's start. Backward: the noised runs return the
    gradient of their initial states, which is injected into the clean run's reverse recurrence at
    the block-start chunks. q, k [B, 2L, Hk, Dk], v [B, 2L, Hv, Dv]; g, beta [B, 2L, Hv]."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, L, block):
        B = q.shape[0]
        C, nb = 32, L // block
        cpb = block // C
        gf, bf = g.float(), beta.float()
        clean = [t[:, L:].contiguous() for t in (q, k, v, gf, bf)]
        o0, S0_in, _ = _C.gdn_fwd(*clean, L // 2, C, True)  # x_0: one causal run of L tokens
        rows = [t[:, :L].reshape(B * nb, block, *t.shape[2:]).contiguous() for t in (q, k, v, gf, bf)]
        S0 = S0_in[:, ::cpb].reshape(B * nb, *S0_in.shape[2:]).contiguous()  # the fork states
        ot, St_in = _C.gdn_fwd_rows(*rows, S0, C)
        _count(6)
        ctx.save_for_backward(*clean, S0_in, *rows, St_in)
        ctx.cfg = (B, L, block, C, nb, cpb)
        ctx.dtypes = (g.dtype, beta.dtype)
        return torch.cat([ot.reshape(B, L, *ot.shape[2:]), o0], 1)

    @staticmethod
    def backward(ctx, do):
        saved = ctx.saved_tensors
        clean, S0_in, rows, St_in = saved[:5], saved[5], saved[6:11], saved[11]
        B, L, block, C, nb, cpb = ctx.cfg
        do = do.to(torch.bfloat16)
        dot = do[:, :L].reshape(B * nb, block, *do.shape[2:]).contiguous()
        dqt, dkt, dvt, dgt, dbt, dS0 = _C.gdn_bwd_rows(dot, *rows, St_in, C, None, True)
        inj = torch.zeros_like(S0_in)
        inj[:, ::cpb] = dS0.reshape(B, nb, *dS0.shape[1:])
        dq0, dk0, dv0, dg0, db0 = _C.gdn_bwd_rows(do[:, L:].contiguous(), *clean, S0_in, C, inj, False)
        _count(8)

        def cat(a, b):
            return torch.cat([a.reshape(B, L, *a.shape[2:]), b], 1)

        dq, dk, dv, dg, db = cat(dqt, dq0), cat(dkt, dk0), cat(dvt, dv0), cat(dgt, dg0), cat(dbt, db0)
        Hk, Hv = clean[0].shape[2], clean[2].shape[2]
        if Hv != Hk:  # per-v-head gradients: sum each repeat group (one pass each)
            dq = _C.group_sum(dq.to(torch.bfloat16).contiguous(), Hk).to(clean[0].dtype)
            dk = _C.group_sum(dk.to(torch.bfloat16).contiguous(), Hk).to(clean[1].dtype)
            _count(2)
        return dq, dk, dv, dg.to(ctx.dtypes[0]), db.to(ctx.dtypes[1]), None, None


def gdn_core_blockdiff(q, k, v, g, beta, L, block, chunk, mode):
    """chunk is the host reference's chunking. The kernels chunk at the block when it is <= 32;
    larger blocks (multiples of 32) run the clean stream and the noised blocks as separate runs
    chunked at 32 (`_GDNCoreBlocks`); the concat fault is one causal run at any block."""
    del chunk
    if L % block:
        raise ValueError(f"native GDN needs the block to divide L (got block={block}, L={L})")
    if mode == "concat":
        return _GDNCore.apply(q, k, v, g, beta, L, block if block <= 32 else 32, True)
    if block <= 32:
        return _GDNCore.apply(q, k, v, g, beta, L, block, False)
    if block % 32:
        raise ValueError(f"native GDN: blocks above 32 must be multiples of 32 (got {block})")
    return _GDNCoreBlocks.apply(q, k, v, g, beta, L, block)


# ----------------------------------------------------------------------------- attention


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, L, block, scale, leak):
        saved = ActStore.take()
        if saved is not None:
            o, lse = saved
        else:
            o, lse = _C.attn_fwd(q, k, v, L, block, scale, leak)
            _count()
            ActStore.put(o, lse)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.cfg = (L, block, scale, leak)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _C.attn_bwd(do, q, k, v, o, lse, *ctx.cfg)
        _count(2)
        return dq, dk, dv, None, None, None, None


def _rows16(t):
    ok = t.stride(-1) == 1 and t.stride(2) == t.shape[3] and t.stride(1) % 8 == 0 and t.data_ptr() % 16 == 0 \
        and t.stride(0) == t.shape[1] * t.stride(1)
    return t if ok else t.contiguous()


def attention_blockdiff(q, k, v, L, block, scale, leak_xt_prefix=False):
    """q [B, 2L, Hq, D], k/v [B, 2L, Hk, D] (strided token rows allowed) -> o [B, 2L, Hq, D]."""
    return _Attention.apply(_rows16(q), _rows16(k), _rows16(v), L, block, float(scale), bool(leak_xt_prefix))


def adamw_step(w, p, g, m, v, lr, b1, b2, eps, wd, coef, bc1, bc2):
    _C.adamw_step(w, p, g.contiguous(), m, v, lr, b1, b2, eps, wd, coef, None, bc1, bc2)
    _count()


def adamw_flat(w, p, g, m, v, lr, b1, b2, eps, wd, coef, bc1, bc2):
    dev_coef = coef.float().reshape(1) if torch.is_tensor(coef) else None
    _C.adamw_step(w, p, g, m, v, lr, b1, b2, eps, wd, 1.0 if dev_coef is not None else float(coef), dev_coef,
                  bc1, bc2)
    _count()


def sumsq_(x, sq, dst=None):
    _C.sumsq_(x, sq, dst)
    _count()


def error_word(reset: bool = False) -> int:
    return int(_C.read_error_word(reset))


def check_errors() -> None:
    e = error_word(reset=True)
    if e:
        raise RuntimeError(f"a bounded device wait expired (error code {e}); see csrc/common.cuh")
