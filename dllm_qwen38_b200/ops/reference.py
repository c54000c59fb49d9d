"""Plain PyTorch implementations of every op the model uses.

These are the CPU path and the numerics oracle for the sm_100a kernels in ``csrc/``. They are
written for clarity, differentiate through autograd, and compute in fp32 wherever the
reference does (`gdn.py:76-84` casts the delta rule to fp32; HF RMSNorm computes in fp32,
HF modeling_qwen3_5.py:711-728).

Layout convention used by the whole framework: both diffusion streams live in ONE tensor
``[B, 2L, ...]`` -- positions ``[0, L)`` are the noised stream x_t and ``[L, 2L)`` the clean
stream x_0 (the order of the reference's ``cat([x_t, x_0])``, `blockdiff.py:179-182`).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

# --------------------------------------------------------------------------- norms


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3.5 RMSNorm with the (1 + w) parameterisation, fp32 math (HF:711-728)."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())
    return y.to(x.dtype)


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """(w * rmsnorm(x)) * silu(z) over the last dim (HF:175-190)."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = w * y.to(x.dtype)
    y = y * F.silu(z.float())
    return y.to(x.dtype)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


# --------------------------------------------------------------------------- dense


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return x @ w.t()


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate) * up


# --------------------------------------------------------------------------- RoPE


def rope_cos_sin(positions: torch.Tensor, rotary_dim: int, theta: float, dtype, device):
    """cos/sin [T, rotary_dim] for text positions (all three MRoPE rows equal -> plain RoPE,
    HF:85-172): inv_freq over the rotary dims, emb = cat(freqs, freqs)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.int64, device=device).float() / rotary_dim))
    freqs = positions.to(device=device, dtype=torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., T, H, Dh]; cos/sin [T, R] with R <= Dh; rotate_half on the first R dims."""
    R = cos.shape[-1]
    c, s = cos[:, None, :], sin[:, None, :]
    xr, xp = x[..., :R], x[..., R:]
    x1, x2 = xr[..., : R // 2], xr[..., R // 2 :]
    rot = torch.cat([-x2, x1], -1)
    return torch.cat([xr * c + rot * s, xp], -1)


# --------------------------------------------------------------------------- masks


def block_causal_allowed(T: int, block: int, device) -> torch.Tensor:
    idx = torch.arange(T, device=device) // block
    return idx[None, :] <= idx[:, None]


def complementary_allowed(L: int, block: int, device, leak_xt_prefix: bool = False) -> torch.Tensor:
    """[2L, 2L] bool over cat([x_t, x_0]) (`blockdiff.py:50-66`):
    x_t i sees x_t j iff same block (M_BD); x_t i sees x_0 j iff block(j) < block(i) (M_OBC);
    x_0 i sees x_0 j iff block(j) <= block(i) (M_BC); x_0 never sees x_t.
    leak_xt_prefix is the deliberate fault: x_t also sees earlier x_t blocks."""
    idx = torch.arange(L, device=device) // block
    bi, bj = idx[:, None], idx[None, :]
    tt = (bj <= bi) if leak_xt_prefix else (bj == bi)
    tc = bj < bi
    cc = bj <= bi
    ct = torch.zeros(L, L, dtype=torch.bool, device=device)
    return torch.cat([torch.cat([tt, tc], 1), torch.cat([ct, cc], 1)], 0)


def additive_mask(allowed: torch.Tensor, dtype) -> torch.Tensor:
    return torch.zeros(allowed.shape, dtype=dtype, device=allowed.device).masked_fill(~allowed, torch.finfo(dtype).min)


# --------------------------------------------------------------------------- attention


def attention(q, k, v, allowed: torch.Tensor, scale: float) -> torch.Tensor:
    """Softmax attention with GQA. q [B, T, Hq, Dh], k/v [B, T, Hk, Dh]; allowed [T, T] bool.
    Softmax in fp32 (HF eager, HF:594-617). Returns [B, T, Hq, Dh]."""
    Hq, Hk = q.shape[2], k.shape[2]
    rep = Hq // Hk
    qh = q.transpose(1, 2).float()
    kh = k.transpose(1, 2).float().repeat_interleave(rep, 1)
    vh = v.transpose(1, 2).float().repeat_interleave(rep, 1)
    s = (qh @ kh.transpose(-1, -2)) * scale
    s = s.masked_fill(~allowed, float("-inf"))
    p = torch.softmax(s, -1)
    p = torch.nan_to_num(p, nan=0.0)  # fully masked rows (none in the contracts used here)
    o = p @ vh
    return o.transpose(1, 2).to(q.dtype)


# --------------------------------------------------------------------------- conv


CONV_FORK, CONV_NOPREFIX, CONV_CONCAT = "fork", "no-prefix", "concat"


def causal_conv_silu(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Depthwise causal conv + SiLU over one stream. x [B, T, C], w [C, K]."""
    K = w.shape[1]
    xt = F.pad(x.transpose(1, 2), (K - 1, 0))
    y = F.conv1d(xt, w[:, None, :].to(x.dtype), groups=w.shape[0])
    return F.silu(y).transpose(1, 2)


def conv_blockdiff(raw: torch.Tensor, w: torch.Tensor, L: int, block: int, mode: str = CONV_FORK) -> torch.Tensor:
    """Short causal conv + SiLU for both streams in the [B, 2L, C] layout.

    x_0 (positions L..2L): plain causal conv from a zero start.
    x_t (positions 0..L), mode "fork": token p of block k reads taps at p-j; taps inside block k
      come from x_t, taps before k*block come from the CLEAN stream (the state fork's conv
      prefix, `blockdiff.py:167-173`), zeros before position 0.
    mode "no-prefix": taps before k*block read zero (the no-conv-prefix fault).
    mode "concat": one causal conv over the 2L sequence (the concat-causal-gdn fault).
    """
    B, T2, C = raw.shape
    assert T2 == 2 * L
    K = w.shape[1]
    if mode == CONV_CONCAT:
        return causal_conv_silu(raw, w)
    xt, x0 = raw[:, :L], raw[:, L:]
    y0 = causal_conv_silu(x0, w)
    nb = L // block
    km1 = K - 1
    rows = xt.reshape(B, nb, block, C)
    if mode == CONV_FORK:
        padded = torch.cat([x0.new_zeros(B, km1, C), x0], 1)  # zero pad = sequence start
        # prefix of block k = clean positions [k*block-km1, k*block) -> padded[k*block : k*block+km1]
        idx = torch.arange(nb, device=raw.device)[:, None] * block + torch.arange(km1, device=raw.device)[None, :]
        prefix = padded[:, idx.reshape(-1)].reshape(B, nb, km1, C)
    elif mode == CONV_NOPREFIX:
        prefix = rows.new_zeros(B, nb, km1, C)
    else:
        raise ValueError(mode)
    seq = torch.cat([prefix, rows], 2).reshape(B * nb, km1 + block, C)
    xpad = seq.transpose(1, 2)
    y = F.conv1d(xpad, w[:, None, :].to(raw.dtype), groups=C)
    yt = F.silu(y).transpose(1, 2).reshape(B, L, C)
    return torch.cat([yt, y0], 1)


# --------------------------------------------------------------------------- GDN


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """beta = sigmoid(b); g = -exp(A_log) * softplus(a + dt_bias) in fp32 (`gdn.py:225-226`)."""
    beta = b.sigmoid()
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, beta


def chunk_gated_delta_rule(q, k, v, g, beta, chunk: int, initial_state=None, state_every: int | None = None,
                           l2_qk: bool = True):
    """Chunked gated delta rule in fp32, vectorised over chunks; only the state recurrence loops.

    q, k: [N, T, H, Dk]; v: [N, T, H, Dv]; g, beta: [N, T, H]; initial_state [N, H, Dk, Dv] or None.
    Returns (o [N, T, H, Dv] in v.dtype, states [N, T/state_every, H, Dk, Dv] fp32 or None), where
    states[:, i] is the state after tokens < (i+1)*state_every. state_every must divide the chunk
    or be a multiple of it. Same math as `gdn.py:48-123` (the UT transform solved exactly).
    """
    dt = v.dtype
    N, T, H, Dk = k.shape
    Dv = v.shape[-1]
    if T % chunk:
        raise ValueError(f"T={T} not a multiple of chunk={chunk}")
    q, k, v, g, beta = (x.float() for x in (q, k, v, g, beta))
    if l2_qk:
        q, k = l2norm(q), l2norm(k)
    q = q * Dk ** -0.5
    nc = T // chunk
    # [N, H, nc, C, D]
    q, k, v = (x.transpose(1, 2).reshape(N, H, nc, chunk, -1) for x in (q, k, v))
    g = g.transpose(1, 2).reshape(N, H, nc, chunk)
    beta = beta.transpose(1, 2).reshape(N, H, nc, chunk)
    gam = g.cumsum(-1)
    tri_incl = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril()
    diff = gam[..., :, None] - gam[..., None, :]
    decay = torch.where(tri_incl, diff, torch.full_like(diff, float("-inf"))).exp()  # Gamma incl diag
    kb = k * beta[..., None]
    A = (kb @ k.transpose(-1, -2)) * decay
    A = torch.tril(A, -1)  # strict lower
    eye = torch.eye(chunk, device=q.device, dtype=q.dtype)
    Lmat = eye + A
    U = torch.linalg.solve_triangular(Lmat, v * beta[..., None], upper=False, unitriangular=True)
    W = torch.linalg.solve_triangular(Lmat, kb * gam.exp()[..., None], upper=False, unitriangular=True)
    qk = (q @ k.transpose(-1, -2)) * decay
    qg = q * gam.exp()[..., None]
    kd = k * (gam[..., -1:] - gam).exp()[..., None]
    cdec = gam[..., -1].exp()
    S = q.new_zeros(N, H, Dk, Dv) if initial_state is None else initial_state.float()
    outs, states = [], []
    if state_every is not None and state_every < chunk:
        if chunk % state_every:
            raise ValueError("state_every must divide chunk")
        sub = chunk // state_every
    else:
        sub = 1
    every_chunks = 1 if (state_every is None or state_every <= chunk) else state_every // chunk
    if state_every is not None and state_every > chunk and state_every % chunk:
        raise ValueError("state_every must be a multiple of chunk")
    for i in range(nc):
        vn = U[:, :, i] - W[:, :, i] @ S
        outs.append(qg[:, :, i] @ S + qk[:, :, i] @ vn)
        if state_every is not None and sub > 1:
            # mid-chunk snapshots: the state after the first j*state_every tokens of this chunk
            for j in range(1, sub):
                e = j * state_every
                gi = gam[:, :, i]
                kdj = k[:, :, i, :e] * (gi[..., e - 1 : e] - gi[..., :e]).exp()[..., None]
                states.append(S * gi[..., e - 1].exp()[..., None, None] + kdj.transpose(-1, -2) @ vn[:, :, :e])
        S = S * cdec[:, :, i, None, None] + kd[:, :, i].transpose(-1, -2) @ vn
        if state_every is not None and (i + 1) % every_chunks == 0:
            states.append(S)
    o = torch.stack(outs, 2).reshape(N, H, T, Dv).transpose(1, 2).to(dt)
    st = torch.stack(states, 1) if state_every is not None else None
    return o, st


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, l2_qk: bool = True):
    """Token-by-token gated delta rule (the decode form, HF:314-353): the independent ground truth.
    Shapes as chunk_gated_delta_rule. Returns (o, final_state)."""
    dt = v.dtype
    N, T, H, Dk = k.shape
    q, k, v, g, beta = (x.float() for x in (q, k, v, g, beta))
    if l2_qk:
        q, k = l2norm(q), l2norm(k)
    q = q * Dk ** -0.5
    S = q.new_zeros(N, H, Dk, v.shape[-1]) if initial_state is None else initial_state.float().clone()
    out = []
    for t in range(T):
        S = S * g[:, t].exp()[..., None, None]
        kv = (S * k[:, t, :, :, None]).sum(-2)
        delta = (v[:, t] - kv) * beta[:, t, :, None]
        S = S + k[:, t, :, :, None] * delta[:, :, None, :]
        out.append((S * q[:, t, :, :, None]).sum(-2))
    return torch.stack(out, 1).to(dt), S


GDN_FORK, GDN_CONCAT = "fork", "concat"


def gdn_core_blockdiff(q, k, v, g, beta, L: int, block: int, chunk: int, mode: str = GDN_FORK):
    """State-fork delta rule over the [B, 2L] two-stream layout (`blockdiff.py:159-177`).

    x_0: one causal pass from a zero state, keeping S_k after every block.
    x_t block k: its own row, starting from S_{k-1} (zero for k = 0).
    mode "concat": one causal pass over the whole 2L sequence (the concat-causal-gdn fault).
    q/k may have fewer heads than v (GQA); they are repeated to the v heads.
    """
    Hk, Hv = k.shape[2], v.shape[2]
    if Hv != Hk:
        q = q.repeat_interleave(Hv // Hk, 2)
        k = k.repeat_interleave(Hv // Hk, 2)
    B = q.shape[0]
    if mode == GDN_CONCAT:
        c = math.gcd(chunk, 2 * L)
        o, _ = chunk_gated_delta_rule(q, k, v, g, beta, c)
        return o
    nb = L // block
    sl0 = slice(L, 2 * L)
    # clean-pass chunk: a multiple of the block that divides L (snapshots land on block ends)
    c0 = block * math.gcd(L // block, max(1, chunk // block))
    o0, st = chunk_gated_delta_rule(q[:, sl0], k[:, sl0], v[:, sl0], g[:, sl0], beta[:, sl0], c0, state_every=block)
    init = torch.cat([torch.zeros_like(st[:, :1]), st[:, :-1]], 1).reshape(B * nb, *st.shape[2:])
    rs = lambda x: x[:, :L].reshape(B * nb, block, *x.shape[2:])  # noqa: E731
    ot, _ = chunk_gated_delta_rule(rs(q), rs(k), rs(v), rs(g), rs(beta), block, initial_state=init)
    return torch.cat([ot.reshape(B, L, *ot.shape[2:]), o0], 1)


# --------------------------------------------------------------------------- loss


def masked_ce_sum(hidden: torch.Tensor, w: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Sum of fp32 cross-entropy of hidden [n, D] projected by w [V, D] against targets [n]."""
    logits = (hidden @ w.t()).float()
    return F.cross_entropy(logits, targets, reduction="sum")
