"""Explicit forward and backward of the chunked gated delta rule (fp32, vectorised over chunks).

This is the specification the CUDA kernels in ``csrc/gdn.cu`` implement, kept as runnable
torch code and checked against autograd in the tests. The reference computes the same rule with
torch ops and two triangular solves per chunk and differentiates it by autograd
(`src/dllm_qwen38/gdn.py:48-123`). Per chunk of C tokens and one head
(q^, k^ are the l2-normalised query/key, q^ scaled by Dk^-1/2; S [Dk, Dv] the state entering the
chunk):

    gamma = cumsum(g),  Gam_ij = exp(gamma_i - gamma_j)  (i >= j)
    A  = strict_lower(diag(beta) k^ k^T * Gam),  T = (I + A)^-1        (UT transform)
    U  = T diag(beta) V,  W = T diag(beta e^gamma) k^
    V' = U - W S
    O  = diag(e^gamma) q^ S + (q^ k^T * Gam * incl_lower) V'
    S' = e^gamma_C S + k^T diag(e^(gamma_C - gamma)) V'

(the chunked form of Yang et al., "Gated Delta Networks" 2024, and the WY/UT representation of
"Parallelizing Linear Transformers with the Delta Rule over Sequence Length", 2024). Only the two
state recurrences are sequential in the chunk index:
    forward : V'_c = U_c - W_c S_c;  S_{c+1} = e^gamma_C S_c + k~_c^T V'_c
    backward: dV'_c = P_c^T dO_c + diag(F_c) k^_c dS_{c+1};  dS_c = e^gamma_C dS_{c+1} + q~_c^T dO_c - W_c^T dV'_c
and both are independent across the Dv columns of the state, which is how the kernels split
them across CTAs.
"""

from __future__ import annotations

import torch

from .reference import l2norm


def _f(x):
    """fp32 math (fp64 kept as is, for gradient checks)."""
    return x if x.dtype == torch.float64 else x.float()


def _chunks(x, N, H, nc, C):
    return x.transpose(1, 2).reshape(N, H, nc, C, *x.shape[3:])


def prep(q, k, v, g, beta, C):
    """Per-chunk quantities; inputs [N, T, H, D] / [N, T, H]. Returns a dict of [N, H, nc, ...]."""
    N, T, H, Dk = k.shape
    nc = T // C
    qf, kf, vf, gf, bf = (_f(x) for x in (q, k, v, g, beta))
    qn, kn = l2norm(qf), l2norm(kf)
    qh = qn * Dk ** -0.5
    Q, K, V = (_chunks(x, N, H, nc, C) for x in (qh, kn, vf))
    gam = _chunks(gf, N, H, nc, C).cumsum(-1)
    B = _chunks(bf, N, H, nc, C)
    incl = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    diff = gam[..., :, None] - gam[..., None, :]
    Gam = torch.where(incl, diff, torch.full_like(diff, float("-inf"))).exp()
    KK = K @ K.transpose(-1, -2)
    A = torch.tril(B[..., :, None] * KK * Gam, -1)
    eye = torch.eye(C, device=q.device, dtype=qf.dtype)
    Tm = torch.linalg.solve_triangular(eye + A, eye.expand_as(A), upper=False, unitriangular=True)
    E = gam.exp()
    F = (gam[..., -1:] - gam).exp()
    Ec = gam[..., -1].exp()
    U = Tm @ (B[..., None] * V)
    W = Tm @ ((B * E)[..., None] * K)
    P = (Q @ K.transpose(-1, -2)) * Gam
    return dict(Q=Q, K=K, V=V, B=B, gam=gam, Gam=Gam, KK=KK, T=Tm, E=E, F=F, Ec=Ec, U=U, W=W, P=P,
                qn=qn, kn=kn, qf=qf, kf=kf)


def forward(q, k, v, g, beta, C, S0=None):
    """Returns (o [N, T, H, Dv] fp32, S_in [N, H, nc, Dk, Dv] (state entering each chunk),
    S_final, cache)."""
    N, T, H, Dk = k.shape
    Dv = v.shape[-1]
    nc = T // C
    c = prep(q, k, v, g, beta, C)
    S = c["Q"].new_zeros(N, H, Dk, Dv) if S0 is None else _f(S0)
    S_in, Vp, O = [], [], []
    for i in range(nc):
        S_in.append(S)
        vp = c["U"][:, :, i] - c["W"][:, :, i] @ S
        Vp.append(vp)
        O.append((c["E"][:, :, i, :, None] * c["Q"][:, :, i]) @ S + c["P"][:, :, i] @ vp)
        S = c["Ec"][:, :, i, None, None] * S + (c["F"][:, :, i, :, None] * c["K"][:, :, i]).transpose(-1, -2) @ vp
    c["Vp"] = torch.stack(Vp, 2)
    S_in = torch.stack(S_in, 2)
    o = torch.stack(O, 2).reshape(N, H, T, Dv).transpose(1, 2)
    return o, S_in, S, c


def backward(q, k, v, g, beta, C, S_in, c, do, dS_final=None, dS_ext=None):
    """Gradients of the chunked rule. do [N, T, H, Dv]; dS_final [N, H, Dk, Dv] (gradient of the
    state after the last chunk); dS_ext [N, H, nc, Dk, Dv]: extra gradient on the state ENTERING
    chunk i (the state fork's injection point). Returns (dq, dk, dv, dg, dbeta, dS0)."""
    N, T, H, Dk = k.shape
    Dv = v.shape[-1]
    nc = T // C
    dO = _chunks(_f(do), N, H, nc, C)
    Q, K, V, Bt, E, F, Ec, W, P, Vp = (c[n] for n in ("Q", "K", "V", "B", "E", "F", "Ec", "W", "P", "Vp"))
    # ---- sequential: dV'_c and dS_{c+1} (state after chunk c) for every chunk
    dS = dO.new_zeros(N, H, Dk, Dv) if dS_final is None else _f(dS_final).clone()
    dVp, dSout = [None] * nc, [None] * nc
    for i in reversed(range(nc)):
        dSout[i] = dS
        dvp = P[:, :, i].transpose(-1, -2) @ dO[:, :, i] + F[:, :, i, :, None] * (K[:, :, i] @ dS)
        dVp[i] = dvp
        dS = Ec[:, :, i, None, None] * dS + (E[:, :, i, :, None] * Q[:, :, i]).transpose(-1, -2) @ dO[:, :, i] \
            - W[:, :, i].transpose(-1, -2) @ dvp
        if dS_ext is not None:
            dS = dS + dS_ext[:, :, i]
    dS0 = dS
    dVp = torch.stack(dVp, 2)
    dSout = torch.stack(dSout, 2)
    # ---- parallel over chunks
    S = S_in
    # O = diag(E) Q S + P V'
    QS = Q @ S
    dQ = E[..., None] * (dO @ S.transpose(-1, -2))
    dE = (QS * dO).sum(-1)
    dP = dO @ Vp.transpose(-1, -2)
    incl = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    dPm = dP * c["Gam"] * incl  # derivative through P = (Q K^T) * Gam
    dQ = dQ + dPm @ K
    dK = dPm.transpose(-1, -2) @ Q
    G1 = dP * P  # d/dgamma through Gam in P
    dgam = G1.sum(-1) - G1.sum(-2)
    # S' = Ec S + K^T diag(F) V'
    dK = dK + F[..., None] * (Vp @ dSout.transpose(-1, -2))
    dF = ((K @ dSout) * Vp).sum(-1)
    dEc = (S * dSout).sum((-1, -2))
    # V' = U - W S
    dU = dVp
    dW = -dVp @ S.transpose(-1, -2)
    # U = T diag(B) V, W = T diag(B E) K
    Tm = c["T"]
    dBv = Tm.transpose(-1, -2) @ dU
    dBk = Tm.transpose(-1, -2) @ dW
    dT = dU @ (Bt[..., None] * V).transpose(-1, -2) + dW @ ((Bt * E)[..., None] * K).transpose(-1, -2)
    dV = Bt[..., None] * dBv
    dB = (dBv * V).sum(-1) + E * (dBk * K).sum(-1)
    dK = dK + (Bt * E)[..., None] * dBk
    dE = dE + Bt * (dBk * K).sum(-1)
    # T = (I + A)^-1 -> dA = -T^T dT T^T (strict lower)
    dA = torch.tril(-Tm.transpose(-1, -2) @ dT @ Tm.transpose(-1, -2), -1)
    # A = strict_lower(B_i KK_ij Gam_ij)
    KK, Gam = c["KK"], c["Gam"]
    dB = dB + (dA * KK * Gam).sum(-1)
    dKK = dA * Bt[..., :, None] * Gam
    dK = dK + dKK @ K + dKK.transpose(-1, -2) @ K
    H2 = dA * Bt[..., :, None] * KK * Gam
    dgam = dgam + H2.sum(-1) - H2.sum(-2)
    # E = e^gam, F = e^(gam_C - gam), Ec = e^gam_C
    dgam = dgam + dE * E - dF * F
    dgam[..., -1] = dgam[..., -1] + (dF * F).sum(-1) + dEc * Ec
    dg = dgam.flip(-1).cumsum(-1).flip(-1)

    def unchunk(x):
        return x.reshape(N, H, T, *x.shape[4:]).transpose(1, 2)

    dqh, dkn, dv = unchunk(dQ), unchunk(dK), unchunk(dV)
    dg, dbeta = unchunk(dg), unchunk(dB)
    # q^ = l2norm(q) * s, k^ = l2norm(k)
    dqn = dqh * Dk ** -0.5

    def l2_bwd(x, dy):
        r = torch.rsqrt((x * x).sum(-1, keepdim=True) + 1e-6)
        return r * dy - x * r ** 3 * (x * dy).sum(-1, keepdim=True)

    dq = l2_bwd(c["qf"], dqn)
    dk = l2_bwd(c["kf"], dkn)
    return dq, dk, dv, dg, dbeta, dS0
