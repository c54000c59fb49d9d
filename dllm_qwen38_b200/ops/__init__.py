"""Op layer: one functional entry per hot op.

Every op has exactly two implementations: the hand-written sm_100a kernel (``csrc/``, loaded
through ``ops._native``) for CUDA tensors, and the fp32 PyTorch reference (``ops.reference``)
for CPU tensors. There is no third path and no silent fallback: a CUDA tensor reaching an op
whose extension is not built raises. Which path ran is recorded per op (``last_impl``), the
same contract as the reference's ``gdn.last_impl`` (`gdn.py:22-45`): reports name the path
they measured instead of assuming it.
"""

from __future__ import annotations

import torch

from . import reference as ref

_LAST: dict[str, str] = {}


def _record(op: str, impl: str) -> None:
    _LAST[op] = impl


def last_impl(op: str | None = None):
    """Which implementation each op used on its most recent call ('native' or 'reference')."""
    return dict(_LAST) if op is None else _LAST.get(op)


def reset_impl_record() -> None:
    _LAST.clear()


def _native():
    from . import _native as nat

    return nat


def use_native(*tensors: torch.Tensor) -> bool:
    """True when the op must run the CUDA kernel (any CUDA input). Raises if it is not built."""
    if any(t is not None and t.is_cuda for t in tensors):
        _native().require()
        return True
    return False


# ----------------------------------------------------------------------------- norms / dense


def rmsnorm(x, w, eps: float):
    if use_native(x):
        _record("rmsnorm", "native")
        return _native().rmsnorm(x, w, eps)
    _record("rmsnorm", "reference")
    return ref.rmsnorm(x, w, eps)


def linear(x, w):
    """y = x @ w^T for x [..., K], w [N, K] (nn.Linear layout)."""
    if use_native(x):
        _record("linear", "native")
        return _native().linear(x, w)
    _record("linear", "reference")
    return ref.linear(x, w)


def swiglu_mlp(x, w_gate, w_up, w_down):
    """down(silu(gate x) * up x)."""
    if use_native(x):
        _record("mlp", "native")
        return _native().swiglu_mlp(x, w_gate, w_up, w_down)
    _record("mlp", "reference")
    return ref.linear(ref.swiglu(ref.linear(x, w_gate), ref.linear(x, w_up)), w_down)


def gated_rmsnorm(x, z, w, eps: float):
    if use_native(x):
        _record("gated_rmsnorm", "native")
        return _native().gated_rmsnorm(x, z, w, eps)
    _record("gated_rmsnorm", "reference")
    return ref.gated_rmsnorm(x, z, w, eps)


# ----------------------------------------------------------------------------- GDN


def conv_blockdiff(raw, w, L: int, block: int, mode: str = ref.CONV_FORK):
    if use_native(raw):
        _record("conv", "native")
        return _native().conv_blockdiff(raw, w, L, block, mode)
    _record("conv", "reference")
    return ref.conv_blockdiff(raw, w, L, block, mode)


def gdn_gates(a, b, A_log, dt_bias):
    if use_native(a):
        _record("gdn_gates", "native")
        return _native().gdn_gates(a, b, A_log, dt_bias)
    _record("gdn_gates", "reference")
    return ref.gdn_gates(a, b, A_log, dt_bias)


def gdn_core_blockdiff(q, k, v, g, beta, L: int, block: int, chunk: int, mode: str = ref.GDN_FORK):
    if use_native(q):
        _record("gdn_core", "native")
        return _native().gdn_core_blockdiff(q, k, v, g, beta, L, block, chunk, mode)
    _record("gdn_core", "reference")
    return ref.gdn_core_blockdiff(q, k, v, g, beta, L, block, chunk, mode)


# ----------------------------------------------------------------------------- attention


def attention_blockdiff(q, k, v, L: int, block: int, scale: float, leak_xt_prefix: bool = False):
    """Complementary-mask attention over the [B, 2L] layout (mask computed, never stored)."""
    if use_native(q):
        _record("attention", "native")
        return _native().attention_blockdiff(q, k, v, L, block, scale, leak_xt_prefix)
    _record("attention", "reference")
    allowed = ref.complementary_allowed(L, block, q.device, leak_xt_prefix)
    return ref.attention(q, k, v, allowed, scale)


def attention_masked(q, k, v, allowed, scale: float):
    """Attention under an explicit [T, T] bool mask (oracles and the plain forward)."""
    _record("attention_masked", "reference")
    return ref.attention(q, k, v, allowed, scale)


def qk_norm_rope(q, k, wq, wk, eps: float, cos, sin):
    """Per-head RMSNorm(1+w) of q and k, then partial RoPE on both."""
    if use_native(q):
        _record("qk_norm_rope", "native")
        return _native().qk_norm_rope(q, k, wq, wk, eps, cos, sin)
    _record("qk_norm_rope", "reference")
    return ref.apply_rope(ref.rmsnorm(q, wq, eps), cos, sin), ref.apply_rope(ref.rmsnorm(k, wk, eps), cos, sin)


# ----------------------------------------------------------------------------- loss


def masked_ce_sum(hidden, w, targets):
    """Sum over rows of fp32 CE(hidden @ w^T, targets); never holds the full-vocab logits on GPU."""
    if use_native(hidden):
        _record("masked_ce", "native")
        return _native().masked_ce_sum(hidden, w, targets)
    _record("masked_ce", "reference")
    return ref.masked_ce_sum(hidden, w, targets)


def embedding(ids, table):
    if use_native(ids):
        _record("embedding", "native")
        return _native().embedding(ids, table)
    _record("embedding", "reference")
    return torch.nn.functional.embedding(ids, table)
