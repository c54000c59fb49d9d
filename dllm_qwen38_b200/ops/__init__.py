"""Op layer: one functional entry per hot op.

Every op has exactly two implementations: the hand-written sm_100a kernel (``csrc/``, loaded
through ``ops._native``) for CUDA tensors, and the fp32 PyTorch reference (``ops.reference``)
for CPU tensors. There is no silent fallback: a CUDA tensor reaching an op whose extension is
not built raises, and torch runs on the device only where a caller asks for it by name
(`torch_on_cuda`, `torch_paths`: the lever benchmark, the fp32 gate on a GPU, `--gdn torch`). Which path ran is recorded per op (``last_impl``), the
same contract as the reference's ``gdn.last_impl`` (`gdn.py:22-45`): reports name the path
they measured instead of assuming it.
"""

from __future__ import annotations

import torch

from . import reference as ref

_LAST: dict[str, str] = {}


def _record(op: str, impl: str) -> None:
    _LAST[op] = impl


_PENDING_TORCH_CUDA: set = set()


def _record_ref(op: str) -> None:
    """Record the torch path: 'torch-cuda' if use_native just routed a CUDA call here, else
    'reference' (host tensors)."""
    if op in _PENDING_TORCH_CUDA:
        _PENDING_TORCH_CUDA.discard(op)
        _LAST[op] = "torch-cuda"
    else:
        _LAST[op] = "reference"


def last_impl(op: str | None = None):
    """Which implementation each op used on its most recent call: 'native' (sm_100a kernel),
    'reference' (fp32 torch on the host) or 'torch-cuda' (torch on the device: an op whose kernel
    is not written yet, or one routed there by `torch_on_cuda` / `torch_paths` for comparison)."""
    return dict(_LAST) if op is None else _LAST.get(op)


def reset_impl_record() -> None:
    _LAST.clear()


def _nat():
    import importlib

    return importlib.import_module(__name__ + "._native")


_LEVERS: set = set()

# every op family with a native kernel (the native kernels compute in bf16; fp32 runs on a CUDA
# device go through torch_on_cuda(*ALL_OPS))
ALL_OPS = ("rmsnorm", "linear", "mlp", "gated_rmsnorm", "conv", "gdn_gates", "gdn_core", "attention",
           "qk_norm_rope", "output_gate", "masked_ce", "embedding")


class torch_on_cuda:
    """Context manager: run the named ops through their torch path on the device (recorded as
    'torch-cuda'). Used by the lever benchmark to measure what each native kernel buys and by the
    command lines' `--gdn torch` / `--attn sdpa`; no default path enters it."""

    def __init__(self, *ops: str):
        self.ops = set(ops)
        self.prev: set = set()

    def __enter__(self):
        self.prev = set(_LEVERS)
        _LEVERS.update(self.ops)
        return self

    def __exit__(self, *exc):
        _LEVERS.clear()
        _LEVERS.update(self.prev)
        return False


GDN_CHOICES = ("native", "auto", "torch")
ATTN_CHOICES = ("native", "sdpa", "eager")


def torch_paths(gdn: str = "native", attn: str = "native") -> torch_on_cuda:
    """The command lines' `--gdn` / `--attn` choices (the reference's flags, `train.py:220-221`,
    `equivalence.py:172`) as one context: gdn 'torch' runs the GDN core through the fp32 torch
    chunked rule on the device; attn 'sdpa' or 'eager' runs the masked attention through torch's
    scaled_dot_product_attention over the boolean complementary mask (one torch path stands for
    both). 'native' / 'auto' keep the sm_100a kernels. Host tensors take the torch path anyway."""
    if gdn not in GDN_CHOICES or attn not in ATTN_CHOICES:
        raise ValueError(f"gdn must be one of {GDN_CHOICES}, attn one of {ATTN_CHOICES}")
    return torch_on_cuda(*((("gdn_core",) if gdn == "torch" else ()) + (("attention",) if attn != "native" else ())))


def use_native(*tensors: torch.Tensor, op: str | None = None) -> bool:
    """True when the op must run the CUDA kernel (any CUDA input). Raises if the extension is not
    built. An op listed in ``ops.cuda.TORCH_ON_CUDA`` has no kernel yet: it runs the reference on
    the device and is recorded as 'torch-cuda' so no report mistakes it for a native path."""
    if any(t is not None and t.is_cuda for t in tensors):
        _nat().require()
        if op is not None and (op in _nat().TORCH_ON_CUDA or op in _LEVERS):
            _PENDING_TORCH_CUDA.add(op)
            return False
        return True
    return False


# ----------------------------------------------------------------------------- norms / dense


def rmsnorm(x, w, eps: float):
    if use_native(x, op="rmsnorm"):
        _record("rmsnorm", "native")
        return _nat().rmsnorm(x, w, eps)
    _record_ref("rmsnorm")
    return ref.rmsnorm(x, w, eps)


def linear(x, w):
    """y = x @ w^T for x [..., K], w [N, K] (nn.Linear layout)."""
    if use_native(x, op="linear"):
        _record("linear", "native")
        return _nat().linear(x, w)
    _record_ref("linear")
    return ref.linear(x, w)


def swiglu_mlp(x, w_gate, w_up, w_down):
    """down(silu(gate x) * up x)."""
    if use_native(x, op="mlp"):
        _record("mlp", "native")
        return _nat().swiglu_mlp(x, w_gate, w_up, w_down)
    _record_ref("mlp")
    return ref.linear(ref.swiglu(ref.linear(x, w_gate), ref.linear(x, w_up)), w_down)


def swiglu_mlp_fused(x, w_gate_up, w_down):
    """down(silu(x Wg^T) * (x Wu^T)) with w_gate_up = [Wg; Wu] one contiguous [2F, D] weight."""
    if use_native(x, op="mlp"):
        _record("mlp", "native")
        return _nat().swiglu_mlp_fused(x, w_gate_up, w_down)
    _record_ref("mlp")
    F = w_gate_up.shape[0] // 2
    return ref.linear(ref.swiglu(ref.linear(x, w_gate_up[:F]), ref.linear(x, w_gate_up[F:])), w_down)


def adamw_flat(w, p, g, m, v, lr, b1, b2, eps, wd, coef, bc1, bc2):
    """Fused AdamW over flat fp32 master w, bf16 param p, grad g, moments m, v. coef is the clip
    coefficient (float or 0-d device tensor, read on the device)."""
    if w.is_cuda:
        _record("adamw", "native")
        return _nat().adamw_flat(w, p, g, m, v, lr, b1, b2, eps, wd, coef, bc1, bc2)
    _record_ref("adamw")
    gg = g.float() * (coef if not torch.is_tensor(coef) else coef.float())
    if wd:
        w.mul_(1 - lr * wd)
    m.mul_(b1).add_(gg, alpha=1 - b1)
    v.mul_(b2).addcmul_(gg, gg, value=1 - b2)
    w.addcdiv_(m, (v / bc2).sqrt_().add_(eps), value=-lr / bc1)
    p.copy_(w)


def sumsq_(x, sq, dst=None):
    """sq += ||x||^2 in fp32 (one read of x); with `dst` (fp32, same size) also dst = float(x)."""
    if x.is_cuda:
        return _nat().sumsq_(x, sq, dst)
    if dst is not None:
        dst.copy_(x)
    sq += x.float().pow(2).sum()


def gated_rmsnorm(x, z, w, eps: float):
    if use_native(x, op="gated_rmsnorm"):
        _record("gated_rmsnorm", "native")
        return _nat().gated_rmsnorm(x, z, w, eps)
    _record_ref("gated_rmsnorm")
    return ref.gated_rmsnorm(x, z, w, eps)


# ----------------------------------------------------------------------------- GDN


def conv_blockdiff(raw, w, L: int, block: int, mode: str = ref.CONV_FORK):
    if use_native(raw, op="conv"):
        _record("conv", "native")
        return _nat().conv_blockdiff(raw, w, L, block, mode)
    _record_ref("conv")
    return ref.conv_blockdiff(raw, w, L, block, mode)


def gdn_gates(a, b, A_log, dt_bias):
    if use_native(a, op="gdn_gates"):
        _record("gdn_gates", "native")
        return _nat().gdn_gates(a, b, A_log, dt_bias)
    _record_ref("gdn_gates")
    return ref.gdn_gates(a, b, A_log, dt_bias)


def gdn_core_blockdiff(q, k, v, g, beta, L: int, block: int, chunk: int, mode: str = ref.GDN_FORK):
    if use_native(q, op="gdn_core"):
        _record("gdn_core", "native")
        return _nat().gdn_core_blockdiff(q, k, v, g, beta, L, block, chunk, mode)
    _record_ref("gdn_core")
    return ref.gdn_core_blockdiff(q, k, v, g, beta, L, block, chunk, mode)


# ----------------------------------------------------------------------------- attention


def attention_blockdiff(q, k, v, L: int, block: int, scale: float, leak_xt_prefix: bool = False):
    """Complementary-mask attention over the [B, 2L] layout (mask computed, never stored)."""
    if use_native(q, op="attention"):
        _record("attention", "native")
        return _nat().attention_blockdiff(q, k, v, L, block, scale, leak_xt_prefix)
    _record_ref("attention")
    allowed = ref.complementary_allowed(L, block, q.device, leak_xt_prefix)
    if q.is_cuda:  # device path until the native kernel covers it: no O(T^2) fp32 scores
        o = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), attn_mask=allowed, scale=scale, enable_gqa=True)
        return o.transpose(1, 2)
    return ref.attention(q, k, v, allowed, scale)


def attention_masked(q, k, v, allowed, scale: float):
    """Attention under an explicit [T, T] bool mask (oracles and the plain forward)."""
    _record_ref("attention_masked")
    return ref.attention(q, k, v, allowed, scale)


def qk_norm_rope(q, k, wq, wk, eps: float, cos, sin):
    """Per-head RMSNorm(1+w) of q and k, then partial RoPE on both."""
    if use_native(q, op="qk_norm_rope"):
        _record("qk_norm_rope", "native")
        return _nat().qk_norm_rope(q, k, wq, wk, eps, cos, sin)
    _record_ref("qk_norm_rope")
    return ref.apply_rope(ref.rmsnorm(q, wq, eps), cos, sin), ref.apply_rope(ref.rmsnorm(k, wk, eps), cos, sin)


def output_gate(o, gate):
    """The attention output gate o * sigmoid(gate) (HF `Qwen3_5Attention`'s gated output)."""
    if use_native(o, op="output_gate"):
        _record("output_gate", "native")
        return _nat().output_gate(o, gate)
    _record_ref("output_gate")
    return o * torch.sigmoid(gate)


# ----------------------------------------------------------------------------- loss


def masked_ce_sum(hidden, w, targets):
    """Sum over rows of fp32 CE(hidden @ w^T, targets); never holds the full-vocab logits on GPU."""
    if use_native(hidden, op="masked_ce"):
        _record("masked_ce", "native")
        return _nat().masked_ce_sum(hidden, w, targets)
    _record_ref("masked_ce")
    return ref.masked_ce_sum(hidden, w, targets)


def embedding(ids, table):
    if use_native(ids, op="embedding"):
        _record("embedding", "native")
        return _nat().embedding(ids, table)
    _record_ref("embedding")
    return torch.nn.functional.embedding(ids, table)
