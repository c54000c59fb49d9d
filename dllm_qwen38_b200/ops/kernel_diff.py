"""Native-vs-reference probe of the state-fork gated delta rule on a real GDN mixer.

The reference's `kernel_diff` (`gdn.py:166-190`) measures the max |difference| of the mixer
output and of the per-block states between its fast kernel and its fp32 torch core, and refuses
to answer when the fast kernel did not run. Same contract here: the fast side is this
repository's sm_100a kernel (`_C.gdn_fwd`), the slow side `ops.reference.chunk_gated_delta_rule`
in fp32 on the same inputs; no answer without the extension on a CUDA device.

    python -m dllm_qwen38_b200.ops.kernel_diff [--model 27b] [--seq-len 2048] [--block 32]
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from . import _native
from . import reference as ref


@torch.no_grad()
def core_diff(q, k, v, g, beta, L: int, block: int, chunk: int = 64) -> dict:
    """q, k [B, 2L, Hk, D], v [B, 2L, Hv, D] (post-conv, pre-norm), g/beta [B, 2L, Hv]."""
    if not q.is_cuda or not _native.available():
        raise RuntimeError("kernel_diff: the native kernel cannot run here (needs CUDA and the built extension)")
    C = _native.require()
    o, S_in, _ = C.gdn_fwd(q, k, v, g.float().contiguous(), beta.float().contiguous(), L, block, False)
    o_ref = ref.gdn_core_blockdiff(q.float(), k.float(), v.float(), g.float(), beta.float(), L, block, chunk)
    Hk, Hv = k.shape[2], v.shape[2]
    qf, kf = q.float(), k.float()
    if Hv != Hk:
        qf, kf = qf.repeat_interleave(Hv // Hk, 2), kf.repeat_interleave(Hv // Hk, 2)
    sl = slice(L, 2 * L)
    c0 = block * math.gcd(L // block, max(1, chunk // block))
    _, st = ref.chunk_gated_delta_rule(qf[:, sl], kf[:, sl], v[:, sl].float(), g[:, sl].float(),
                                       beta[:, sl].float(), c0, state_every=block)
    entry = torch.cat([torch.zeros_like(st[:, :1]), st[:, :-1]], 1)  # state entering block k
    scale = float(o_ref.abs().max())
    return {"out_max_abs_diff": float((o.float() - o_ref).abs().max()), "out_max_abs": scale,
            "states_max_abs_diff": float((S_in - entry).abs().max()), "states_max_abs": float(entry.abs().max()),
            "impl": "native"}


@torch.no_grad()
def mixer_diff(mixer, hidden: torch.Tensor, L: int, block: int, chunk: int = 64) -> dict:
    """Run a GDN mixer's projections, conv (state fork) and gates with reference ops on
    `hidden` [B, 2L, D], then compare the two cores."""
    m = mixer
    w = torch.cat([m.in_proj_qkv.weight, m.in_proj_z.weight, m.in_proj_b.weight, m.in_proj_a.weight], 0)
    proj = hidden @ w.t()
    raw, _, b, a = torch.split(proj, [m.conv_dim, m.value_dim, m.num_v_heads, m.num_v_heads], dim=-1)
    mixed = ref.conv_blockdiff(raw, m.conv1d.weight[:, 0, :], L, block, ref.CONV_FORK)
    q, k, v = torch.split(mixed, [m.key_dim, m.key_dim, m.value_dim], dim=-1)
    B, T, _ = hidden.shape
    q = q.reshape(B, T, m.num_k_heads, m.head_k_dim).contiguous()
    k = k.reshape(B, T, m.num_k_heads, m.head_k_dim).contiguous()
    v = v.reshape(B, T, m.num_v_heads, m.head_v_dim).contiguous()
    g, beta = ref.gdn_gates(a, b, m.A_log, m.dt_bias)
    return core_diff(q, k, v, g, beta, L, block, chunk)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="27b")
    p.add_argument("--seq-len", type=int, default=2048)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    from ..config import LINEAR, preset
    from ..models.qwen35 import build_model

    cfg = preset(a.model, layers=1)
    if cfg.layer_types[0] != LINEAR:
        raise SystemExit("the first layer of this preset is not a GDN layer")
    model = build_model(cfg, seed=a.seed, device="cuda", dtype=torch.bfloat16)
    gen = torch.Generator(device="cuda").manual_seed(a.seed)
    ids = torch.randint(0, cfg.mask_id, (1, 2 * a.seq_len), device="cuda", generator=gen)
    h = model.text_model.embed_tokens(ids)
    layer = model.text_model.layers[0]
    n = ref.rmsnorm(h, layer.input_layernorm.weight, layer.input_layernorm.eps)
    res = mixer_diff(layer.linear_attn, n, a.seq_len, a.block)
    print(json.dumps({"kernel_diff": res, "model": a.model, "seq_len": a.seq_len, "block": a.block}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
