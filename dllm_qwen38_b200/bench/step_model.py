"""Speed-of-light model of one training step, family by family (CPU only; no GPU needed).

    python -m dllm_qwen38_b200.bench.step_model [--layers 16] [--seq-len 4096] [--kept 14]

For the flagship step (`bench.py`: one sequence per GPU, two complementary views of the x_t || x_0
layout, so every layer sees R = 4 L token rows; the lm_head scores the L masked rows of the two
views together) it counts the work each kernel family must do at least and divides by the pool's
measured peaks (`MEASURED_PEAKS.json`: cuBLAS bf16 rate sustained under the power cap for the
tensor-core families, STREAM-style copy bandwidth for the memory-bound ones). Set against the
step profiler's per-family times (`bench.step_profile`) this says how far each family sits from
its roofline.

Counted work (no kernel detail, only what the math needs):
  GEMM       2 R P per forward pass over a layer's dense weights P, 4 R P for its backward
             (input and weight gradients), plus the forward again for the layers whose GEMM
             outputs are not kept; lm_head 6 L D V.
  attention  the complementary mask's allowed (query, key) pairs per view, block^2 nb (nb + 1)
             for nb = L / block, times 4 Dh per pair and query head forward and 10 Dh backward
             (scores recomputed, dP, dV, dQ, dK); outputs are kept, so no forward recompute.
  AdamW      28 bytes per parameter (fp32 master, m, v read and written; bf16 gradient read and
             parameter written).
  norms      RMSNorm: 4 bytes per element forward (read x, write y), 6 backward; gated RMSNorm
             (x, z): 6 forward, 10 backward; the final norm and the q/k norms included.
  SwiGLU     the derivative kernel: 10 bytes per element of the [R, F] activation.
  CE rows    the [L, V] bf16 logits read twice and written once: 6 L V bytes.
  embedding  the backward's [R, D] row gradients read once and the table rows written once
             (at most min(R, V) distinct ids; all V when R >= V).
  GDN core   the larger of two floors. FLOPs of the chunk algebra per (chunk of C tokens, v-head)
             with Dk = Dv = D: 6 C D^2 (W S, Q S, the state update) + 10 C^2 D (K K^T, T V, T K,
             Q K^T, its product with V') + 2/3 C^3 (the triangular inverse) for a clean chunk, less
             the state update for a noised block; backward twice the forward. Bytes: q, k, v, g,
             beta read and o written forward; those inputs, dO read and dq, dk, dv, dg, dbeta written
             backward (no saved states counted).

With --gpus N (the sharded engine, one sequence per GPU) the per-GPU work above stays, AdamW
covers 1/N of the parameters, and two NVLink rows are added: every unit's parameters gathered
twice per step (forward, and again for the backward's GEMMs) and its gradient reduce-scattered
once, (N - 1) / N of the bf16 bytes arriving at each GPU, at the pool's measured peer copy rate
(770 GB/s per direction). Those transfers overlap the compute, so they are a floor of their own,
not an addition to the step's.

The causal conv is left out; the GDN floor ignores that each head's chunks form a chain of L / C
dependent steps, which is what actually bounds its kernels (their per-phase profile is in
`profiles/gdn_tc_27b_shapes.md`).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks(path: str | None = None) -> dict:
    """{'tflops': sustained bf16 TF/s, 'gbs': copy GB/s, 'source': ...} from MEASURED_PEAKS.json,
    else the pool's earlier measurement (1.4 PF/s sustained, 6.65 TB/s)."""
    path = path or os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"tflops": float(p["bf16_tflops_sustained"]), "gbs": float(p["hbm_gbs"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"tflops": 1400.0, "gbs": 6650.0, "source": "fallback"}


def dense_params(cfg, kind: str) -> int:
    """Weights of one layer that its GEMMs multiply (projections and MLP)."""
    D, F = cfg.hidden_size, cfg.intermediate_size
    n = 3 * D * F
    if kind == "linear_attention":
        n += D * cfg.conv_dim + D * cfg.value_dim + 2 * D * cfg.linear_num_value_heads + cfg.value_dim * D
    else:
        Hq, Hk, Dh = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        n += D * Hq * Dh * 2 + 2 * D * Hk * Dh + Hq * Dh * D
    return n


def step_work(cfg, L: int, block: int, kept: int, gpus: int = 1) -> dict:
    """{family: (flops, bytes)} for one GPU's share of one step (one sequence of length L per GPU)."""
    D, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    R = 4 * L
    kinds = list(cfg.layer_types)
    gemm = 0.0
    for i, kind in enumerate(kinds):
        P = dense_params(cfg, kind)
        gemm += (2 + 4) * R * P + (0 if i < kept else 2 * R * P)
    gemm += 6.0 * L * D * V
    nb = L // block
    pairs = block * block * nb * (nb + 1)  # per view
    n_attn = sum(1 for k in kinds if k != "linear_attention")
    attn = 2 * pairs * cfg.num_attention_heads * cfg.head_dim * (4 + 10) * n_attn
    adamw_b = 28.0 * cfg.param_count() / gpus
    norm_b = 0.0
    for kind in kinds:
        norm_b += 2 * (4 + 6) * R * D  # input and post-attention RMSNorm
        if kind == "linear_attention":
            norm_b += (6 + 10) * R * cfg.value_dim  # gated RMSNorm over the value heads
        else:
            norm_b += (4 + 6) * R * (cfg.num_attention_heads + cfg.num_key_value_heads) * cfg.head_dim
    norm_b += (4 + 6) * L * D  # final norm over the scored rows
    swiglu_b = 10.0 * R * F * len(kinds)
    ce_b = 6.0 * L * V
    embed_b = 2.0 * R * D + 2.0 * min(R, V) * D
    n_gdn = sum(1 for k in kinds if k == "linear_attention")
    C, Dg, Hv, Hk = block, cfg.linear_key_head_dim, cfg.linear_num_value_heads, cfg.linear_num_key_heads
    clean = 6 * C * Dg * Dg + 10 * C * C * Dg + (2 / 3) * C ** 3
    noised = clean - 2 * C * Dg * Dg
    per_view = (L // C) * Hv * (clean + noised)
    gdn_f = 3 * 2 * per_view * n_gdn  # two views, forward + backward (twice the forward)
    T2 = 2 * L  # tokens per view
    io_fwd = T2 * (2 * Hk * Dg * 2 + Hv * Dg * 2 + 2 * Hv * 4 + Hv * Dg * 2)  # q, k, v, g, beta in; o out
    io_bwd = io_fwd + T2 * (2 * Hk * Dg * 2 + Hv * Dg * 2 + 2 * Hv * 4)  # + dq, dk, dv, dg, dbeta
    gdn_b = 2 * (io_fwd + io_bwd) * n_gdn
    return {"GEMM (tcgen05)": (gemm, 0.0), "attention": (attn, 0.0), "AdamW": (0.0, adamw_b),
            "norms": (0.0, norm_b), "SwiGLU element-wise": (0.0, swiglu_b), "CE rows": (0.0, ce_b),
            "embedding": (0.0, embed_b), "GDN core": (gdn_f, gdn_b)}


def comm_bytes(cfg, gpus: int) -> dict:
    """Bytes arriving at each GPU over NVLink per step of the sharded engine (bf16 parameters and
    gradients): {'all-gather': ..., 'reduce-scatter': ...}; empty on one GPU."""
    if gpus <= 1:
        return {}
    share = (gpus - 1) / gpus * 2.0 * cfg.param_count()
    return {"FSDP all-gather (NVLink, overlapped)": 2 * share, "FSDP reduce-scatter (NVLink, overlapped)": share}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="27b")
    p.add_argument("--layers", type=int, default=16)
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--kept", type=int, default=None, help="layers whose GEMM outputs are kept (default: all)")
    p.add_argument("--peaks", default=None, help="a MEASURED_PEAKS.json (default: the repository's)")
    p.add_argument("--gpus", type=int, default=1, help="ranks of the sharded engine (one sequence each)")
    p.add_argument("--nvlink-gbs", type=float, default=770.0,
                   help="peer copy GB/s per direction (the pool's measured figure)")
    a = p.parse_args(argv)
    sys.path.insert(0, ROOT)
    from ..config import preset

    cfg = preset(a.model, layers=a.layers)
    kept = cfg.num_hidden_layers if a.kept is None else a.kept
    pk = peaks(a.peaks)
    work = step_work(cfg, a.seq_len, a.block, kept, a.gpus)
    print(f"{a.model}, {cfg.num_hidden_layers} layers, seq {a.seq_len}, GEMM outputs kept for {kept}; peaks "
          f"({pk['source']}): {pk['tflops']:.1f} TF/s bf16 sustained, {pk['gbs']:.1f} GB/s copy")
    total = 0.0
    for fam, (flops, byts) in work.items():
        ms = 1e3 * max(flops / (pk["tflops"] * 1e12), byts / (pk["gbs"] * 1e9))
        total += ms
        what = "  ".join(x for x in (f"{flops / 1e12:7.2f} TFLOP" if flops else "",
                                     f"{byts / 1e9:7.2f} GB" if byts else "") if x)
        print(f"  {ms:9.2f} ms  {what:24s}  {fam}")
    print(f"  {total:9.2f} ms  total of the modelled families (per GPU, {a.gpus} GPU{'s' if a.gpus > 1 else ''})")
    for what, byts in comm_bytes(cfg, a.gpus).items():
        print(f"  {1e3 * byts / (a.nvlink_gbs * 1e9):9.2f} ms  {byts / 1e9:7.2f} GB{'':15s}  {what}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
