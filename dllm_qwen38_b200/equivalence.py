"""Equivalence gate for the state fork, with deliberate faults as negative controls.

The state fork computes every noised block from the clean stream's recurrent state at the block's
start instead of running the block-causal mask over the whole x_t||x_0 sequence. This module
measures whether that shortcut is exact. It builds an oracle that knows nothing about forking:
for each block it reruns an ordinary, unforked forward over the clean prefix followed by that
block's noised tokens (fp32 reference ops, delta rule one token at a time, on an fp32 copy of
the weights), then reports

  * the largest logit difference between the candidate's noised stream and that oracle, and the
    same for the clean stream against a plain causal forward;
  * three visibility probes made by editing the input: a noised block must not change when the
    previous noised block or its own clean block is rewritten, and must change (by at least a
    floor, 10x the tolerance by default) when the previous clean block is rewritten;
  * for each fault in `FAULTS` (run the DeltaNet causally over the concatenation, let noised
    tokens see their own clean block, start each block's convolution without the clean prefix),
    whether the first measure moves beyond the tolerance. A fault that stays inside it means the
    gate could not have caught that bug.

The process status is the verdict: 0 when every measure is within bounds and every fault is
caught, 1 otherwise, 2 when the run itself failed (model not loadable, bad arguments). With
``--device cuda --dtype bfloat16`` the candidate runs on the sm_100a kernels, which carry the
fault switches themselves; ``--dtype float32`` on a GPU runs the candidate through the fp32 torch
ops there (the kernels compute in bf16). Tolerances follow the dtype: 1e-3 for fp32, 0.25 for
bf16.

    python -m dllm_qwen38_b200.equivalence [--model tiny] [--block 32 --nblocks 4] [--device cuda]

Contract kept with the reference (`src/dllm_qwen38/equivalence.py:75-219`): check and fault
names, output lines, tolerances and exit codes.
"""

from __future__ import annotations

import argparse
import copy
import json
import sys
import time

import torch

from . import ops
from .models.blockdiff import FAULTS, BreakMode, block_diffusion_forward
from .models.oracle import reference_block_logits, reference_clean_logits


def _maxdiff(a, b) -> float:
    return float((a.float().cpu() - b.float().cpu()).abs().max())


def run(model, *, block: int, nblocks: int, layers: int | None, tol: float, change_floor: float, seed: int,
        device: str, oracle_model=None, batch: int = 1, oracle_gdn: str = "recurrent") -> dict:
    """Checks + faults on `model` (on `device`); the oracle runs on `oracle_model` (default: the
    same model) on its own device, in fp32 reference ops."""
    oracle_model = oracle_model or model
    odev = next(oracle_model.parameters()).device
    torch.manual_seed(seed)
    L = block * nblocks
    vocab = model.config.vocab_size
    x0 = torch.randint(0, vocab, (batch, L))
    xt = x0.clone()
    mask_id = vocab - 1  # visibility does not depend on which id plays [MASK]
    xt[torch.rand(batch, L) < 0.5] = mask_id
    dx0, dxt = x0.to(device), xt.to(device)

    def cand(a, b, fault=None):
        with torch.no_grad():
            return block_diffusion_forward(model, a.to(device), b.to(device), block, layers=layers, fault=fault)[0]

    checks: list = []
    t0 = time.time()
    with torch.no_grad():
        lt, l0 = block_diffusion_forward(model, dx0, dxt, block, layers=layers)
        ref_t = reference_block_logits(oracle_model, x0.to(odev), xt.to(odev), block, layers=layers, gdn=oracle_gdn)
        ref_0 = reference_clean_logits(oracle_model, x0.to(odev), block, layers=layers, gdn=oracle_gdn)
    impl = ops.last_impl()
    d = _maxdiff(lt, ref_t)
    checks.append({"name": "noised-stream-vs-oracle", "max_abs_diff": d, "tol": tol, "pass": d <= tol})
    d = _maxdiff(l0, ref_0)
    checks.append({"name": "clean-stream-vs-oracle", "max_abs_diff": d, "tol": tol, "pass": d <= tol})
    if nblocks >= 2:
        worst_xt, worst_x0k, weakest = 0.0, 0.0, float("inf")
        for k in range(1, nblocks):
            sl, prev = slice(k * block, (k + 1) * block), slice((k - 1) * block, k * block)
            xt2 = xt.clone()
            xt2[:, prev] = torch.randint(0, vocab, (batch, block))
            worst_xt = max(worst_xt, _maxdiff(lt[:, sl], cand(x0, xt2)[:, sl]))
            x02 = x0.clone()
            x02[:, sl] = torch.randint(0, vocab, (batch, block))
            worst_x0k = max(worst_x0k, _maxdiff(lt[:, sl], cand(x02, xt)[:, sl]))
            x03 = x0.clone()
            x03[:, prev] = torch.randint(0, vocab, (batch, block))
            weakest = min(weakest, _maxdiff(lt[:, sl], cand(x03, xt)[:, sl]))
        checks.append({"name": "xt-block-k-ignores-xt-block-k-1", "max_abs_diff": worst_xt, "tol": tol, "pass": worst_xt <= tol})
        checks.append({"name": "xt-block-k-ignores-x0-block-k", "max_abs_diff": worst_x0k, "tol": tol, "pass": worst_x0k <= tol})
        checks.append({"name": "xt-block-k-reacts-to-x0-block-k-1", "min_abs_diff": weakest, "floor": change_floor,
                       "pass": weakest >= change_floor})
    faults = []
    for name in FAULTS:
        d = _maxdiff(cand(x0, xt, BreakMode(name)), ref_t)
        faults.append({"fault": name, "max_abs_diff": d, "tol": tol, "detected": d > tol})
    cfg = model.config
    n_layers = layers if layers is not None else cfg.num_hidden_layers
    return {
        "block": block, "nblocks": nblocks, "seq_len": L, "batch": batch, "layers": n_layers,
        "layer_types": list(cfg.layer_types[:n_layers]),
        "dtype": str(model.text_model.embed_tokens.weight.dtype), "device": device,
        "seconds": round(time.time() - t0, 2), "checks": checks, "faults": faults,
        "checks_passed": sum(c["pass"] for c in checks), "checks_total": len(checks),
        "faults_detected": sum(f["detected"] for f in faults), "faults_total": len(faults),
        "candidate_impl": impl, "oracle": f"reference-ops/{oracle_gdn}",
    }


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="tiny", help="preset (tiny, tiny_ref, 0.8b, 27b) or HF checkpoint dir")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--nblocks", type=int, default=4)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--tol", type=float, default=None, help="max |dlogit| (default fp32 1e-3, bf16 0.25)")
    p.add_argument("--change-floor", type=float, default=None, help="default 10 x tol")
    p.add_argument("--dtype", default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--device", default="cpu")
    p.add_argument("--attn", default="native", choices=["native", "sdpa", "eager"],
                   help="candidate attention on a GPU: native (sm_100a kernel) or torch's attention over "
                        "the boolean mask (sdpa / eager); on the CPU the candidate runs the fp32 torch ops")
    p.add_argument("--oracle-gdn", default="recurrent", choices=["recurrent", "chunk"])
    p.add_argument("--oracle-device", default=None, help="where the fp32 oracle runs (default: --device)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--json", default=None)
    a = p.parse_args(argv)
    dtype = torch.float32 if a.dtype == "float32" else torch.bfloat16
    tol = a.tol if a.tol is not None else (1e-3 if dtype == torch.float32 else 0.25)
    floor = a.change_floor if a.change_floor is not None else 10 * tol
    if a.nblocks < 1:
        print("COULD-NOT-MEASURE nblocks < 1", file=sys.stderr)
        return 2
    try:
        from .io.hf_load import load_model, spare_rows

        model, tok = load_model(a.model, dtype=dtype, device=a.device, layers=a.layers, seed=a.seed)
        spare = spare_rows(model, tok) if tok is not None else None
    except Exception as e:  # noqa: BLE001
        print(f"COULD-NOT-MEASURE model load failed: {type(e).__name__}: {e}", file=sys.stderr)
        return 2
    if a.layers is not None and a.layers > model.config.num_hidden_layers:
        print("COULD-NOT-MEASURE --layers exceeds the model", file=sys.stderr)
        return 2
    oracle_model = model
    odev = a.oracle_device or a.device
    if a.device != "cpu" or dtype != torch.float32:  # the oracle: fp32 reference ops on its own copy
        oracle_model = copy.deepcopy(model).to(odev, torch.float32)
    from . import ops

    # the sm_100a kernels compute in bf16: an fp32 gate on a GPU runs the fp32 torch ops there
    ctx = ops.torch_on_cuda(*ops.ALL_OPS) if (a.device != "cpu" and dtype == torch.float32) else \
        ops.torch_paths(attn=a.attn)
    with ctx:
        rep = run(model, block=a.block, nblocks=a.nblocks, layers=None, tol=tol, change_floor=floor, seed=a.seed,
                  device=a.device, oracle_model=oracle_model, batch=a.batch, oracle_gdn=a.oracle_gdn)
    rep["model"] = a.model
    if spare:
        rep["vocab"] = spare
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rep, f, indent=1)
    for c in rep["checks"]:
        val = c.get("max_abs_diff", c.get("min_abs_diff"))
        print(f"{'PASS' if c['pass'] else 'FAIL'}\t{c['name']}\t{val:.3e}")
    for f in rep["faults"]:
        print(f"{'DETECTED' if f['detected'] else 'UNDETECTED'}\tfault:{f['fault']}\t{f['max_abs_diff']:.3e}")
    print(f"CHECKS\t{rep['checks_passed']}/{rep['checks_total']}\tFAULTS-DETECTED\t{rep['faults_detected']}/{rep['faults_total']}"
          f"\tmodel={rep['model']} layers={rep['layers']} L={rep['seq_len']} dtype={rep['dtype']} oracle={rep['oracle']} {rep['seconds']}s")
    if spare:
        print(f"VOCAB\tembedding_rows={spare['embedding_rows']}\ttokenizer_len={spare['tokenizer_len']}\tspare_rows={spare['spare_rows']}")
    ok = rep["checks_passed"] == rep["checks_total"] and rep["faults_detected"] == rep["faults_total"]
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
