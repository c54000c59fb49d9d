"""The state-fork equivalence gate through the sm_100a kernels (bf16), on the 27B layer shapes.

The candidate forward runs on the native kernels only (no torch fallback on the device): the
conv, GDN and attention kernels take the fault flags themselves, so the three deliberate faults
are injected inside the kernels. The oracle is the fp32 per-block recompute on the reference ops
(token-by-token delta rule) on its own fp32 copy of the weights. The gate is the reference's bf16
one (`equivalence.py:163-219` there): every check within 0.25 of the oracle, the reaction check
above 10 x that, and every fault pushing the noised stream beyond 0.25.
"""

import copy

import pytest
import torch

from dllm_qwen38_b200 import ops
from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.equivalence import run
from dllm_qwen38_b200.models.blockdiff import FAULTS
from dllm_qwen38_b200.models.qwen35 import build_model

pytestmark = pytest.mark.gpu

NATIVE_OPS = ("rmsnorm", "linear", "mlp", "gated_rmsnorm", "conv", "gdn_gates", "gdn_core", "attention",
              "qk_norm_rope", "output_gate", "embedding")


def _gate(cfg, block, nblocks, batch=1, seed=0):
    model = build_model(cfg, seed=seed, device="cuda", dtype=torch.bfloat16)
    oracle = copy.deepcopy(model).to("cuda", torch.float32)
    rep = run(model, block=block, nblocks=nblocks, layers=None, tol=0.25, change_floor=2.5, seed=seed,
              device="cuda", oracle_model=oracle, batch=batch)
    impl = ops.last_impl()
    return rep, impl


def _assert_gate(rep, impl):
    for op in NATIVE_OPS:
        if op in rep["candidate_impl"]:
            assert rep["candidate_impl"][op] == "native", (op, rep["candidate_impl"])
            assert impl[op] == "native", (op, impl)  # the fault runs too
    failed = [(c["name"], c.get("max_abs_diff", c.get("min_abs_diff"))) for c in rep["checks"] if not c["pass"]]
    assert failed == [], rep["checks"]
    assert rep["checks"][0]["max_abs_diff"] <= 0.25 and rep["checks"][1]["max_abs_diff"] <= 0.25
    undetected = [(f["fault"], f["max_abs_diff"]) for f in rep["faults"] if not f["detected"]]
    assert undetected == [], rep["faults"]
    assert rep["checks_total"] == 5 and rep["faults_total"] == len(FAULTS) == 3


def test_equivalence_gate_native_kernels_27b_shapes():
    """27B shapes (hidden 5120, GDN 16/48 heads of 128, attention 24/4 of 256, vocab 248320),
    first 4 layers (3 GDN + 1 attention), L 128 = 4 blocks of 32, bf16 on the native kernels."""
    rep, impl = _gate(preset("27b", layers=4), block=32, nblocks=4)
    print({c["name"]: c.get("max_abs_diff", c.get("min_abs_diff")) for c in rep["checks"]},
          {f["fault"]: f["max_abs_diff"] for f in rep["faults"]})
    _assert_gate(rep, impl)


def test_equivalence_gate_native_kernels_block16_batch2():
    """A second block size and batch 2 on the 0.8B layer shapes (GDN 16/16 heads of 128,
    attention 8/2 of 256), 4 layers, 6 blocks of 16."""
    rep, impl = _gate(preset("0.8b", layers=4), block=16, nblocks=6, batch=2, seed=1)
    _assert_gate(rep, impl)
