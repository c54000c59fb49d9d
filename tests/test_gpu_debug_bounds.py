"""The debug-bounds build (`_C_dbg`: the same kernels compiled with -DBDLLM_DEBUG_BOUNDS) and the
determinism of the kernels designed to be deterministic.

Debug build, in a child interpreter with BDLLM_DEBUG_BOUNDS=1 (the loader reads it once):
  * a block-diffusion forward + backward of a small hybrid model through the checked kernels
    records no failed check (indices, TMA x alignment, 16-byte vector stores, non-finite epilogue
    values) and matches the normal build's loss;
  * a CE target outside the vocabulary is recorded (line, index = target, limit = vocab) and its
    read skipped (loss NaN). The bad target sits in row 0 of a two-row logits tensor, so even an
    unchecked read of it would stay inside the allocation;
  * a non-finite RMSNorm input row trips the norm's sentinel.
Nothing here faults or waits: every case is an ordinary in-bounds launch.

Determinism: GEMM (both tile shapes), attention forward, state-fork GDN forward, causal conv,
RMSNorm and CE rows run twice on the same inputs and must be bit-equal."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, torch
from dllm_qwen38_b200.ops import _native
C = _native.require()
from dllm_qwen38_b200.config import preset
from dllm_qwen38_b200.models.blockdiff import block_diffusion_forward
from dllm_qwen38_b200.models.qwen35 import build_model
from dllm_qwen38_b200.ops import cuda as Cu
from dllm_qwen38_b200.train.objective import complementary_step_inputs, masked_ce_from_hidden

out = {"module": _native.module_name(), "debug": bool(C.debug_bounds_build())}
dev = "cuda:0"
torch.cuda.set_device(0)
cfg = preset("tiny", hidden_size=256, intermediate_size=512, linear_key_head_dim=64, linear_value_head_dim=64,
             head_dim=64)
model = build_model(cfg, seed=0, device=dev, dtype=torch.bfloat16)
g = torch.Generator(device=dev).manual_seed(0)
x0 = torch.randint(0, cfg.vocab_size - 1, (2, 128), device=dev, generator=g)
x0_2, xt_2, m_2 = complementary_step_inputs(x0, torch.zeros(2, dtype=torch.long, device=dev), 32, cfg.mask_id, g)
ht, _ = block_diffusion_forward(model, x0_2, xt_2, 32, output="hidden")
loss, n = masked_ce_from_hidden(ht, model.lm_head.weight, x0_2, m_2)
loss.backward()
torch.cuda.synchronize()
out["loss"] = float(loss)
out["clean"] = [list(r) for r in _native.bounds_report(True)]
out["error_word"] = int(C.read_error_word(True))

V = 1024
logits = torch.randn(2, V, device=dev).bfloat16()
tgt = torch.tensor([V + 5, 3], device=dev)
lo = C.ce_rows_(logits, tgt)
torch.cuda.synchronize()
out["ce_loss"] = [float(v) for v in lo]
out["ce"] = [list(r) for r in _native.bounds_report(True)]

x = torch.randn(4, 256, device=dev).bfloat16()
x[2, 7] = float("nan")
C.rmsnorm_fwd(x, torch.ones(256, device=dev), 1e-6)
torch.cuda.synchronize()
out["norm"] = [list(r) for r in _native.bounds_report(True)]
print("RESULT " + json.dumps(out))
"""


def _child(debug: bool) -> dict:
    env = dict(os.environ, BDLLM_DEBUG_BOUNDS="1" if debug else "0", PYTHONPATH=ROOT)
    p = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]
    line = [ln for ln in p.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


def test_debug_bounds_build_records_and_skips():
    if not os.path.exists(os.path.join(ROOT, "dllm_qwen38_b200")) or not any(
            f.startswith("_C_dbg") for f in os.listdir(os.path.join(ROOT, "dllm_qwen38_b200"))):
        pytest.fail("the debug-bounds extension _C_dbg is not built (setup.py build_ext --inplace)")
    dbg, rel = _child(True), _child(False)
    assert dbg["module"] == "_C_dbg" and dbg["debug"], dbg
    assert rel["module"] == "_C" and not rel["debug"], rel
    # a clean run trips nothing and computes what the normal build computes
    assert dbg["clean"] == [] and dbg["error_word"] == 0, dbg
    assert abs(dbg["loss"] - rel["loss"]) <= 1e-3 * max(1.0, abs(rel["loss"])), (dbg["loss"], rel["loss"])
    # the out-of-range target: recorded in misc.cu with (index, limit) = (V + 5, V), read skipped
    assert len(dbg["ce"]) == 1, dbg["ce"]
    f, line, idx, lim, count = dbg["ce"][0]
    assert f.endswith("misc.cu") and idx == 1024 + 5 and lim == 1024 and count == 1, dbg["ce"]
    assert dbg["ce_loss"][0] != dbg["ce_loss"][0] and dbg["ce_loss"][1] == dbg["ce_loss"][1]  # NaN, finite
    # the NaN row: the norm's sentinel, index = row 2
    assert len(dbg["norm"]) == 1 and dbg["norm"][0][0].endswith("norm.cu") and dbg["norm"][0][2] == 2, dbg["norm"]
    # the normal build records nothing
    assert rel["clean"] == [] and rel["ce"] == [] and rel["norm"] == []


def _twice(fn):
    a = fn()
    torch.cuda.synchronize()
    b = fn()
    torch.cuda.synchronize()
    return a, b


def _bit_equal(a, b):
    if isinstance(a, (tuple, list)):
        return all(_bit_equal(x, y) for x, y in zip(a, b))
    return torch.equal(a.view(torch.uint8) if a.dtype != torch.bool else a, b.view(torch.uint8) if b.dtype != torch.bool else b)


def test_deterministic_kernels_are_bit_equal():
    from dllm_qwen38_b200.ops import cuda as Cu

    torch.manual_seed(0)
    dev = "cuda"
    x = torch.randn(1000, 1536, device=dev).bfloat16()
    w = torch.randn(2304, 1536, device=dev).bfloat16() * 0.05
    cases = {"gemm": lambda: Cu.gemm_nt(x, w)}
    B, L, Hq, Hk, D = 1, 256, 8, 2, 128
    q = torch.randn(B, 2 * L, Hq, D, device=dev).bfloat16()
    k = torch.randn(B, 2 * L, Hk, D, device=dev).bfloat16()
    v = torch.randn(B, 2 * L, Hk, D, device=dev).bfloat16()
    cases["attn_fwd"] = lambda: Cu._C.attn_fwd(q, k, v, L, 32, D ** -0.5, False)
    Hv, Dg = 4, 128
    gq = torch.nn.functional.normalize(torch.randn(B, 2 * L, 2, Dg, device=dev), dim=-1).bfloat16()
    gk = torch.nn.functional.normalize(torch.randn(B, 2 * L, 2, Dg, device=dev), dim=-1).bfloat16()
    gv = torch.randn(B, 2 * L, Hv, Dg, device=dev).bfloat16()
    gg = -torch.rand(B, 2 * L, Hv, device=dev) * 0.5
    gb = torch.rand(B, 2 * L, Hv, device=dev)
    cases["gdn_fwd"] = lambda: Cu.gdn_core_blockdiff(gq, gk, gv, gg, gb, L, 32, 64, "fork")
    raw = torch.randn(B, 2 * L, 512, device=dev).bfloat16()
    cw = torch.randn(512, 4, device=dev) * 0.3
    cases["conv"] = lambda: Cu.conv_blockdiff(raw, cw, L, 32, "fork")
    nx = torch.randn(300, 1024, device=dev).bfloat16()
    nw = torch.randn(1024, device=dev).bfloat16() * 0.1
    cases["rmsnorm"] = lambda: Cu.rmsnorm(nx, nw, 1e-6)
    lg = torch.randn(64, 4096, device=dev).bfloat16()
    tg = torch.randint(0, 4096, (64,), device=dev)
    cases["ce_rows"] = lambda: (Cu._C.ce_rows_(lg.clone(), tg),)
    with torch.no_grad():
        for name, fn in cases.items():
            a, b = _twice(fn)
            assert _bit_equal(a, b), name
