"""Host-side pieces of the benchmarks: the clock / throttle summary that every timed result
carries, and the kernel-family grouping of the step profiler. CPU only."""

from dllm_qwen38_b200.bench.step_profile import FAMILIES, family
from dllm_qwen38_b200.utils.clocks import ClockSampler, summarize

HEADER_FREE_ROWS = """\
0, 1590, 1965, 978.12, 0x0000000000000004, Not Active, Not Active, Not Active, Active
0, 1575, 1965, 990.40, 0x0000000000000004, Not Active, Not Active, Not Active, Active
0, 1605, 1965, 985.00, 0x0000000000000004, Not Active, Not Active, Not Active, Active
0, 345, 1965, 120.00, 0x0000000000000001, Not Active, Not Active, Not Active, Not Active
"""


def test_clock_summary_takes_the_busy_median_and_active_reasons():
    s = summarize(HEADER_FREE_ROWS)
    # the idle sample (345 MHz, below half the peak) is left out of the median under load
    assert s["sm_mhz"] == 1590.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["samples"] == 4 and s["power_w_max"] == 990.4


def test_clock_summary_reports_thermal_reasons_and_empty_input():
    row = "0, 1200, 1965, 700, 0x40, Not Active, Active, Not Active, Not Active\n"
    assert summarize(row)["reasons"] == ["hw_thermal_slowdown"]
    assert summarize("")["reasons"] == ["no samples"]
    assert summarize("garbage\n0, n/a, n/a, n/a, x, a, b, c, d\n")["sm_mhz"] is None


def test_clock_sampler_without_nvidia_smi(monkeypatch):
    import shutil

    monkeypatch.setattr(shutil, "which", lambda name: None)
    s = ClockSampler().start()
    assert s.stop()["reasons"] == ["nvidia-smi unavailable"]


def test_step_profile_families():
    assert family("void bdllm::gemm2_kernel<3, false, false, 512>(...)") == "GEMM (tcgen05)"
    assert family("gdn::bwd_chunk_tc_kernel(...)") == "state-fork GDN"
    assert family("bdllm::out_gate_bwd_kernel(...)") == "attention"
    assert family("bdllm::colsum_kernel(...)") == "norms"
    assert family("void at::native::vectorized_elementwise_kernel<...>") == "torch element-wise / copies"
    assert family("something_unknown") == "other"
    # the first matching fragment wins, so each fragment is listed once
    frags = [f for f, _ in FAMILIES]
    assert len(frags) == len(set(frags))


def test_lever_legs_name_real_op_families():
    from dllm_qwen38_b200 import ops
    from dllm_qwen38_b200.bench.levers import LEGS

    names = [n for n, _, _ in LEGS]
    assert names[0] == "native" and len(names) == len(set(names))
    for _, off, opts in LEGS:
        assert set(off) <= set(ops.ALL_OPS), off
        assert set(opts) <= {"checkpointing", "batch_mult"}


def test_step_model_gemm_work_matches_the_bench_flop_count():
    """The speed-of-light model's GEMM FLOPs (all GEMM outputs kept) agree with the FLOPs the
    bench's MFU divides by, less its attention term; not keeping a layer adds its forward again."""
    import importlib.util
    import os

    from dllm_qwen38_b200.bench.step_model import dense_params, step_work
    from dllm_qwen38_b200.config import preset

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_main", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cfg = preset("27b", layers=16)
    L = 4096
    work = step_work(cfg, L, 32, kept=16)
    n_attn = sum(1 for t in cfg.layer_types if t == "full_attention")
    bench_gemm = bench.model_flops_per_step(cfg, L, 1) - 12.0 * cfg.head_dim * cfg.num_attention_heads * L * L * 2 * n_attn
    assert abs(work["GEMM (tcgen05)"][0] / bench_gemm - 1) < 0.01
    fewer = step_work(cfg, L, 32, kept=15)["GEMM (tcgen05)"][0] - work["GEMM (tcgen05)"][0]
    assert fewer == 2 * 4 * L * dense_params(cfg, cfg.layer_types[15])


def test_step_model_gdn_floor_scales_with_gdn_layers():
    from dllm_qwen38_b200.bench.step_model import step_work
    from dllm_qwen38_b200.config import preset

    w16 = step_work(preset("27b", layers=16), 4096, 32, kept=16)["GDN core"]
    w8 = step_work(preset("27b", layers=8), 4096, 32, kept=8)["GDN core"]
    assert 3.4e12 < w16[0] < 3.6e12 and w16[1] > 0
    assert abs(w16[0] / w8[0] - 2.0) < 1e-9 and abs(w16[1] / w8[1] - 2.0) < 1e-9  # 12 vs 6 GDN layers


def test_step_model_sharded_engine_terms():
    from dllm_qwen38_b200.bench.step_model import comm_bytes, step_work
    from dllm_qwen38_b200.config import preset

    cfg = preset("27b", layers=16)
    assert comm_bytes(cfg, 1) == {}
    c2, c8 = comm_bytes(cfg, 2), comm_bytes(cfg, 8)
    ag2, rs2 = c2.values()
    ag8, rs8 = c8.values()
    assert ag2 == 2 * rs2 and ag8 == 2 * rs8
    assert abs(rs8 / rs2 - (7 / 8) / (1 / 2)) < 1e-12  # (N - 1) / N of the bf16 parameter bytes
    assert abs(rs2 - cfg.param_count()) < 1  # half of 2 bytes per parameter arrives at each of 2 GPUs
    one, eight = step_work(cfg, 4096, 32, 16, 1), step_work(cfg, 4096, 32, 16, 8)
    assert eight["AdamW"][1] * 8 == one["AdamW"][1] and eight["GEMM (tcgen05)"] == one["GEMM (tcgen05)"]
