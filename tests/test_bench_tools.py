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
