"""`python -m dllm_qwen38_b200`: the framework's command lines, one line each."""

from __future__ import annotations

import sys

COMMANDS = (
    ("equivalence", "state-fork equivalence gate with its three faults (exit 0 / 1 / 2)"),
    ("train.single", "single-device block-diffusion training (synthetic rule, random or chat data)"),
    ("train.fsdp_train", "sharded training under torchrun: DCP checkpoints, resume, self-test, REPORT line"),
    ("eval.gsm8k", "GSM8K subset, autoregressive baseline or block-diffusion decoding"),
    ("bench.decode", "decode throughput: native engine, tensor-parallel under torchrun, or the golden decoder"),
    ("bench.kernels", "one kernel against its roofline (gemm, gdn, attn, ce, conv, norms, adamw, ...)"),
    ("bench.levers", "the training step with one native kernel family swapped for torch at a time"),
    ("bench.step_profile", "one training step's device time by kernel family (torch profiler)"),
    ("bench.step_model", "the training step's speed of light by kernel family (no GPU needed)"),
    ("bench.collectives", "fused all-gather / reduce-scatter paths against their roofline (torchrun)"),
    ("ops.kernel_diff", "native GDN kernel against the fp32 reference on a real mixer"),
    ("io.ckpt", "convert a checkpoint of the sharded engine to the reference's per-parameter layout"),
    ("launch", "run any of these on local GPUs with logs and a report"),
    ("weight_space.server", "loopback completion server over the block-diffusion decoder"),
    ("weight_space.bench", "GSM8K-train development runs against that server and their paired comparison"),
)


def main(argv=None) -> int:
    width = max(len(c) for c, _ in COMMANDS)
    print("python -m dllm_qwen38_b200.<command> --help for each; the flagship benchmark is `python bench.py`.\n")
    for cmd, what in COMMANDS:
        print(f"  {cmd:<{width}}  {what}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
