"""Block-diffusion decode throughput: generated tokens per second.

    python -m dllm_qwen38_b200.bench.decode [--model 27b] [--batch 1] [--new-tokens 1024]
        [--prompt-len 512] [--impl native|reference] [--layers N]

Config (the inference benchmark config): block 32, sub-block 8, confidence threshold 0.9,
prompts of random ids, random weights (seed 0), bf16, one GPU. The native arm is this repository's
cached decoder (`infer/cached.py`); the reference arm is the reference's own golden decoder
(`decode.py:35-99`, full forward per denoising step, no cache) on an HF `Qwen3_5TextModel` holding
the same random weights, batch rows decoded one after another (the reference decoder is
unbatched). Timed with CUDA events around the whole generation, after one warm-up generation.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="27b")
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--new-tokens", type=int, default=1024)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--sub-block", type=int, default=8)
    p.add_argument("--threshold", type=float, default=0.9)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--engine", default="native", choices=["native", "cached"],
                   help="native: static caches + device commit + CUDA graphs; cached: the torch cached decoder")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--ref-blocks", type=int, default=None,
                   help="reference arm: decode only this many blocks (its per-step cost grows with the prefix, so "
                        "a shorter run overstates its rate)")
    a = p.parse_args(argv)
    sys.path.insert(0, ROOT)
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model

    cfg = preset(a.model, layers=a.layers)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:  # tensor parallel: one process per GPU (torchrun)
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", torch.cuda.current_device()))
        if a.impl != "native":
            raise SystemExit("the reference decoder is single-GPU")
    dev = "cuda"
    g = torch.Generator().manual_seed(a.seed)
    prompts = [torch.randint(0, cfg.mask_id, (a.prompt_len,), generator=g).tolist() for _ in range(a.batch)]
    room = a.block - a.prompt_len % a.block
    n_blocks = 1 if a.new_tokens <= room else 1 + (a.new_tokens - room + a.block - 1) // a.block
    kw = dict(n_blocks=n_blocks, block=a.block, mask_id=cfg.mask_id, threshold=a.threshold, sub_block=a.sub_block)
    if a.impl == "native":
        model = build_model(cfg, seed=a.seed, device=dev, dtype=torch.bfloat16)
    if a.impl == "native" and a.engine == "cached":
        from dllm_qwen38_b200.infer import cached

        def run():
            out = cached.generate(model, prompts, **kw)
            return sum(t.generated for t in out), sum(t.forwards for t in out)
    elif a.impl == "native" and world > 1:
        from dllm_qwen38_b200.infer.tp import TPDecodeEngine

        eng = TPDecodeEngine(model, a.batch, a.prompt_len + (n_blocks + 1) * a.block, a.block,
                             threshold=a.threshold, sub_block=a.sub_block, graphs=not a.no_graphs)
        del model
        torch.cuda.empty_cache()

        def run():
            out = eng.generate(prompts, n_blocks=n_blocks)
            return sum(t.generated for t in out), sum(t.forwards for t in out)
    elif a.impl == "native":
        from dllm_qwen38_b200.infer.engine import DecodeEngine

        eng = DecodeEngine(model, a.batch, a.prompt_len + (n_blocks + 1) * a.block, a.block, threshold=a.threshold,
                           sub_block=a.sub_block, graphs=not a.no_graphs)

        def run():
            out = eng.generate(prompts, n_blocks=n_blocks)
            return sum(t.generated for t in out), sum(t.forwards for t in out)
    else:
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "dllm_qwen38")):
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not installed"}))
            return 0
        sys.path.insert(0, ref_root)
        import dllm_qwen38.gdn as rgdn
        from dllm_qwen38 import decode as rdecode
        from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

        import bench as flagship

        flagship._install_conv_adapter(rgdn)
        c = cfg
        hc = Qwen3_5TextConfig(
            vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
            num_hidden_layers=c.num_hidden_layers, layer_types=list(c.layer_types),
            num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
            head_dim=c.head_dim, linear_num_key_heads=c.linear_num_key_heads,
            linear_num_value_heads=c.linear_num_value_heads, linear_key_head_dim=c.linear_key_head_dim,
            linear_value_head_dim=c.linear_value_head_dim, linear_conv_kernel_dim=c.linear_conv_kernel_dim,
            rms_norm_eps=c.rms_norm_eps, max_position_embeddings=8192,
            rope_parameters={"rope_type": "default", "rope_theta": c.rope_theta, "mrope_section": [11, 11, 10],
                             "partial_rotary_factor": c.partial_rotary_factor},
            attn_implementation="sdpa")
        torch.manual_seed(a.seed)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)  # build in bf16 directly (27B in fp32 would not fit twice)
        try:
            with torch.device(dev):
                hm = Qwen3_5TextModel(hc).eval()
                head = torch.nn.Linear(c.hidden_size, c.vocab_size, bias=False)
        finally:
            torch.set_default_dtype(prev)
        if a.ref_blocks:
            kw["n_blocks"] = min(kw["n_blocks"], a.ref_blocks)

        def run():
            gen = fw = 0
            for pr in prompts:
                tr = rdecode.generate(hm, head, pr, **kw)
                gen += tr.generated
                fw += tr.forwards
            return gen, fw

    if a.impl == "native":
        run()  # warm-up (graph capture, tensor maps)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gen, fw = run()
    e1.record()
    torch.cuda.synchronize()
    s = e0.elapsed_time(e1) / 1e3
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the slowest rank's device time
        s = float(t.item())
        if hasattr(eng, "timing") and os.environ.get("BDLLM_TP_TIMING") == "1":
            print(json.dumps({"rank": rank, "tp_timing_ms": eng.timing()}), flush=True)
        eng.close()
        dist.destroy_process_group()
        if rank != 0:
            return 0
    print(json.dumps({"metric": "dLLM decode tok/s", "value": round(gen / s, 2), "unit": "tok/s", "impl": a.impl, "engine": a.engine if a.impl == "native" else "golden",
                      "generated": gen, "forwards": fw, "seconds": round(s, 3), "batch": a.batch, "n_gpus": world,
                      "parallelism": f"tp{world}" if world > 1 else "single",
                      "config": {"model": a.model, "layers": cfg.num_hidden_layers, "prompt_len": a.prompt_len,
                                 "new_tokens": a.new_tokens, "block": a.block, "sub_block": a.sub_block,
                                 "threshold": a.threshold, "data": "random ids, random weights"}}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
