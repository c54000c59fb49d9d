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
    a = p.parse_args(argv)
    sys.path.insert(0, ROOT)
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model

    cfg = preset(a.model, layers=a.layers)
    dev = "cuda"
    model = build_model(cfg, seed=a.seed, device=dev, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(a.seed)
    prompts = [torch.randint(0, cfg.mask_id, (a.prompt_len,), generator=g).tolist() for _ in range(a.batch)]
    room = a.block - a.prompt_len % a.block
    n_blocks = 1 if a.new_tokens <= room else 1 + (a.new_tokens - room + a.block - 1) // a.block
    kw = dict(n_blocks=n_blocks, block=a.block, mask_id=cfg.mask_id, threshold=a.threshold, sub_block=a.sub_block)
    if a.impl == "native":
        from dllm_qwen38_b200.infer import cached

        def run():
            out = cached.generate(model, prompts, **kw)
            return sum(t.generated for t in out), sum(t.forwards for t in out)
    else:
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "dllm_qwen38")):
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not installed"}))
            return 0
        sys.path.insert(0, ref_root)
        import dllm_qwen38.gdn as rgdn
        from dllm_qwen38 import decode as rdecode

        sys.path.insert(0, ROOT)
        import bench as flagship

        flagship._install_conv_adapter(rgdn)
        from dllm_qwen38_b200.models.oracle import hf_text_model

        hm = hf_text_model(model.to("cpu", torch.float32)).to(dev, torch.bfloat16)
        head = torch.nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False).to(dev, torch.bfloat16)
        with torch.no_grad():
            head.weight.copy_(model.lm_head.weight.to(dev, torch.bfloat16))
        del model

        def run():
            gen = fw = 0
            for pr in prompts:
                tr = rdecode.generate(hm, head, pr, **kw)
                gen += tr.generated
                fw += tr.forwards
            return gen, fw

    run()  # warm-up
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gen, fw = run()
    e1.record()
    torch.cuda.synchronize()
    s = e0.elapsed_time(e1) / 1e3
    print(json.dumps({"metric": "dLLM decode tok/s", "value": round(gen / s, 2), "unit": "tok/s", "impl": a.impl,
                      "generated": gen, "forwards": fw, "seconds": round(s, 3), "batch": a.batch,
                      "config": {"model": a.model, "layers": cfg.num_hidden_layers, "prompt_len": a.prompt_len,
                                 "new_tokens": a.new_tokens, "block": a.block, "sub_block": a.sub_block,
                                 "threshold": a.threshold, "data": "random ids, random weights"}}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
