"""Single-device block-diffusion training loop (the reference's `train.py`).

Data sources: ``synthetic`` -- a deterministic token rule x_{i+1} = (7 x_i + 3) mod V that the
tiny model must learn and the decoder must then reproduce (`train.py:34-47`); or an HF chat
dataset rendered with the model's chat template (prompt tokens clean and unscored,
`train.py:50-111`; needs the `datasets` package and network access).

Throughput is reported in the reference's unit: unique sequence tokens (batch x L) per second,
not counting the two complementary views or the x_t||x_0 doubling (`train.py:164`).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import torch

from ..config import preset
from ..infer.golden import generate
from ..models.blockdiff import block_diffusion_forward
from ..models.qwen35 import build_model
from .. import ops
from .objective import complementary_step_inputs, masked_ce_from_hidden
from .optim import MasterAdamW


def synthetic_rule(start: int, n: int, vocab: int, a: int = 7, c: int = 3) -> list:
    out, x = [], start
    for _ in range(n):
        out.append(x)
        x = (x * a + c) % vocab
    return out


def synthetic_batches(B: int, L: int, vocab: int, block: int, seed: int):
    """Yields (x0 [B, L], prompt_len [B] = block, valid_len [B] = L) forever."""
    g = torch.Generator().manual_seed(seed)
    while True:
        starts = torch.randint(0, vocab, (B,), generator=g).tolist()
        x0 = torch.tensor([synthetic_rule(s, L, vocab) for s in starts])
        yield x0, torch.full((B,), block), torch.full((B,), L)


def random_batches(B: int, L: int, vocab: int, seed: int, prompt: int = 0):
    """Uniform random ids (the benchmark's synthetic data): prompt_len = `prompt`, valid = L."""
    g = torch.Generator().manual_seed(seed)
    while True:
        yield torch.randint(0, vocab, (B, L), generator=g), torch.full((B,), prompt), torch.full((B,), L)


def _messages(row: dict):
    """Chat rows: a `messages` list, or Nemotron-style `input` (a Python-literal message list or a
    string) plus `output` (`train.py:94-111`)."""
    if isinstance(row.get("messages"), list):
        return row["messages"]
    inp, out = row.get("input"), row.get("output")
    if isinstance(inp, str) and inp.lstrip().startswith("[{"):
        import ast

        try:
            inp = ast.literal_eval(inp)
        except (ValueError, SyntaxError):
            return None
    if isinstance(inp, list) and isinstance(out, str):
        return list(inp) + [{"role": "assistant", "content": out}]
    if isinstance(inp, str) and isinstance(out, str):
        return [{"role": "user", "content": inp}, {"role": "assistant", "content": out}]
    return None


def chat_batches(dataset: str, split: str, tokenizer, B: int, L: int, block: int, seed: int, streaming: bool = True):
    """Cycling chat-data batches (`train.py:50-91`): (x0, prompt_len, valid_len)."""
    from datasets import load_dataset  # optional dependency

    pad = tokenizer.pad_token_id if tokenizer.pad_token_id is not None else 0
    buf_x, buf_p, buf_v = [], [], []
    pass_n = 0
    while True:
        ds = load_dataset(dataset, "SFT" if "Nemotron" in dataset else None, split=split, streaming=streaming)
        if streaming:
            ds = ds.shuffle(seed=seed + pass_n, buffer_size=2000)
        added = yielded = 0
        for row in ds:
            msgs = _messages(row)
            if msgs is None:
                continue
            prompt = tokenizer.apply_chat_template(msgs[:-1], tokenize=True, add_generation_prompt=True)
            full = tokenizer.apply_chat_template(msgs, tokenize=True)
            if hasattr(prompt, "get"):
                prompt, full = prompt.get("input_ids", prompt), full.get("input_ids", full)
            if len(prompt) >= L or len(full) <= len(prompt):
                continue
            ids = list(full[:L])
            valid = len(ids)
            buf_x.append(ids + [pad] * (L - valid))
            buf_p.append(len(prompt))
            buf_v.append(valid)
            added += 1
            if len(buf_x) == B:
                yield torch.tensor(buf_x), torch.tensor(buf_p), torch.tensor(buf_v)
                buf_x, buf_p, buf_v = [], [], []
                yielded += 1
        if added == 0 or (yielded == 0 and pass_n >= 1):
            raise RuntimeError(f"{dataset}/{split}: usable rows can't fill one batch (added {added}, yielded {yielded})")
        pass_n += 1


def train(model, batches, *, block: int, mask_id: int, steps: int, lr: float, device: str, log_every: int = 10,
          seed: int = 0, grad_clip: float = 1.0, checkpointing: bool = False, log=print) -> dict:
    params = model.unique_parameters()
    for p in params:
        p.requires_grad_(True)
    opt = MasterAdamW(params, lr=lr, betas=(0.9, 0.95), weight_decay=0.0)
    gen = torch.Generator(device=device).manual_seed(seed)
    losses, seq_tokens, skipped = [], 0, 0
    if device.startswith("cuda"):
        torch.cuda.reset_peak_memory_stats()
    model.train()
    t0 = time.time()
    for step in range(1, steps + 1):
        x0, prompt_len, valid_len = next(batches)
        x0, prompt_len, valid_len = x0.to(device), prompt_len.to(device), valid_len.to(device)
        x0_2, xt_2, m_2 = complementary_step_inputs(x0, prompt_len, block, mask_id, gen, valid_len)
        ht, _ = block_diffusion_forward(model, x0_2, xt_2, block, output="hidden", checkpointing=checkpointing)
        loss, n = masked_ce_from_hidden(ht, model.lm_head.weight, x0_2, m_2)
        if n == 0:
            skipped += 1  # an averaged nothing is a silent green (`objective.py:60-69`)
            continue
        opt.zero_grad()
        loss.backward()
        opt.step(clip=grad_clip)
        losses.append(float(loss.detach()))
        seq_tokens += x0.numel()
        if step % log_every == 0 or step == steps:
            el = time.time() - t0
            log(f"step {step}\tloss {losses[-1]:.4f}\ttargets {n}\tseq-tok/s {seq_tokens / el:.0f}\telapsed {el:.0f}s")
    model.eval()
    el = time.time() - t0
    return {
        "steps": steps,
        "skipped_steps": skipped,
        "loss_first": losses[0] if losses else None,
        "loss_last": losses[-1] if losses else None,
        "loss_mean_last10": sum(losses[-10:]) / max(1, len(losses[-10:])),
        "seq_tokens": seq_tokens,
        "seq_tokens_per_s": seq_tokens / el if el else 0.0,
        "seconds": el,
        "peak_mem_gib": round(torch.cuda.max_memory_allocated() / 2**30, 2) if device.startswith("cuda") else None,
        "losses": losses,
        "checkpointing": checkpointing,
        "impl": ops.last_impl(),
    }


def synthetic_eval(model, *, block: int, mask_id: int, vocab: int, seed: int, threshold: float, n_prompts: int = 8,
                   n_blocks: int = 2) -> dict:
    """Decode with the golden decoder and score against the rule (`train.py:188-202`)."""
    g = torch.Generator().manual_seed(seed + 12345)
    correct = total = forwards = gen_tokens = 0
    for _ in range(n_prompts):
        start = int(torch.randint(0, vocab, (1,), generator=g))
        truth = synthetic_rule(start, block * (1 + n_blocks), vocab)
        tr = generate(model, truth[:block], n_blocks=n_blocks, block=block, mask_id=mask_id, threshold=threshold)
        out = tr.tokens[block:]
        correct += sum(int(a == b) for a, b in zip(out, truth[block:]))
        total += len(out)
        forwards += tr.forwards
        gen_tokens += tr.generated
    return {"rule_accuracy": correct / total, "generated": total, "forwards": forwards,
            "tokens_per_forward": gen_tokens / forwards}


def save_safetensors(model, path: str) -> None:
    """`model.safetensors` with keys text_model.* / lm_head.* (`train.py:270-276`)."""
    from safetensors.torch import save_file

    state = {f"text_model.{k}": v.detach().cpu().contiguous() for k, v in model.text_model.state_dict().items()}
    state["lm_head.weight"] = model.lm_head.weight.detach().cpu().contiguous().clone()
    save_file(state, path)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="tiny_ref", help="preset name (tiny_ref, tiny, 0.8b, 27b) or an HF checkpoint dir")
    p.add_argument("--data", default="synthetic", help="'synthetic', 'random', or an HF dataset id")
    p.add_argument("--split", default="chat")
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--lr", type=float, default=1e-5)
    p.add_argument("--layers", type=int, default=None)
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    p.add_argument("--dtype", default=None, choices=["float32", "bfloat16"], help="default: bf16 on cuda, fp32 on cpu")
    p.add_argument("--grad-checkpoint", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--threshold", type=float, default=0.9)
    p.add_argument("--out", default=None)
    p.add_argument("--no-eval", action="store_true")
    p.add_argument("--threads", type=int, default=None)
    a = p.parse_args(argv)
    if a.threads:
        torch.set_num_threads(a.threads)
    if a.seq_len % a.block:
        print("COULD-NOT-MEASURE seq-len must be a multiple of block", file=sys.stderr)
        return 2
    dtype = {"float32": torch.float32, "bfloat16": torch.bfloat16}.get(a.dtype) or (
        torch.bfloat16 if a.device.startswith("cuda") else torch.float32)
    try:
        from ..io.hf_load import load_model

        model, tok = load_model(a.model, dtype=dtype, device=a.device, layers=a.layers, seed=a.seed)
    except Exception as e:  # noqa: BLE001 - could-not-measure has its own exit code
        print(f"COULD-NOT-MEASURE model load failed: {type(e).__name__}: {e}", file=sys.stderr)
        return 2
    cfg = model.config
    vocab = cfg.vocab_size
    mask_id = cfg.mask_id if tok is None else len(tok)
    if a.data == "synthetic":
        batches = synthetic_batches(a.batch, a.seq_len, vocab if tok is None else len(tok), a.block, a.seed)
    elif a.data == "random":
        batches = random_batches(a.batch, a.seq_len, mask_id, a.seed)
    else:
        if tok is None:
            print("COULD-NOT-MEASURE a chat dataset needs a tokenizer (HF checkpoint dir)", file=sys.stderr)
            return 2
        batches = chat_batches(a.data, a.split, tok, a.batch, a.seq_len, a.block, a.seed)
    rep = train(model, batches, block=a.block, mask_id=mask_id, steps=a.steps, lr=a.lr, device=a.device, seed=a.seed,
                checkpointing=a.grad_checkpoint)
    rep.update({"model": a.model, "data": a.data, "block": a.block, "seq_len": a.seq_len, "batch": a.batch, "lr": a.lr,
                "device": a.device, "dtype": str(dtype)})
    if a.data == "synthetic" and not a.no_eval:
        rep["eval"] = synthetic_eval(model, block=a.block, mask_id=mask_id, vocab=vocab if tok is None else len(tok),
                                     seed=a.seed, threshold=a.threshold)
    if a.out:
        os.makedirs(a.out, exist_ok=True)
        save_safetensors(model, os.path.join(a.out, "model.safetensors"))
        with open(os.path.join(a.out, "report.json"), "w") as f:
            json.dump(rep, f, indent=1, default=str)
    lf, ll = rep["loss_first"], rep["loss_last"]
    print(f"TRAIN\tsteps {rep['steps']}\tskipped {rep['skipped_steps']}\tloss {lf if lf is None else round(lf, 4)} -> "
          f"{ll if ll is None else round(ll, 4)}\tseq-tok/s {rep['seq_tokens_per_s']:.0f}\tpeak_mem_gib {rep['peak_mem_gib']}\t{rep['seconds']:.0f}s")
    if "eval" in rep:
        e = rep["eval"]
        print(f"EVAL\trule_accuracy {e['rule_accuracy']:.3f}\tgenerated {e['generated']}\ttokens_per_forward {e['tokens_per_forward']:.2f}")
    return 0 if (ll is not None and math.isfinite(ll)) else 1


if __name__ == "__main__":
    sys.exit(main())
