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

from ..infer.golden import generate
from ..models.blockdiff import block_diffusion_forward
from .. import ops
from .objective import complementary_step_inputs, masked_ce_from_hidden
from .optim import MasterAdamW


def synthetic_rule(start: int, n: int, vocab: int, a: int = 7, c: int = 3) -> list:
    """The affine token rule x_{i+1} = (a x_i + c) mod vocab from `start`, n tokens (the
    reference's synthetic task, `train.py:33-38`)."""
    return _affine_rows(torch.tensor([start]), n, vocab, a, c)[0].tolist()


def _affine_rows(starts: torch.Tensor, n: int, vocab: int, a: int = 7, c: int = 3) -> torch.Tensor:
    """[len(starts), n] int64: every row follows the affine rule from its start, all rows at once."""
    cols = [starts.to(torch.int64)]
    for _ in range(n - 1):
        cols.append((cols[-1] * a + c) % vocab)
    return torch.stack(cols, 1)


def synthetic_batches(B: int, L: int, vocab: int, block: int, seed: int):
    """Yields (x0 [B, L], prompt_len [B] = block, valid_len [B] = L) forever: one start id per row
    from a generator seeded with `seed` (the same seed gives the reference's rows), the first
    block as the unscored prompt."""
    g = torch.Generator().manual_seed(seed)
    prompt, valid = torch.full((B,), block), torch.full((B,), L)
    while True:
        yield _affine_rows(torch.randint(0, vocab, (B,), generator=g), L, vocab), prompt, valid


def random_batches(B: int, L: int, vocab: int, seed: int, prompt: int = 0):
    """Uniform random ids (the benchmark's synthetic data): prompt_len = `prompt`, valid = L."""
    g = torch.Generator().manual_seed(seed)
    while True:
        yield torch.randint(0, vocab, (B, L), generator=g), torch.full((B,), prompt), torch.full((B,), L)


# ---------------------------------------------------------------------------- chat data


def _literal_list(text: str):
    """A message list written as a Python literal (single quotes), or None."""
    import ast

    try:
        val = ast.literal_eval(text)
    except (ValueError, SyntaxError):
        return None
    return val if isinstance(val, list) else None


def _messages(row: dict):
    """Normalise one dataset row to a chat message list ending with the assistant turn, or None.

    Accepted shapes: {"messages": [...]}; {"input": <message list, or that list as a Python
    literal string, or a plain user string>, "output": <assistant text>} (the Nemotron SFT rows
    the reference trains on, `train.py:94-111`)."""
    if isinstance(row.get("messages"), list):
        return row["messages"]
    reply = row.get("output")
    if not isinstance(reply, str):
        return None
    turns = row.get("input")
    if isinstance(turns, str) and turns.lstrip().startswith("[{"):
        turns = _literal_list(turns)
        if turns is None:
            return None
    if isinstance(turns, str):
        turns = [{"role": "user", "content": turns}]
    if not isinstance(turns, list):
        return None
    return [*turns, {"role": "assistant", "content": reply}]


def _token_list(encoded) -> list:
    """apply_chat_template may return a list of ids or a mapping holding them."""
    return list(encoded["input_ids"]) if hasattr(encoded, "keys") else list(encoded)


def encode_chat(tokenizer, msgs: list, L: int):
    """(ids truncated to L, prompt token count) for one conversation; None when the prompt alone
    fills L or the reply adds no token (nothing to score)."""
    prompt = _token_list(tokenizer.apply_chat_template(msgs[:-1], tokenize=True, add_generation_prompt=True))
    full = _token_list(tokenizer.apply_chat_template(msgs, tokenize=True))
    if len(prompt) >= L or len(full) <= len(prompt):
        return None
    return full[:L], len(prompt)


def _chat_rows(dataset: str, split: str, tokenizer, L: int, seed: int, streaming: bool):
    """Encoded (ids, prompt_len) rows forever, one shuffled pass of the split after another (pass
    p shuffled with seed + p, 2000-row buffer); yields None at the end of each pass so the batcher
    can tell whether a pass produced anything."""
    from datasets import load_dataset  # optional dependency

    name = "SFT" if "Nemotron" in dataset else None
    p = 0
    while True:
        ds = load_dataset(dataset, name, split=split, streaming=streaming)
        if streaming:
            ds = ds.shuffle(seed=seed + p, buffer_size=2000)
        for row in ds:
            msgs = _messages(row)
            enc = encode_chat(tokenizer, msgs, L) if msgs else None
            if enc is not None:
                yield enc
        yield None
        p += 1


def chat_batches(dataset: str, split: str, tokenizer, B: int, L: int, block: int, seed: int, streaming: bool = True):
    """Cycling chat-data batches (x0 [B, L] right-padded, prompt_len [B], valid_len [B]): the
    prompt tokens stay clean and unscored. Stops with RuntimeError when a whole pass has no usable
    row, or when a second pass still has not filled one batch (the split is too small for B)."""
    pad = tokenizer.pad_token_id if tokenizer.pad_token_id is not None else 0
    x0 = torch.full((B, L), pad, dtype=torch.long)
    plen = torch.zeros(B, dtype=torch.long)
    vlen = torch.zeros(B, dtype=torch.long)
    fill = usable = batches = passes = 0
    for item in _chat_rows(dataset, split, tokenizer, L, seed, streaming):
        if item is None:  # end of a pass
            if usable == 0 or (batches == 0 and passes >= 1):
                raise RuntimeError(f"{dataset}/{split}: not enough usable rows for a batch of {B} "
                                   f"({usable} usable rows, {batches} batches in pass {passes})")
            usable = batches = 0
            passes += 1
            continue
        ids, n_prompt = item
        x0[fill].fill_(pad)
        x0[fill, : len(ids)] = torch.tensor(ids)
        plen[fill], vlen[fill] = n_prompt, len(ids)
        fill += 1
        usable += 1
        if fill == B:
            yield x0.clone(), plen.clone(), vlen.clone()
            fill = 0
            batches += 1


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
    p.add_argument("--gdn", default="native", choices=["native", "auto", "torch", "fla"],
                   help="GDN core: native (= auto) runs the sm_100a kernels on CUDA; torch runs the fp32 torch "
                        "chunked rule on the device (the reference's torch path, for comparison); fla is not "
                        "part of this framework")
    p.add_argument("--attn", default="native", choices=list(ops.ATTN_CHOICES),
                   help="masked attention: native runs the sm_100a kernels; sdpa / eager run torch's "
                        "attention over the boolean mask on the device (for comparison)")
    a = p.parse_args(argv)
    if a.gdn == "fla":
        print("COULD-NOT-MEASURE --gdn fla: fla's Triton kernel is not part of this framework (the native "
              "tcgen05 kernel replaces it); use --gdn native, or --gdn torch for the torch chunked rule",
              file=sys.stderr)
        return 2
    with ops.torch_paths(a.gdn, a.attn):
        return _run(a)


def _run(a) -> int:
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
