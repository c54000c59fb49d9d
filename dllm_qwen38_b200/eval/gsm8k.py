"""GSM8K subset evaluation: the same problems, prompt and scorer for the autoregressive baseline
and for the block-diffusion decoder (the measurement behind the reference's stop rule,
`gsm8k_eval.py:1-40`).

Contract kept identical to the reference so that scores are comparable across the two code
bases (the subset, the demos, the prompt text and the scorer are the measurement itself):
  * subset: `random.Random(20260913).sample(range(n_rows), n)`, sorted (`gsm8k_eval.py:61-67`);
    demos: `random.Random(20260914).sample(range(len(train)), shots)` from the TRAIN split
    (`gsm8k_eval.py:152-155`); fingerprint: sha256 over stripped questions with \\x00 after each
    subset question and \\x01 after each demo question, first 16 hex digits (`:70-79`);
  * prompt: one user message = instruction + "Question: ...\\nAnswer: <cot> #### <final>" demos
    + the live question, through the chat template with the generation prompt and thinking off
    (`:155-201`);
  * scoring: text after the last think-close tag (nothing when a trace opened and never closed),
    then the last "#### <number>", else the last number; Decimal equality after stripping "$"
    and ","; an unparseable gold answer is skipped, not wrong (`:85-149`);
  * decode budget: n_blocks = the fewest blocks whose capacity covers max_new (`:207-216`),
    generation cut at the first EOS (`:219-224`);
  * results: one JSONL line per problem keyed by subset position, appended; a rerun skips done
    problems and tolerates a torn last line (`:430-446`).

Differences by design: the dLLM path runs this repository's cached decoder (identical token
stream to the golden decoder; `--decoder golden` selects the no-cache one), restores either a
checkpoint of this repository's sharded engine, a reference FSDP checkpoint, or a safetensors
export; datasets are read from local JSONL/Parquet files (no network).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import random
import re
import time
from decimal import Decimal, InvalidOperation

SUBSET_SEED = 20260913
DEMO_SEED = 20260914
INSTRUCTION = ("Solve the math word problem. Think step by step, then give the final numeric answer "
               "on its own last line as '#### <answer>'.\n\n")
THINK_OPEN = "<" + "think" + ">"
THINK_CLOSE = "<" + "/think" + ">"

# ----------------------------------------------------------------------------- subset


def subset_indices(n_rows: int, n: int, seed: int = SUBSET_SEED) -> list:
    return sorted(random.Random(seed).sample(range(n_rows), min(n, n_rows)))


def subset_rows(rows, n: int, seed: int = SUBSET_SEED) -> list:
    return [rows[i] for i in subset_indices(len(rows), n, seed)]


def subset_fingerprint(items, demos) -> str:
    h = hashlib.sha256()
    for it in items:
        h.update(it["question"].strip().encode() + b"\x00")
    for q, _ in demos:
        h.update(q.strip().encode() + b"\x01")
    return h.hexdigest()[:16]


# ----------------------------------------------------------------------------- scoring


def to_decimal(s: str):
    t = s.strip().strip("$").strip().replace(",", "")
    try:
        return Decimal(t)
    except (InvalidOperation, ValueError):
        return None


def gold_value(answer: str):
    head, sep, tail = answer.rpartition("####")
    return to_decimal(tail) if sep else None


_MARKED = re.compile(r"####\s*\$?\s*([\-0-9.,]+)")
_NUMBER = re.compile(r"(-?\d[\d,]*(?:\.\d+)?)")


def post_think(text: str) -> str:
    """The text after the last think-close tag; "" for a trace that opened and never closed."""
    if THINK_CLOSE in text:
        return text.rpartition(THINK_CLOSE)[2]
    return "" if THINK_OPEN in text else text


def extract_pred(text: str) -> tuple:
    """(number string or "", method in {"####", "last_number", "none"})."""
    body = post_think(text)
    marked = _MARKED.findall(body)
    if marked:
        return marked[-1], "####"
    nums = _NUMBER.findall(body)
    return (nums[-1], "last_number") if nums else ("", "none")


def score(pred_text: str, answer: str) -> tuple:
    """(ok, pred, method); ok is None when the gold answer cannot be parsed (skipped)."""
    gold = gold_value(answer)
    raw, method = extract_pred(pred_text)
    if gold is None:
        return None, raw, method
    p = to_decimal(raw)
    return (p is not None and p == gold), raw, method


def accuracy(results) -> dict:
    scored = [(ok, m) for ok, m in results if ok is not None]
    by_method = {}
    for _, m in scored:
        by_method[m] = by_method.get(m, 0) + 1
    n_ok = sum(1 for ok, _ in scored if ok)
    return {"acc": round(n_ok / len(scored), 4) if scored else None, "n": len(scored),
            "skipped": sum(1 for ok, _ in results if ok is None), "by_method": by_method}


# ----------------------------------------------------------------------------- prompt


def fewshot_demos(train_rows, shots: int, seed: int = DEMO_SEED) -> list:
    pick = random.Random(seed).sample(range(len(train_rows)), shots)
    return [(train_rows[i]["question"], train_rows[i]["answer"]) for i in pick]


def fewshot_block(demos, item) -> str:
    parts = []
    for q, a in demos:
        if "####" in a:
            cot, _, final = a.rpartition("####")
        else:
            cot, final = a.strip(), ""
        parts.append(f"Question: {q}\nAnswer: {cot.strip()} #### {final.strip()}".rstrip())
    parts.append(f"Question: {item['question']}\nAnswer:")
    return "\n\n".join(parts)


def user_message(item, demos) -> str:
    return INSTRUCTION + fewshot_block(demos, item)


def prompt_ids(tok, item, demos) -> list:
    """Chat-templated prompt ids as a flat list of ints, whatever container the tokenizer
    returns (list, nested list, tensor, or a mapping with "input_ids")."""
    out = tok.apply_chat_template([{"role": "user", "content": user_message(item, demos)}], tokenize=True,
                                  add_generation_prompt=True, enable_thinking=False)
    if hasattr(out, "get") and not isinstance(out, (list, tuple)):
        out = out.get("input_ids", out)
    try:
        first = out[0]
    except (TypeError, IndexError, KeyError):
        first = None
    if isinstance(first, (list, tuple)) or (hasattr(first, "dim") and first.dim() > 0):
        if len(out) != 1:
            raise ValueError(f"chat template returned {len(out)} prompt rows for one conversation")
        out = first
    return [int(t) for t in out]


# ----------------------------------------------------------------------------- decode helpers


def blocks_for(max_new: int, prompt_len: int, block: int) -> int:
    """Fewest blocks whose capacity (room in the prompt's last block + whole blocks) >= max_new."""
    room = block - prompt_len % block
    return 1 if max_new <= room else 1 + -(-(max_new - room) // block)


def cut_at_eos(tokens, eos_ids) -> list:
    for i, t in enumerate(tokens):
        if t in eos_ids:
            return list(tokens[:i])
    return list(tokens)


# ----------------------------------------------------------------------------- data


def load_split(path: str) -> list:
    """Rows {"question", "answer"} from a .jsonl / .json / .parquet file."""
    if path.endswith(".parquet"):
        import pyarrow.parquet as pq

        return pq.read_table(path).to_pylist()
    with open(path) as f:
        if path.endswith(".json"):
            return json.load(f)
        return [json.loads(ln) for ln in f if ln.strip()]


def load_gsm8k(data_dir: str) -> tuple:
    def find(split):
        for ext in (".jsonl", ".json", ".parquet"):
            for name in (f"{split}{ext}", f"main/{split}{ext}", f"{split}-00000-of-00001{ext}",
                         f"main/{split}-00000-of-00001{ext}"):
                p = os.path.join(data_dir, name)
                if os.path.exists(p):
                    return p
        raise FileNotFoundError(f"no GSM8K {split} split under {data_dir}")

    return load_split(find("train")), load_split(find("test"))


def read_results(path: str) -> dict:
    done = {}
    if os.path.exists(path):
        with open(path) as f:
            for ln in f:
                try:
                    r = json.loads(ln)
                    done[int(r["idx"])] = r
                except (json.JSONDecodeError, KeyError, ValueError, TypeError):
                    continue  # a torn last line from an interrupted append
    return done


def append_result(path: str, r: dict) -> None:
    with open(path, "a") as f:
        f.write(json.dumps(r) + "\n")


# ----------------------------------------------------------------------------- runners


def run_one_dllm(model, tok, ids, *, block: int, threshold: float, sub_block, max_new: int, mask_id: int,
                 eos_id, decoder: str = "cached"):
    """One problem through the block-diffusion decoder; (text, trace meta)."""
    if decoder == "golden":
        from ..infer.golden import generate
    else:
        from ..infer.cached import generate

    t0 = time.time()
    nb = blocks_for(max_new, len(ids), block)
    tr = generate(model, ids, n_blocks=nb, block=block, mask_id=mask_id, threshold=threshold, sub_block=sub_block,
                  eos_id=eos_id, temperature=0.0)
    gen = cut_at_eos(tr.tokens[len(ids):], {eos_id} if eos_id is not None else set())
    text = tok.decode(gen, skip_special_tokens=True)
    return text, {"forwards": tr.forwards, "generated": tr.generated, "n_blocks": nb,
                  "steps_per_block": tr.steps_per_block, "wall_s": round(time.time() - t0, 1)}


def run_ar_batch(model, tok, ids_list, max_new: int, device: str) -> list:
    """Greedy left-padded AR generation with an HF causal LM; masks built from lengths."""
    import torch

    width = max(len(x) for x in ids_list)
    pad = tok.pad_token_id if tok.pad_token_id is not None else tok.eos_token_id
    ids = torch.full((len(ids_list), width), pad, dtype=torch.long, device=device)
    att = torch.zeros_like(ids)
    for i, x in enumerate(ids_list):
        ids[i, width - len(x):] = torch.tensor(x, device=device)
        att[i, width - len(x):] = 1
    out = model.generate(input_ids=ids, attention_mask=att, max_new_tokens=max_new, do_sample=False, num_beams=1,
                         pad_token_id=pad)
    return [tok.decode(out[i, width:], skip_special_tokens=True) for i in range(len(ids_list))]


def load_dllm_model(model_dir: str, ckpt: str | None, device: str, layers=None):
    """Model weights for the dLLM path: HF safetensors dir, then (optionally) a checkpoint of this
    repository's engine (``step-N`` dir), a reference FSDP checkpoint, or a safetensors export."""
    import torch

    from ..io import ckpt as ck
    from ..io.hf_load import load_model

    model = load_model(model_dir, dtype=torch.bfloat16, device="cpu", layers=layers)
    info = {}
    if ckpt:
        if ckpt.endswith(".safetensors"):
            from safetensors.torch import load_file

            ck.restore_into(model, load_file(ckpt), ctx=ckpt)
        else:
            tensors, step, seq = ck.any_dcp_tensors(ckpt, model.config)
            ck.restore_into(model, tensors, ctx=ckpt)
            info = {"dcp_step": step, "dcp_seq_tokens": seq}
    return model.to(device), info


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="dllm_qwen38_b200.eval.gsm8k", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--mode", required=True, choices=["ar", "dllm"])
    p.add_argument("--model", required=True, help="local HF model dir (config, tokenizer, safetensors)")
    p.add_argument("--data-dir", required=True, help="dir with GSM8K train/test .jsonl/.json/.parquet")
    p.add_argument("--ckpt-dir", default=None)
    p.add_argument("--gstep", type=int, default=None)
    p.add_argument("--ckpt", default=None, help="explicit checkpoint dir or .safetensors (overrides --ckpt-dir)")
    p.add_argument("--n", type=int, default=500)
    p.add_argument("--shots", type=int, default=4)
    p.add_argument("--threshold", type=float, default=0.9)
    p.add_argument("--sub-block", type=int, default=None)
    p.add_argument("--max-new", type=int, default=1024)
    p.add_argument("--block", type=int, default=32)
    p.add_argument("--decoder", default="cached", choices=["cached", "golden"])
    p.add_argument("--ar-batch", type=int, default=8)
    p.add_argument("--limit", type=int, default=0)
    p.add_argument("--max-hours", type=float, default=0.0)
    p.add_argument("--report-every", type=int, default=20)
    p.add_argument("--device", default="cuda")
    p.add_argument("--results-dir", default=None)
    p.add_argument("--out", default=".")
    a = p.parse_args(argv)

    import torch
    from transformers import AutoTokenizer

    from ..train.objective import mask_token_id

    os.makedirs(a.out, exist_ok=True)
    rdir = a.results_dir or a.out
    os.makedirs(rdir, exist_ok=True)
    tok = AutoTokenizer.from_pretrained(a.model)
    train_rows, test_rows = load_gsm8k(a.data_dir)
    demos = fewshot_demos(train_rows, a.shots)
    items = subset_rows(test_rows, a.n)
    fp = subset_fingerprint(items, demos)
    path = os.path.join(rdir, f"{a.mode}-n{a.n}-fp{fp}.jsonl")
    done = read_results(path)
    pending = [(i, it) for i, it in enumerate(items) if i not in done]
    if a.limit:
        pending = pending[: a.limit]
    rep = {"mode": a.mode, "model": a.model, "n_subset": len(items), "shots": a.shots, "subset_fingerprint": fp,
           "results_file": path, "done_before": len(done), "to_run": len(pending),
           "params": {k: getattr(a, k) for k in ("threshold", "sub_block", "max_new", "block", "decoder", "ar_batch",
                                                 "limit", "max_hours")}}
    t0 = time.time()
    deadline = t0 + a.max_hours * 3600 if a.max_hours else None

    def progress(tag):
        acc = accuracy([(r["ok"], r["method"]) for r in done.values()])
        print(f"PROGRESS\t{tag}\t{len(done)}/{len(items)}\tacc={acc['acc']}\tn={acc['n']}\t"
              f"skipped={acc['skipped']}\telapsed_s={time.time() - t0:.0f}", flush=True)

    if a.mode == "ar":
        from transformers import AutoModelForCausalLM

        m = AutoModelForCausalLM.from_pretrained(a.model, dtype=torch.bfloat16).to(a.device).eval()
        tok.padding_side = "left"
        bs = max(1, a.ar_batch)
        with torch.inference_mode():
            for b0 in range(0, len(pending), bs):
                if deadline is not None and time.time() > deadline and b0 > 0:
                    break
                chunk = pending[b0 : b0 + bs]
                ids_list = [prompt_ids(tok, it, demos) for _, it in chunk]
                tb = time.time()
                texts = run_ar_batch(m, tok, ids_list, a.max_new, a.device)
                wall = (time.time() - tb) / len(chunk)
                for (idx, it), ids, text in zip(chunk, ids_list, texts):
                    ok, pred, method = score(text, it["answer"])
                    r = {"idx": idx, "question": it["question"], "prompt_len": len(ids), "pred": pred,
                         "method": method, "ok": ok, "wall_s": round(wall, 2), "max_new": a.max_new}
                    append_result(path, r)
                    done[idx] = r
                progress("AR")
    else:
        from ..io.ckpt import latest_checkpoint

        ckpt = a.ckpt
        if ckpt is None and a.ckpt_dir:
            g = a.gstep if a.gstep is not None else latest_checkpoint(a.ckpt_dir)
            if g is None:
                raise SystemExit(f"no step-* checkpoint in {a.ckpt_dir}")
            ckpt = os.path.join(a.ckpt_dir, f"step-{g:08d}")
        rep["ckpt"] = ckpt
        model, info = load_dllm_model(a.model, ckpt, a.device)
        rep.update(info)
        mid = mask_token_id(model, tok)
        with torch.inference_mode():
            for i, (idx, it) in enumerate(pending):
                if deadline is not None and time.time() > deadline and i > 0:
                    break
                ids = prompt_ids(tok, it, demos)
                text, meta = run_one_dllm(model, tok, ids, block=a.block, threshold=a.threshold, sub_block=a.sub_block,
                                          max_new=a.max_new, mask_id=mid, eos_id=tok.eos_token_id, decoder=a.decoder)
                ok, pred, method = score(text, it["answer"])
                r = {"idx": idx, "question": it["question"], "prompt_len": len(ids), "pred": pred, "method": method,
                     "ok": ok, "wall_s": meta.pop("wall_s"), "trace": meta}
                append_result(path, r)
                done[idx] = r
                if i % a.report_every == 0 or i + 1 == len(pending):
                    progress("DLLM")
    rep.update({"done": len(done), "subset_scored": accuracy([(r["ok"], r["method"]) for r in done.values()]),
                "wall_s": round(time.time() - t0, 1)})
    with open(os.path.join(a.out, "report.json"), "w") as f:
        json.dump(rep, f, indent=1)
    print(f"REPORT\t{json.dumps(rep, default=str)}", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
