"""GSM8K harness: scorer, subset, prompt, decode budget, results file and checkpoint restore (CPU)."""

from collections import UserDict

import pytest
import torch

from dllm_qwen38_b200.eval import gsm8k as E

OPEN, CLOSE = E.THINK_OPEN, E.THINK_CLOSE


def test_post_think():
    assert E.post_think("aaa" + CLOSE + "bbb") == "bbb"
    assert E.post_think(OPEN + "t1" + CLOSE + "mid" + CLOSE + "end") == "end"
    assert E.post_think(OPEN + "trace with 17") == ""
    assert E.post_think("plain #### 5") == "plain #### 5"


def test_score_and_accuracy():
    gold = "she has 3 bags\n#### 72"
    text = OPEN + "plan, #### 999" + CLOSE + " final #### 72"
    assert E.score(text, gold) == (True, "72", "####")
    assert E.score(text.replace("#### 72", "#### 71"), gold) == (False, "71", "####")
    a = E.accuracy([(True, "####"), (False, "####"), (None, "none")])
    assert a == {"acc": 0.5, "n": 2, "skipped": 1, "by_method": {"####": 2}}
    assert E.accuracy([]) == {"acc": None, "n": 0, "skipped": 0, "by_method": {}}


def test_extract_pred_edges():
    assert E.extract_pred("so #### 1,234 total") == ("1,234", "####")
    assert E.extract_pred("count #### 18.") == ("18.", "####")
    assert E.extract_pred("owes #### -3") == ("-3", "####")
    assert E.extract_pred("costs #### $3.50") == ("3.50", "####")
    assert E.extract_pred("#### 1 ... #### 77") == ("77", "####")
    assert E.extract_pred("the answer is 42.") == ("42", "last_number")
    assert E.extract_pred("no digits at all?") == ("", "none")
    assert E.extract_pred(OPEN + "5 apples then 12") == ("", "none")
    assert E.extract_pred(OPEN + "5 apples" + CLOSE + "done") == ("", "none")


def test_score_equivalences_and_unparseable_gold():
    assert E.score("#### 1,234", "receipt\n#### 1234")[0] is True
    assert E.score("#### $3.5", "x\n#### 3.50")[0] is True
    assert E.score("#### 4", "no marker")[0] is None
    assert E.score("#### 4", "x\n#### abc")[0] is None
    assert E.gold_value("step\n#### 42") == 42 and E.gold_value("#### $7") == 7 and E.gold_value("####") is None


def test_subset_and_fingerprint():
    n1 = E.subset_indices(1319, 500)
    assert n1 == E.subset_indices(1319, 500) and len(n1) == 500 and n1 == sorted(n1)
    assert 0 <= n1[0] and n1[-1] < 1319
    assert E.subset_indices(1319, 500, seed=1) != n1
    rows = [{"question": f"q{i}"} for i in range(1319)]
    picked = E.subset_rows(rows, 500)
    assert [r["question"] for r in picked] == [f"q{i}" for i in n1]
    demos = [("d1", "a1"), ("d2", "a2")]
    fp = E.subset_fingerprint(picked, demos)
    assert fp == E.subset_fingerprint(picked, demos)
    assert fp != E.subset_fingerprint(picked, demos[:1]) and fp != E.subset_fingerprint(picked[:499], demos)


def test_demos_and_prompt_block():
    train = [{"question": f"q{i}", "answer": f"cot {i}\n#### {i}"} for i in range(50)]
    d1 = E.fewshot_demos(train, 4)
    assert d1 == E.fewshot_demos(train, 4) and len(d1) == 4 and E.fewshot_demos(train, 4, seed=7) != d1
    demos = [("qA", "two steps\n#### 12"), ("qB", "plain")]
    block = E.fewshot_block(demos, {"question": "zzz-live"})
    assert block.count("Question: ") == 3 and block.strip().endswith("Answer:")
    assert "#### 12" in block and "Answer: plain" in block
    assert block.index("zzz-live") > block.index("qB")
    assert E.user_message({"question": "x"}, demos).startswith("Solve the math word problem")


def test_blocks_for_capacity():
    for pl in (0, 1, 7, 8, 15, 32, 33, 1700):
        for mn in (1, 24, 32, 100, 512, 1024, 2000):
            nb = E.blocks_for(mn, pl, 32)
            room = 32 - pl % 32
            assert room + (nb - 1) * 32 >= mn
            assert nb == 1 or room + (nb - 2) * 32 < mn
    assert E.blocks_for(28, 160, 32) == 1 and E.blocks_for(33, 160, 32) == 2 and E.blocks_for(1024, 1700, 32) == 33


def test_prompt_ids_shapes():
    item = {"question": "qq"}
    want = [11, 12, 13]

    class BatchEnc(UserDict):
        pass

    class Tok:
        def __init__(self, ret):
            self.ret = ret

        def apply_chat_template(self, conv, tokenize=True, **kw):
            assert kw.get("add_generation_prompt") is True and kw.get("enable_thinking") is False
            assert conv == [{"role": "user", "content": E.user_message(item, [])}]
            return self.ret

    assert E.prompt_ids(Tok(BatchEnc(input_ids=want, attention_mask=[1, 1, 1])), item, []) == want
    assert E.prompt_ids(Tok(BatchEnc(input_ids=[want])), item, []) == want
    assert E.prompt_ids(Tok({"input_ids": want}), item, []) == want
    assert E.prompt_ids(Tok(want), item, []) == want
    assert E.prompt_ids(Tok(torch.tensor([[31, 32, 33]])), item, []) == [31, 32, 33]
    with pytest.raises(ValueError, match="2 prompt rows"):
        E.prompt_ids(Tok([[21], [22]]), item, [])


def test_cut_at_eos():
    assert E.cut_at_eos([1, 2, 3], {5}) == [1, 2, 3]
    assert E.cut_at_eos([1, 2, 5, 2, 5], {5}) == [1, 2]
    assert E.cut_at_eos([5, 9], {5, 9}) == []


def test_results_file_resumes_and_skips_torn_line(tmp_path):
    p = str(tmp_path / "r.jsonl")
    E.append_result(p, {"idx": 0, "ok": True, "method": "####"})
    E.append_result(p, {"idx": 3, "ok": False, "method": "last_number"})
    with open(p, "a") as f:
        f.write('{"idx": 4, "ok": tr')  # interrupted append
    done = E.read_results(p)
    assert sorted(done) == [0, 3]


def test_load_split_formats(tmp_path):
    import json

    import pyarrow as pa
    import pyarrow.parquet as pq

    rows = [{"question": "a", "answer": "x\n#### 1"}, {"question": "b", "answer": "y\n#### 2"}]
    (tmp_path / "train.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    pq.write_table(pa.Table.from_pylist(rows), str(tmp_path / "test.parquet"))
    tr, te = E.load_gsm8k(str(tmp_path))
    assert tr == rows and te == rows


def test_engine_checkpoint_restores_full_model(tmp_path):
    """A checkpoint of the sharded engine reads back as full parameters under our keys."""
    import copy

    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.io import ckpt
    from dllm_qwen38_b200.models.qwen35 import build_model
    from dllm_qwen38_b200.parallel.fsdp import FSDPTrainer

    cfg = preset("tiny_ref")
    m = build_model(cfg, seed=0)
    ref = copy.deepcopy(m)
    tr = FSDPTrainer(m, block=8, mask_id=cfg.mask_id, lr=1e-3)
    x0 = torch.randint(0, cfg.mask_id, (2, 32), generator=torch.Generator().manual_seed(0))
    tr.step(x0, torch.zeros(2, dtype=torch.long), torch.full((2,), 32, dtype=torch.long))
    ckpt.save_engine(tr.engine, str(tmp_path), 1, 64)
    tensors, step, seq = ckpt.any_dcp_tensors(ckpt.ckpt_path(str(tmp_path), 1), cfg)
    assert (step, seq) == (1, 64)
    full = tr.engine.full_state()
    assert set(tensors) == set(full)
    for k in full:
        assert torch.equal(tensors[k], full[k]), k
    ckpt.restore_into(ref, tensors)
    assert torch.equal(ref.lm_head.weight, full["lm_head.weight"])


def test_run_one_dllm_seam():
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model

    torch.set_num_threads(1)
    cfg = preset("tiny_ref")
    model = build_model(cfg, seed=0)

    class Tok:
        eos_token_id = 3

        def decode(self, ids, skip_special_tokens=True):
            return ",".join(str(i) for i in ids)

    ids = [10, 11, 12, 13, 14]
    with torch.inference_mode():
        for decoder in ("cached", "golden"):
            text, meta = E.run_one_dllm(model, Tok(), ids, block=8, threshold=0.9, sub_block=None, max_new=24,
                                        mask_id=cfg.mask_id, eos_id=None, decoder=decoder)
            assert meta["n_blocks"] == 4 and meta["generated"] == 27 and len(meta["steps_per_block"]) == 4
