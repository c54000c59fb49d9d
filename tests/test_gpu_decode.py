"""Decode kernels (conv with cached tail, GDN rows from a cached state, attention over a KV cache,
confidence, commit rule) against fp32 references, and the native decode engine against the
torch cached decoder."""

import pytest
import torch

from dllm_qwen38_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _C():
    from dllm_qwen38_b200.ops import _native

    return _native.require()


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def test_conv_tail_matches_reference_and_updates_tail():
    C = _C()
    torch.manual_seed(0)
    B, T, Ch = 3, 32, 256
    raw = torch.randn(B, T, Ch, device="cuda").bfloat16()
    tail = torch.randn(B, 3, Ch, device="cuda").bfloat16()
    w = torch.randn(Ch, 4, device="cuda") * 0.3
    seq = torch.cat([tail, raw], 1).float()
    want = ref.causal_conv_silu(seq, w)[:, 3:]
    t2 = tail.clone()
    y = C.conv_tail(raw, t2, w, False)
    assert _rel(y, want) < 1e-2 and torch.equal(t2, tail)
    y2 = C.conv_tail(raw, t2, w, True)
    assert torch.equal(y, y2) and torch.equal(t2, raw[:, -3:])


@pytest.mark.parametrize("Hk,Hv,D", [(2, 4, 64), (2, 6, 128)])
def test_gdn_rows_from_cached_state(Hk, Hv, D):
    C = _C()
    torch.manual_seed(0)
    B, T = 2, 32
    q = torch.randn(B, T, Hk, D, device="cuda").bfloat16()
    k = torch.randn(B, T, Hk, D, device="cuda").bfloat16()
    v = torch.randn(B, T, Hv, D, device="cuda").bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(B, T, Hv, device="cuda"))
    beta = torch.sigmoid(torch.randn(B, T, Hv, device="cuda"))
    S0 = torch.randn(B, Hv, D, D, device="cuda") * 0.1
    rep = Hv // Hk
    o_ref, st = ref.chunk_gated_delta_rule(q.float().repeat_interleave(rep, 2), k.float().repeat_interleave(rep, 2),
                                           v.float(), g, beta, T, initial_state=S0, state_every=T)
    (o,) = C.gdn_rows(q, k, v, g, beta, S0, None, T)
    assert _rel(o, o_ref) < 2e-2
    S = S0.clone()
    (o2,) = C.gdn_rows(q, k, v, g, beta, S, S, T)  # in place
    assert torch.equal(o, o2)
    assert _rel(S, st[:, -1]) < 2e-2


def test_attn_prefix_over_cache():
    C = _C()
    torch.manual_seed(0)
    B, T, Hq, Hk, D, Tmax, Tk = 2, 32, 6, 2, 128, 256, 160
    q = torch.randn(B, T, Hq, D, device="cuda").bfloat16()
    Kc = torch.randn(B, Tmax, Hk, D, device="cuda").bfloat16()
    Vc = torch.randn(B, Tmax, Hk, D, device="cuda").bfloat16()
    tk = torch.tensor([Tk], dtype=torch.int32, device="cuda")
    o = C.attn_prefix(q, Kc, Vc, 0, tk, D ** -0.5)
    allowed = torch.ones(T, Tk, dtype=torch.bool, device="cuda")
    rep = Hq // Hk
    qh = q.float().transpose(1, 2)
    kh = Kc[:, :Tk].float().transpose(1, 2).repeat_interleave(rep, 1)
    vh = Vc[:, :Tk].float().transpose(1, 2).repeat_interleave(rep, 1)
    want = (torch.softmax(qh @ kh.transpose(-1, -2) * D ** -0.5, -1) @ vh).transpose(1, 2)
    del allowed
    assert _rel(o, want) < 1e-2
    o2 = C.attn_prefix(q, Kc, Vc, Tk, None, D ** -0.5)
    assert torch.equal(o, o2)


def test_confidence_and_commit_rule_match_golden():
    from dllm_qwen38_b200.infer.golden import select_commits

    C = _C()
    torch.manual_seed(0)
    B, T, V = 4, 32, 5000
    conf = torch.empty(B * T, device="cuda")
    pick = torch.empty(B * T, dtype=torch.long, device="cuda")
    lb = (torch.randn(B * T, V, device="cuda") * 3).bfloat16()  # bf16 rows: ties possible
    for rows in (lb, lb[:, :4999]):  # the 16-byte vector path, and the element path (V % 8 != 0)
        C.confidence(rows, conf, pick)
        cm = torch.softmax(rows.float(), -1).max(-1).values
        assert torch.allclose(conf, cm, rtol=1e-4, atol=1e-6)
        assert torch.equal(pick, rows.float().argmax(-1))  # the first index of the maximum
    logits = torch.randn(B * T, V, device="cuda") * 3  # fp32 rows: the argmax is unique
    C.confidence(logits, conf, pick)
    cm, pm = torch.softmax(logits, -1).max(-1)
    assert torch.allclose(conf, cm, rtol=1e-4, atol=1e-6) and torch.equal(pick, pm)
    for sub in (0, 8):
        for thr in (0.05, 0.9):
            masked = torch.rand(B, T, device="cuda") < 0.7
            masked[0] = False  # a finished row
            ids = torch.full((B, T), -1, dtype=torch.long, device="cuda")
            m2, ids2 = masked.clone(), ids.clone()
            fw = torch.zeros(B, dtype=torch.int32, device="cuda")
            left = torch.zeros(B, dtype=torch.int32, device="cuda")
            C.commit(conf, pick, m2, ids2, thr, sub, fw, left)
            for r in range(B):
                if not bool(masked[r].any()):
                    assert int(fw[r]) == 0 and int(left[r]) == 0 and torch.equal(m2[r], masked[r])
                    continue
                commit, pk = select_commits(logits[r * T : (r + 1) * T], masked[r], thr, sub or None, 0.0)
                assert torch.equal(m2[r], masked[r] & ~commit), (r, sub, thr)
                assert torch.equal(ids2[r][commit], pk[commit])
                assert int(fw[r]) == 1 and int(left[r]) == int((masked[r] & ~commit).sum())


def _small_model():
    from dllm_qwen38_b200.config import preset
    from dllm_qwen38_b200.models.qwen35 import build_model

    cfg = preset("tiny", hidden_size=256, intermediate_size=512, linear_key_head_dim=64, linear_value_head_dim=64,
                 head_dim=64)
    return build_model(cfg, seed=0, device="cuda", dtype=torch.bfloat16)


def test_engine_block_pass_matches_cached_decoder():
    from dllm_qwen38_b200.infer import cached
    from dllm_qwen38_b200.infer.engine import DecodeEngine

    model = _small_model()
    cfg = model.config
    B, T = 2, 32
    g = torch.Generator(device="cuda").manual_seed(1)
    prompt = torch.randint(0, cfg.mask_id, (B, 64), device="cuda", generator=g)
    eng = DecodeEngine(model, B, 256, T, graphs=False)
    eng.prefill(prompt)
    cache = cached.BlockCache()
    with torch.no_grad():
        cached.prefill(model, cache, prompt, T)
        blk = torch.randint(0, cfg.mask_id, (B, T), device="cuda", generator=g)
        eng.ids.copy_(blk)
        eng.masked.zero_()
        eng.masked[:, 10:] = True
        eng._set_block(64)
        h_eng = eng._block_pass(commit=False)
        h_ref = cached.block_pass(model, cache, torch.where(eng.masked, cfg.mask_id, blk), 64, commit=False)
    assert _rel(h_eng.view(B, T, -1), h_ref) < 3e-2


def test_engine_graphs_reproduce_eager_and_accounting():
    from dllm_qwen38_b200.infer.engine import DecodeEngine

    model = _small_model()
    cfg = model.config
    g = torch.Generator().manual_seed(3)
    prompts = torch.randint(0, cfg.mask_id, (2, 40), generator=g).tolist()
    out = {}
    for graphs in (False, True):
        eng = DecodeEngine(model, 2, 256, 32, threshold=0.9, sub_block=8, graphs=graphs)
        out[graphs] = eng.generate(prompts, n_blocks=3)
    for a, b in zip(out[False], out[True]):
        assert a.tokens == b.tokens and a.forwards == b.forwards and a.steps_per_block == b.steps_per_block
        assert a.generated == (32 - 40 % 32) + 2 * 32
        assert a.forwards >= 3
