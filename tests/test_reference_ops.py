"""The fp32 reference ops against independent formulations."""

import torch

from dllm_qwen38_b200.ops import reference as ref


def _gdn_inputs(N=2, T=32, H=3, D=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(N, T, H, D, generator=g) for _ in range(3))
    return q, k, v, -torch.rand(N, T, H, generator=g), torch.rand(N, T, H, generator=g)


def test_chunked_delta_rule_equals_token_recurrence_for_every_chunk_size():
    q, k, v, g, b = _gdn_inputs()
    o1, s1 = ref.recurrent_gated_delta_rule(q, k, v, g, b)
    for c in (32, 16, 8, 4):
        o2, st = ref.chunk_gated_delta_rule(q, k, v, g, b, c, state_every=32)
        assert float((o1 - o2).abs().max()) < 1e-5, c
        assert float((st[:, -1] - s1).abs().max()) < 1e-5, c


def test_mid_chunk_and_multi_chunk_state_snapshots():
    q, k, v, g, b = _gdn_inputs()
    for chunk, every in ((32, 8), (16, 8), (8, 16), (8, 8)):
        _, st = ref.chunk_gated_delta_rule(q, k, v, g, b, chunk, state_every=every)
        assert st.shape[1] == 32 // every
        for i in range(32 // every):
            e = (i + 1) * every
            _, s = ref.recurrent_gated_delta_rule(q[:, :e], k[:, :e], v[:, :e], g[:, :e], b[:, :e])
            assert float((st[:, i] - s).abs().max()) < 1e-5, (chunk, every, i)


def test_initial_state_continues_the_recurrence():
    q, k, v, g, b = _gdn_inputs()
    o_full, _ = ref.recurrent_gated_delta_rule(q, k, v, g, b)
    _, s16 = ref.recurrent_gated_delta_rule(q[:, :16], k[:, :16], v[:, :16], g[:, :16], b[:, :16])
    o2, _ = ref.chunk_gated_delta_rule(q[:, 16:], k[:, 16:], v[:, 16:], g[:, 16:], b[:, 16:], 8, initial_state=s16)
    assert float((o_full[:, 16:] - o2).abs().max()) < 1e-5


def test_conv_fork_equals_explicit_prefix_concat():
    torch.manual_seed(0)
    B, L, C, K, block = 2, 24, 6, 4, 8
    raw = torch.randn(B, 2 * L, C)
    w = torch.randn(C, K)
    y = ref.conv_blockdiff(raw, w, L, block)
    x0 = raw[:, L:]
    assert torch.allclose(y[:, L:], ref.causal_conv_silu(x0, w), atol=1e-6)
    for kb in range(L // block):
        seq = torch.cat([x0[:, : kb * block], raw[:, kb * block : (kb + 1) * block]], 1)
        want = ref.causal_conv_silu(seq, w)[:, -block:]
        assert torch.allclose(y[:, kb * block : (kb + 1) * block], want, atol=1e-6), kb
    y2 = ref.conv_blockdiff(raw, w, L, block, ref.CONV_NOPREFIX)
    assert not torch.allclose(y2[:, block : 2 * block], y[:, block : 2 * block])


def test_complementary_mask_components():
    L, block = 12, 4
    a = ref.complementary_allowed(L, block, "cpu")
    blk = torch.arange(L) // block
    for i in range(L):
        for j in range(L):
            assert bool(a[i, j]) == bool(blk[j] == blk[i])  # M_BD
            assert bool(a[i, L + j]) == bool(blk[j] < blk[i])  # M_OBC
            assert bool(a[L + i, L + j]) == bool(blk[j] <= blk[i])  # M_BC
            assert not bool(a[L + i, j])  # x_0 never sees x_t
    leak = ref.complementary_allowed(L, block, "cpu", leak_xt_prefix=True)
    assert bool(leak[block, 0]) and not bool(a[block, 0])


def test_kernel_diff_refuses_without_the_native_kernel():
    import pytest

    from dllm_qwen38_b200.ops import kernel_diff

    q = torch.zeros(1, 64, 1, 16)
    g = torch.zeros(1, 64, 1)
    with pytest.raises(RuntimeError, match="cannot run"):
        kernel_diff.core_diff(q, q, q, g, g, 32, 32)


def test_no_states_requested_gives_the_same_output_and_no_states():
    """Without `state_every` the chunked rule returns the same output and no snapshots (the
    reference's need_states=False contract, `gdn.py:57,112,118-123`)."""
    q, k, v, g, b = _gdn_inputs()
    o_with, st = ref.chunk_gated_delta_rule(q, k, v, g, b, 8, state_every=8)
    o_without, none = ref.chunk_gated_delta_rule(q, k, v, g, b, 8)
    assert none is None and st is not None
    assert torch.equal(o_with, o_without)
