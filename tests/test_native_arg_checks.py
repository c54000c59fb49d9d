"""Host-side argument checks of the native element-wise, norm, conv, CE and optimizer entry points.

The kernels move data in 16-byte vectors and index their inputs by the shapes they are given, so
each wrapper checks that its tensors agree in shape and type before anything is launched (and
copies an input whose view offset breaks the 16-byte alignment). These checks run on the host:
CPU tensors with mismatched shapes must raise the wrapper's error, never reach a kernel. No GPU
is needed.
"""

import pytest
import torch

bf = torch.bfloat16


@pytest.fixture(scope="module")
def C():
    try:
        from dllm_qwen38_b200 import _C
    except ImportError as e:  # the extension is built by the package build; nothing to check without it
        pytest.skip(f"native extension not built: {e}")
    return _C


def z(*shape, dtype=torch.float32):
    return torch.zeros(*shape, dtype=dtype)


CASES = [
    ("out_gate_fwd", lambda C: C.out_gate_fwd(z(4, 8, dtype=bf), z(4, 16, dtype=bf)), "one shape"),
    ("out_gate_bwd", lambda C: C.out_gate_bwd(z(4, 8, dtype=bf), z(4, 8, dtype=bf), z(4, 16, dtype=bf)), "one shape"),
    ("out_gate_bwd dy", lambda C: C.out_gate_bwd(z(3, 8, dtype=bf), z(4, 8, dtype=bf), z(4, 8, dtype=bf)),
     "as many elements"),
    ("dswiglu rows", lambda C: C.dswiglu(z(4, 8, dtype=bf), z(3, 16, dtype=bf)), "rows differ"),
    ("dswiglu width", lambda C: C.dswiglu(z(4, 8, dtype=bf), z(4, 12, dtype=bf)), "shapes"),
    ("swiglu_act", lambda C: C.swiglu_act(z(4, 8, dtype=bf)), "F % 8"),
    ("conv weight", lambda C: C.conv_fwd(z(1, 8, 16, dtype=bf), z(16, 3), 4, 2, 0), "kernel size 4"),
    ("conv length", lambda C: C.conv_fwd(z(1, 6, 16, dtype=bf), z(16, 4), 4, 2, 0), "[B, 2L, C]"),
    ("conv dy", lambda C: C.conv_bwd(z(1, 8, 8, dtype=bf), z(1, 8, 16, dtype=bf), z(16, 4), 4, 2, 0), "conv: dy"),
    ("ce targets", lambda C: C.ce_rows_(z(4, 16, dtype=bf), z(3, dtype=torch.long)), "one target per row"),
    ("ce dtype", lambda C: C.ce_rows_(z(4, 16), z(4, dtype=torch.long)), "bf16 logits"),
    ("adamw lengths", lambda C: C.adamw_step(z(8), z(8, dtype=bf), z(7), z(8), z(8), 1e-3, 0.9, 0.95, 1e-8, 0.0,
                                             1.0, None, 1.0, 1.0), "one length"),
    ("adamw moments", lambda C: C.adamw_step(z(8), z(8, dtype=bf), z(8), z(8, dtype=bf), z(8), 1e-3, 0.9, 0.95,
                                             1e-8, 0.0, 1.0, None, 1.0, 1.0), "moments"),
    ("embed width", lambda C: C.embed_fwd(z(4, dtype=torch.long), z(16, 12, dtype=bf)), "D % 8"),
    ("embed_bwd_sorted", lambda C: C.embed_bwd_sorted(z(16, 8, dtype=bf), z(4, dtype=torch.long),
                                                      z(3, dtype=torch.long), z(4, 8, dtype=bf)), "sorted ids"),
    ("gates heads", lambda C: C.gdn_gates_fwd(z(4, 6, dtype=bf), z(4, 6, dtype=bf), z(5), z(6)), "A_log"),
    ("gates b", lambda C: C.gdn_gates_fwd(z(4, 6, dtype=bf), z(4, 5, dtype=bf), z(6), z(6)), "one shape"),
    ("gates bwd", lambda C: C.gdn_gates_bwd(z(3, 6), z(4, 6), z(4, 6, dtype=bf), z(4, 6, dtype=bf), z(6), z(6)),
     "one shape"),
    ("rmsnorm_bwd", lambda C: C.rmsnorm_bwd(z(4, 16, dtype=bf), z(5, 16, dtype=bf), z(16), 1e-6), "dy of x's size"),
    ("gated z", lambda C: C.gated_rmsnorm_fwd(z(4, 32, dtype=bf), z(3, 32, dtype=bf), z(32), 1e-6), "z of x's size"),
    ("gated bwd", lambda C: C.gated_rmsnorm_bwd(z(3, 32, dtype=bf), z(4, 32, dtype=bf), z(4, 32, dtype=bf), z(32),
                                                1e-6), "dy of x's size"),
    ("qk cos", lambda C: C.qk_norm_rope_fwd(z(1, 4, 2, 16, dtype=bf), z(16), z(4, 3, dtype=bf), z(4, 3, dtype=bf),
                                            1e-6), "R even"),
    ("qk cos rows", lambda C: C.qk_norm_rope_fwd(z(1, 4, 2, 16, dtype=bf), z(16), z(5, 4, dtype=bf),
                                                 z(5, 4, dtype=bf), 1e-6), "[T2, R]"),
    ("qk dout", lambda C: C.qk_norm_rope_bwd(z(1, 4, 2, 8, dtype=bf), z(1, 4, 2, 16, dtype=bf), z(16),
                                             z(4, 4, dtype=bf), z(4, 4, dtype=bf), 1e-6), "dout of src's size"),
]


@pytest.mark.parametrize("name,call,fragment", CASES, ids=[c[0] for c in CASES])
def test_wrapper_rejects_mismatched_arguments(C, name, call, fragment):
    with pytest.raises(RuntimeError) as e:
        call(C)
    assert fragment in str(e.value), (name, str(e.value).splitlines()[0])


def _views():
    """Small tensors laid out like the training step's: the gate and q as strided halves of a
    q|gate projection, the conv input as the leading columns of a wider projection row."""
    qg = z(2, 8, 3, 32, dtype=bf)
    q, gate = torch.split(qg, 16, dim=-1)
    proj = z(2, 16, 48, dtype=bf)
    return q, gate, proj[..., :32], proj[..., 32:38], proj[..., 38:44]


ACCEPTED = [
    ("out_gate_fwd", lambda C, v: C.out_gate_fwd(z(2, 8, 3, 16, dtype=bf), v[1])),
    ("out_gate_bwd", lambda C, v: C.out_gate_bwd(z(2, 8, 3, 16), z(2, 8, 3, 16, dtype=bf), v[1])),
    ("conv_fwd", lambda C, v: C.conv_fwd(v[2], z(32, 4, dtype=bf), 8, 4, 0)),
    ("conv_bwd", lambda C, v: C.conv_bwd(z(2, 16, 32, dtype=bf), v[2], z(32, 4, dtype=bf), 8, 4, 0)),
    ("dswiglu", lambda C, v: C.dswiglu(z(10, 16), z(10, 32, dtype=bf))),
    ("swiglu_act", lambda C, v: C.swiglu_act(z(2, 5, 32, dtype=bf))),
    ("ce_rows_", lambda C, v: C.ce_rows_(z(4, 16, dtype=bf), z(4, dtype=torch.long))),
    ("adamw", lambda C, v: C.adamw_step(z(8), z(8, dtype=bf), z(8, dtype=bf), z(8), z(8), 1e-3, 0.9, 0.95, 1e-8,
                                        0.0, 1.0, z(1), 1.0, 1.0)),
    ("embed_fwd", lambda C, v: C.embed_fwd(z(6, dtype=torch.long), z(16, 8, dtype=bf))),
    ("embed_bwd_sorted", lambda C, v: C.embed_bwd_sorted(z(16, 8, dtype=bf), z(6, dtype=torch.long),
                                                         z(6, dtype=torch.long), z(6, 8, dtype=bf))),
    ("gdn_gates_fwd", lambda C, v: C.gdn_gates_fwd(v[4], v[3], z(6), z(6))),
    ("gdn_gates_bwd", lambda C, v: C.gdn_gates_bwd(z(2, 16, 6), z(2, 16, 6), v[4], v[3], z(6), z(6))),
    ("qk_norm_rope_fwd", lambda C, v: C.qk_norm_rope_fwd(v[0], z(16), z(8, 4, dtype=bf), z(8, 4, dtype=bf), 1e-6)),
    ("rmsnorm_fwd", lambda C, v: C.rmsnorm_fwd(z(2, 16, 32, dtype=bf), z(32), 1e-6)),
    ("rmsnorm_bwd", lambda C, v: C.rmsnorm_bwd(z(2, 16, 32), z(2, 16, 32, dtype=bf), z(32), 1e-6)),
    ("gated_rmsnorm_fwd", lambda C, v: C.gated_rmsnorm_fwd(z(2, 8, 3, 32, dtype=bf), _z_view(), z(32), 1e-6)),
    ("gated_rmsnorm_bwd", lambda C, v: C.gated_rmsnorm_bwd(z(2, 8, 3, 32), z(2, 8, 3, 32, dtype=bf), _z_view(),
                                                          z(32), 1e-6)),
    ("group_sum", lambda C, v: C.group_sum(z(2, 8, 6, 16, dtype=bf), 2)),
]


def _z_view():
    """z as GDN's projection leaves it: [B, T, H, D] columns of a wider row (token stride > H D)."""
    return z(2, 8, 3 * 32 + 40, dtype=bf)[..., 8 : 8 + 3 * 32].reshape(2, 8, 3, 32)


@pytest.mark.parametrize("name,call", ACCEPTED, ids=[c[0] for c in ACCEPTED])
def test_wrapper_accepts_the_step_layouts(C, name, call):
    """Well-formed host tensors with the step's layouts pass every check and only stop at the CUDA
    device guard (these tensors are on the host), so no check rejects what the engine passes."""
    with pytest.raises(RuntimeError) as e:
        call(C, _views())
    assert "CUDA" in str(e.value) and "Impl" in str(e.value), (name, str(e.value).splitlines()[0])


def _gdn_views(B=1, L=64, Hk=2, Hv=4, D=16):
    """q, k, v as the state-fork GDN reads them: head-packed column blocks of the post-conv row
    [B, 2L, 2 Hk D + Hv D]; g, beta fp32 [B, 2L, Hv]."""
    mixed = z(B, 2 * L, 2 * Hk * D + Hv * D, dtype=bf)
    q = mixed[..., : Hk * D].reshape(B, 2 * L, Hk, D)
    k = mixed[..., Hk * D : 2 * Hk * D].reshape(B, 2 * L, Hk, D)
    v = mixed[..., 2 * Hk * D :].reshape(B, 2 * L, Hv, D)
    return q, k, v, z(B, 2 * L, Hv), z(B, 2 * L, Hv)


def _attn_views(B=1, L=64, Hq=4, Hk=2, D=64):
    """q, k normalised copies [B, 2L, H, D]; v a column block of the q|gate, k, v projection row."""
    proj = z(B, 2 * L, 2 * Hq * D + 2 * Hk * D, dtype=bf)
    v = proj[..., 2 * Hq * D + Hk * D :].reshape(B, 2 * L, Hk, D)
    return z(B, 2 * L, Hq, D, dtype=bf), z(B, 2 * L, Hk, D, dtype=bf), v


DEVICE_CHECKED = [
    ("gdn_fwd", lambda C: C.gdn_fwd(*_gdn_views(), 64, 32, False)),
    ("gdn_fwd concat", lambda C: C.gdn_fwd(*_gdn_views(), 64, 32, True)),
    ("gdn_bwd", lambda C: C.gdn_bwd(z(1, 128, 4, 16), *_gdn_views(), z(1, 2, 4, 16, 16), 64, 32, False)),
    ("gdn_rows", lambda C: C.gdn_rows(*_gdn_views(B=2, L=16), z(2, 4, 16, 16), None, 32)),
    ("gdn_fwd_tc", lambda C: C.gdn_fwd_tc(*_gdn_views(L=128, D=128), 128)),
    ("attn_fwd", lambda C: C.attn_fwd(*_attn_views(), 64, 32, 0.125, False)),
    ("attn_bwd", lambda C: C.attn_bwd(z(1, 128, 4, 64), *_attn_views(), z(1, 128, 4, 64, dtype=bf), z(1, 4, 128),
                                      64, 32, 0.125, False)),
    ("attn_prefix", lambda C: C.attn_prefix(z(2, 32, 4, 64, dtype=bf), z(2, 96, 2, 64, dtype=bf),
                                            z(2, 96, 2, 64, dtype=bf), 64, None, 0.125)),
]


@pytest.mark.parametrize("name,call", DEVICE_CHECKED, ids=[c[0] for c in DEVICE_CHECKED])
def test_gdn_and_attention_wrappers_accept_the_step_layouts(C, name, call):
    with pytest.raises(RuntimeError) as e:
        call(C)
    assert "CUDA" in str(e.value) and "Impl" in str(e.value), (name, str(e.value).splitlines()[0])


def _k_with_four_heads():
    """k read from the same row as q (same token stride) but with four heads against q's two."""
    q, _, v, g, b = _gdn_views()
    mixed_row = q.as_strided((1, 128, 128), (q.stride(0), q.stride(1), 1))
    return q, mixed_row[..., 32:96].reshape(1, 128, 4, 16), v, g, b


MISMATCHED = [
    ("gdn k heads", lambda C: C.gdn_fwd(*_k_with_four_heads(), 64, 32, False), "q, k [B, 2L, Hk, Dk]"),
    ("gdn gates", lambda C: C.gdn_fwd(*_gdn_views()[:3], z(1, 128, 3), z(1, 128, 3), 64, 32, False), "g, beta"),
    ("gdn dout", lambda C: C.gdn_bwd(z(1, 64, 4, 16), *_gdn_views(), z(1, 2, 4, 16, 16), 64, 32, False),
     "gdn_bwd: dout"),
    ("gdn states", lambda C: C.gdn_bwd(z(1, 128, 4, 16), *_gdn_views(), z(1, 3, 4, 16, 16), 64, 32, False),
     "gdn_bwd: S_in"),
    ("attn v length", lambda C: C.attn_fwd(*_attn_views()[:2], z(1, 64, 2, 64, dtype=bf), 64, 32, 0.125, False),
     "one batch, length and head dim"),
    ("attn lse", lambda C: C.attn_bwd(z(1, 128, 4, 64), *_attn_views(), z(1, 128, 4, 64, dtype=bf), z(1, 4, 64),
                                      64, 32, 0.125, False), "fp32 lse"),
]


@pytest.mark.parametrize("name,call,fragment", MISMATCHED, ids=[c[0] for c in MISMATCHED])
def test_gdn_and_attention_wrappers_reject_mismatches(C, name, call, fragment):
    with pytest.raises(RuntimeError) as e:
        call(C)
    assert fragment in str(e.value), (name, str(e.value).splitlines()[0])


def test_decode_conv_tail_accepts_the_engine_layout(C):
    """The decode engine's conv input: the conv columns of the in-projection row [B, T, C] (token
    stride wider than C), a bf16 tail [B, 3, C] and fp32 taps [C, 4]."""
    proj = z(2, 32, 64 + 24, dtype=bf)
    with pytest.raises(RuntimeError) as e:
        C.conv_tail(proj[..., :64], z(2, 3, 64, dtype=bf), z(64, 4), True)
    assert "CUDA" in str(e.value) and "Impl" in str(e.value), str(e.value).splitlines()[0]
    with pytest.raises(RuntimeError, match="tail"):
        C.conv_tail(proj[..., :64], z(2, 2, 64, dtype=bf), z(64, 4), True)
