"""The no-allocation GDN forward entry point, called through its exported C symbol.

For callers that cannot allocate device memory (hosts that reserve all of a GPU's memory through
their own allocator, or loops that must not pay cudaMalloc's synchronisation), the library exports
`bdllm_gdn_forward_noalloc`, which takes caller-owned inputs and outputs and draws its working
memory from a fixed array inside the library. These tests call it through ctypes and compare each
result with the regular (allocating) entry point, which runs the same deterministic kernels, so the
outputs must be bit-identical. The file name sorts last so that a run stopping at the first failure
has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, BAD_ARGUMENT, TOO_LARGE = 0, 1, 2


def _lib():
    from dllm_qwen38_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.bdllm_gdn_forward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return _C, fn


def _inputs(B, L, Hk, Hv, D, seed, packed=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T2 = 2 * L
    if packed:  # q | k | v in one row, as the fused input projection writes them
        mixed = torch.randn(B, T2, 2 * Hk * D + Hv * D, device="cuda", dtype=torch.bfloat16, generator=g)
        q = mixed[..., : Hk * D].reshape(B, T2, Hk, D)
        k = mixed[..., Hk * D : 2 * Hk * D].reshape(B, T2, Hk, D)
        v = mixed[..., 2 * Hk * D :].reshape(B, T2, Hv, D)
    else:  # three separate buffers (q and k with token stride Hk * D)
        q = torch.randn(B, T2, Hk, D, device="cuda", dtype=torch.bfloat16, generator=g)
        k = torch.randn(B, T2, Hk, D, device="cuda", dtype=torch.bfloat16, generator=g)
        v = torch.randn(B, T2, Hv, D, device="cuda", dtype=torch.bfloat16, generator=g)
    gate = -torch.rand(B, T2, Hv, device="cuda", generator=g) * 0.5
    beta = torch.rand(B, T2, Hv, device="cuda", generator=g)
    return q, k, v, gate, beta


def _call(fn, q, k, v, gate, beta, o, B, L, Hk, Hv, D, block, *, q_ptr=None):
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(q.data_ptr() if q_ptr is None else q_ptr, k.data_ptr(), v.data_ptr(), q.stride(1), v.stride(1),
            gate.data_ptr(), beta.data_ptr(), o.data_ptr(), B, L, Hk, Hv, D, block, stream, err, len(err))
    return rc, err.value.decode()


def _check(C, fn, B, L, block, Hk, Hv, D, seed, packed=True):
    q, k, v, gate, beta = _inputs(B, L, Hk, Hv, D, seed, packed)
    ref_o = C.gdn_fwd(q, k, v, gate, beta, L, block, False)[0]
    o = torch.full((B, 2 * L, Hv, D), float("nan"), device="cuda", dtype=torch.bfloat16)
    rc, msg = _call(fn, q, k, v, gate, beta, o, B, L, Hk, Hv, D, block)
    torch.cuda.synchronize()
    assert rc == OK, msg
    assert torch.equal(o, ref_o), float((o.float() - ref_o.float()).abs().max())


@pytest.mark.parametrize("B,L,block,Hk,Hv,D", [(2, 64, 16, 2, 4, 32), (1, 128, 32, 2, 6, 128),
                                                (2, 96, 32, 1, 2, 16), (1, 64, 8, 2, 4, 64)])
def test_noalloc_matches_allocating_entry_point_twice(B, L, block, Hk, Hv, D):
    C, fn = _lib()
    for call in range(2):  # the second call reuses scratch left by the first
        _check(C, fn, B, L, block, Hk, Hv, D, seed=10 + call)


def test_noalloc_small_call_after_a_large_one_and_separate_q_k_buffers():
    C, fn = _lib()
    _check(C, fn, 1, 512, 32, 4, 8, 128, seed=1)  # fills half of the scratch array
    _check(C, fn, 1, 32, 16, 1, 2, 32, seed=2, packed=False)  # a smaller problem over stale scratch
    _check(C, fn, 1, 512, 32, 4, 8, 128, seed=3, packed=False)


def test_noalloc_rejects_bad_arguments_without_launching():
    _, fn = _lib()
    B, L, block, Hk, Hv, D = 1, 64, 32, 2, 4, 32
    q, k, v, gate, beta = _inputs(B, L, Hk, Hv, D, seed=0)
    o = torch.zeros(B, 2 * L, Hv, D, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    cases = [
        dict(D=48),  # unsupported head dim
        dict(block=24),  # block does not divide L
        dict(block=64),  # block above 32
        dict(Hv=3),  # Hv not a multiple of Hk
        dict(q_ptr=q.data_ptr() + 2),  # q offset by one bf16 element: not 16-byte aligned
    ]
    for c in cases:
        args = dict(B=B, L=L, Hk=Hk, Hv=Hv, D=D, block=block)
        q_ptr = c.pop("q_ptr", None)
        args.update(c)
        rc, msg = _call(fn, q, k, v, gate, beta, o, args["B"], args["L"], args["Hk"], args["Hv"], args["D"],
                        args["block"], q_ptr=q_ptr)
        assert rc == BAD_ARGUMENT and msg, (c, rc, msg)
    torch.cuda.synchronize()
    assert int(o.abs().sum()) == 0  # nothing was written


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    _, fn = _lib()
    B, L, block, Hk, Hv, D = 8, 4096, 32, 16, 48, 128
    t = torch.empty(8, device="cuda", dtype=torch.bfloat16)
    f = torch.empty(8, device="cuda")
    err = ctypes.create_string_buffer(256)
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), 2 * Hk * D + Hv * D, 2 * Hk * D + Hv * D, f.data_ptr(),
            f.data_ptr(), t.data_ptr(), B, L, Hk, Hv, D, block, torch.cuda.current_stream().cuda_stream, err, 256)
    assert rc == TOO_LARGE and b"scratch" in err.value
