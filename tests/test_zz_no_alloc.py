"""The no-allocation GDN forward entry point, called through its exported C symbol.

For callers that cannot allocate device memory (hosts that reserve all of a GPU's memory through
their own allocator, or loops that must not pay cudaMalloc's synchronisation), the library exports
`bdllm_gdn_forward_noalloc`, which takes caller-owned inputs and outputs and draws its working
memory from a fixed array inside the library. This test calls it twice in a row through ctypes and
compares each result with the regular (allocating) entry point. The file name sorts last so that
a run stopping at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from dllm_qwen38_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.bdllm_gdn_forward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return _C, fn


def _inputs(B, L, Hk, Hv, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T2 = 2 * L
    mixed = torch.randn(B, T2, 2 * Hk * D + Hv * D, device="cuda", dtype=torch.bfloat16, generator=g)
    q = mixed[..., : Hk * D].reshape(B, T2, Hk, D)
    k = mixed[..., Hk * D : 2 * Hk * D].reshape(B, T2, Hk, D)
    v = mixed[..., 2 * Hk * D :].reshape(B, T2, Hv, D)
    gate = -torch.rand(B, T2, Hv, device="cuda", generator=g) * 0.5
    beta = torch.rand(B, T2, Hv, device="cuda", generator=g)
    return mixed, q, k, v, gate, beta


def _call(fn, q, k, v, gate, beta, o, B, L, Hk, Hv, D, block):
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(1), v.stride(1), gate.data_ptr(), beta.data_ptr(),
            o.data_ptr(), B, L, Hk, Hv, D, block, stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("B,L,block,Hk,Hv,D", [(2, 64, 16, 2, 4, 32), (1, 128, 32, 2, 6, 128)])
def test_noalloc_matches_allocating_entry_point_twice(B, L, block, Hk, Hv, D):
    C, fn = _lib()
    for call in range(2):  # the second call reuses scratch left by the first
        mixed, q, k, v, gate, beta = _inputs(B, L, Hk, Hv, D, seed=10 + call)
        ref_o = C.gdn_fwd(q, k, v, gate, beta, L, block, False)[0]
        o = torch.full((B, 2 * L, Hv, D), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc, msg = _call(fn, q, k, v, gate, beta, o, B, L, Hk, Hv, D, block)
        torch.cuda.synchronize()
        assert rc == 0, msg
        rel = float((o.float() - ref_o.float()).norm() / ref_o.float().norm())
        assert rel < 1e-2, (call, rel)


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    _, fn = _lib()
    B, L, block, Hk, Hv, D = 8, 4096, 32, 16, 48, 128
    t = torch.empty(8, device="cuda", dtype=torch.bfloat16)
    f = torch.empty(8, device="cuda")
    err = ctypes.create_string_buffer(256)
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), 2 * Hk * D + Hv * D, 2 * Hk * D + Hv * D, f.data_ptr(),
            f.data_ptr(), t.data_ptr(), B, L, Hk, Hv, D, block, torch.cuda.current_stream().cuda_stream, err, 256)
    assert rc == 2 and b"scratch" in err.value
