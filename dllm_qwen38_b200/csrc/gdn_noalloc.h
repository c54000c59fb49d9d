// No-allocation entry point for the state-fork gated delta rule forward.
//
// This entry point has no counterpart in the reference project; it exists for callers of this
// library that cannot allocate device memory. Examples: a host application that reserves all of a
// GPU's memory up front through its own allocator (a stray cudaMalloc there fails, or fragments a
// pool the application manages), and latency-sensitive loops that must not pay cudaMalloc/cudaFree,
// which can synchronise the device. Such a caller passes its own input and output buffers; the
// temporary working memory the kernels need comes from a fixed array compiled into this library.
//
// Limits and behaviour (see gdn.cu for the implementation):
//   * Scratch is one file-scope __device__ array of BDLLM_GDN_NOALLOC_SCRATCH_BYTES (32 MiB).
//     Every GPU that loads the library holds this array until the process exits.
//   * Problems whose scratch exceeds that size are rejected with BDLLM_NOALLOC_TOO_LARGE; the
//     scratch a call needs is 4 * B * (L / block) * Hv * (4 * block * D + D * D + 1) bytes plus
//     alignment padding (D = head dim, Dk == Dv).
//   * The first call on a device looks up that device's address of the array
//     (cudaGetSymbolAddress) with the device current; make that first call before any stream
//     capture. Later calls on the device only launch kernels.
//   * All calls share the one array and it keeps the last call's contents. Calls whose kernels
//     overlap on the GPU (different streams without ordering, or concurrent host threads) race on
//     it. Nothing in it has to start at zero: every element a call reads was written earlier in
//     the same call.
//   * The call allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine.
//   * Pointer rules: q, k, v and o 16-byte aligned, g and beta 4-byte aligned; anything else is
//     refused with BDLLM_NOALLOC_BAD_ARGUMENT before a launch. q and k may be separate buffers or
//     slices of one packed row; they share the token stride ld_qk (>= Hk * D).
//   * A CUDA error already pending on the calling thread when the call starts is left in place
//     (not consumed) and the call returns BDLLM_NOALLOC_CUDA_ERROR without launching.
//   * Only the main library (_C) exports this symbol; the debug-bounds build (_C_dbg) leaves it
//     out, so loading both still holds one scratch array per GPU.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define BDLLM_GDN_NOALLOC_SCRATCH_BYTES (32u << 20)

enum {
  BDLLM_NOALLOC_OK = 0,
  BDLLM_NOALLOC_BAD_ARGUMENT = 1,  // shape, stride or alignment not supported
  BDLLM_NOALLOC_TOO_LARGE = 2,     // the problem's scratch exceeds the fixed array
  BDLLM_NOALLOC_CUDA_ERROR = 3,    // set-up or launch failed (cudaGetLastError has the code)
};

#ifdef __cplusplus
extern "C" {
#endif

// Forward of the state-fork chunked gated delta rule over the [B, 2L] two-stream layout
// (positions [0, L) the noised stream, [L, 2L) the clean stream), chunk = block.
//   q, k : bf16, element (b, t, h, d) at base + (b * 2L + t) * ld_qk + h * D + d   (Hk heads)
//   v    : bf16, element (b, t, h, d) at base + (b * 2L + t) * ld_v + h * D + d    (Hv heads)
//   g    : fp32 [B, 2L, Hv] log-decay gates;  beta : fp32 [B, 2L, Hv]
//   o    : bf16 [B, 2L, Hv, D] output (written)
// Supported: D in {16, 32, 64, 128}, block <= 32 dividing L, Hv a multiple of Hk, ld_* multiples
// of 8 with ld_qk >= Hk * D and ld_v >= Hv * D. Returns one of the BDLLM_NOALLOC_* codes; on a
// non-zero code `err` (if not null, of `err_len` bytes) receives a one-line reason.
int bdllm_gdn_forward_noalloc(const void* q, const void* k, const void* v, int64_t ld_qk, int64_t ld_v,
                              const float* g, const float* beta, void* o, int B, int L, int Hk, int Hv, int D,
                              int block, cudaStream_t stream, char* err, int err_len);

#ifdef __cplusplus
}
#endif
