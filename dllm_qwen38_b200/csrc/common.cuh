// Shared device helpers for the sm_100a kernels: bounded mbarrier waits, TMA tile loads,
// tcgen05 (TMEM alloc / MMA / commit / load), and the device-side error word.
//
// Every spin-wait in this library is bounded by %globaltimer. A wait that expires records an
// error code in the global error word (read by the host through bdllm_error_word()) and returns
// false; the kernel then stops issuing work, drains what it already issued (again bounded),
// frees its TMEM and returns. Nothing here traps.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef BDLLM_WAIT_NS
#define BDLLM_WAIT_NS 4000000000ull  // 4 s: far beyond any legitimate single wait
#endif

namespace bdllm {

// error codes written to the error word (first writer wins)
enum : int {
  ERR_NONE = 0,
  ERR_GEMM_WAIT = 1,
  ERR_GDN_WAIT = 2,
  ERR_ATTN_WAIT = 3,
  ERR_COMM_WAIT = 4,
  ERR_BOUNDS = 5,
};

// The error word lives in one device int allocated by the host (error_word_ptr()); every kernel
// that waits receives its address.
__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

int* error_word_ptr();     // host: lazily allocated device int, per device
void bind_context(int dev);  // host: make the device's primary context current in this thread

// ------------------------------------------------------------------ debug-bounds build
// The `_C_dbg` extension is this library compiled with -DBDLLM_DEBUG_BOUNDS. There,
// BDLLM_CHECK(cond, idx, lim) evaluates an index / alignment condition before an access; a failing
// check records (line, idx, lim) in its translation unit's record (the first failure keeps its
// line, index and limit; every failure is counted) and evaluates to false, so the caller skips the
// access. Nothing traps: a kernel with a skipped TMA load runs into its bounded mbarrier wait and
// returns. The host collects every unit's record through bounds_report(). In the normal build the
// macro is the constant `true` and costs nothing.
struct BoundsRec {
  unsigned long long line, idx, lim, count;
};
using BoundsReader = void (*)(BoundsRec*, bool);
struct BoundsUnit {
  const char* file;
  BoundsReader read;
};
inline BoundsUnit* bounds_units(int* n_out) {  // one registry for the whole shared object
  static BoundsUnit units[32];
  static int n = 0;
  if (n_out == nullptr) return units + (n < 32 ? n++ : 31);
  *n_out = n;
  return units;
}

#ifdef BDLLM_DEBUG_BOUNDS
namespace dbg {
static __device__ BoundsRec g_rec;
static void read_rec(BoundsRec* out, bool reset) {
  cudaMemcpyFromSymbol(out, g_rec, sizeof(BoundsRec));
  if (reset) {
    BoundsRec z{};
    cudaMemcpyToSymbol(g_rec, &z, sizeof(BoundsRec));
  }
}
static const int g_registered = (*bounds_units(nullptr) = BoundsUnit{__BASE_FILE__, &read_rec}, 0);
static __device__ __noinline__ void fail(int line, long long idx, long long lim) {
  if (atomicCAS(&g_rec.line, 0ull, (unsigned long long)line) == 0ull) {
    g_rec.idx = (unsigned long long)idx;
    g_rec.lim = (unsigned long long)lim;
  }
  atomicAdd(&g_rec.count, 1ull);
}
}  // namespace dbg
#define BDLLM_DEBUG_BUILD 1
#define BDLLM_CHECK(cond, idx, lim) \
  ((cond) ? true : (::bdllm::dbg::fail(__LINE__, (long long)(idx), (long long)(lim)), false))
#else
#define BDLLM_DEBUG_BUILD 0
#define BDLLM_CHECK(cond, idx, lim) true
#endif
// index i in [0, n)
#define BDLLM_IDX(i, n) BDLLM_CHECK((long long)(i) >= 0 && (long long)(i) < (long long)(n), (i), (n))

// NaN / Inf sentinel of an epilogue (debug build): true when all n values are finite
__device__ __forceinline__ bool all_finite(const float* v, int n) {
  bool ok = true;
  for (int i = 0; i < n; ++i) ok &= isfinite(v[i]);
  return ok;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false (and records `code` in the
// error word `err`) on timeout, or returns false when `abort` (shared flag) is raised by another warp.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++it & 255u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (globaltimer() - t0 > BDLLM_WAIT_NS) {
        record_error(err, code);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------ TMA
// Every tensor map of this library is bf16: a tiled load's x coordinate must be a multiple of 8
// elements (16 bytes). The debug build checks it and skips a load that breaks it.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  if (!BDLLM_CHECK((x & 7) == 0, x, 8)) return;
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  if (!BDLLM_CHECK((x & 7) == 0, x, 8)) return;
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate)
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive on `bar` once all previously issued tcgen05 async ops of this thread complete
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns -> 32 registers per thread (thread i = lane base + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (tcgen05): start >> 4 in [0,14), LBO >> 4 in [16,30),
// SBO >> 4 in [32,46), constant 1 at bit 46, swizzle mode in [61,64) (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t swz = 2) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)swz << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, M x N tile, operand majors.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

}  // namespace bdllm
