// State-fork chunked gated delta rule, forward and backward, over the [B, 2L] two-stream layout.
// (Reference: torch ops with triangular solves and a Python chunk loop, `src/dllm_qwen38/gdn.py:48-123`,
// run twice for the fork, `blockdiff.py:159-177`, and differentiated by autograd.)
//
// Math (per chunk of C tokens and one v-head; the torch specification with the same names is
// dllm_qwen38_b200/ops/gdn_chunked.py and is checked against autograd):
//   gam = cumsum(g), Gam_ij = exp(gam_i - gam_j) (i >= j), E = e^gam, F = e^(gam_C - gam)
//   A = strict_lower(beta_i k^_i.k^_j Gam_ij), T = (I + A)^-1
//   U = T diag(beta) V, W = T diag(beta E) k^, V' = U - W S
//   O = diag(E) q^ S + (q^ k^T * Gam * incl) V',  S' = e^gam_C S + (diag(F) k^)^T V'
// Chunk = block here, so the state entering clean chunk k is exactly S_{k-1}, the state a noised
// block k starts from (the state fork).
//
// Kernels:
//   fwd_prep   clean chunks, parallel: U, W, K~ = diag(F) k^, e^gam_C            -> scratch
//   fwd_recur  sequential over chunks, one CTA per (b, head, 32 value columns): S_in[c], V'_c
//   fwd_out    every chunk of both streams, parallel: O (noised blocks do their own UT transform
//              and start from S_in[k] of the clean stream)
//   bwd_noised noised blocks: all input gradients and dS_inj[k] = d(loss)/d(S_in[k])
//   bwd_prep   clean chunks: P^T dO, K~, q~ = diag(E) q^, W, e^gam_C                -> scratch
//   bwd_recur  reverse recurrence: dS_out[c] (gradient of the state after chunk c), dV'_c
//   bwd_chunk  clean chunks, parallel: input gradients
// The per-chunk products run on tensor cores (mma.sync TF32 with fp32 accumulation) when they tile
// into 16 x 32 x 8, and in fp32 on CUDA cores otherwise (small test shapes).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
void make_map_bf16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                   uint32_t box_outer);
void gdn_bwd_recurrence_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                           const at::Tensor& beta, const at::Tensor& dout, int64_t L, __nv_bfloat16* dS_out,
                           float* dVp);
namespace gdn {

constexpr int NT = 512;

struct Args {
  // inputs ([B, 2L, heads, dim] strided views; row stride = token stride)
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ldqk, ldv;  // token strides (elements)
  const float* g;     // [B, 2L, Hv]
  const float* beta;  // [B, 2L, Hv]
  int B, L, Hk, Hv, C, nb;
  float scale;        // Dk^-1/2
  // forward scratch / outputs
  float* U;     // [B, nb, Hv, C, Dv]
  float* W;     // [B, nb, Hv, C, Dk]
  float* Kt;    // [B, nb, Hv, C, Dk]
  float* Ec;    // [B, nb, Hv]
  float* S_in;  // [B, nb, Hv, Dk, Dv]
  float* Vp;    // [B, nb, Hv, C, Dv]
  __nv_bfloat16* o;  // [B, 2L, Hv, Dv]
  int concat;        // 1: one causal run over the 2L sequence (the concat fault), no fork
  const float* S0;   // optional [B, Hv, Dk, Dv] state before the first chunk (decode rows)
  float* S_final;    // optional [B, Hv, Dk, Dv] state after the last chunk (may alias S0)
  // backward
  const __nv_bfloat16* dout;  // [B, 2L, Hv, Dv]
  float* dS_inj;   // [B, nb, Hv, Dk, Dv]
  float* dS_out;   // [B, nb, Hv, Dk, Dv]
  float* dVp;      // [B, nb, Hv, C, Dv]
  float* PtdO;     // [B, nb, Hv, C, Dv]
  float* Qt;       // [B, nb, Hv, C, Dk]
  __nv_bfloat16* dq;  // [B, 2L, Hv, Dk]  (per v-head; GQA sum done by the caller)
  __nv_bfloat16* dk;  // [B, 2L, Hv, Dk]
  __nv_bfloat16* dv;  // [B, 2L, Hv, Dv]
  float* dg;          // [B, 2L, Hv]
  float* dbeta;       // [B, 2L, Hv]
  long long* phase;   // optional: clock64() at phase boundaries of CTA (0, 0) (BDLLM_GDN_PHASES=1)
  float* dS0;         // optional [B, Hv, Dk, Dv]: gradient of the state before the first chunk (rows)
};

// records the SM clock at phase boundary `k` (thread 0 of CTA (0, 0) only; no-op without a buffer)
__device__ __forceinline__ void mark(const Args& a, int k) {
  if (a.phase != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) a.phase[k] = clock64();
}

// ------------------------------------------------------------------ small matmul in smem
// For every output (m, n) of an M x N product sum_k A(m,k) B(k,n), call epi(m, n, value).
// A(m,k) = AT ? A[k*lda + m] : A[m*lda + k];  B(k,n) = BT ? B[n*ldb + k] : B[k*ldb + n].
template <int TM, int TN, bool AT, bool BT, typename Epi>
__device__ __forceinline__ void mm(int M, int N, int K, const float* A, int lda, const float* B, int ldb, Epi epi) {
  const int tiles_n = N / TN, tiles = (M / TM) * tiles_n;
  for (int t = threadIdx.x; t < tiles; t += NT) {
    const int m0 = (t / tiles_n) * TM, n0 = (t % tiles_n) * TN;
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
    for (int kk = 0; kk < K; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = AT ? A[kk * lda + m0 + i] : A[(m0 + i) * lda + kk];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = BT ? B[(n0 + j) * ldb + kk] : B[kk * ldb + n0 + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] += a[i] * b[j];
    }
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) epi(m0 + i, n0 + j, acc[i][j]);
  }
}

// Tensor-core path: each warp owns 16 x 32 output tiles and runs mma.sync m16n8k8 with TF32
// operands (rounded from the fp32 shared tiles, cvt.rna) and fp32 accumulation. Fragment layout
// (g = lane / 4, t = lane % 4): A a0 (g, t) a1 (g+8, t) a2 (g, t+4) a3 (g+8, t+4); B b0 (t, g)
// b1 (t+4, g); C c0 (g, 2t) c1 (g, 2t+1) c2 (g+8, 2t) c3 (g+8, 2t+1).
__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

template <bool AT, bool BT, typename Epi>
__device__ __forceinline__ void mm_tc(int M, int N, int K, const float* A, int lda, const float* B, int ldb, Epi epi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tiles_n = N / 32, tiles = (M / 16) * tiles_n;
  for (int tile = warp; tile < tiles; tile += NT / 32) {
    const int m0 = (tile / tiles_n) * 16, n0 = (tile % tiles_n) * 32;
    float c[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
    for (int k0 = 0; k0 < K; k0 += 8) {
      auto Aget = [&](int m, int k) { return AT ? A[k * lda + m] : A[m * lda + k]; };
      const uint32_t a0 = tf32(Aget(m0 + g, k0 + t)), a1 = tf32(Aget(m0 + g + 8, k0 + t));
      const uint32_t a2 = tf32(Aget(m0 + g, k0 + t + 4)), a3 = tf32(Aget(m0 + g + 8, k0 + t + 4));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + j * 8 + g;
        const uint32_t b0 = tf32(BT ? B[n * ldb + k0 + t] : B[(k0 + t) * ldb + n]);
        const uint32_t b1 = tf32(BT ? B[n * ldb + k0 + t + 4] : B[(k0 + t + 4) * ldb + n]);
        asm volatile(
            "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[j][0]), "+f"(c[j][1]), "+f"(c[j][2]), "+f"(c[j][3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j * 8 + 2 * t;
      epi(m0 + g, n, c[j][0]);
      epi(m0 + g, n + 1, c[j][1]);
      epi(m0 + g + 8, n, c[j][2]);
      epi(m0 + g + 8, n + 1, c[j][3]);
    }
  }
}

#define M_TILES_OK(M, N, K) ((M) % 16 == 0 && (N) % 32 == 0 && (K) % 8 == 0)

// mm_tc over warps [w0, w0 + nw) only (the other warps skip it)
template <bool AT, bool BT, typename Epi>
__device__ __forceinline__ void mm_tc_part(int M, int N, int K, const float* A, int lda, const float* B, int ldb,
                                           Epi epi, int w0, int nw) {
  const int warp = (threadIdx.x >> 5) - w0, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (warp < 0 || warp >= nw) return;
  const int tiles_n = N / 32, tiles = (M / 16) * tiles_n;
  for (int tile = warp; tile < tiles; tile += nw) {
    const int m0 = (tile / tiles_n) * 16, n0 = (tile % tiles_n) * 32;
    float c[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
    for (int k0 = 0; k0 < K; k0 += 8) {
      auto Aget = [&](int m, int k) { return AT ? A[k * lda + m] : A[m * lda + k]; };
      const uint32_t a0 = tf32(Aget(m0 + g, k0 + t)), a1 = tf32(Aget(m0 + g + 8, k0 + t));
      const uint32_t a2 = tf32(Aget(m0 + g, k0 + t + 4)), a3 = tf32(Aget(m0 + g + 8, k0 + t + 4));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + j * 8 + g;
        const uint32_t b0 = tf32(BT ? B[n * ldb + k0 + t] : B[(k0 + t) * ldb + n]);
        const uint32_t b1 = tf32(BT ? B[n * ldb + k0 + t + 4] : B[(k0 + t + 4) * ldb + n]);
        asm volatile(
            "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[j][0]), "+f"(c[j][1]), "+f"(c[j][2]), "+f"(c[j][3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + j * 8 + 2 * t;
      epi(m0 + g, n, c[j][0]);
      epi(m0 + g, n + 1, c[j][1]);
      epi(m0 + g + 8, n, c[j][2]);
      epi(m0 + g + 8, n + 1, c[j][3]);
    }
  }
}

// tensor cores when the shape tiles into 16 x 32 x 8, else fp32 CUDA cores (4x4 register tiles)
template <bool AT, bool BT, typename Epi>
__device__ __forceinline__ void matmul(int M, int N, int K, const float* A, int lda, const float* B, int ldb,
                                       Epi epi) {
  if (M % 16 == 0 && N % 32 == 0 && K % 8 == 0)
    mm_tc<AT, BT>(M, N, K, A, lda, B, ldb, epi);
  else if (M % 4 == 0 && N % 4 == 0)
    mm<4, 4, AT, BT>(M, N, K, A, lda, B, ldb, epi);
  else if (N % 4 == 0)
    mm<1, 4, AT, BT>(M, N, K, A, lda, B, ldb, epi);
  else
    mm<1, 1, AT, BT>(M, N, K, A, lda, B, ldb, epi);
}

// out[m] += sum_n f(m, n, (A B)_mn) for an M x N product. On tensor cores the four lanes that share
// a row reduce with shuffles first, so each warp tile issues one shared atomic per row.
template <bool AT, bool BT, typename F>
__device__ __forceinline__ void matmul_rowsum(int M, int N, int K, const float* A, int lda, const float* B, int ldb,
                                              F f, float* out) {
  if (M % 16 == 0 && N % 32 == 0 && K % 8 == 0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tiles_n = N / 32, tiles = (M / 16) * tiles_n;
    for (int tile = warp; tile < tiles; tile += NT / 32) {
      const int m0 = (tile / tiles_n) * 16, n0 = (tile % tiles_n) * 32;
      float c[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
      for (int k0 = 0; k0 < K; k0 += 8) {
        auto Aget = [&](int m, int k) { return AT ? A[k * lda + m] : A[m * lda + k]; };
        const uint32_t a0 = tf32(Aget(m0 + g, k0 + t)), a1 = tf32(Aget(m0 + g + 8, k0 + t));
        const uint32_t a2 = tf32(Aget(m0 + g, k0 + t + 4)), a3 = tf32(Aget(m0 + g + 8, k0 + t + 4));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int n = n0 + j * 8 + g;
          const uint32_t b0 = tf32(BT ? B[n * ldb + k0 + t] : B[(k0 + t) * ldb + n]);
          const uint32_t b1 = tf32(BT ? B[n * ldb + k0 + t + 4] : B[(k0 + t + 4) * ldb + n]);
          asm volatile(
              "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
              "{%0,%1,%2,%3};"
              : "+f"(c[j][0]), "+f"(c[j][1]), "+f"(c[j][2]), "+f"(c[j][3])
              : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
        }
      }
      float r0 = 0.f, r1 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + j * 8 + 2 * t;
        r0 += f(m0 + g, n, c[j][0]) + f(m0 + g, n + 1, c[j][1]);
        r1 += f(m0 + g + 8, n, c[j][2]) + f(m0 + g + 8, n + 1, c[j][3]);
      }
      r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
      r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
      r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
      r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
      if (t == 0) {
        atomicAdd(&out[m0 + g], r0);
        atomicAdd(&out[m0 + g + 8], r1);
      }
    }
  } else {
    matmul<AT, BT>(M, N, K, A, lda, B, ldb, [&](int m, int n, float x) { atomicAdd(&out[m], f(m, n, x)); });
  }
}

// out[i] += sum_d X[i][d] * Y[i][d] over C rows of D, warp per row
// Two independent products at once, each on half of the warps (for shapes whose tile count is at
// most half the warps, so neither half idles); sequential when a shape does not tile.
template <bool AT1, bool BT1, bool AT2, bool BT2, typename E1, typename E2>
__device__ __forceinline__ void matmul_pair(int M1, int N1, int K1, const float* A1, int lda1, const float* B1,
                                            int ldb1, E1 e1, int M2, int N2, int K2, const float* A2, int lda2,
                                            const float* B2, int ldb2, E2 e2) {
  const bool tc = M1 % 16 == 0 && N1 % 32 == 0 && K1 % 8 == 0 && M2 % 16 == 0 && N2 % 32 == 0 && K2 % 8 == 0;
  if (!tc) {
    matmul<AT1, BT1>(M1, N1, K1, A1, lda1, B1, ldb1, e1);
    matmul<AT2, BT2>(M2, N2, K2, A2, lda2, B2, ldb2, e2);
    return;
  }
  constexpr int H = NT / 64;
  mm_tc_part<AT1, BT1>(M1, N1, K1, A1, lda1, B1, ldb1, e1, 0, H);
  mm_tc_part<AT2, BT2>(M2, N2, K2, A2, lda2, B2, ldb2, e2, H, H);
}

// matmul_rowsum for two products at once (each on half of the warps)
template <bool AT1, bool BT1, bool AT2, bool BT2, typename F1, typename F2>
__device__ __forceinline__ void matmul_rowsum_pair(int M1, int N1, int K1, const float* A1, int lda1, const float* B1,
                                                   int ldb1, F1 f1, float* out1, int M2, int N2, int K2,
                                                   const float* A2, int lda2, const float* B2, int ldb2, F2 f2,
                                                   float* out2) {
  const bool tc = M1 % 16 == 0 && N1 % 32 == 0 && K1 % 8 == 0 && M2 % 16 == 0 && N2 % 32 == 0 && K2 % 8 == 0;
  if (!tc) {
    matmul_rowsum<AT1, BT1>(M1, N1, K1, A1, lda1, B1, ldb1, f1, out1);
    matmul_rowsum<AT2, BT2>(M2, N2, K2, A2, lda2, B2, ldb2, f2, out2);
    return;
  }
  constexpr int H = NT / 64;
  const int lane = threadIdx.x & 31;
  auto row_acc = [&](auto f, float* out) {
    return [&, f, out](int m, int n, float x) {
      // the four lanes of a quad share row m: reduce over the quad, one atomic per row and column pair
      float v = f(m, n, x);
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if ((lane & 3) == 0) atomicAdd(&out[m], v);
    };
  };
  mm_tc_part<AT1, BT1>(M1, N1, K1, A1, lda1, B1, ldb1, row_acc(f1, out1), 0, H);
  mm_tc_part<AT2, BT2>(M2, N2, K2, A2, lda2, B2, ldb2, row_acc(f2, out2), H, H);
}

__device__ __forceinline__ void rowdot(int C, int D, const float* X, int ldx, const float* Y, int ldy, float* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < C; i += NT / 32) {
    float acc = 0.f;
    for (int d = lane; d < D; d += 32) acc += X[i * ldx + d] * Y[i * ldy + d];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[i] += acc;
  }
}

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// token index (into [B, 2L]) of token i of chunk `c` of the given stream.
// stream 0 = noised (x_t, positions [0, L)), stream 1 = clean (x_0, positions [L, 2L)); in concat
// mode stream 1 is the whole 2L sequence run causally (the concat-causal-gdn fault).
__device__ __forceinline__ int64_t tok(const Args& a, int b, int stream, int c, int i) {
  const int64_t t = (int64_t)b * 2 * a.L + ((stream && !a.concat) ? a.L : 0) + (int64_t)c * a.C + i;
  if (!BDLLM_IDX(t, (int64_t)a.B * 2 * a.L)) return 0;  // debug build: recorded, redirected to row 0
  return t;
}

// 16-byte asynchronous global -> shared copies (operand prefetch in the recurrences)
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// ------------------------------------------------------------------ shared-tile strides
// Row strides of the fp32 shared tiles are padded by 4 floats: with that, every TF32 fragment read
// pattern of mm_tc (lanes spanning 8 rows x 4 columns or 4 rows x 8 columns) hits 32 distinct banks.
template <int D>
struct Ld {
  static constexpr int v = D + 4;
};
constexpr int LDC = 36;  // [C][C] tiles (C <= 32)

// ------------------------------------------------------------------ per-chunk loads
// sQ/sK [C][Dk] l2-normalised (q scaled), sV [C][Dv], sgam[C] = cumsum g, sbeta[C].
template <int Dk, int Dv>
__device__ void load_chunk(const Args& a, int b, int stream, int c, int h, float* sQ, float* sK, float* sV,
                           float* sgam, float* sbeta, bool need_q, bool need_v) {
  constexpr int KD = Ld<Dk>::v, VD = Ld<Dv>::v;
  const int C = a.C;
  const int hk = h / (a.Hv / a.Hk);
  for (int idx = threadIdx.x; idx < C * (Dk / 8); idx += NT) {
    const int i = idx / (Dk / 8), d = (idx % (Dk / 8)) * 8;
    const int64_t t = tok(a, b, stream, c, i);
    uint4 kk = *reinterpret_cast<const uint4*>(a.k + t * a.ldqk + hk * Dk + d);
    const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kk);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(k2[e]);
      sK[i * KD + d + 2 * e] = f.x, sK[i * KD + d + 2 * e + 1] = f.y;
    }
    if (need_q) {
      uint4 qq = *reinterpret_cast<const uint4*>(a.q + t * a.ldqk + hk * Dk + d);
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qq);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(q2[e]);
        sQ[i * KD + d + 2 * e] = f.x, sQ[i * KD + d + 2 * e + 1] = f.y;
      }
    }
  }
  if (need_v)
    for (int idx = threadIdx.x; idx < C * (Dv / 8); idx += NT) {
      const int i = idx / (Dv / 8), d = (idx % (Dv / 8)) * 8;
      uint4 vv = *reinterpret_cast<const uint4*>(a.v + tok(a, b, stream, c, i) * a.ldv + h * Dv + d);
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&vv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(v2[e]);
        sV[i * VD + d + 2 * e] = f.x, sV[i * VD + d + 2 * e + 1] = f.y;
      }
    }
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    float gv = 0.f, bv = 0.f;
    if (i < C) {
      const int64_t t = tok(a, b, stream, c, i);
      gv = a.g[t * a.Hv + h];
      bv = a.beta[t * a.Hv + h];
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {  // inclusive prefix sum over the chunk (C <= 32)
      float y = __shfl_up_sync(0xffffffffu, gv, o);
      if (i >= o) gv += y;
    }
    if (i < C) sgam[i] = gv, sbeta[i] = bv;
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int r = warp; r < (need_q ? 2 * C : C); r += NT / 32) {  // l2 normalisation, warp per row
    float* row = (r < C) ? sK + r * KD : sQ + (r - C) * KD;
    float ss = 0.f;
    for (int d = lane; d < Dk; d += 32) ss += row[d] * row[d];
    ss = wsum(ss);
    const float inv = rsqrtf(ss + 1e-6f) * (r < C ? 1.f : a.scale);
    for (int d = lane; d < Dk; d += 32) row[d] *= inv;
  }
  __syncthreads();
}

// sT = (I + A)^-1 with A = strict_lower(beta_i KK_ij Gam_ij); sKK = k^ k^T must be ready.
// All [C][C] tiles use row stride LDC.
__device__ void ut_transform(int C, const float* sKK, const float* sgam, const float* sbeta, float* sA, float* sT) {
  for (int idx = threadIdx.x; idx < C * C; idx += NT) {
    const int i = idx / C, j = idx % C;
    sA[i * LDC + j] = j < i ? sbeta[i] * sKK[i * LDC + j] * __expf(sgam[i] - sgam[j]) : 0.f;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // forward substitution, lane = column of T: the column lives in registers (t[i] for rows i),
    // row i needs sum_{j<i} A_ij t_j: fully unrolled with four independent partial sums, A read as
    // broadcast shared loads. Rows / columns >= C have A = 0 and are not stored.
    const int col = threadIdx.x;
    float t[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
      const float* Ai = sA + i * LDC;
#pragma unroll
      for (int j = 0; j + 3 < i; j += 4) {
        p0 += Ai[j] * t[j];
        p1 += Ai[j + 1] * t[j + 1];
        p2 += Ai[j + 2] * t[j + 2];
        p3 += Ai[j + 3] * t[j + 3];
      }
#pragma unroll
      for (int j = i & ~3; j < i; ++j) p0 += Ai[j] * t[j];
      t[i] = (i < C ? ((i == col) ? 1.f : 0.f) - ((p0 + p1) + (p2 + p3)) : 0.f);
    }
    if (col < C)
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < C) sT[i * LDC + col] = t[i];
  }
  __syncthreads();
}

// ------------------------------------------------------------------ forward smem layout
template <int Dk, int Dv>
struct Smem {
  static constexpr int KD = Ld<Dk>::v, VD = Ld<Dv>::v, MD = (KD > VD ? KD : VD);
  float *Q, *K, *V, *W, *X, *Y, *S, *KK, *A, *T, *P, *gam, *beta;
  __device__ Smem(float* base, int) {
    float* p = base;
    Q = p; p += 32 * KD;
    K = p; p += 32 * KD;
    V = p; p += 32 * VD;
    W = p; p += 32 * KD;
    X = p; p += 32 * MD;
    Y = p; p += 32 * MD;
    S = p; p += Dk * VD;
    KK = p; p += 32 * LDC;
    A = p; p += 32 * LDC;
    T = p; p += 32 * LDC;
    P = p; p += 32 * LDC;
    gam = p; p += 32;
    beta = p; p += 32;
  }
  static constexpr int floats = 3 * 32 * KD + 32 * VD + 2 * 32 * MD + Dk * VD + 4 * 32 * LDC + 64;
};

// ================================================================== forward
// prep for clean chunk c: U, W, K~, Ec to scratch.
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) fwd_prep_kernel(Args a) {
  extern __shared__ float sm[];
  Smem<Dk, Dv> s(sm, a.C);
  constexpr int KD = Ld<Dk>::v, VD = Ld<Dv>::v;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv, C = a.C;
  load_chunk<Dk, Dv>(a, b, 1, c, h, s.Q, s.K, s.V, s.gam, s.beta, false, true);
  matmul<false, true>(C, C, Dk, s.K, KD, s.K, KD, [&](int i, int j, float x) { s.KK[i * LDC + j] = x; });
  __syncthreads();
  ut_transform(C, s.KK, s.gam, s.beta, s.A, s.T);
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  float* U = a.U + base * C * Dv;
  float* Wg = a.W + base * C * Dk;
  float* Kt = a.Kt + base * C * Dk;
  // U = T diag(beta) V ; W = T diag(beta E) k^
  for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
    const int i = idx / Dv, d = idx % Dv;
    s.X[i * VD + d] = s.beta[i] * s.V[i * VD + d];
  }
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk, d = idx % Dk;
    s.Y[i * KD + d] = s.beta[i] * __expf(s.gam[i]) * s.K[i * KD + d];
    Kt[i * Dk + d] = __expf(s.gam[C - 1] - s.gam[i]) * s.K[i * KD + d];
  }
  __syncthreads();
  matmul<false, false>(C, Dv, C, s.T, LDC, s.X, VD, [&](int i, int d, float x) { U[i * Dv + d] = x; });
  matmul<false, false>(C, Dk, C, s.T, LDC, s.Y, KD, [&](int i, int d, float x) { Wg[i * Dk + d] = x; });
  if (threadIdx.x == 0) a.Ec[base] = __expf(s.gam[C - 1]);
}

// sequential state recurrence: CTA per (b, h, 32 value columns). The chunk operands (W, K~ and
// the U columns) are double-buffered: chunk c+1's are copied in (cp.async) while chunk c is
// computed.
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) fwd_recur_kernel(Args a) {
  extern __shared__ float sm[];
  constexpr int KD = Ld<Dk>::v;
  const int C = a.C;
  // buffer k: W and K~ [C][KD] each, then the U columns [C][LDC]
  constexpr int BUF = 2 * 32 * KD + 32 * LDC;
  auto sWb = [&](int k) { return sm + k * BUF; };
  auto sKtb = [&](int k) { return sm + k * BUF + 32 * KD; };
  auto sUb = [&](int k) { return sm + k * BUF + 2 * 32 * KD; };
  float* sVp = sm + 2 * BUF;       // [C][LDC]
  float* sS = sVp + 32 * LDC;      // [Dk][LDC]
  const int bh = blockIdx.x, b = bh / a.Hv, h = bh % a.Hv;
  const int col0 = blockIdx.y * 32;
  const int ncols = min(32, Dv - col0);
  auto prefetch = [&](int c, int buf) {
    const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
    const float* Wg = a.W + base * C * Dk;
    const float* Kt = a.Kt + base * C * Dk;
    const float* U = a.U + base * C * Dv;
    for (int idx = threadIdx.x; idx < C * (Dk / 4); idx += NT) {
      const int i = idx / (Dk / 4), q = (idx % (Dk / 4)) * 4;
      cp16(sWb(buf) + i * KD + q, Wg + i * Dk + q);
      cp16(sKtb(buf) + i * KD + q, Kt + i * Dk + q);
    }
    for (int idx = threadIdx.x; idx < C * 8; idx += NT) {
      const int i = idx / 8, q = (idx % 8) * 4;
      if (q < ncols) cp16(sUb(buf) + i * LDC + q, U + i * Dv + col0 + q);
    }
    cp_commit();
  };
  for (int idx = threadIdx.x; idx < Dk * LDC; idx += NT) {
    const int r = idx / LDC, cc = idx % LDC;
    sS[idx] = (a.S0 != nullptr && cc < ncols) ? a.S0[((int64_t)bh * Dk + r) * Dv + col0 + cc] : 0.f;
  }
  if (a.nb > 0) prefetch(0, 0);
  __syncthreads();
  for (int c = 0; c < a.nb; ++c) {
    const int buf = c & 1;
    const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
    float* Sin = a.S_in + base * Dk * Dv;
    for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) {
      const int r = idx / 32, cc = idx % 32;
      if (cc < ncols) Sin[r * Dv + col0 + cc] = sS[r * LDC + cc];
    }
    cp_wait_all();
    __syncthreads();  // chunk c's operands are in buffer buf; buffer buf^1 is no longer read
    if (c + 1 < a.nb) prefetch(c + 1, buf ^ 1);
    const float* sW = sWb(buf);
    const float* sKt = sKtb(buf);
    const float* sU = sUb(buf);
    float* Vp = a.Vp + base * C * Dv;
    matmul<false, false>(C, 32, Dk, sW, KD, sS, LDC, [&](int i, int j, float x) {  // V' = U - W S
      if (j < ncols) {
        const float v = sU[i * LDC + j] - x;
        sVp[i * LDC + j] = v;
        Vp[i * Dv + col0 + j] = v;
      } else {
        sVp[i * LDC + j] = 0.f;
      }
    });
    __syncthreads();
    const float ec = a.Ec[base];
    matmul<true, false>(Dk, 32, C, sKt, KD, sVp, LDC, [&](int r, int j, float x) {  // S = Ec S + K~^T V'
      sS[r * LDC + j] = ec * sS[r * LDC + j] + x;
    });
    __syncthreads();
  }
  cp_wait_all();
  if (a.S_final != nullptr)
    for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) {
      const int r = idx / 32, cc = idx % 32;
      if (cc < ncols) a.S_final[((int64_t)bh * Dk + r) * Dv + col0 + cc] = sS[r * LDC + cc];
    }
}

// output for chunk blockIdx.x of the noised stream (x < nb) or clean stream (x >= nb).
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) fwd_out_kernel(Args a) {
  extern __shared__ float sm[];
  Smem<Dk, Dv> s(sm, a.C);
  constexpr int KD = Ld<Dk>::v, VD = Ld<Dv>::v;
  const int C = a.C;
  const int stream = (a.concat || blockIdx.x >= a.nb) ? 1 : 0;
  const int c = blockIdx.x - ((stream && !a.concat) ? a.nb : 0);
  const int bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv;
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  const float* Sin = a.S_in + base * Dk * Dv;
  for (int idx = threadIdx.x; idx < Dk * (Dv / 4); idx += NT) {  // asynchronous: first used for V' / O
    const int r = idx / (Dv / 4), d = (idx % (Dv / 4)) * 4;
    cp16(s.S + r * VD + d, Sin + r * Dv + d);
  }
  cp_commit();
  load_chunk<Dk, Dv>(a, b, stream, c, h, s.Q, s.K, s.V, s.gam, s.beta, true, stream == 0);
  matmul<false, true>(C, C, Dk, s.Q, KD, s.K, KD, [&](int i, int j, float x) {  // P = q^ k^T * Gam (incl)
    s.P[i * LDC + j] = j <= i ? x * __expf(s.gam[i] - s.gam[j]) : 0.f;
  });
  if (stream == 0)
    matmul<false, true>(C, C, Dk, s.K, KD, s.K, KD, [&](int i, int j, float x) { s.KK[i * LDC + j] = x; });
  __syncthreads();
  float* sVp = s.X;  // [C][VD]
  if (stream == 0) {
    ut_transform(C, s.KK, s.gam, s.beta, s.A, s.T);
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
      const int i = idx / Dv, d = idx % Dv;
      s.V[i * VD + d] *= s.beta[i];
    }
    for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
      const int i = idx / Dk, d = idx % Dk;
      s.Y[i * KD + d] = s.beta[i] * __expf(s.gam[i]) * s.K[i * KD + d];
    }
    __syncthreads();
    matmul<false, false>(C, Dk, C, s.T, LDC, s.Y, KD, [&](int i, int d, float x) { s.W[i * KD + d] = x; });
    matmul<false, false>(C, Dv, C, s.T, LDC, s.V, VD, [&](int i, int d, float x) { sVp[i * VD + d] = x; });
    cp_wait_all();
    __syncthreads();
    matmul<false, false>(C, Dv, Dk, s.W, KD, s.S, VD, [&](int i, int d, float x) { sVp[i * VD + d] -= x; });
  } else {
    const float* Vp = a.Vp + base * C * Dv;
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
      const int i = idx / Dv, d = idx % Dv;
      sVp[i * VD + d] = Vp[idx];
    }
  }
  cp_wait_all();
  __syncthreads();
  // O = diag(E) q^ S + P V'
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk, d = idx % Dk;
    s.Q[i * KD + d] *= __expf(s.gam[i]);
  }
  __syncthreads();
  float* sO = s.Y;
  matmul<false, false>(C, Dv, C, s.P, LDC, sVp, VD, [&](int i, int d, float x) { sO[i * VD + d] = x; });
  __syncthreads();
  matmul<false, false>(C, Dv, Dk, s.Q, KD, s.S, VD, [&](int i, int d, float x) { sO[i * VD + d] += x; });
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * (Dv / 8); idx += NT) {  // 16-byte bf16 stores
    const int i = idx / (Dv / 8), d = (idx % (Dv / 8)) * 8;
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) o2[e] = __floats2bfloat162_rn(sO[i * VD + d + 2 * e], sO[i * VD + d + 2 * e + 1]);
    (void)BDLLM_CHECK(all_finite(sO + i * VD + d, 8), i, C);  // sentinel: non-finite output
    *reinterpret_cast<uint4*>(a.o + tok(a, b, stream, c, i) * (int64_t)a.Hv * Dv + h * Dv + d) = o;
  }
}

// ================================================================== backward
// With R = diag(beta) (V - diag(E) k^ S) the UT identities give V' = T R and dT = dV' R^T, so the
// chunk backward needs, besides the inputs: R0 = V - diag(E) k^ S (stored), dR = T^T dV'.
//   dV = diag(beta) dR;  dbeta_i = sum_b dR_ib R0_ib + sum_j dA_ij KK_ij Gam_ij
//   dk^ += -diag(beta E) dR S^T + (dP*Gam)^T q^ + diag(F) V' dS_out^T + dKK k^ + dKK^T k^
//   dq^  = diag(E) dO S^T + (dP*Gam) k^,  dP = dO V'^T
//   dE_i = sum_b (q^ S)_ib dO_ib - beta_i sum_b dR_ib (k^ S)_ib,  dF_i = sum_b (k^ dS_out)_ib V'_ib
//   dA = strict_lower(-T^T dT T^T),  dKK = dA * beta_i * Gam
//   dS_in = e^gam_C dS_out + (diag(E) q^)^T dO - k^T diag(beta E) dR
// The T-path (dT, dA, dKK) runs right after dR, after which the dV' tile is dead and holds the
// dq^ accumulator: 8 [C][D] tiles + S + 5 [C][C] tiles fit in 227 KB with padded strides.
template <int Dk, int Dv>
struct BSmem {
  static constexpr int KD = Ld<Dk>::v, VD = Ld<Dv>::v;
  float *Q, *K, *R0, *dO, *Vp, *dVp, *dR, *dK, *S, *KK, *T, *P, *X, *Y, *gam, *beta, *dgam, *dE, *dF, *red;
  float* dQ;  // aliases dVp once the T-path is done
  __device__ BSmem(float* base) {
    float* p = base;
    Q = p; p += 32 * KD;
    K = p; p += 32 * KD;
    R0 = p; p += 32 * VD;
    dO = p; p += 32 * VD;
    Vp = p; p += 32 * VD;
    dVp = p; p += 32 * (VD > KD ? VD : KD);
    dR = p; p += 32 * VD;
    dK = p; p += 32 * KD;
    S = p; p += Dk * VD;
    KK = p; p += 32 * LDC;
    T = p; p += 32 * LDC;
    P = p; p += 32 * LDC;
    X = p; p += 32 * LDC;
    Y = p; p += 32 * LDC;
    gam = p; p += 32;
    beta = p; p += 32;
    dgam = p; p += 32;
    dE = p; p += 32;
    dF = p; p += 32;
    red = p; p += 32;
    dQ = dVp;
  }
  static constexpr int floats =
      3 * 32 * KD + 4 * 32 * VD + 32 * (VD > KD ? VD : KD) + Dk * VD + 5 * 32 * LDC + 6 * 32;
};

// mode 0: noised block (dS_out = 0, dV' = P^T dO, writes dS_inj[c]); mode 1: clean chunk
// (dV' and dS_out from the reverse recurrence).
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) bwd_chunk_kernel(Args a, int mode) {
  extern __shared__ float sm[];
  BSmem<Dk, Dv> s(sm);
  constexpr int KD = Ld<Dk>::v, VD = Ld<Dv>::v;
  const int C = a.C;
  const int stream = mode == 0 ? 0 : 1;
  const int c = blockIdx.x;
  const int bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv;
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  mark(a, 0);
  // ---- loads: S (asynchronously: first needed after the UT transform), q^, k^, V (into R0), gam,
  // beta, dO
  const float* Sin = a.S_in + base * Dk * Dv;
  for (int idx = threadIdx.x; idx < Dk * (Dv / 4); idx += NT) {
    const int r = idx / (Dv / 4), d = (idx % (Dv / 4)) * 4;
    cp16(s.S + r * VD + d, Sin + r * Dv + d);
  }
  cp_commit();
  load_chunk<Dk, Dv>(a, b, stream, c, h, s.Q, s.K, s.R0, s.gam, s.beta, true, true);
  for (int idx = threadIdx.x; idx < C * (Dv / 8); idx += NT) {  // 16-byte loads
    const int i = idx / (Dv / 8), d = (idx % (Dv / 8)) * 8;
    const uint4 raw = *reinterpret_cast<const uint4*>(a.dout + tok(a, b, stream, c, i) * (int64_t)a.Hv * Dv + h * Dv + d);
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(r2[e]);
      s.dO[i * VD + d + 2 * e] = f.x, s.dO[i * VD + d + 2 * e + 1] = f.y;
    }
  }
  if (threadIdx.x < 32) {
    s.dgam[threadIdx.x] = 0.f, s.dE[threadIdx.x] = 0.f, s.dF[threadIdx.x] = 0.f, s.red[threadIdx.x] = 0.f;
  }
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk, d = idx % Dk;
    s.dK[i * KD + d] = 0.f;
  }
  __syncthreads();
  mark(a, 1);  // loads done
  // ---- KK, P (with Gam, incl), T
  matmul<false, true>(C, C, Dk, s.K, KD, s.K, KD, [&](int i, int j, float x) { s.KK[i * LDC + j] = x; });
  matmul<false, true>(C, C, Dk, s.Q, KD, s.K, KD, [&](int i, int j, float x) {
    s.P[i * LDC + j] = j <= i ? x * __expf(s.gam[i] - s.gam[j]) : 0.f;
  });
  __syncthreads();
  mark(a, 2);  // KK, P
  ut_transform(C, s.KK, s.gam, s.beta, s.X, s.T);  // X is scratch for A here
  cp_wait_all();
  __syncthreads();
  mark(a, 3);  // UT transform (and the state tile landed)
  // ---- R0 = V - diag(E) k^ S (in place over V)
  matmul<false, false>(C, Dv, Dk, s.K, KD, s.S, VD, [&](int i, int d, float x) {
    s.R0[i * VD + d] -= __expf(s.gam[i]) * x;
  });
  __syncthreads();
  // ---- V' = (T diag(beta)) R0
  for (int idx = threadIdx.x; idx < C * C; idx += NT) {
    const int i = idx / C, j = idx % C;
    s.X[i * LDC + j] = s.T[i * LDC + j] * s.beta[j];
  }
  __syncthreads();
  // ---- V' and dV' (noised blocks: P^T dO, computed next to V' on the other half of the warps)
  if (mode == 0) {
    matmul_pair<false, false, true, false>(
        C, Dv, C, s.X, LDC, s.R0, VD, [&](int i, int d, float x) { s.Vp[i * VD + d] = x; },
        C, Dv, C, s.P, LDC, s.dO, VD, [&](int i, int d, float x) { s.dVp[i * VD + d] = x; });
    __syncthreads();
    mark(a, 4);  // R0, V', dV'
  } else {
    matmul<false, false>(C, Dv, C, s.X, LDC, s.R0, VD, [&](int i, int d, float x) { s.Vp[i * VD + d] = x; });
    __syncthreads();
    mark(a, 4);  // R0, V'
    const float* gdv = a.dVp + base * C * Dv;
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
      const int i = idx / Dv, d = idx % Dv;
      s.dVp[i * VD + d] = gdv[idx];
    }
  }
  __syncthreads();
  // ---- dR = T^T dV' ; dV = diag(beta) dR -> global
  matmul<true, false>(C, Dv, C, s.T, LDC, s.dVp, VD, [&](int i, int d, float x) { s.dR[i * VD + d] = x; });
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * (Dv / 8); idx += NT) {  // dv = diag(beta) dR, 16-byte stores
    const int i = idx / (Dv / 8), d = (idx % (Dv / 8)) * 8;
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
    const float bi = s.beta[i];
#pragma unroll
    for (int e = 0; e < 4; ++e) o2[e] = __floats2bfloat162_rn(bi * s.dR[i * VD + d + 2 * e], bi * s.dR[i * VD + d + 2 * e + 1]);
    *reinterpret_cast<uint4*>(a.dv + tok(a, b, stream, c, i) * (int64_t)a.Hv * Dv + h * Dv + d) = o;
  }
  __syncthreads();
  mark(a, 5);  // dV', dR, dv
  // ---- T-path: dT = dV' R^T (R = diag(beta) R0) -> Y ; dA = strict_lower(-T^T dT T^T) -> Y
  matmul<false, true>(C, C, Dv, s.dVp, VD, s.R0, VD, [&](int i, int j, float x) { s.Y[i * LDC + j] = x * s.beta[j]; });
  __syncthreads();
  matmul<false, true>(C, C, C, s.Y, LDC, s.T, LDC, [&](int i, int j, float x) { s.X[i * LDC + j] = x; });
  __syncthreads();
  matmul<true, false>(C, C, C, s.T, LDC, s.X, LDC, [&](int i, int j, float x) { s.Y[i * LDC + j] = j < i ? -x : 0.f; });
  __syncthreads();
  // dbeta += sum_j dA_ij KK_ij Gam_ij ; dKK = dA * beta_i * Gam (-> X) ; H2 = dA beta KK Gam (-> P2)
  // with dgam += rowsum(H2) - colsum(H2): one thread per row, then one per column (no atomics)
  for (int idx = threadIdx.x; idx < C * C; idx += NT) {
    const int i = idx / C, j = idx % C;
    const float gm = j < i ? __expf(s.gam[i] - s.gam[j]) : 0.f;
    const float dA = s.Y[i * LDC + j];
    s.X[i * LDC + j] = dA * s.beta[i] * gm;
    s.Y[i * LDC + j] = dA * s.KK[i * LDC + j] * gm;  // dA KK Gam (H2 / beta_i)
  }
  __syncthreads();
  if (threadIdx.x < C) {
    const int i = threadIdx.x;
    float rs = 0.f, cs = 0.f;
    for (int j = 0; j < C; ++j) rs += s.Y[i * LDC + j], cs += s.beta[j] * s.Y[j * LDC + i];
    s.red[i] += rs;
    s.dgam[i] += s.beta[i] * rs - cs;
  }
  __syncthreads();
  mark(a, 6);  // T-path, dKK, dbeta / dgam rows
  // dK += dKK k^ + dKK^T k^ = (dKK + dKK^T) k^ (Y is free again); dV' is dead from here on: its
  // tile becomes the dq^ accumulator
  for (int idx = threadIdx.x; idx < C * C; idx += NT) {
    const int i = idx / C, j = idx % C;
    s.Y[i * LDC + j] = s.X[i * LDC + j] + s.X[j * LDC + i];
  }
  __syncthreads();
  matmul<false, false>(C, Dk, C, s.Y, LDC, s.K, KD, [&](int i, int d, float x) { s.dK[i * KD + d] += x; });
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk, d = idx % Dk;
    s.dQ[i * KD + d] = 0.f;
  }
  __syncthreads();
  mark(a, 7);  // dK from dKK
  // ---- products with S: dQ += diag(E) dO S^T ; dK -= diag(beta E) dR S^T ; dE terms ; dbeta part
  matmul_pair<false, true, false, true>(
      C, Dk, Dv, s.dO, VD, s.S, VD, [&](int i, int d, float x) { s.dQ[i * KD + d] += __expf(s.gam[i]) * x; },
      C, Dk, Dv, s.dR, VD, s.S, VD,
      [&](int i, int d, float x) { s.dK[i * KD + d] -= s.beta[i] * __expf(s.gam[i]) * x; });
  matmul_rowsum_pair<false, false, false, false>(
      C, Dv, Dk, s.Q, KD, s.S, VD, [&](int i, int d, float x) { return x * s.dO[i * VD + d]; }, s.dE,
      C, Dv, Dk, s.K, KD, s.S, VD, [&](int i, int d, float x) { return -s.beta[i] * x * s.dR[i * VD + d]; }, s.dE);
  __syncthreads();
  rowdot(C, Dv, s.dR, VD, s.R0, VD, s.red);
  __syncthreads();
  mark(a, 8);  // products with S
  // ---- dP = dO V'^T ; dPm = dP * Gam (incl) -> X ; G1 = dP * P -> Y ; dgam += rowsum(G1) - colsum(G1)
  matmul<false, true>(C, C, Dv, s.dO, VD, s.Vp, VD, [&](int i, int j, float x) {
    const float gm = j <= i ? __expf(s.gam[i] - s.gam[j]) : 0.f;
    s.X[i * LDC + j] = x * gm;
    s.Y[i * LDC + j] = x * s.P[i * LDC + j];
  });
  __syncthreads();
  if (threadIdx.x < C) {
    const int i = threadIdx.x;
    float rs = 0.f, cs = 0.f;
    for (int j = 0; j < C; ++j) rs += s.Y[i * LDC + j], cs += s.Y[j * LDC + i];
    s.dgam[i] += rs - cs;
  }
  __syncthreads();
  matmul_pair<false, false, true, false>(
      C, Dk, C, s.X, LDC, s.K, KD, [&](int i, int d, float x) { s.dQ[i * KD + d] += x; },
      C, Dk, C, s.X, LDC, s.Q, KD, [&](int i, int d, float x) { s.dK[i * KD + d] += x; });
  __syncthreads();
  mark(a, 9);  // dP path
  // ---- state gradient
  if (mode == 0) {
    // dS_inj = (diag(E) q^)^T dO - k^T diag(beta E) dR ; dO and dR are consumed (scaled in place)
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
      const int i = idx / Dv, d = idx % Dv;
      const float e = __expf(s.gam[i]);
      s.dO[i * VD + d] *= e;
      s.dR[i * VD + d] *= s.beta[i] * e;
    }
    __syncthreads();
    matmul<true, false>(Dk, Dv, C, s.Q, KD, s.dO, VD, [&](int r, int d, float x) { s.S[r * VD + d] = x; });
    __syncthreads();
    float* dSi = a.dS_inj + base * Dk * Dv;
    matmul<true, false>(Dk, Dv, C, s.K, KD, s.dR, VD, [&](int r, int d, float x) { s.S[r * VD + d] -= x; });
    __syncthreads();
    for (int idx = threadIdx.x; idx < Dk * (Dv / 4); idx += NT) {  // 16-byte stores
      const int r = idx / (Dv / 4), d = (idx % (Dv / 4)) * 4;
      *reinterpret_cast<float4*>(dSi + r * Dv + d) = *reinterpret_cast<const float4*>(s.S + r * VD + d);
    }
    __syncthreads();
  } else {
    // dEc = sum S * dS_out and S <- dS_out in one pass (each thread reads its four S values before
    // overwriting them)
    const float* dSo = a.dS_out + base * Dk * Dv;
    float part = 0.f;
    for (int idx = threadIdx.x; idx < Dk * (Dv / 4); idx += NT) {
      const int r = idx / (Dv / 4), d = (idx % (Dv / 4)) * 4;
      float4* sp = reinterpret_cast<float4*>(s.S + r * VD + d);
      const float4 o = *reinterpret_cast<const float4*>(dSo + r * Dv + d);
      const float4 v = *sp;
      part += v.x * o.x + v.y * o.y + v.z * o.z + v.w * o.w;
      *sp = o;
    }
    part = wsum(part);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s.dgam[C - 1], part * __expf(s.gam[C - 1]));  // dEc * Ec
    __syncthreads();
    // dK += diag(F) V' dS_out^T ; dF_i = sum_b (k^ dS_out)_ib V'_ib (on the two halves of the warps)
    if (M_TILES_OK(C, Dk, Dv) && M_TILES_OK(C, Dv, Dk)) {
      constexpr int H = NT / 64;
      const int lane = threadIdx.x & 31;
      mm_tc_part<false, true>(C, Dk, Dv, s.Vp, VD, s.S, VD, [&](int i, int d, float x) {
        s.dK[i * KD + d] += __expf(s.gam[C - 1] - s.gam[i]) * x;
      }, 0, H);
      mm_tc_part<false, false>(C, Dv, Dk, s.K, KD, s.S, VD, [&](int i, int d, float x) {
        float v = x * s.Vp[i * VD + d];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if ((lane & 3) == 0) atomicAdd(&s.dF[i], v);
      }, H, H);
    } else {
      matmul<false, true>(C, Dk, Dv, s.Vp, VD, s.S, VD, [&](int i, int d, float x) {
        s.dK[i * KD + d] += __expf(s.gam[C - 1] - s.gam[i]) * x;
      });
      matmul_rowsum<false, false>(C, Dv, Dk, s.K, KD, s.S, VD,
                                   [&](int i, int d, float x) { return x * s.Vp[i * VD + d]; }, s.dF);
    }
    __syncthreads();
  }
  mark(a, 10);  // state gradient
  // ---- gates: dgam += dE E - dF F ; dgam[C-1] += sum dF F ; dg = reverse cumsum ; dbeta
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    float dgi = 0.f, fsum = 0.f;
    if (i < C) {
      const float E = __expf(s.gam[i]), F = __expf(s.gam[C - 1] - s.gam[i]);
      dgi = s.dgam[i] + s.dE[i] * E - s.dF[i] * F;
      fsum = s.dF[i] * F;
    }
    fsum = wsum(fsum);
    if (i == C - 1) dgi += fsum;
    float v = dgi;  // reverse inclusive cumsum: dg_i = sum_{j >= i} dgam_j
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y = __shfl_down_sync(0xffffffffu, v, o);
      if (i + o < 32) v += y;
    }
    if (i < C) {
      const int64_t t = tok(a, b, stream, c, i);
      a.dg[t * a.Hv + h] = v;
      a.dbeta[t * a.Hv + h] = s.red[i];
    }
  }
  mark(a, 11);  // gates
  // ---- l2norm backward (warp per row): dq = l2_bwd(q_raw, scale * dQ), dk = l2_bwd(k_raw, dK)
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int hk = h / (a.Hv / a.Hk);
  for (int r = warp; r < 2 * C; r += NT / 32) {
    const bool isq = r >= C;
    const int i = isq ? r - C : r;
    const int64_t t = tok(a, b, stream, c, i);
    const __nv_bfloat16* src = (isq ? a.q : a.k) + t * a.ldqk + hk * Dk;
    const float* dy = (isq ? s.dQ : s.dK) + i * KD;
    const float sc = isq ? a.scale : 1.f;
    float ss = 0.f, xd = 0.f;
    for (int d = lane; d < Dk; d += 32) {
      const float x = __bfloat162float(src[d]);
      ss += x * x;
      xd += x * dy[d] * sc;
    }
    ss = wsum(ss);
    xd = wsum(xd);
    const float rr = rsqrtf(ss + 1e-6f);
    __nv_bfloat16* out = (isq ? a.dq : a.dk) + (t * a.Hv + h) * (int64_t)Dk;
    for (int d = lane; d < Dk; d += 32) {
      const float x = __bfloat162float(src[d]);
      out[d] = __float2bfloat16(rr * dy[d] * sc - x * rr * rr * rr * xd);
    }
  }
  __syncthreads();
  mark(a, 12);  // l2norm backward, stores
}


// clean chunks: what the reverse recurrence needs -> PtdO [C][Dv], Kt [C][Dk], Qt [C][Dk], W [C][Dk], Ec
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) bwd_prep_kernel(Args a) {
  extern __shared__ float sm[];
  Smem<Dk, Dv> s(sm, a.C);
  constexpr int KD = Ld<Dk>::v, VD = Ld<Dv>::v;
  const int C = a.C;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv;
  load_chunk<Dk, Dv>(a, b, 1, c, h, s.Q, s.K, s.V, s.gam, s.beta, true, false);
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
    const int i = idx / Dv, d = idx % Dv;
    s.X[i * VD + d] = __bfloat162float(a.dout[tok(a, b, 1, c, i) * (int64_t)a.Hv * Dv + h * Dv + d]);
  }
  matmul<false, true>(C, C, Dk, s.K, KD, s.K, KD, [&](int i, int j, float x) { s.KK[i * LDC + j] = x; });
  matmul<false, true>(C, C, Dk, s.Q, KD, s.K, KD, [&](int i, int j, float x) {
    s.P[i * LDC + j] = j <= i ? x * __expf(s.gam[i] - s.gam[j]) : 0.f;
  });
  __syncthreads();
  ut_transform(C, s.KK, s.gam, s.beta, s.A, s.T);
  float* PtdO = a.PtdO + base * C * Dv;
  matmul<true, false>(C, Dv, C, s.P, LDC, s.X, VD, [&](int i, int d, float x) { PtdO[i * Dv + d] = x; });
  float* Kt = a.Kt + base * C * Dk;
  float* Qt = a.Qt + base * C * Dk;
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk, d = idx % Dk;
    Kt[idx] = __expf(s.gam[C - 1] - s.gam[i]) * s.K[i * KD + d];
    Qt[idx] = __expf(s.gam[i]) * s.Q[i * KD + d];
    s.Y[i * KD + d] = s.beta[i] * __expf(s.gam[i]) * s.K[i * KD + d];
  }
  __syncthreads();
  float* Wg = a.W + base * C * Dk;
  matmul<false, false>(C, Dk, C, s.T, LDC, s.Y, KD, [&](int i, int d, float x) { Wg[i * Dk + d] = x; });
  if (threadIdx.x == 0) a.Ec[base] = __expf(s.gam[C - 1]);
}

// reverse recurrence, CTA per (b, h, 32 value columns):
//   dS_out[c] = dS ; dV'_c = PtdO_c + K~_c dS ; dS = Ec dS + q~_c^T dO_c - W_c^T dV'_c (+ dS_inj[c])
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) bwd_recur_kernel(Args a, int has_inj) {
  extern __shared__ float sm[];
  constexpr int KD = Ld<Dk>::v;
  const int C = a.C;
  // double-buffered chunk operands: W, K~, q~ [C][KD], P^T dO columns [C][LDC] (fp32) and the dO
  // columns as raw bf16 [C][32]
  constexpr int BUF = 3 * 32 * KD + 32 * LDC + 32 * 16;
  auto sWb = [&](int k) { return sm + k * BUF; };
  auto sKtb = [&](int k) { return sm + k * BUF + 32 * KD; };
  auto sQtb = [&](int k) { return sm + k * BUF + 2 * 32 * KD; };
  auto sPb = [&](int k) { return sm + k * BUF + 3 * 32 * KD; };
  auto sOb = [&](int k) { return reinterpret_cast<__nv_bfloat16*>(sm + k * BUF + 3 * 32 * KD + 32 * LDC); };
  float* p = sm + 2 * BUF;
  float* sdVp = p;               // [C][LDC]
  float* sdO = sdVp + 32 * LDC;  // [C][LDC]
  float* sS = sdO + 32 * LDC;    // [Dk][LDC]
  const int bh = blockIdx.x, b = bh / a.Hv, h = bh % a.Hv;
  const int col0 = blockIdx.y * 32;
  const int ncols = min(32, Dv - col0);
  auto prefetch = [&](int c, int buf) {
    const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
    const float* Wg = a.W + base * C * Dk;
    const float* Kt = a.Kt + base * C * Dk;
    const float* Qt = a.Qt + base * C * Dk;
    const float* Pt = a.PtdO + base * C * Dv;
    for (int idx = threadIdx.x; idx < C * (Dk / 4); idx += NT) {
      const int i = idx / (Dk / 4), q = (idx % (Dk / 4)) * 4;
      cp16(sWb(buf) + i * KD + q, Wg + i * Dk + q);
      cp16(sKtb(buf) + i * KD + q, Kt + i * Dk + q);
      cp16(sQtb(buf) + i * KD + q, Qt + i * Dk + q);
    }
    for (int idx = threadIdx.x; idx < C * 8; idx += NT) {
      const int i = idx / 8, q = (idx % 8) * 4;
      if (q < ncols) cp16(sPb(buf) + i * LDC + q, Pt + i * Dv + col0 + q);
    }
    for (int idx = threadIdx.x; idx < C * 4; idx += NT) {
      const int i = idx / 4, q = (idx % 4) * 8;
      if (q < ncols)
        cp16(sOb(buf) + i * 32 + q, a.dout + tok(a, b, 1, c, i) * (int64_t)a.Hv * Dv + h * Dv + col0 + q);
    }
    cp_commit();
  };
  for (int idx = threadIdx.x; idx < Dk * LDC; idx += NT) sS[idx] = 0.f;
  if (a.nb > 0) prefetch(a.nb - 1, (a.nb - 1) & 1);
  __syncthreads();
  for (int c = a.nb - 1; c >= 0; --c) {
    const int buf = c & 1;
    const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
    float* dSo = a.dS_out + base * Dk * Dv;
    for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) {
      const int r = idx / 32, cc = idx % 32;
      if (cc < ncols) dSo[r * Dv + col0 + cc] = sS[r * LDC + cc];
    }
    cp_wait_all();
    __syncthreads();  // chunk c's operands are in buffer buf; buffer buf^1 is no longer read
    if (c > 0) prefetch(c - 1, buf ^ 1);
    for (int idx = threadIdx.x; idx < C * 32; idx += NT) {
      const int i = idx / 32, cc = idx % 32;
      sdO[i * LDC + cc] = cc < ncols ? __bfloat162float(sOb(buf)[i * 32 + cc]) : 0.f;
    }
    const float* sW = sWb(buf);
    const float* sKt = sKtb(buf);
    const float* sQt = sQtb(buf);
    const float* sP = sPb(buf);
    float* dVp = a.dVp + base * C * Dv;
    matmul<false, false>(C, 32, Dk, sKt, KD, sS, LDC, [&](int i, int j, float x) {
      if (j < ncols) {
        const float v = sP[i * LDC + j] + x;
        sdVp[i * LDC + j] = v;
        dVp[i * Dv + col0 + j] = v;
      } else {
        sdVp[i * LDC + j] = 0.f;
      }
    });
    __syncthreads();
    const float ec = a.Ec[base];
    const float* inj = has_inj ? a.dS_inj + base * Dk * Dv : nullptr;
    matmul<true, false>(Dk, 32, C, sQt, KD, sdO, LDC, [&](int r, int j, float x) {
      sS[r * LDC + j] = ec * sS[r * LDC + j] + x;
    });
    __syncthreads();
    matmul<true, false>(Dk, 32, C, sW, KD, sdVp, LDC, [&](int r, int j, float x) {
      float v = sS[r * LDC + j] - x;
      if (inj != nullptr && j < ncols) v += inj[r * Dv + col0 + j];
      sS[r * LDC + j] = v;
    });
    __syncthreads();
  }
  cp_wait_all();
  if (a.dS0 != nullptr)  // the gradient of the state entering chunk 0 (the row's initial state)
    for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) {
      const int r = idx / 32, cc = idx % 32;
      if (cc < ncols) a.dS0[((int64_t)bh * Dk + r) * Dv + col0 + cc] = sS[r * LDC + cc];
    }
}

// ------------------------------------------------------------------------------------- tcgen05 backward
#include "gdn_bwd_tc.cuh"

// ------------------------------------------------------------------------------------- host

template <typename K>
static void launch(K kern, dim3 grid, int smem_floats, const Args& a) {
  const int bytes = smem_floats * 4;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  kern<<<grid, NT, bytes, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
template <typename K>
static void launch2(K kern, dim3 grid, int smem_floats, const Args& a, int x) {
  const int bytes = smem_floats * 4;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  kern<<<grid, NT, bytes, at::cuda::getCurrentCUDAStream()>>>(a, x);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static Args make_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                      const at::Tensor& beta, int64_t L, int64_t C, bool concat) {
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "gdn: q, k, v [B, 2L, H, D]");
  TORCH_CHECK(q.stride(-1) == 1 && k.stride(-1) == 1 && v.stride(-1) == 1, "gdn: unit inner stride");
  TORCH_CHECK(q.stride(1) == k.stride(1) && q.stride(2) == q.size(3) && k.stride(2) == k.size(3) &&
                  v.stride(2) == v.size(3),
              "gdn: heads must be packed within a token row");
  TORCH_CHECK(q.size(0) == 1 || (q.stride(0) == q.size(1) * q.stride(1) && v.stride(0) == v.size(1) * v.stride(1)),
              "gdn: batch and token dims must merge");  // (a single batch row has no batch stride)
  TORCH_CHECK(g.is_contiguous() && beta.is_contiguous() && g.scalar_type() == at::kFloat &&
                  beta.scalar_type() == at::kFloat,
              "gdn: g, beta fp32 contiguous [B, 2L, Hv]");
  TORCH_CHECK(C <= 32 && C >= 1 && (2 * L) % C == 0 && (concat || L % C == 0),
              "gdn: chunk (= block) must be <= 32 and divide L");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "gdn: bf16 q, k, v");
  TORCH_CHECK(q.size(1) == 2 * L && k.sizes() == q.sizes() && v.size(0) == q.size(0) && v.size(1) == q.size(1) &&
                  v.size(2) % q.size(2) == 0,
              "gdn: q, k [B, 2L, Hk, Dk] and v [B, 2L, Hv, Dv] with Hv a multiple of Hk");
  TORCH_CHECK(g.numel() == q.size(0) * q.size(1) * v.size(2) && beta.numel() == g.numel(), "gdn: g, beta [B, 2L, Hv]");
  Args a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.ldqk = q.stride(1);
  a.ldv = v.stride(1);
  a.g = g.data_ptr<float>();
  a.beta = beta.data_ptr<float>();
  a.B = q.size(0);
  a.L = (int)L;
  a.Hk = q.size(2);
  a.Hv = v.size(2);
  a.C = (int)C;
  a.concat = concat ? 1 : 0;
  a.nb = (int)((concat ? 2 * L : L) / C);
  a.scale = 1.f / sqrtf((float)q.size(3));
  return a;
}

// Forward. Returns {o, S_in, Vp}; S_in [B, nb, Hv, Dk, Dv] fp32 (state entering each clean chunk),
// Vp [B, nb, Hv, C, Dv] fp32 (clean V').
template <int Dk, int Dv>
static std::vector<at::Tensor> forward_t(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                         const at::Tensor& g, const at::Tensor& beta, int64_t L, int64_t C,
                                         bool concat) {
  Args a = make_args(q, k, v, g, beta, L, C, concat);
  c10::cuda::CUDAGuard guard(q.device());  // (after the host checks, which host tests reach)
  auto f32 = q.options().dtype(at::kFloat);
  auto U = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto W = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Kt = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Ec = at::empty({a.B, a.nb, a.Hv}, f32);
  auto S_in = at::empty({a.B, a.nb, a.Hv, Dk, Dv}, f32);
  auto Vp = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto o = at::empty({a.B, 2 * L, a.Hv, Dv}, q.options());
  a.U = U.data_ptr<float>();
  a.W = W.data_ptr<float>();
  a.Kt = Kt.data_ptr<float>();
  a.Ec = Ec.data_ptr<float>();
  a.S_in = S_in.data_ptr<float>();
  a.Vp = Vp.data_ptr<float>();
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  const int BH = a.B * a.Hv;
  launch(fwd_prep_kernel<Dk, Dv>, dim3(a.nb, BH), Smem<Dk, Dv>::floats, a);
  launch(fwd_recur_kernel<Dk, Dv>, dim3(BH, (Dv + 31) / 32), 4 * 32 * Ld<Dk>::v + 3 * 32 * LDC + Dk * LDC, a);
  // noised blocks (x < nb) only exist with the fork
  const int ngrid = concat ? a.nb : 2 * a.nb;
  launch(fwd_out_kernel<Dk, Dv>, dim3(ngrid, BH), Smem<Dk, Dv>::floats, a);
  return {o, S_in, Vp};
}

// Decode rows: q, k [B, T, Hk, Dk], v [B, T, Hv, Dv] (T even, chunked by C), one causal run per
// row starting from S0 [B, Hv, Dk, Dv] (fp32); writes the final state into S_final when given
// (S_final may be S0: each CTA reads its slice before it writes it). Returns o [B, T, Hv, Dv].
template <int Dk, int Dv>
static std::vector<at::Tensor> rows_t(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                      const at::Tensor& g, const at::Tensor& beta, const at::Tensor& S0,
                                      const c10::optional<at::Tensor>& S_final, int64_t C, bool want_states = false) {
  const int64_t T = q.size(1);
  TORCH_CHECK(T % 2 == 0 && T % C == 0, "gdn_rows: T even and a multiple of the chunk");
  Args a = make_args(q, k, v, g, beta, T / 2, C, true);
  TORCH_CHECK(S0.is_contiguous() && S0.scalar_type() == at::kFloat && S0.numel() == (int64_t)a.B * a.Hv * Dk * Dv,
              "gdn_rows: S0 fp32 [B, Hv, Dk, Dv]");
  c10::cuda::CUDAGuard guard(q.device());
  auto f32 = q.options().dtype(at::kFloat);
  auto U = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto W = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Kt = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Ec = at::empty({a.B, a.nb, a.Hv}, f32);
  auto S_in = at::empty({a.B, a.nb, a.Hv, Dk, Dv}, f32);
  auto Vp = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto o = at::empty({a.B, T, a.Hv, Dv}, q.options());
  a.U = U.data_ptr<float>();
  a.W = W.data_ptr<float>();
  a.Kt = Kt.data_ptr<float>();
  a.Ec = Ec.data_ptr<float>();
  a.S_in = S_in.data_ptr<float>();
  a.Vp = Vp.data_ptr<float>();
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.S0 = S0.data_ptr<float>();
  if (S_final.has_value()) {
    TORCH_CHECK(S_final->is_contiguous() && S_final->scalar_type() == at::kFloat && S_final->numel() == S0.numel(),
                "gdn_rows: S_final like S0");
    a.S_final = S_final->data_ptr<float>();
  }
  const int BH = a.B * a.Hv;
  launch(fwd_prep_kernel<Dk, Dv>, dim3(a.nb, BH), Smem<Dk, Dv>::floats, a);
  launch(fwd_recur_kernel<Dk, Dv>, dim3(BH, (Dv + 31) / 32), 4 * 32 * Ld<Dk>::v + 3 * 32 * LDC + Dk * LDC, a);
  launch(fwd_out_kernel<Dk, Dv>, dim3(a.nb, BH), Smem<Dk, Dv>::floats, a);
  if (want_states) return {o, S_in};
  return {o};
}

// Backward. Returns {dq, dk (per v-head), dv, dg, dbeta}.
template <int Dk, int Dv>
static std::vector<at::Tensor> backward_t(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                          const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta,
                                          const at::Tensor& S_in, int64_t L, int64_t C, bool concat,
                                          const c10::optional<at::Tensor>& inj = c10::nullopt,
                                          bool want_dS0 = false) {
  Args a = make_args(q, k, v, g, beta, L, C, concat);
  auto f32 = q.options().dtype(at::kFloat);
  TORCH_CHECK(dout.numel() == (int64_t)a.B * 2 * L * a.Hv * Dv, "gdn_bwd: dout [B, 2L, Hv, Dv]");
  TORCH_CHECK(S_in.is_contiguous() && (S_in.scalar_type() == at::kFloat || S_in.scalar_type() == at::kBFloat16) &&
                  S_in.numel() == (int64_t)a.B * a.nb * a.Hv * Dk * Dv,
              "gdn_bwd: S_in [B, nb, Hv, Dk, Dv] (fp32, or bf16 from the tensor-core forward)");
  c10::cuda::CUDAGuard guard(q.device());
  auto d = dout.to(at::kBFloat16).contiguous();
  if (reinterpret_cast<uintptr_t>(d.data_ptr()) % 16 != 0) d = d.clone();  // read in 16-byte vectors and TMA tiles
  a.dout = reinterpret_cast<const __nv_bfloat16*>(d.data_ptr());
  // bf16 S_in: the tensor-core forward's S^T rows; the whole backward then runs on tcgen05
  const bool bf16_states = S_in.scalar_type() == at::kBFloat16;
  a.S_in = bf16_states ? nullptr : const_cast<float*>(S_in.data_ptr<float>());
  auto dq = at::empty({a.B, 2 * L, a.Hv, Dk}, q.options());
  auto dk = at::empty({a.B, 2 * L, a.Hv, Dk}, q.options());
  auto dv = at::empty({a.B, 2 * L, a.Hv, Dv}, q.options());
  auto dg = at::empty({a.B, 2 * L, a.Hv}, f32);
  auto db = at::empty({a.B, 2 * L, a.Hv}, f32);
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  a.dg = dg.data_ptr<float>();
  a.dbeta = db.data_ptr<float>();
  // concat runs take optional injected state gradients (one [Dk, Dv] per chunk entry, e.g. from
  // rows that start from those states) and may return the gradient of their initial state
  TORCH_CHECK(!inj.has_value() || (concat && inj->is_contiguous() && inj->scalar_type() == at::kFloat &&
                                   inj->numel() == (int64_t)a.B * a.nb * a.Hv * Dk * Dv),
              "gdn_bwd: injected state gradients fp32 [B, nb, Hv, Dk, Dv] (concat runs)");
  auto dS_inj = concat ? (inj.has_value() ? *inj : at::Tensor()) : at::empty({a.B, a.nb, a.Hv, Dk, Dv}, f32);
  auto dS0 = want_dS0 ? at::empty({a.B, a.Hv, Dk, Dv}, f32) : at::Tensor();
  a.dS0 = want_dS0 ? dS0.data_ptr<float>() : nullptr;
  auto dS_out = at::empty({a.B, a.nb, a.Hv, Dk, Dv}, bf16_states ? q.options().dtype(at::kBFloat16) : f32);
  auto dVp = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto PtdO = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto Qt = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Kt = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto W = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Ec = at::empty({a.B, a.nb, a.Hv}, f32);
  a.dS_inj = dS_inj.defined() ? dS_inj.data_ptr<float>() : nullptr;
  a.dS_out = bf16_states ? nullptr : dS_out.data_ptr<float>();
  a.dVp = dVp.data_ptr<float>();
  a.PtdO = PtdO.data_ptr<float>();
  a.Qt = Qt.data_ptr<float>();
  a.Kt = Kt.data_ptr<float>();
  a.W = W.data_ptr<float>();
  a.Ec = Ec.data_ptr<float>();
  const int BH = a.B * a.Hv;
  // BDLLM_GDN_PHASES=1: clock64() at the phase boundaries of the chunk kernel's first CTA, printed
  // per launch (diagnostics; one device-to-host read per launch)
  static const bool phases = getenv("BDLLM_GDN_PHASES") != nullptr;
  at::Tensor ph;
  auto report = [&](const char* what) {
    if (!phases) return;
    auto h = ph.cpu();
    const int64_t* t = h.data_ptr<int64_t>();
    fprintf(stderr, "[gdn phases] %s:", what);
    for (int i = 1; i < 13; ++i) fprintf(stderr, " %lld", (long long)(t[i] - t[i - 1]));
    fprintf(stderr, " | total %lld cycles\n", (long long)(t[12] - t[0]));
  };
  if (phases) {
    ph = at::zeros({16}, q.options().dtype(at::kLong));
    a.phase = reinterpret_cast<long long*>(ph.data_ptr<int64_t>());
  }
  // the whole backward on tcgen05 when the forward saved bf16 S^T rows (head dim 128, chunk 32, the
  // fork layout, L a multiple of 128: the tensor-core forward's domain): chunk kernels fed by TMA
  // (q, k, v, dO tiles of 32 tokens; S^T and dS_out^T tiles) and the reverse recurrence, which adds
  // the noised blocks' state gradients itself
  const bool tc = bf16_states;
  TORCH_CHECK(!tc || (Dk == 128 && Dv == 128 && !concat && C == 32 && L % 128 == 0 && a.ldqk % 8 == 0 &&
                      a.ldv % 8 == 0 && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(k.data_ptr()) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(v.data_ptr()) % 16 == 0),
              "gdn_bwd: bf16 states come from the tensor-core forward (head dim 128, block 32, L % 128 == 0)");
  struct alignas(64) TcMaps {
    CUtensorMap mq, mk, mv, mdo, ms, mds, mdq, mdk, mdv;
  };
  static thread_local TcMaps tm;
  auto chunk_tc = [&](int mode) {
    void* kargs[12];
    int* err = error_word_ptr();
    Args ac = a;
    kargs[0] = &tm.mq, kargs[1] = &tm.mk, kargs[2] = &tm.mv, kargs[3] = &tm.mdo, kargs[4] = &tm.ms,
    kargs[5] = &tm.mds, kargs[6] = &tm.mdq, kargs[7] = &tm.mdk, kargs[8] = &tm.mdv, kargs[9] = &ac,
    kargs[10] = &mode, kargs[11] = &err;
    C10_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(bwd_chunk_tc_kernel), dim3(a.nb, BH),
                                    dim3(btc::NTH), kargs, btc::L::BYTES, at::cuda::getCurrentCUDAStream()));
  };
  if (tc) {
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(bwd_chunk_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          btc::L::BYTES));
      attr = true;
    }
    const uint64_t rows = (uint64_t)a.B * 2 * L;
    make_map_bf16(&tm.mq, q.data_ptr(), (uint64_t)a.Hk * Dk, rows, a.ldqk, 64, 32);
    make_map_bf16(&tm.mk, k.data_ptr(), (uint64_t)a.Hk * Dk, rows, a.ldqk, 64, 32);
    make_map_bf16(&tm.mv, v.data_ptr(), (uint64_t)a.Hv * Dv, rows, a.ldv, 64, 32);
    make_map_bf16(&tm.mdo, d.data_ptr(), (uint64_t)a.Hv * Dv, rows, (uint64_t)a.Hv * Dv, 64, 32);
    const uint64_t srows = (uint64_t)a.B * a.nb * a.Hv * Dk;
    make_map_bf16(&tm.ms, S_in.data_ptr(), Dv, srows, Dv, 64, 128);
    make_map_bf16(&tm.mds, dS_out.data_ptr(), Dv, srows, Dv, 64, 128);
    // outputs [B * 2L, Hv * D] (per v-head dq and dk): 32-row boxes stored from the staged tiles
    make_map_bf16(&tm.mdq, dq.data_ptr(), (uint64_t)a.Hv * Dk, rows, (uint64_t)a.Hv * Dk, 64, 32);
    make_map_bf16(&tm.mdk, dk.data_ptr(), (uint64_t)a.Hv * Dk, rows, (uint64_t)a.Hv * Dk, 64, 32);
    make_map_bf16(&tm.mdv, dv.data_ptr(), (uint64_t)a.Hv * Dv, rows, (uint64_t)a.Hv * Dv, 64, 32);
  }
  if (!concat) {
    if (tc)
      chunk_tc(0);
    else
      launch2(bwd_chunk_kernel<Dk, Dv>, dim3(a.nb, BH), BSmem<Dk, Dv>::floats, a, 0);
    report("noised");
  }
  if (tc) {
    gdn_bwd_recurrence_tc(q, k, v, g, beta, d, L, reinterpret_cast<__nv_bfloat16*>(dS_out.data_ptr()), a.dVp);
  } else {
    Args a2 = a;
    a2.phase = nullptr;
    launch(bwd_prep_kernel<Dk, Dv>, dim3(a.nb, BH), Smem<Dk, Dv>::floats, a2);
    launch2(bwd_recur_kernel<Dk, Dv>, dim3(BH, (Dv + 31) / 32),
            2 * (3 * 32 * Ld<Dk>::v + 32 * LDC + 32 * 16) + 2 * 32 * LDC + Dk * LDC, a2,
            a.dS_inj != nullptr ? 1 : 0);
  }
  if (tc)
    chunk_tc(1);
  else
    launch2(bwd_chunk_kernel<Dk, Dv>, dim3(a.nb, BH), BSmem<Dk, Dv>::floats, a, 1);
  report("clean");
  if (want_dS0) return {dq, dk, dv, dg, db, dS0};
  return {dq, dk, dv, dg, db};
}

}  // namespace gdn

#define GDN_DISPATCH(FN, ...)                                                 \
  const int Dk = q.size(3), Dv = v.size(3);                                   \
  TORCH_CHECK(Dk == Dv, "gdn: Dk == Dv supported");                           \
  switch (Dk) {                                                               \
    case 16: return gdn::FN<16, 16>(__VA_ARGS__);                             \
    case 32: return gdn::FN<32, 32>(__VA_ARGS__);                             \
    case 64: return gdn::FN<64, 64>(__VA_ARGS__);                             \
    case 128: return gdn::FN<128, 128>(__VA_ARGS__);                          \
    default: TORCH_CHECK(false, "gdn: head dim ", Dk, " not in {16, 32, 64, 128}"); \
  }

std::vector<at::Tensor> gdn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                const at::Tensor& beta, int64_t L, int64_t C, bool concat) {
  GDN_DISPATCH(forward_t, q, k, v, g, beta, L, C, concat)
  return {};
}

std::vector<at::Tensor> gdn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                const at::Tensor& g, const at::Tensor& beta, const at::Tensor& S_in, int64_t L,
                                int64_t C, bool concat) {
  GDN_DISPATCH(backward_t, dout, q, k, v, g, beta, S_in, L, C, concat)
  return {};
}

std::vector<at::Tensor> gdn_rows(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                 const at::Tensor& beta, const at::Tensor& S0, const c10::optional<at::Tensor>& S_final,
                                 int64_t C) {
  GDN_DISPATCH(rows_t, q, k, v, g, beta, S0, S_final, C)
  return {};
}

// rows with an initial state, for training: {o, S_in} (S_in: the state entering each chunk)
std::vector<at::Tensor> gdn_fwd_rows(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                     const at::Tensor& g, const at::Tensor& beta, const at::Tensor& S0, int64_t C) {
  GDN_DISPATCH(rows_t, q, k, v, g, beta, S0, c10::nullopt, C, true)
  return {};
}

// backward of one causal run per row (q [B, T, ...], T = 2 * (T / 2)) with optional injected
// chunk-entry state gradients; want_dS0 adds the gradient of the initial state as a sixth output
std::vector<at::Tensor> gdn_bwd_rows(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                     const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta,
                                     const at::Tensor& S_in, int64_t C, const c10::optional<at::Tensor>& inj,
                                     bool want_dS0) {
  const int64_t half = q.size(1) / 2;
  GDN_DISPATCH(backward_t, dout, q, k, v, g, beta, S_in, half, C, true, inj, want_dS0)
  return {};
}

}  // namespace bdllm

// ============================================================================ no-allocation entry
// The forward above, with its working memory taken from a fixed array instead of allocated
// tensors. Declared (and its contract described) in gdn_noalloc.h. Left out of the debug-bounds
// build (_C_dbg), so a process that loads both libraries holds one scratch array, not two.
#ifndef BDLLM_DEBUG_BOUNDS
#include <atomic>
#include <cstdio>

#include "gdn_noalloc.h"

namespace {

static __device__ __align__(256) unsigned char g_gdn_noalloc_scratch[BDLLM_GDN_NOALLOC_SCRATCH_BYTES];

// this device's address of the array, looked up on the first call made with the device current
static std::atomic<void*> g_gdn_noalloc_addr[64];

int noalloc_fail(char* err, int err_len, int code, const char* msg) {
  if (err != nullptr && err_len > 0) snprintf(err, (size_t)err_len, "%s", msg);
  return code;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

template <int D>
int noalloc_run(bdllm::gdn::Args a, unsigned char* base, size_t cap, cudaStream_t stream, char* err, int err_len) {
  using namespace bdllm::gdn;
  const size_t units = (size_t)a.B * a.nb * a.Hv;
  const size_t C = (size_t)a.C;
  size_t off = 0;
  auto take = [&](size_t floats) {
    float* p = reinterpret_cast<float*>(base + off);
    off = align256(off + floats * sizeof(float));
    return p;
  };
  a.U = take(units * C * D);
  a.W = take(units * C * D);
  a.Kt = take(units * C * D);
  a.Ec = take(units);
  a.S_in = take(units * D * D);
  a.Vp = take(units * C * D);
  if (off > cap) {
    char msg[160];
    snprintf(msg, sizeof msg, "problem needs %zu bytes of scratch; the fixed array holds %zu", off, cap);
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_TOO_LARGE, msg);
  }
  const int BH = a.B * a.Hv;
  const int big = Smem<D, D>::floats * 4;
  const int rec = (4 * 32 * Ld<D>::v + 3 * 32 * LDC + D * LDC) * 4;
  if (cudaFuncSetAttribute(fwd_prep_kernel<D, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess ||
      cudaFuncSetAttribute(fwd_recur_kernel<D, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, rec) != cudaSuccess ||
      cudaFuncSetAttribute(fwd_out_kernel<D, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "cudaFuncSetAttribute failed");
  // no error was pending on entry, so one seen after a launch is that launch's own
  fwd_prep_kernel<D, D><<<dim3(a.nb, BH), NT, big, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "launch of the chunk-preparation kernel failed");
  fwd_recur_kernel<D, D><<<dim3(BH, (D + 31) / 32), NT, rec, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "launch of the state recurrence kernel failed");
  fwd_out_kernel<D, D><<<dim3(2 * a.nb, BH), NT, big, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "launch of the output kernel failed");
  return BDLLM_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int bdllm_gdn_forward_noalloc(
    const void* q, const void* k, const void* v, int64_t ld_qk, int64_t ld_v, const float* g, const float* beta,
    void* o, int B, int L, int Hk, int Hv, int D, int block, cudaStream_t stream, char* err, int err_len) {
  if (q == nullptr || k == nullptr || v == nullptr || g == nullptr || beta == nullptr || o == nullptr)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_BAD_ARGUMENT, "null pointer argument");
  if (B < 1 || L < 1 || Hk < 1 || Hv < 1 || Hv % Hk != 0 || block < 1 || block > 32 || L % block != 0)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_BAD_ARGUMENT, "need block <= 32 dividing L and Hv % Hk == 0");
  if (D != 16 && D != 32 && D != 64 && D != 128)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_BAD_ARGUMENT, "head dim must be 16, 32, 64 or 128");
  if (ld_qk % 8 != 0 || ld_v % 8 != 0 || ld_qk < (int64_t)Hk * D || ld_v < (int64_t)Hv * D)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_BAD_ARGUMENT, "token strides too small or not multiples of 8");
  // the kernels move q, k, v and o in 16-byte vectors and g, beta as 4-byte floats
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o)) & 15u)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_BAD_ARGUMENT, "q, k, v and o must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(beta)) & 3u)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_BAD_ARGUMENT, "g and beta must be 4-byte aligned");
  // an error left pending by earlier work on this thread belongs to its owner: report it without
  // consuming it, and launch nothing
  if (cudaPeekAtLastError() != cudaSuccess)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "a CUDA error was already pending on entry");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "cudaGetDevice failed");
  void* base = g_gdn_noalloc_addr[dev].load(std::memory_order_acquire);
  if (base == nullptr) {  // first call on this device: look up the array's device address
    if (cudaGetSymbolAddress(&base, g_gdn_noalloc_scratch) != cudaSuccess || base == nullptr)
      return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "cudaGetSymbolAddress failed");
    g_gdn_noalloc_addr[dev].store(base, std::memory_order_release);
  }
  bdllm::gdn::Args a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k = reinterpret_cast<const __nv_bfloat16*>(k);
  a.v = reinterpret_cast<const __nv_bfloat16*>(v);
  a.ldqk = ld_qk;
  a.ldv = ld_v;
  a.g = g;
  a.beta = beta;
  a.B = B;
  a.L = L;
  a.Hk = Hk;
  a.Hv = Hv;
  a.C = block;
  a.concat = 0;
  a.nb = L / block;
  a.scale = 1.f / sqrtf((float)D);
  a.o = reinterpret_cast<__nv_bfloat16*>(o);
  unsigned char* s = reinterpret_cast<unsigned char*>(base);
  const size_t cap = BDLLM_GDN_NOALLOC_SCRATCH_BYTES;
  switch (D) {
    case 16: return noalloc_run<16>(a, s, cap, stream, err, err_len);
    case 32: return noalloc_run<32>(a, s, cap, stream, err, err_len);
    case 64: return noalloc_run<64>(a, s, cap, stream, err, err_len);
    default: return noalloc_run<128>(a, s, cap, stream, err, err_len);
  }
}
#endif  // BDLLM_DEBUG_BOUNDS
