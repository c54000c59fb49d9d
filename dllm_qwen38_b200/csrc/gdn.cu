// State-fork chunked gated delta rule, forward and backward, over the [B, 2L] two-stream layout.
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
// Math is fp32 in shared memory with 4x4 register tiles (CUDA cores).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
namespace gdn {

constexpr int NT = 256;

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
};

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

// tile selection: 4 when the dimension allows it
template <bool AT, bool BT, typename Epi>
__device__ __forceinline__ void matmul(int M, int N, int K, const float* A, int lda, const float* B, int ldb,
                                       Epi epi) {
  if (M % 4 == 0 && N % 4 == 0)
    mm<4, 4, AT, BT>(M, N, K, A, lda, B, ldb, epi);
  else if (N % 4 == 0)
    mm<1, 4, AT, BT>(M, N, K, A, lda, B, ldb, epi);
  else
    mm<1, 1, AT, BT>(M, N, K, A, lda, B, ldb, epi);
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
  return (int64_t)b * 2 * a.L + ((stream && !a.concat) ? a.L : 0) + (int64_t)c * a.C + i;
}

// ------------------------------------------------------------------ per-chunk loads
// sQ/sK [C][Dk] l2-normalised (q scaled), sV [C][Dv], sgam[C] = cumsum g, sbeta[C].
template <int Dk, int Dv>
__device__ void load_chunk(const Args& a, int b, int stream, int c, int h, float* sQ, float* sK, float* sV,
                           float* sgam, float* sbeta, bool need_q, bool need_v) {
  const int C = a.C;
  const int hk = h / (a.Hv / a.Hk);
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk, d = idx % Dk;
    const int64_t t = tok(a, b, stream, c, i);
    sK[i * Dk + d] = __bfloat162float(a.k[t * a.ldqk + hk * Dk + d]);
    if (need_q) sQ[i * Dk + d] = __bfloat162float(a.q[t * a.ldqk + hk * Dk + d]);
  }
  if (need_v)
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
      const int i = idx / Dv, d = idx % Dv;
      sV[i * Dv + d] = __bfloat162float(a.v[tok(a, b, stream, c, i) * a.ldv + h * Dv + d]);
    }
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    float gv = 0.f, bv = 0.f;
    if (i < C) {
      const int64_t t = tok(a, b, stream, c, i);
      gv = a.g[t * a.Hv + h];
      bv = a.beta[t * a.Hv + h];
    }
    // inclusive prefix sum over the chunk (C <= 32)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y = __shfl_up_sync(0xffffffffu, gv, o);
      if (i >= o) gv += y;
    }
    if (i < C) sgam[i] = gv, sbeta[i] = bv;
  }
  __syncthreads();
  // l2 normalisation, one warp per row
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int r = warp; r < (need_q ? 2 * C : C); r += NT / 32) {
    float* row = (r < C) ? sK + r * Dk : sQ + (r - C) * Dk;
    float ss = 0.f;
    for (int d = lane; d < Dk; d += 32) ss += row[d] * row[d];
    ss = wsum(ss);
    const float inv = rsqrtf(ss + 1e-6f) * (r < C ? 1.f : a.scale);
    for (int d = lane; d < Dk; d += 32) row[d] *= inv;
  }
  __syncthreads();
}

// sT = (I + A)^-1 with A = strict_lower(beta_i KK_ij Gam_ij); sKK = k^ k^T must be ready.
__device__ void ut_transform(int C, const float* sKK, const float* sgam, const float* sbeta, float* sA, float* sT) {
  for (int idx = threadIdx.x; idx < C * C; idx += NT) {
    const int i = idx / C, j = idx % C;
    sA[idx] = j < i ? sbeta[i] * sKK[idx] * __expf(sgam[i] - sgam[j]) : 0.f;
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // forward substitution, lane = column (C <= 32)
    const int col = threadIdx.x;
    for (int i = 0; i < C; ++i) {
      float v = (i == col) ? 1.f : 0.f;
      for (int j = 0; j < i; ++j) v -= sA[i * C + j] * sT[j * C + col];
      if (col < C) sT[i * C + col] = v;
      __syncwarp();
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------ smem layout helper
template <int Dk, int Dv>
struct Smem {
  float *Q, *K, *V, *W, *X, *Y, *S, *KK, *A, *T, *P, *gam, *beta, *red;
  __device__ Smem(float* base, int C) {
    float* p = base;
    Q = p; p += 32 * Dk;
    K = p; p += 32 * Dk;
    V = p; p += 32 * Dv;
    W = p; p += 32 * Dk;
    X = p; p += 32 * (Dk > Dv ? Dk : Dv);
    Y = p; p += 32 * (Dk > Dv ? Dk : Dv);
    S = p; p += Dk * Dv;
    KK = p; p += 32 * 32;
    A = p; p += 32 * 32;
    T = p; p += 32 * 32;
    P = p; p += 32 * 32;
    gam = p; p += 32;
    beta = p; p += 32;
    red = p; p += 4 * 32;
  }
  static constexpr int floats = 6 * 32 * 128 + Dk * Dv + 4 * 1024 + 64 + 128;
};

// ================================================================== forward
// prep for clean chunk c: U, W, K~, Ec to scratch.
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) fwd_prep_kernel(Args a) {
  extern __shared__ float sm[];
  Smem<Dk, Dv> s(sm, a.C);
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv, C = a.C;
  load_chunk<Dk, Dv>(a, b, 1, c, h, s.Q, s.K, s.V, s.gam, s.beta, false, true);
  matmul<false, true>(C, C, Dk, s.K, Dk, s.K, Dk, [&](int i, int j, float x) { s.KK[i * C + j] = x; });
  __syncthreads();
  ut_transform(C, s.KK, s.gam, s.beta, s.A, s.T);
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  float* U = a.U + base * C * Dv;
  float* Wg = a.W + base * C * Dk;
  float* Kt = a.Kt + base * C * Dk;
  // U = T diag(beta) V ; W = T diag(beta E) k^
  for (int idx = threadIdx.x; idx < C * Dv; idx += NT) s.X[idx] = s.beta[idx / Dv] * s.V[idx];
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk;
    s.Y[idx] = s.beta[i] * __expf(s.gam[i]) * s.K[idx];
    Kt[idx] = __expf(s.gam[C - 1] - s.gam[i]) * s.K[idx];
  }
  __syncthreads();
  matmul<false, false>(C, Dv, C, s.T, C, s.X, Dv, [&](int i, int d, float x) { U[i * Dv + d] = x; });
  matmul<false, false>(C, Dk, C, s.T, C, s.Y, Dk, [&](int i, int d, float x) { Wg[i * Dk + d] = x; });
  if (threadIdx.x == 0) a.Ec[base] = __expf(s.gam[C - 1]);
}

// sequential state recurrence: CTA per (b, h, 32 value columns); the state slice lives in
// registers (Dk x 32 / NT per thread), the chunk operands stream through smem.
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) fwd_recur_kernel(Args a) {
  extern __shared__ float sm[];
  const int C = a.C;
  float* sW = sm;              // [C][Dk]
  float* sKt = sW + 32 * Dk;   // [C][Dk]
  float* sVp = sKt + 32 * Dk;  // [C][32]
  float* sS = sVp + 32 * 32;   // [Dk][32]
  const int bh = blockIdx.x, b = bh / a.Hv, h = bh % a.Hv;
  const int col0 = blockIdx.y * 32;
  const int ncols = min(32, Dv - col0);
  for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) sS[idx] = 0.f;
  __syncthreads();
  for (int c = 0; c < a.nb; ++c) {
    const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
    float* Sin = a.S_in + base * Dk * Dv;
    for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) {
      const int r = idx / 32, cc = idx % 32;
      if (cc < ncols) Sin[r * Dv + col0 + cc] = sS[idx];
    }
    const float* Wg = a.W + base * C * Dk;
    const float* Kt = a.Kt + base * C * Dk;
    const float* U = a.U + base * C * Dv;
    for (int idx = threadIdx.x; idx < C * Dk; idx += NT) sW[idx] = Wg[idx], sKt[idx] = Kt[idx];
    __syncthreads();
    // V' = U - W S   [C x ncols]
    float* Vp = a.Vp + base * C * Dv;
    matmul<false, false>(C, 32, Dk, sW, Dk, sS, 32, [&](int i, int j, float x) {
      if (j < ncols) {
        const float v = U[i * Dv + col0 + j] - x;
        sVp[i * 32 + j] = v;
        Vp[i * Dv + col0 + j] = v;
      } else {
        sVp[i * 32 + j] = 0.f;
      }
    });
    __syncthreads();
    // S = Ec S + K~^T V'   [Dk x 32]
    const float ec = a.Ec[base];
    matmul<true, false>(Dk, 32, C, sKt, Dk, sVp, 32, [&](int r, int j, float x) {
      sS[r * 32 + j] = ec * sS[r * 32 + j] + x;
    });
    __syncthreads();
  }
}

// output for chunk blockIdx.x of the noised stream (x < nb) or clean stream (x >= nb).
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) fwd_out_kernel(Args a) {
  extern __shared__ float sm[];
  Smem<Dk, Dv> s(sm, a.C);
  const int C = a.C;
  const int stream = (a.concat || blockIdx.x >= a.nb) ? 1 : 0;
  const int c = blockIdx.x - ((stream && !a.concat) ? a.nb : 0);
  const int bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv;
  load_chunk<Dk, Dv>(a, b, stream, c, h, s.Q, s.K, s.V, s.gam, s.beta, true, stream == 0);
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  const float* Sin = a.S_in + base * Dk * Dv;
  for (int idx = threadIdx.x; idx < Dk * Dv; idx += NT) s.S[idx] = Sin[idx];
  // P = q^ k^T * Gam (incl)
  matmul<false, true>(C, C, Dk, s.Q, Dk, s.K, Dk, [&](int i, int j, float x) {
    s.P[i * C + j] = j <= i ? x * __expf(s.gam[i] - s.gam[j]) : 0.f;
  });
  if (stream == 0) {
    matmul<false, true>(C, C, Dk, s.K, Dk, s.K, Dk, [&](int i, int j, float x) { s.KK[i * C + j] = x; });
  }
  __syncthreads();
  float* sVp = s.X;  // [C][Dv]
  if (stream == 0) {
    ut_transform(C, s.KK, s.gam, s.beta, s.A, s.T);
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) s.V[idx] *= s.beta[idx / Dv];
    for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
      const int i = idx / Dk;
      s.Y[idx] = s.beta[i] * __expf(s.gam[i]) * s.K[idx];
    }
    __syncthreads();
    matmul<false, false>(C, Dk, C, s.T, C, s.Y, Dk, [&](int i, int d, float x) { s.W[i * Dk + d] = x; });
    matmul<false, false>(C, Dv, C, s.T, C, s.V, Dv, [&](int i, int d, float x) { sVp[i * Dv + d] = x; });
    __syncthreads();
    matmul<false, false>(C, Dv, Dk, s.W, Dk, s.S, Dv, [&](int i, int d, float x) { sVp[i * Dv + d] -= x; });
  } else {
    const float* Vp = a.Vp + base * C * Dv;
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) sVp[idx] = Vp[idx];
  }
  __syncthreads();
  // O = diag(E) q^ S + P V'
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) s.Q[idx] *= __expf(s.gam[idx / Dk]);
  __syncthreads();
  float* sO = s.Y;
  matmul<false, false>(C, Dv, C, s.P, C, sVp, Dv, [&](int i, int d, float x) { sO[i * Dv + d] = x; });
  __syncthreads();
  matmul<false, false>(C, Dv, Dk, s.Q, Dk, s.S, Dv, [&](int i, int d, float x) {
    a.o[tok(a, b, stream, c, i) * (int64_t)a.Hv * Dv + h * Dv + d] = __float2bfloat16(x + sO[i * Dv + d]);
  });
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
template <int Dk, int Dv>
struct BSmem {
  float *Q, *K, *R0, *dO, *Vp, *dVp, *dR, *dQ, *dK, *S, *KK, *T, *P, *X, *gam, *beta, *dgam, *dE, *dF, *red;
  __device__ BSmem(float* base) {
    float* p = base;
    Q = p; p += 32 * Dk;
    K = p; p += 32 * Dk;
    R0 = p; p += 32 * Dv;
    dO = p; p += 32 * Dv;
    Vp = p; p += 32 * Dv;
    dVp = p; p += 32 * Dv;
    dR = p; p += 32 * Dv;
    dQ = p; p += 32 * Dk;
    dK = p; p += 32 * Dk;
    S = p; p += Dk * Dv;
    KK = p; p += 32 * 32;
    T = p; p += 32 * 32;
    P = p; p += 32 * 32;
    X = p; p += 32 * 32;
    gam = p; p += 32;
    beta = p; p += 32;
    dgam = p; p += 32;
    dE = p; p += 32;
    dF = p; p += 32;
    red = p; p += 32;
  }
  static constexpr int floats = 4 * 32 * Dk + 5 * 32 * Dv + Dk * Dv + 4 * 1024 + 6 * 32;
};

// mode 0: noised block (dS_out = 0, dV' = P^T dO, writes dS_inj[c]); mode 1: clean chunk
// (dV' and dS_out from the reverse recurrence).
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) bwd_chunk_kernel(Args a, int mode) {
  extern __shared__ float sm[];
  BSmem<Dk, Dv> s(sm);
  const int C = a.C;
  const int stream = mode == 0 ? 0 : 1;
  const int c = blockIdx.x;
  const int bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv;
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  // ---- loads: q^, k^, V (into R0), gam, beta, S, dO
  load_chunk<Dk, Dv>(a, b, stream, c, h, s.Q, s.K, s.R0, s.gam, s.beta, true, true);
  const float* Sin = a.S_in + base * Dk * Dv;
  for (int idx = threadIdx.x; idx < Dk * Dv; idx += NT) s.S[idx] = Sin[idx];
  for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
    const int i = idx / Dv, d = idx % Dv;
    s.dO[idx] = __bfloat162float(a.dout[tok(a, b, stream, c, i) * (int64_t)a.Hv * Dv + h * Dv + d]);
  }
  if (threadIdx.x < 32) {
    s.dgam[threadIdx.x] = 0.f, s.dE[threadIdx.x] = 0.f, s.dF[threadIdx.x] = 0.f, s.red[threadIdx.x] = 0.f;
  }
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) s.dQ[idx] = 0.f, s.dK[idx] = 0.f;
  // ---- KK, P (with Gam, incl), T
  matmul<false, true>(C, C, Dk, s.K, Dk, s.K, Dk, [&](int i, int j, float x) { s.KK[i * C + j] = x; });
  matmul<false, true>(C, C, Dk, s.Q, Dk, s.K, Dk, [&](int i, int j, float x) {
    s.P[i * C + j] = j <= i ? x * __expf(s.gam[i] - s.gam[j]) : 0.f;
  });
  __syncthreads();
  ut_transform(C, s.KK, s.gam, s.beta, s.X, s.T);  // X is scratch for A here
  // ---- R0 = V - diag(E) k^ S (in place over V)
  matmul<false, false>(C, Dv, Dk, s.K, Dk, s.S, Dv, [&](int i, int d, float x) {
    s.R0[i * Dv + d] -= __expf(s.gam[i]) * x;
  });
  __syncthreads();
  // ---- V' = (T diag(beta)) R0
  for (int idx = threadIdx.x; idx < C * C; idx += NT) s.X[idx] = s.T[idx] * s.beta[idx % C];
  __syncthreads();
  matmul<false, false>(C, Dv, C, s.X, C, s.R0, Dv, [&](int i, int d, float x) { s.Vp[i * Dv + d] = x; });
  __syncthreads();
  // ---- dV'
  if (mode == 0) {
    matmul<true, false>(C, Dv, C, s.P, C, s.dO, Dv, [&](int i, int d, float x) { s.dVp[i * Dv + d] = x; });
  } else {
    const float* gdv = a.dVp + base * C * Dv;
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) s.dVp[idx] = gdv[idx];
  }
  __syncthreads();
  // ---- dR = T^T dV' ; dV = diag(beta) dR -> global
  matmul<true, false>(C, Dv, C, s.T, C, s.dVp, Dv, [&](int i, int d, float x) {
    s.dR[i * Dv + d] = x;
    a.dv[tok(a, b, stream, c, i) * (int64_t)a.Hv * Dv + h * Dv + d] = __float2bfloat16(s.beta[i] * x);
  });
  __syncthreads();
  // ---- products with S: dQ += diag(E) dO S^T ; dK -= diag(beta E) dR S^T ; dE terms ; dbeta part
  matmul<false, true>(C, Dk, Dv, s.dO, Dv, s.S, Dv, [&](int i, int d, float x) {
    s.dQ[i * Dk + d] += __expf(s.gam[i]) * x;
  });
  matmul<false, true>(C, Dk, Dv, s.dR, Dv, s.S, Dv, [&](int i, int d, float x) {
    s.dK[i * Dk + d] -= s.beta[i] * __expf(s.gam[i]) * x;
  });
  matmul<false, false>(C, Dv, Dk, s.Q, Dk, s.S, Dv, [&](int i, int d, float x) {
    atomicAdd(&s.dE[i], x * s.dO[i * Dv + d]);
  });
  matmul<false, false>(C, Dv, Dk, s.K, Dk, s.S, Dv, [&](int i, int d, float x) {
    atomicAdd(&s.dE[i], -s.beta[i] * x * s.dR[i * Dv + d]);
  });
  for (int idx = threadIdx.x; idx < C * Dv; idx += NT) atomicAdd(&s.red[idx / Dv], s.dR[idx] * s.R0[idx]);
  __syncthreads();
  // ---- dP = dO V'^T ; dPm = dP * Gam (incl) -> X ; dgam += rowsum(dP*P) - colsum(dP*P)
  matmul<false, true>(C, C, Dv, s.dO, Dv, s.Vp, Dv, [&](int i, int j, float x) {
    const float gm = j <= i ? __expf(s.gam[i] - s.gam[j]) : 0.f;
    s.X[i * C + j] = x * gm;
    const float g1 = x * s.P[i * C + j];
    atomicAdd(&s.dgam[i], g1);
    atomicAdd(&s.dgam[j], -g1);
  });
  __syncthreads();
  // dQ += dPm k^ ; dK += dPm^T q^
  matmul<false, false>(C, Dk, C, s.X, C, s.K, Dk, [&](int i, int d, float x) { s.dQ[i * Dk + d] += x; });
  matmul<true, false>(C, Dk, C, s.X, C, s.Q, Dk, [&](int i, int d, float x) { s.dK[i * Dk + d] += x; });
  __syncthreads();
  // ---- state gradient
  if (mode == 0) {
    // dS_inj = (diag(E) q^)^T dO - k^T diag(beta E) dR ; dO and dR are consumed here (scaled in place)
    for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
      const int i = idx / Dv;
      const float e = __expf(s.gam[i]);
      s.dO[idx] *= e;
      s.dR[idx] *= s.beta[i] * e;
    }
    __syncthreads();
    matmul<true, false>(Dk, Dv, C, s.Q, Dk, s.dO, Dv, [&](int r, int d, float x) { s.S[r * Dv + d] = x; });
    __syncthreads();
    float* dSi = a.dS_inj + base * Dk * Dv;
    matmul<true, false>(Dk, Dv, C, s.K, Dk, s.dR, Dv, [&](int r, int d, float x) {
      dSi[r * Dv + d] = s.S[r * Dv + d] - x;
    });
    __syncthreads();
  } else {
    // dEc = sum S * dS_out (S still in smem, dS_out from global) ; then S <- dS_out
    const float* dSo = a.dS_out + base * Dk * Dv;
    float part = 0.f;
    for (int idx = threadIdx.x; idx < Dk * Dv; idx += NT) part += s.S[idx] * dSo[idx];
    part = wsum(part);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s.dgam[C - 1], part * __expf(s.gam[C - 1]));  // dEc * Ec
    __syncthreads();
    for (int idx = threadIdx.x; idx < Dk * Dv; idx += NT) s.S[idx] = dSo[idx];
    __syncthreads();
    // dK += diag(F) V' dS_out^T ; dF_i = sum_b (k^ dS_out)_ib V'_ib
    matmul<false, true>(C, Dk, Dv, s.Vp, Dv, s.S, Dv, [&](int i, int d, float x) {
      s.dK[i * Dk + d] += __expf(s.gam[C - 1] - s.gam[i]) * x;
    });
    matmul<false, false>(C, Dv, Dk, s.K, Dk, s.S, Dv, [&](int i, int d, float x) {
      atomicAdd(&s.dF[i], x * s.Vp[i * Dv + d]);
    });
    __syncthreads();
  }
  // ---- dT = dV' R^T with R = diag(beta) R0 -> P (P no longer needed)
  matmul<false, true>(C, C, Dv, s.dVp, Dv, s.R0, Dv, [&](int i, int j, float x) { s.P[i * C + j] = x * s.beta[j]; });
  __syncthreads();
  // dA = strict_lower(-T^T dT T^T): M = dT T^T -> X, then -T^T M -> P (masked)
  matmul<false, true>(C, C, C, s.P, C, s.T, C, [&](int i, int j, float x) { s.X[i * C + j] = x; });
  __syncthreads();
  matmul<true, false>(C, C, C, s.T, C, s.X, C, [&](int i, int j, float x) { s.P[i * C + j] = j < i ? -x : 0.f; });
  __syncthreads();
  // dbeta += sum_j dA_ij KK_ij Gam_ij ; dKK = dA * beta_i * Gam (-> X) ; dgam from H2
  for (int idx = threadIdx.x; idx < C * C; idx += NT) {
    const int i = idx / C, j = idx % C;
    const float gm = j < i ? __expf(s.gam[i] - s.gam[j]) : 0.f;
    const float dA = s.P[idx];
    const float h2 = dA * s.beta[i] * s.KK[idx] * gm;
    atomicAdd(&s.red[i], dA * s.KK[idx] * gm);
    atomicAdd(&s.dgam[i], h2);
    atomicAdd(&s.dgam[j], -h2);
    s.X[idx] = dA * s.beta[i] * gm;
  }
  __syncthreads();
  // dK += dKK k^ + dKK^T k^
  matmul<false, false>(C, Dk, C, s.X, C, s.K, Dk, [&](int i, int d, float x) { s.dK[i * Dk + d] += x; });
  __syncthreads();
  matmul<true, false>(C, Dk, C, s.X, C, s.K, Dk, [&](int i, int d, float x) { s.dK[i * Dk + d] += x; });
  __syncthreads();
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
  // ---- l2norm backward (warp per row): dq = l2_bwd(q_raw, scale * dQ), dk = l2_bwd(k_raw, dK)
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int hk = h / (a.Hv / a.Hk);
  for (int r = warp; r < 2 * C; r += NT / 32) {
    const bool isq = r >= C;
    const int i = isq ? r - C : r;
    const int64_t t = tok(a, b, stream, c, i);
    const __nv_bfloat16* src = (isq ? a.q : a.k) + t * a.ldqk + hk * Dk;
    const float* dy = (isq ? s.dQ : s.dK) + i * Dk;
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
}

// clean chunks: what the reverse recurrence needs -> PtdO [C][Dv], Kt [C][Dk], Qt [C][Dk], W [C][Dk], Ec
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) bwd_prep_kernel(Args a) {
  extern __shared__ float sm[];
  Smem<Dk, Dv> s(sm, a.C);
  const int C = a.C;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv;
  load_chunk<Dk, Dv>(a, b, 1, c, h, s.Q, s.K, s.V, s.gam, s.beta, true, false);
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  for (int idx = threadIdx.x; idx < C * Dv; idx += NT) {
    const int i = idx / Dv, d = idx % Dv;
    s.X[idx] = __bfloat162float(a.dout[tok(a, b, 1, c, i) * (int64_t)a.Hv * Dv + h * Dv + d]);
  }
  matmul<false, true>(C, C, Dk, s.K, Dk, s.K, Dk, [&](int i, int j, float x) { s.KK[i * C + j] = x; });
  matmul<false, true>(C, C, Dk, s.Q, Dk, s.K, Dk, [&](int i, int j, float x) {
    s.P[i * C + j] = j <= i ? x * __expf(s.gam[i] - s.gam[j]) : 0.f;
  });
  __syncthreads();
  ut_transform(C, s.KK, s.gam, s.beta, s.A, s.T);
  float* PtdO = a.PtdO + base * C * Dv;
  matmul<true, false>(C, Dv, C, s.P, C, s.X, Dv, [&](int i, int d, float x) { PtdO[i * Dv + d] = x; });
  float* Kt = a.Kt + base * C * Dk;
  float* Qt = a.Qt + base * C * Dk;
  for (int idx = threadIdx.x; idx < C * Dk; idx += NT) {
    const int i = idx / Dk;
    Kt[idx] = __expf(s.gam[C - 1] - s.gam[i]) * s.K[idx];
    Qt[idx] = __expf(s.gam[i]) * s.Q[idx];
    s.Y[idx] = s.beta[i] * __expf(s.gam[i]) * s.K[idx];
  }
  __syncthreads();
  float* Wg = a.W + base * C * Dk;
  matmul<false, false>(C, Dk, C, s.T, C, s.Y, Dk, [&](int i, int d, float x) { Wg[i * Dk + d] = x; });
  if (threadIdx.x == 0) a.Ec[base] = __expf(s.gam[C - 1]);
}

// reverse recurrence, CTA per (b, h, 32 value columns):
//   dS_out[c] = dS ; dV'_c = PtdO_c + K~_c dS ; dS = Ec dS + q~_c^T dO_c - W_c^T dV'_c (+ dS_inj[c])
template <int Dk, int Dv>
__global__ void __launch_bounds__(NT) bwd_recur_kernel(Args a, int has_inj) {
  extern __shared__ float sm[];
  const int C = a.C;
  float* sW = sm;               // [C][Dk]
  float* sKt = sW + 32 * Dk;    // [C][Dk]
  float* sQt = sKt + 32 * Dk;   // [C][Dk]
  float* sdVp = sQt + 32 * Dk;  // [C][32]
  float* sdO = sdVp + 32 * 32;  // [C][32]
  float* sS = sdO + 32 * 32;    // [Dk][32]
  const int bh = blockIdx.x, b = bh / a.Hv, h = bh % a.Hv;
  const int col0 = blockIdx.y * 32;
  const int ncols = min(32, Dv - col0);
  for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) sS[idx] = 0.f;
  __syncthreads();
  for (int c = a.nb - 1; c >= 0; --c) {
    const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
    float* dSo = a.dS_out + base * Dk * Dv;
    for (int idx = threadIdx.x; idx < Dk * 32; idx += NT) {
      const int r = idx / 32, cc = idx % 32;
      if (cc < ncols) dSo[r * Dv + col0 + cc] = sS[idx];
    }
    const float* Wg = a.W + base * C * Dk;
    const float* Kt = a.Kt + base * C * Dk;
    const float* Qt = a.Qt + base * C * Dk;
    for (int idx = threadIdx.x; idx < C * Dk; idx += NT) sW[idx] = Wg[idx], sKt[idx] = Kt[idx], sQt[idx] = Qt[idx];
    for (int idx = threadIdx.x; idx < C * 32; idx += NT) {
      const int i = idx / 32, cc = idx % 32;
      sdO[idx] = cc < ncols ? __bfloat162float(a.dout[tok(a, b, 1, c, i) * (int64_t)a.Hv * Dv + h * Dv + col0 + cc])
                            : 0.f;
    }
    __syncthreads();
    const float* PtdO = a.PtdO + base * C * Dv;
    float* dVp = a.dVp + base * C * Dv;
    matmul<false, false>(C, 32, Dk, sKt, Dk, sS, 32, [&](int i, int j, float x) {
      if (j < ncols) {
        const float v = PtdO[i * Dv + col0 + j] + x;
        sdVp[i * 32 + j] = v;
        dVp[i * Dv + col0 + j] = v;
      } else {
        sdVp[i * 32 + j] = 0.f;
      }
    });
    __syncthreads();
    const float ec = a.Ec[base];
    const float* inj = has_inj ? a.dS_inj + base * Dk * Dv : nullptr;
    // dS = Ec dS + Qt^T dO - W^T dV' (+ inj): two products into registers via the epilogue
    matmul<true, false>(Dk, 32, C, sQt, Dk, sdO, 32, [&](int r, int j, float x) {
      sS[r * 32 + j] = ec * sS[r * 32 + j] + x;
    });
    __syncthreads();
    matmul<true, false>(Dk, 32, C, sW, Dk, sdVp, 32, [&](int r, int j, float x) {
      float v = sS[r * 32 + j] - x;
      if (inj != nullptr && j < ncols) v += inj[r * Dv + col0 + j];
      sS[r * 32 + j] = v;
    });
    __syncthreads();
  }
}

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
  TORCH_CHECK(q.stride(0) == q.size(1) * q.stride(1) && v.stride(0) == v.size(1) * v.stride(1),
              "gdn: batch and token dims must merge");
  TORCH_CHECK(g.is_contiguous() && beta.is_contiguous() && g.scalar_type() == at::kFloat &&
                  beta.scalar_type() == at::kFloat,
              "gdn: g, beta fp32 contiguous [B, 2L, Hv]");
  TORCH_CHECK(C <= 32 && C >= 1 && (2 * L) % C == 0 && L % C == 0, "gdn: chunk (= block) must be <= 32 and divide L");
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
  launch(fwd_recur_kernel<Dk, Dv>, dim3(BH, (Dv + 31) / 32), 3 * 32 * Dk + 32 * 32 + Dk * 32, a);
  // noised blocks (x < nb) only exist with the fork
  const int ngrid = concat ? a.nb : 2 * a.nb;
  launch(fwd_out_kernel<Dk, Dv>, dim3(ngrid, BH), Smem<Dk, Dv>::floats, a);
  return {o, S_in, Vp};
}

// Backward. Returns {dq, dk (per v-head), dv, dg, dbeta}.
template <int Dk, int Dv>
static std::vector<at::Tensor> backward_t(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                          const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta,
                                          const at::Tensor& S_in, int64_t L, int64_t C, bool concat) {
  Args a = make_args(q, k, v, g, beta, L, C, concat);
  auto f32 = q.options().dtype(at::kFloat);
  auto d = dout.to(at::kBFloat16).contiguous();
  a.dout = reinterpret_cast<const __nv_bfloat16*>(d.data_ptr());
  a.S_in = const_cast<float*>(S_in.data_ptr<float>());
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
  auto dS_inj = concat ? at::Tensor() : at::empty({a.B, a.nb, a.Hv, Dk, Dv}, f32);
  auto dS_out = at::empty({a.B, a.nb, a.Hv, Dk, Dv}, f32);
  auto dVp = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto PtdO = at::empty({a.B, a.nb, a.Hv, C, Dv}, f32);
  auto Qt = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Kt = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto W = at::empty({a.B, a.nb, a.Hv, C, Dk}, f32);
  auto Ec = at::empty({a.B, a.nb, a.Hv}, f32);
  a.dS_inj = concat ? nullptr : dS_inj.data_ptr<float>();
  a.dS_out = dS_out.data_ptr<float>();
  a.dVp = dVp.data_ptr<float>();
  a.PtdO = PtdO.data_ptr<float>();
  a.Qt = Qt.data_ptr<float>();
  a.Kt = Kt.data_ptr<float>();
  a.W = W.data_ptr<float>();
  a.Ec = Ec.data_ptr<float>();
  const int BH = a.B * a.Hv;
  if (!concat) launch2(bwd_chunk_kernel<Dk, Dv>, dim3(a.nb, BH), BSmem<Dk, Dv>::floats, a, 0);
  launch(bwd_prep_kernel<Dk, Dv>, dim3(a.nb, BH), Smem<Dk, Dv>::floats, a);
  launch2(bwd_recur_kernel<Dk, Dv>, dim3(BH, (Dv + 31) / 32), 3 * 32 * Dk + 2 * 32 * 32 + Dk * 32, a,
          concat ? 0 : 1);
  launch2(bwd_chunk_kernel<Dk, Dv>, dim3(a.nb, BH), BSmem<Dk, Dv>::floats, a, 1);
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
  c10::cuda::CUDAGuard guard(q.device());
  GDN_DISPATCH(forward_t, q, k, v, g, beta, L, C, concat)
  return {};
}

std::vector<at::Tensor> gdn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                const at::Tensor& g, const at::Tensor& beta, const at::Tensor& S_in, int64_t L,
                                int64_t C, bool concat) {
  c10::cuda::CUDAGuard guard(q.device());
  GDN_DISPATCH(backward_t, dout, q, k, v, g, beta, S_in, L, C, concat)
  return {};
}

}  // namespace bdllm

// ============================================================================ no-allocation entry
// The forward above, with its working memory taken from a fixed array instead of allocated
// tensors. Declared (and its contract described) in gdn_noalloc.h.
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
  const int rec = (3 * 32 * D + 32 * 32 + D * 32) * 4;
  if (cudaFuncSetAttribute(fwd_prep_kernel<D, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess ||
      cudaFuncSetAttribute(fwd_recur_kernel<D, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, rec) != cudaSuccess ||
      cudaFuncSetAttribute(fwd_out_kernel<D, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "cudaFuncSetAttribute failed");
  fwd_prep_kernel<D, D><<<dim3(a.nb, BH), NT, big, stream>>>(a);
  fwd_recur_kernel<D, D><<<dim3(BH, (D + 31) / 32), NT, rec, stream>>>(a);
  fwd_out_kernel<D, D><<<dim3(2 * a.nb, BH), NT, big, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_CUDA_ERROR, "kernel launch failed");
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
  if (ld_qk % 8 != 0 || ld_v % 8 != 0 || ld_qk < 2 * (int64_t)Hk * D || ld_v < (int64_t)Hv * D)
    return noalloc_fail(err, err_len, BDLLM_NOALLOC_BAD_ARGUMENT, "token strides too small or not multiples of 8");
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
