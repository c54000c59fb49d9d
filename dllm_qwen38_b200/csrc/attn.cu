// Complementary-mask flash attention over the [B, 2L] two-stream layout, GQA, forward and
// backward. The mask is a predicate on positions (never stored):
//   x_t row i sees x_t key j iff block(j) == block(i)   (block(j) <= block(i) for the mask-leak fault)
//   x_t row i sees x_0 key j iff block(j) <  block(i)
//   x_0 row i sees x_0 key j iff block(j) <= block(i);   x_0 never sees x_t
// Key tiles that no row of a query tile may see are skipped (about half of the 2L x 2L pairs).
// (The reference builds a dense [2L, 2L] additive mask, `src/dllm_qwen38/blockdiff.py:50-66`, and runs
// HF eager or SDPA attention over it, `blockdiff.py:178-182`.)
//
// Tiles of 64 query rows x 64 keys, 4 warps (16 rows each), bf16 mma.sync m16n8k16 with fp32
// accumulation, online softmax in base 2. Shared tiles are 16-byte-chunk XOR-swizzled for
// conflict-free ldmatrix. Forward writes O and the per-row log2-sum-exp; backward is two kernels:
// dQ per query tile (with Delta = rowsum(dO * O)), and dK/dV per key tile looping over the query
// heads of its GQA group (for head dim 256 the dK/dV accumulators are split across two CTAs by
// head-dim halves).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
bool attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                 int64_t L, int64_t block, double scale, bool leak);
bool attn_bwd_tc(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                 const at::Tensor& o, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
                 at::Tensor& dv, int64_t L, int64_t block, double scale, bool leak);

namespace attn {

constexpr int TILE = 64;
constexpr int NTH = 128;
constexpr float NEG_INF = -INFINITY;

struct Args {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_tok, k_tok, v_tok;  // token strides (elements); heads packed at stride D
  __nv_bfloat16* o;             // [B, T2, Hq, D]
  float* lse2;                  // [B, Hq, T2]  log2-sum-exp of the scaled scores
  const __nv_bfloat16* o_in;    // forward output (backward)
  const __nv_bfloat16* dout;    // [B, T2, Hq, D]
  float* delta;                 // [B, Hq, T2]
  __nv_bfloat16* dq;            // [B, T2, Hq, D]
  __nv_bfloat16* dk;            // [B, T2, Hk, D]
  __nv_bfloat16* dv;            // [B, T2, Hk, D]
  int B, T2, L, Hq, Hk, block, leak;  // leak 2: every key visible (decode over a KV cache)
  float scale, scale_log2;
  // forward only: keys may be a separate, longer sequence (a KV cache) with their own batch
  // strides; the key count is Tk, or *tk_dev when set (read on the device, graph-capturable)
  int Tk;
  int64_t q_bat, k_bat, v_bat;
  const int* tk_dev;
};

constexpr int LEAK_ALL = 2;

__device__ __forceinline__ bool allowed(int i, int j, int L, int block, int leak) {
  const bool it = i < L, jt = j < L;
  const int bi = (it ? i : i - L) / block, bj = (jt ? j : j - L) / block;
  if (it) return jt ? (leak ? bj <= bi : bj == bi) : (bj < bi);
  return jt ? false : (bj <= bi);
}

// may any row in [i0, i1] see any key in [j0, j1]?
__device__ __forceinline__ bool tile_may(int i0, int i1, int j0, int j1, int L, int block, int leak) {
  bool any = false;
  if (i0 < L) {
    const int qb0 = i0 / block, qb1 = min(i1, L - 1) / block;
    if (j0 < L) {
      const int kb0 = j0 / block, kb1 = min(j1, L - 1) / block;
      any |= leak ? (kb0 <= qb1) : (kb0 <= qb1 && kb1 >= qb0);
    }
    if (j1 >= L) any |= ((max(j0, L) - L) / block) < qb1;
  }
  if (i1 >= L && j1 >= L) any |= ((max(j0, L) - L) / block) <= (i1 - L) / block;
  return any;
}

// --------------------------------------------------------------- smem tiles and fragments
template <int D>
__device__ __forceinline__ int sw(int r, int c8) {  // element offset of 16-byte chunk c8 of row r
  constexpr int M = (D / 8 >= 8) ? 7 : (D / 8 - 1);
  return r * D + ((c8 ^ (r & M)) << 3);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = smem_u32(dst);
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// 64 rows x D of a [B*T2, ...] tensor with token stride `tok` (elements) starting at row r0
template <int D, int ROWS = TILE>
__device__ __forceinline__ void load_tile(__nv_bfloat16* s, const __nv_bfloat16* base, int64_t tok, int r0, int T2) {
  constexpr int CH = D / 8;
  for (int idx = threadIdx.x; idx < ROWS * CH; idx += NTH) {
    const int r = idx / CH, c8 = idx % CH;
    const bool ok = r0 + r < T2;
    const __nv_bfloat16* src = base + (int64_t)(ok ? r0 + r : 0) * tok + c8 * 8;
    cp_async16(s + sw<D>(r, c8), src, ok);
  }
}

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// A fragment (16 x 16) at rows r0.., cols k0.. of a swizzled [64][D] tile
template <int D>
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], const __nv_bfloat16* s, int r0, int k0) {
  const int lane = threadIdx.x & 31, mi = lane >> 3;
  ldsm4(a, s + sw<D>(r0 + (mi & 1) * 8 + (lane & 7), (k0 >> 3) + (mi >> 1)));
}
// two B fragments (n-tiles n0.. and n0+8..) for a K x N operand stored as rows n (cols = k)
template <int D>
__device__ __forceinline__ void frag_b_rows(uint32_t (&b)[4], const __nv_bfloat16* s, int n0, int k0) {
  const int lane = threadIdx.x & 31, mi = lane >> 3;
  ldsm4(b, s + sw<D>(n0 + (mi >> 1) * 8 + (lane & 7), (k0 >> 3) + (mi & 1)));
}
// two B fragments (n-tiles n0.. and n0+8..) for a K x N operand stored as rows k (cols = n)
template <int D>
__device__ __forceinline__ void frag_b_cols(uint32_t (&b)[4], const __nv_bfloat16* s, int k0, int n0) {
  const int lane = threadIdx.x & 31, mi = lane >> 3;
  ldsm4t(b, s + sw<D>(k0 + (mi & 1) * 8 + (lane & 7), (n0 >> 3) + (mi >> 1)));
}

// S[16 x 8*NN] (NN n-tiles) = A(rows of sa starting at ra, all D) * B(rows of sb)^T
template <int D, int NN = 8>
__device__ __forceinline__ void qk_tile(float (&s)[NN][4], const __nv_bfloat16* sa, int ra, const __nv_bfloat16* sb) {
#pragma unroll
  for (int n = 0; n < NN; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < D; kk += 16) {
    uint32_t a[4];
    frag_a<D>(a, sa, ra, kk);
#pragma unroll
    for (int p = 0; p < NN / 2; ++p) {
      uint32_t b[4];
      frag_b_rows<D>(b, sb, p * 16, kk);
      mma(s[2 * p], a, b[0], b[1]);
      mma(s[2 * p + 1], a, b[2], b[3]);
    }
  }
}

// acc[DA/8][4] += P(16 x 8*NN, from registers) * B(rows k of sb = 8*NN keys, cols d0..d0+DA)
template <int D, int DA, int NN = 8>
__device__ __forceinline__ void pv_tile(float (&acc)[DA / 8][4], const float (&p)[NN][4], const __nv_bfloat16* sb,
                                        int d0) {
#pragma unroll
  for (int kp = 0; kp < NN / 2; ++kp) {
    uint32_t a[4] = {pack(p[2 * kp][0], p[2 * kp][1]), pack(p[2 * kp][2], p[2 * kp][3]),
                     pack(p[2 * kp + 1][0], p[2 * kp + 1][1]), pack(p[2 * kp + 1][2], p[2 * kp + 1][3])};
#pragma unroll
    for (int dp = 0; dp < DA / 16; ++dp) {
      uint32_t b[4];
      frag_b_cols<D>(b, sb, kp * 16, d0 + dp * 16);
      mma(acc[2 * dp], a, b[0], b[1]);
      mma(acc[2 * dp + 1], a, b[2], b[3]);
    }
  }
}

// ================================================================== forward
template <int D>
__global__ void __launch_bounds__(NTH, 1) fwd_kernel(Args a) {
  extern __shared__ __align__(128) __nv_bfloat16 sm[];
  __nv_bfloat16* sQ = sm;
  __nv_bfloat16* sK = sm + TILE * D;
  __nv_bfloat16* sV = sm + 2 * TILE * D;
  const int i0 = blockIdx.x * TILE;
  const int b = blockIdx.y / a.Hq, h = blockIdx.y % a.Hq, hk = h / (a.Hq / a.Hk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const __nv_bfloat16* qb = a.q + (int64_t)b * a.q_bat + h * D;
  const __nv_bfloat16* kb = a.k + (int64_t)b * a.k_bat + hk * D;
  const __nv_bfloat16* vb = a.v + (int64_t)b * a.v_bat + hk * D;
  const int Tk = a.tk_dev != nullptr ? *a.tk_dev : a.Tk;
  const bool all = a.leak == LEAK_ALL;
  load_tile<D>(sQ, qb, a.q_tok, i0, a.T2);
  cp_commit();
  const int r0 = i0 + warp * 16 + g, r1 = r0 + 8;
  float m[2] = {NEG_INF, NEG_INF}, l[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const int i1 = min(i0 + TILE - 1, a.T2 - 1);
  for (int j0 = 0; j0 < Tk; j0 += TILE) {
    if (!all && !tile_may(i0, i1, j0, min(j0 + TILE - 1, Tk - 1), a.L, a.block, a.leak)) continue;
    __syncthreads();
    load_tile<D>(sK, kb, a.k_tok, j0, Tk);
    load_tile<D>(sV, vb, a.v_tok, j0, Tk);
    cp_commit();
    cp_wait_all();
    __syncthreads();
    float s[8][4];
    qk_tile<D>(s, sQ, warp * 16, sK);
    float mx[2] = {NEG_INF, NEG_INF};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = e < 2 ? r0 : r1, col = j0 + n * 8 + t4 * 2 + (e & 1);
        float v = s[n][e] * a.scale_log2;
        if (row >= a.T2 || col >= Tk || !(all || allowed(row, col, a.L, a.block, a.leak))) v = NEG_INF;
        s[n][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], mu[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mn = fmaxf(m[r], mx[r]);
      mu[r] = mn == NEG_INF ? 0.f : mn;
      alpha[r] = exp2f(m[r] - mu[r]);
      m[r] = mn;
    }
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[n][e] - mu[e >> 1]);
        s[n][e] = p;
        rs[e >> 1] += p;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l[r] = l[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= alpha[0], o[n][1] *= alpha[0];
      o[n][2] *= alpha[1], o[n][3] *= alpha[1];
    }
    pv_tile<D, D>(o, s, sV, 0);
  }
  // finalize
  const float inv0 = l[0] > 0.f ? 1.f / l[0] : 0.f, inv1 = l[1] > 0.f ? 1.f / l[1] : 0.f;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int col = n * 8 + t4 * 2;
    if (r0 < a.T2)
      *reinterpret_cast<__nv_bfloat162*>(a.o + ((int64_t)b * a.T2 + r0) * a.Hq * D + h * D + col) =
          __floats2bfloat162_rn(o[n][0] * inv0, o[n][1] * inv0);
    if (r1 < a.T2)
      *reinterpret_cast<__nv_bfloat162*>(a.o + ((int64_t)b * a.T2 + r1) * a.Hq * D + h * D + col) =
          __floats2bfloat162_rn(o[n][2] * inv1, o[n][3] * inv1);
  }
  if (t4 == 0) {
    float* lse = a.lse2 + ((int64_t)b * a.Hq + h) * a.T2;
    if (r0 < a.T2) lse[r0] = m[0] + log2f(fmaxf(l[0], 1e-30f));
    if (r1 < a.T2) lse[r1] = m[1] + log2f(fmaxf(l[1], 1e-30f));
  }
}

// ================================================================== backward: dQ
// key tiles of TK = 32 rows: Q, dO (64 rows) + K, V (32 rows) = 96 KB at D = 256, two CTAs per SM
constexpr int TK = 32;
template <int D>
__global__ void __launch_bounds__(NTH, 2) bwd_dq_kernel(Args a) {
  extern __shared__ __align__(128) __nv_bfloat16 sm[];
  __nv_bfloat16* sQ = sm;
  __nv_bfloat16* sdO = sm + TILE * D;
  __nv_bfloat16* sK = sm + 2 * TILE * D;
  __nv_bfloat16* sV = sm + 2 * TILE * D + TK * D;
  const int i0 = blockIdx.x * TILE;
  const int b = blockIdx.y / a.Hq, h = blockIdx.y % a.Hq, hk = h / (a.Hq / a.Hk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const __nv_bfloat16* qb = a.q + (int64_t)b * a.T2 * a.q_tok + h * D;
  const __nv_bfloat16* kb = a.k + (int64_t)b * a.T2 * a.k_tok + hk * D;
  const __nv_bfloat16* vb = a.v + (int64_t)b * a.T2 * a.v_tok + hk * D;
  const int64_t otok = (int64_t)a.Hq * D;
  const __nv_bfloat16* dob = a.dout + (int64_t)b * a.T2 * otok + h * D;
  load_tile<D>(sQ, qb, a.q_tok, i0, a.T2);
  load_tile<D>(sdO, dob, otok, i0, a.T2);
  cp_commit();
  // Delta = rowsum(dO * O), one warp per row (16 rows per warp)
  float* delta = a.delta + ((int64_t)b * a.Hq + h) * a.T2;
  const __nv_bfloat16* ob = a.o_in + (int64_t)b * a.T2 * otok + h * D;
  for (int rr = 0; rr < 16; ++rr) {
    const int row = i0 + warp * 16 + rr;
    float acc = 0.f;
    if (row < a.T2)
      for (int d = lane; d < D; d += 32)
        acc += __bfloat162float(dob[(int64_t)row * otok + d]) * __bfloat162float(ob[(int64_t)row * otok + d]);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 16);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 8);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 4);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 2);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
    if (lane == 0 && row < a.T2) delta[row] = acc;
  }
  __syncwarp();
  const int r0 = i0 + warp * 16 + g, r1 = r0 + 8;
  const float* lse = a.lse2 + ((int64_t)b * a.Hq + h) * a.T2;
  const float l0 = r0 < a.T2 ? lse[r0] : 0.f, l1 = r1 < a.T2 ? lse[r1] : 0.f;
  const float d0 = r0 < a.T2 ? delta[r0] : 0.f, d1 = r1 < a.T2 ? delta[r1] : 0.f;
  float dq[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;
  const int i1 = min(i0 + TILE - 1, a.T2 - 1);
  for (int j0 = 0; j0 < a.T2; j0 += TK) {
    if (!tile_may(i0, i1, j0, min(j0 + TK - 1, a.T2 - 1), a.L, a.block, a.leak)) continue;
    __syncthreads();
    load_tile<D, TK>(sK, kb, a.k_tok, j0, a.T2);
    load_tile<D, TK>(sV, vb, a.v_tok, j0, a.T2);
    cp_commit();
    cp_wait_all();
    __syncthreads();
    float s[TK / 8][4], dp[TK / 8][4];
    qk_tile<D, TK / 8>(s, sQ, warp * 16, sK);
    qk_tile<D, TK / 8>(dp, sdO, warp * 16, sV);
#pragma unroll
    for (int n = 0; n < TK / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = e < 2 ? r0 : r1, col = j0 + n * 8 + t4 * 2 + (e & 1);
        const bool ok = row < a.T2 && col < a.T2 && allowed(row, col, a.L, a.block, a.leak);
        const float p = ok ? exp2f(s[n][e] * a.scale_log2 - (e < 2 ? l0 : l1)) : 0.f;
        s[n][e] = p * (dp[n][e] - (e < 2 ? d0 : d1));  // dS
      }
    pv_tile<D, D, TK / 8>(dq, s, sK, 0);
  }
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int col = n * 8 + t4 * 2;
    if (r0 < a.T2)
      *reinterpret_cast<__nv_bfloat162*>(a.dq + ((int64_t)b * a.T2 + r0) * otok + h * D + col) =
          __floats2bfloat162_rn(dq[n][0] * a.scale, dq[n][1] * a.scale);
    if (r1 < a.T2)
      *reinterpret_cast<__nv_bfloat162*>(a.dq + ((int64_t)b * a.T2 + r1) * otok + h * D + col) =
          __floats2bfloat162_rn(dq[n][2] * a.scale, dq[n][3] * a.scale);
  }
}

// ================================================================== backward: dK, dV
// CTA = 64 keys of one kv head; blockIdx.z selects the head-dim slice [z*DA, (z+1)*DA) of dK/dV.
// query tiles of TQ = 32 rows: K, V (64 rows) + Q, dO (32 rows) = 96 KB at D = 256, two CTAs per SM
constexpr int TQ = 32;
template <int D, int DA>
__global__ void __launch_bounds__(NTH, 2) bwd_dkv_kernel(Args a) {
  extern __shared__ __align__(128) __nv_bfloat16 sm[];
  __nv_bfloat16* sK = sm;
  __nv_bfloat16* sV = sm + TILE * D;
  __nv_bfloat16* sQ = sm + 2 * TILE * D;
  __nv_bfloat16* sdO = sm + 2 * TILE * D + TQ * D;
  float* sL = reinterpret_cast<float*>(sm + 2 * TILE * D + 2 * TQ * D);  // [TQ] lse2
  float* sD = sL + TQ;                                                   // [TQ] delta
  const int j0 = blockIdx.x * TILE;
  const int b = blockIdx.y / a.Hk, hk = blockIdx.y % a.Hk;
  const int d0 = blockIdx.z * DA;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const __nv_bfloat16* kb = a.k + (int64_t)b * a.T2 * a.k_tok + hk * D;
  const __nv_bfloat16* vb = a.v + (int64_t)b * a.T2 * a.v_tok + hk * D;
  load_tile<D>(sK, kb, a.k_tok, j0, a.T2);
  load_tile<D>(sV, vb, a.v_tok, j0, a.T2);
  cp_commit();
  const int k0 = j0 + warp * 16 + g, k1 = k0 + 8;  // this thread's key rows
  float dk[DA / 8][4], dv[DA / 8][4];
#pragma unroll
  for (int n = 0; n < DA / 8; ++n) {
    dk[n][0] = dk[n][1] = dk[n][2] = dk[n][3] = 0.f;
    dv[n][0] = dv[n][1] = dv[n][2] = dv[n][3] = 0.f;
  }
  const int j1 = min(j0 + TILE - 1, a.T2 - 1);
  const int rep = a.Hq / a.Hk;
  const int64_t otok = (int64_t)a.Hq * D;
  for (int hq = hk * rep; hq < (hk + 1) * rep; ++hq) {
    const __nv_bfloat16* qb = a.q + (int64_t)b * a.T2 * a.q_tok + hq * D;
    const __nv_bfloat16* dob = a.dout + (int64_t)b * a.T2 * otok + hq * D;
    const float* lse = a.lse2 + ((int64_t)b * a.Hq + hq) * a.T2;
    const float* delta = a.delta + ((int64_t)b * a.Hq + hq) * a.T2;
    for (int i0 = 0; i0 < a.T2; i0 += TQ) {
      if (!tile_may(i0, min(i0 + TQ - 1, a.T2 - 1), j0, j1, a.L, a.block, a.leak)) continue;
      __syncthreads();
      load_tile<D, TQ>(sQ, qb, a.q_tok, i0, a.T2);
      load_tile<D, TQ>(sdO, dob, otok, i0, a.T2);
      cp_commit();
      for (int r = threadIdx.x; r < TQ; r += NTH) {
        sL[r] = i0 + r < a.T2 ? lse[i0 + r] : 0.f;
        sD[r] = i0 + r < a.T2 ? delta[i0 + r] : 0.f;
      }
      cp_wait_all();
      __syncthreads();
      float s[TQ / 8][4], dp[TQ / 8][4];
      qk_tile<D, TQ / 8>(s, sK, warp * 16, sQ);   // S^T: rows = keys, cols = queries
      qk_tile<D, TQ / 8>(dp, sV, warp * 16, sdO);  // dP^T = V dO^T
#pragma unroll
      for (int n = 0; n < TQ / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = e < 2 ? k0 : k1, qi = n * 8 + t4 * 2 + (e & 1), row = i0 + qi;
          const bool ok = key < a.T2 && row < a.T2 && allowed(row, key, a.L, a.block, a.leak);
          const float p = ok ? exp2f(s[n][e] * a.scale_log2 - sL[qi]) : 0.f;
          s[n][e] = p;                       // P^T
          dp[n][e] = p * (dp[n][e] - sD[qi]);  // dS^T
        }
      pv_tile<D, DA, TQ / 8>(dv, s, sdO, d0);
      pv_tile<D, DA, TQ / 8>(dk, dp, sQ, d0);
    }
  }
#pragma unroll
  for (int n = 0; n < DA / 8; ++n) {
    const int col = d0 + n * 8 + t4 * 2;
    const int64_t ktok = (int64_t)a.Hk * D;
    if (k0 < a.T2) {
      *reinterpret_cast<__nv_bfloat162*>(a.dk + ((int64_t)b * a.T2 + k0) * ktok + hk * D + col) =
          __floats2bfloat162_rn(dk[n][0] * a.scale, dk[n][1] * a.scale);
      *reinterpret_cast<__nv_bfloat162*>(a.dv + ((int64_t)b * a.T2 + k0) * ktok + hk * D + col) =
          __floats2bfloat162_rn(dv[n][0], dv[n][1]);
    }
    if (k1 < a.T2) {
      *reinterpret_cast<__nv_bfloat162*>(a.dk + ((int64_t)b * a.T2 + k1) * ktok + hk * D + col) =
          __floats2bfloat162_rn(dk[n][2] * a.scale, dk[n][3] * a.scale);
      *reinterpret_cast<__nv_bfloat162*>(a.dv + ((int64_t)b * a.T2 + k1) * ktok + hk * D + col) =
          __floats2bfloat162_rn(dv[n][2], dv[n][3]);
    }
  }
}

// ------------------------------------------------------------------------------------- host
// a contiguous tensor at a 16-byte aligned base (rows move in 16-byte vectors and TMA tiles): the
// input itself, or a copy when a view's offset breaks the alignment
static at::Tensor aligned_rows(const at::Tensor& t) {
  auto c = t.contiguous();
  return reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0 ? c : c.clone();
}

static void check_qkv(const at::Tensor& t, int64_t D) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.dim() == 4, "attn: bf16 [B, T2, H, D]");
  TORCH_CHECK(t.stride(3) == 1 && t.stride(2) == D && t.stride(0) == t.size(1) * t.stride(1),
              "attn: heads packed in a token row, batch and token dims mergeable");
  TORCH_CHECK(t.stride(1) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "attn: 16-byte aligned rows");
}

static Args make_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t L, int64_t block,
                      double scale, bool leak) {
  const int D = q.size(3);
  check_qkv(q, D);
  check_qkv(k, D);
  check_qkv(v, D);
  Args a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.q_tok = q.stride(1);
  a.k_tok = k.stride(1);
  a.v_tok = v.stride(1);
  a.B = q.size(0);
  a.T2 = q.size(1);
  a.L = (int)L;
  a.Hq = q.size(2);
  a.Hk = k.size(2);
  a.block = (int)block;
  a.leak = leak ? 1 : 0;
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  TORCH_CHECK(a.T2 == 2 * L && a.Hq % a.Hk == 0 && block >= 1, "attn: shapes");
  TORCH_CHECK(k.size(0) == a.B && v.size(0) == a.B && k.size(1) == a.T2 && v.size(1) == a.T2 &&
                  v.size(2) == a.Hk && k.size(3) == D && v.size(3) == D,
              "attn: q, k and v of one batch, length and head dim; k and v of one head count");
  a.Tk = a.T2;
  a.q_bat = (int64_t)a.T2 * a.q_tok;
  a.k_bat = (int64_t)a.T2 * a.k_tok;
  a.v_bat = (int64_t)a.T2 * a.v_tok;
  a.tk_dev = nullptr;
  return a;
}

template <typename K>
static void go(K kern, dim3 grid, int bytes, const Args& a) {
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  kern<<<grid, NTH, bytes, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// q [B, Tq, Hq, D] attends to every key of k/v [B, Tmax, Hk, D] rows [0, Tk) (Tk from `tk`, a
// device int32, when given; else `tk_host`). Output [B, Tq, Hq, D]; no lse.
template <int D>
static at::Tensor prefix_t(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t tk_host,
                           const c10::optional<at::Tensor>& tk, double scale) {
  TORCH_CHECK(q.stride(3) == 1 && q.stride(2) == D && k.stride(3) == 1 && k.stride(2) == D && v.stride(3) == 1 &&
                  v.stride(2) == D,
              "attn_prefix: heads packed in a token row");
  for (const at::Tensor* t : {&q, &k, &v})
    TORCH_CHECK(t->stride(1) % 8 == 0 && t->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "attn_prefix: 16-byte aligned rows");
  Args a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.q_tok = q.stride(1), a.k_tok = k.stride(1), a.v_tok = v.stride(1);
  a.q_bat = q.stride(0), a.k_bat = k.stride(0), a.v_bat = v.stride(0);
  a.B = q.size(0), a.T2 = q.size(1), a.L = a.T2, a.Hq = q.size(2), a.Hk = k.size(2), a.block = 1;
  a.leak = LEAK_ALL;
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.Tk = (int)tk_host;
  a.tk_dev = nullptr;
  if (tk.has_value()) {
    TORCH_CHECK(tk->is_cuda() && tk->scalar_type() == at::kInt, "attn_prefix: tk is a device int32");
    a.tk_dev = tk->data_ptr<int>();
  } else {
    TORCH_CHECK(tk_host >= 1 && tk_host <= k.size(1) && tk_host <= v.size(1), "attn_prefix: 1 <= Tk <= cache rows");
  }
  TORCH_CHECK(a.Hq % a.Hk == 0 && k.size(0) == a.B && v.size(0) == a.B && v.size(2) == a.Hk && q.size(3) == D &&
                  k.size(3) == D && v.size(3) == D,
              "attn_prefix: shapes");
  for (const at::Tensor* t : {&q, &k, &v})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 4, "attn_prefix: bf16 [B, T, H, D]");
  c10::cuda::CUDAGuard guard(q.device());
  auto o = at::empty({a.B, a.T2, a.Hq, D}, q.options());
  auto lse = at::empty({a.B, a.Hq, a.T2}, q.options().dtype(at::kFloat));
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse2 = lse.data_ptr<float>();
  go(fwd_kernel<D>, dim3((a.T2 + TILE - 1) / TILE, a.B * a.Hq), 3 * TILE * D * 2, a);
  return o;
}

// BDLLM_ATTN_TC=0 keeps the mma.sync forward for head dims the tcgen05 kernel covers
static bool tc_forward_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("BDLLM_ATTN_TC");
    on = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  return on == 1;
}

// BDLLM_ATTN_TC_BWD=0 keeps the mma.sync backward
static bool tc_backward_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("BDLLM_ATTN_TC_BWD");
    on = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  return on == 1 && tc_forward_enabled();
}

template <int D>
static std::vector<at::Tensor> fwd_t(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t L,
                                     int64_t block, double scale, bool leak) {
  Args a = make_args(q, k, v, L, block, scale, leak);
  c10::cuda::CUDAGuard guard(q.device());  // (after the host checks, which host tests reach)
  auto o = at::empty({a.B, a.T2, a.Hq, D}, q.options());
  auto lse = at::empty({a.B, a.Hq, a.T2}, q.options().dtype(at::kFloat));
  if ((D == 128 || D == 256) && tc_forward_enabled() && attn_fwd_tc(q, k, v, o, lse, L, block, scale, leak))
    return {o, lse};
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse2 = lse.data_ptr<float>();
  go(fwd_kernel<D>, dim3((a.T2 + TILE - 1) / TILE, a.B * a.Hq), 3 * TILE * D * 2, a);
  return {o, lse};
}

template <int D>
static std::vector<at::Tensor> bwd_t(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                     const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, int64_t L,
                                     int64_t block, double scale, bool leak) {
  Args a = make_args(q, k, v, L, block, scale, leak);
  TORCH_CHECK(dout.numel() == q.numel() && o.sizes() == q.sizes() && o.scalar_type() == at::kBFloat16 &&
                  lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == (int64_t)a.B * a.Hq * a.T2,
              "attn: dout and bf16 o of q's shape, fp32 lse [B, Hq, T2]");
  c10::cuda::CUDAGuard guard(q.device());
  auto d = aligned_rows(dout.to(at::kBFloat16));
  auto oc = aligned_rows(o);
  auto delta = at::empty({a.B, a.Hq, a.T2}, q.options().dtype(at::kFloat));
  auto dq = at::empty({a.B, a.T2, a.Hq, D}, q.options());
  auto dk = at::empty({a.B, a.T2, a.Hk, D}, q.options());
  auto dv = at::empty({a.B, a.T2, a.Hk, D}, q.options());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(d.data_ptr());
  a.o_in = reinterpret_cast<const __nv_bfloat16*>(oc.data_ptr());
  a.lse2 = const_cast<float*>(lse.data_ptr<float>());
  a.delta = delta.data_ptr<float>();
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  if ((D == 128 || D == 256) && tc_backward_enabled() &&
      attn_bwd_tc(d, q, k, v, oc, lse, delta, dq, dk, dv, L, block, scale, leak))
    return {dq, dk, dv};
  const int nt = (a.T2 + TILE - 1) / TILE;
  go(bwd_dq_kernel<D>, dim3(nt, a.B * a.Hq), (2 * TILE + 2 * TK) * D * 2, a);
  constexpr int DA = D > 128 ? D / 2 : D;
  go(bwd_dkv_kernel<D, DA>, dim3(nt, a.B * a.Hk, D / DA), (2 * TILE + 2 * TQ) * D * 2 + 2 * TQ * 4, a);
  return {dq, dk, dv};
}

}  // namespace attn

#define ATTN_DISPATCH(FN, ...)                                                       \
  switch (q.size(3)) {                                                               \
    case 16: return attn::FN<16>(__VA_ARGS__);                                       \
    case 32: return attn::FN<32>(__VA_ARGS__);                                       \
    case 64: return attn::FN<64>(__VA_ARGS__);                                       \
    case 128: return attn::FN<128>(__VA_ARGS__);                                     \
    case 256: return attn::FN<256>(__VA_ARGS__);                                     \
    default: TORCH_CHECK(false, "attn: head dim ", q.size(3), " not supported");     \
  }

std::vector<at::Tensor> attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t L,
                                 int64_t block, double scale, bool leak) {
  ATTN_DISPATCH(fwd_t, q, k, v, L, block, scale, leak)
  return {};
}

std::vector<at::Tensor> attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                 const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, int64_t L,
                                 int64_t block, double scale, bool leak) {
  ATTN_DISPATCH(bwd_t, dout, q, k, v, o, lse, L, block, scale, leak)
  return {};
}

}  // namespace bdllm

namespace bdllm {
at::Tensor attn_prefix(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t tk_host,
                       const c10::optional<at::Tensor>& tk, double scale) {
  ATTN_DISPATCH(prefix_t, q, k, v, tk_host, tk, scale)
  return {};
}
}  // namespace bdllm
