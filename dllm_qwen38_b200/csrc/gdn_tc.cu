// State-fork chunked gated delta rule, forward, on the 5th-generation tensor cores (tcgen05 +
// TMEM, operands staged by TMA). Head dim 128, chunk = block = 32, the fork layout [B, 2L]
// (positions [0, L) the noised stream x_t, [L, 2L) the clean stream x_0). Same contract as
// gdn.cu's forward_t for the output: returns o [B, 2L, Hv, 128] bf16, and the state entering each
// clean chunk (= the state each noised block forks from) as S_in^T [B, nb, Hv, 128 (v), 128 (k)]
// bf16, the layout the tensor-core backward loads by TMA (row v of S^T is what one epilogue
// thread holds, so each thread stores one contiguous row).
// (Reference path replaced: `src/dllm_qwen38/gdn.py:48-123` and the fork in `blockdiff.py:159-177`.)
//
// Math per chunk (one v-head; q^, k^ l2-normalised, q^ scaled by 128^-1/2; gam = cumsum g):
//   A = strict_lower(beta_i k^_i.k^_j e^(gam_i - gam_j)), T = (I + A)^-1
//   U = T diag(beta) v,  W = T diag(beta e^gam) k^,  q~ = diag(e^gam) q^,  K~ = diag(e^(gam_C - gam)) k^
//   P = (q^ k^T) * e^(gam_i - gam_j) * [i >= j]
//   V' = U - W S,  O = q~ S + P V',  S_next = e^gam_C S + K~^T V'
// Everything except the two S-dependent lines is independent across chunks.
//
// Kernel 1, prep_kernel (parallel; one CTA = 4 chunks = 128 tokens of one k-head, all its v-heads):
//   TMA loads the q, k tiles [128 tokens x 128] and, per v-head, the v tile; rows are
//   l2-normalised in shared memory; tcgen05 computes k^ k^T and q^ k^T as 128 x 128 x 128 MMAs
//   into TMEM (only the four 32 x 32 diagonal blocks are used: the chunks of the tile); one warp
//   per chunk gates them into A and P and solves T by forward substitution (lane = column of T);
//   T is laid out block-diagonally as a 128 x 128 bf16 A operand, so U = T (beta v) and
//   W = T (beta e^gam k^) are two M 128 x N 128 x K 128 MMAs for the four chunks at once.
//   Writes U, W, q~, K~ [32, 128] and P [32, 64] (32 used) bf16 per chunk-head, e^gam_C fp32.
// Kernel 2, recur_kernel (one CTA per (batch, v-head), sequential over chunk index c): the state
//   lives transposed, S^T [v = 128 TMEM lanes x k], as fp32 registers of 8 epilogue warps and as
//   a bf16 copy in TMEM that is the A operand (M = 128) of every state product:
//     MMA 1: D_w = S^T W_c^T, D_q = S^T q~_c^T, D_wn = S^T W_n^T, D_qn = S^T q~_n^T  (N 32, K 128)
//     E1   : V'^T = U^T - D_w (clean and noised), bf16 into TMEM as the next A operand
//     MMA 2: dS^T = V'^T K~_c (N 128, K 32), D_q += V'^T P_c^T, D_qn += V'_n^T P_n^T  (N 32, K 32)
//     E2   : S^T = e^gam_C S^T + dS^T (fp32 registers), S_in[c+1] to global, bf16 S^T to TMEM,
//            o of clean chunk c and noised block c from D_q / D_qn
//   warp 8 streams each chunk's operand tiles (clean and noised) by TMA into a 2-stage ring;
//   warp 9 issues the MMAs. Clean chunk c and noised block c share S_c, so each state is used
//   in place and never read back from memory.
// Every mbarrier wait is bounded; on expiry the CTA records ERR_GDN_WAIT, drains what it issued
// and frees its TMEM. No multicast loads (every TMA reads this GPU's own memory).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
void make_map_bf16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                   uint32_t box_outer);

namespace gdn_tc {

constexpr int D = 128;   // head dim (k and v)
constexpr int C = 32;    // chunk
constexpr int TT = 128;  // tokens per prep tile (4 chunks)

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void tmem_ld32r(uint32_t taddr, uint32_t (&r)[32]) {
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
}
__device__ __forceinline__ void tmem_ld16r(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st32r(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st8r(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]: A (M 128 x K 16, bf16) read from TMEM, row i in lane i,
// consecutive K pairs packed in consecutive 32-bit columns (8 columns per instruction)
__device__ __forceinline__ void mma_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Byte offset of element (row r, col c) of a K-major bf16 tile of R rows x 128 columns held as
// two TMA boxes [R rows][64 cols] with the 128-byte swizzle (16-byte chunk index XOR row % 8).
template <int R>
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((c >> 6) * (R * 128) + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + ((c & 7) << 1));
}
// byte offset of the 16-byte chunk j (columns 8j..8j+7) of row r in the same layout
template <int R>
__device__ __forceinline__ uint32_t sw_chunk(int r, int j) {
  return (uint32_t)((j >> 3) * (R * 128) + r * 128 + (((j & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, err, ERR_GDN_WAIT, abort);
  return __all_sync(0xffffffffu, ok);
}

// ============================================================================ kernel 1: prep
struct PArgs {
  const float* g;     // [B, 2L, Hv]
  const float* beta;  // [B, 2L, Hv]
  __nv_bfloat16* U;   // [NCH * 32, 128]  (chunk-head ch = ((b * 2 + s) * Hv + h) * nb + c)
  __nv_bfloat16* W;
  __nv_bfloat16* Q;   // q~
  __nv_bfloat16* K;   // K~ (clean stream only)
  __nv_bfloat16* P;   // [NCH * 32, 64] (optional)
  float* Ec;          // [NCH] e^gam_C
  __nv_bfloat16* Pt;  // [NCH * 32, 64] P transposed per chunk (optional: the backward's operand)
  int B, L, Hk, Hv, nb;
  float scale;
  int* err;
};

constexpr int P_THREADS = 256;
constexpr int TILE_BYTES = TT * D * 2;  // 32 KB
struct PSmem {
  static constexpr int Q = 0, K = TILE_BYTES, V = 2 * TILE_BYTES, BK = 3 * TILE_BYTES, T = 4 * TILE_BYTES;
  static constexpr int A = 5 * TILE_BYTES;                // fp32 [4][32][33]
  static constexpr int GAM = A + 4 * 32 * 33 * 4;         // fp32 [128]
  static constexpr int BETA = GAM + TT * 4;               // fp32 [128]
  static constexpr int BAR = BETA + TT * 4;               // mbarriers
  static constexpr int BYTES = BAR + 64 + 1024;           // + alignment slack
};
constexpr uint32_t IDESC_128 = idesc_bf16(128, 128, 0, 0);      // A, B K-major
constexpr uint32_t IDESC_128_BMN = idesc_bf16(128, 128, 0, 1);  // B N-contiguous

__global__ void __launch_bounds__(P_THREADS, 1)
    prep_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                const __grid_constant__ CUtensorMap mv, PArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm + PSmem::Q;
  uint8_t* sK = sm + PSmem::K;
  uint8_t* sV = sm + PSmem::V;
  uint8_t* sBK = sm + PSmem::BK;
  uint8_t* sT = sm + PSmem::T;
  float* sA = reinterpret_cast<float*>(sm + PSmem::A);
  float* sgam = reinterpret_cast<float*>(sm + PSmem::GAM);
  float* sbeta = reinterpret_cast<float*>(sm + PSmem::BETA);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + PSmem::BAR);
  uint64_t* qk_full = bars;      // q, k tiles landed
  uint64_t* v_full = bars + 1;   // v tile landed (once per v-head)
  uint64_t* mma_a = bars + 2;    // k k^T and q k^T done
  uint64_t* mma_b = bars + 3;    // U and W done (once per v-head)
  uint64_t* drain = bars + 4;    // every MMA issued has completed (exit path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 6);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, hk = blockIdx.y, bs = blockIdx.z;  // bs = b * 2 + stream
  const int b = bs >> 1, s = bs & 1;
  const int R = a.Hv / a.Hk;
  const int64_t row0 = (int64_t)b * 2 * a.L + (int64_t)s * a.L + (int64_t)tile * TT;  // first token

  if (threadIdx.x == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mq);
    prefetch_tmap(&mk);
    prefetch_tmap(&mv);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // the off-diagonal blocks of T stay zero for every v-head
  for (int i = threadIdx.x; i < TILE_BYTES / 16; i += P_THREADS) reinterpret_cast<uint4*>(sT)[i] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t KK_COL = 0, QK_COL = 128, U_COL = 256, W_COL = 384;

  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(qk_full, 2 * TILE_BYTES);
    for (int c = 0; c < 2; ++c) {
      tma_load_2d(sQ + c * TT * 128, &mq, qk_full, hk * D + c * 64, (int)row0);
      tma_load_2d(sK + c * TT * 128, &mk, qk_full, hk * D + c * 64, (int)row0);
    }
    mbar_arrive_expect_tx(v_full, TILE_BYTES);
    for (int c = 0; c < 2; ++c) tma_load_2d(sV + c * TT * 128, &mv, v_full, hk * R * D + c * 64, (int)row0);
  }
  bool ok = mbar_wait(qk_full, 0, a.err, ERR_GDN_WAIT, abort_flag);
  ok = __syncthreads_and(ok);
  if (ok) {
    // l2 normalisation in place: threads 0-127 the k rows, 128-255 the q rows (q also scaled)
    const int r = threadIdx.x & 127;
    uint8_t* tileb = threadIdx.x < 128 ? sK : sQ;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint4 u = *reinterpret_cast<const uint4*>(tileb + sw_chunk<TT>(r, j));
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p[e]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    const float inv = rsqrtf(ss + 1e-6f) * (threadIdx.x < 128 ? 1.f : a.scale);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      uint4 u = *reinterpret_cast<const uint4*>(tileb + sw_chunk<TT>(r, j));
      __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p[e]);
        p[e] = __floats2bfloat162_rn(f.x * inv, f.y * inv);
      }
      *reinterpret_cast<uint4*>(tileb + sw_chunk<TT>(r, j)) = u;
    }
    fence_proxy_async();  // the generic-proxy writes must be visible to the tensor core reads
  }
  __syncthreads();
  if (ok && threadIdx.x == 0) {
    tc_fence_after();
    const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk >> 2) * (TT * 128) + (kk & 3) * 32;
      mma_bf16(tmem + KK_COL, smem_desc(k_addr + off, 16, 1024), smem_desc(k_addr + off, 16, 1024), IDESC_128,
               kk > 0 ? 1u : 0u);
      mma_bf16(tmem + QK_COL, smem_desc(q_addr + off, 16, 1024), smem_desc(k_addr + off, 16, 1024), IDESC_128,
               kk > 0 ? 1u : 0u);
    }
    mma_commit(mma_a);
  }
  if (ok) ok = warp_wait(mma_a, 0, a.err, abort_flag);
  ok = __syncthreads_and(ok);
  tc_fence_after();
  int v_loads = 1;  // v tiles armed so far (the first v-head's was armed with q and k)

  const int64_t nb = a.nb;
  for (int j = 0; j < R && ok; ++j) {
    const int h = hk * R + j;
    const int64_t chrow = (((int64_t)bs * a.Hv + h) * nb + (int64_t)tile * 4) * C;  // first output row
    // ---- gates: warp w < 4 = chunk w, lane = token: gam = inclusive cumsum of g within the chunk
    if (warp < 4) {
      const int t = warp * 32 + lane;
      const int64_t tokn = row0 + t;
      float gv = a.g[tokn * a.Hv + h];
      const float bv = a.beta[tokn * a.Hv + h];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, gv, o);
        if (lane >= o) gv += y;
      }
      sgam[t] = gv;
      sbeta[t] = bv;
      if (lane == 31) a.Ec[(((int64_t)bs * a.Hv + h) * nb + tile * 4 + warp)] = __expf(gv);
    }
    __syncthreads();
    // ---- A (warps 0-3, from k^ k^T) and P (warps 4-7, from q^ k^T): warp = chunk, lane = row
    {
      const int ch = warp & 3, t = ch * 32 + lane;
      const float gi = sgam[t];
      uint32_t r[32];
      const uint32_t lane_base = (uint32_t)(ch * 32) << 16;
      if (warp < 4) {
        tmem_ld32r(tmem + lane_base + KK_COL + ch * 32, r);
        const float bi = sbeta[t];
        float* Arow = sA + (ch * 32 + lane) * 33;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          Arow[jj] = jj < lane ? bi * __uint_as_float(r[jj]) * __expf(gi - sgam[ch * 32 + jj]) : 0.f;
      } else {
        tmem_ld32r(tmem + lane_base + QK_COL + ch * 32, r);
        uint32_t pk[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j0 = 2 * jj, j1 = 2 * jj + 1;
          const float p0 = j0 <= lane ? __uint_as_float(r[j0]) * __expf(gi - sgam[ch * 32 + j0]) : 0.f;
          const float p1 = j1 <= lane ? __uint_as_float(r[j1]) * __expf(gi - sgam[ch * 32 + j1]) : 0.f;
          pk[jj] = pack2(p0, p1);
        }
        if (a.P != nullptr) {
          uint4* dst = reinterpret_cast<uint4*>(a.P + (chrow + t) * 64);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        }
        if (a.Pt != nullptr) {  // Pt[chunk row j][lane] = P[lane][j]
          __nv_bfloat16* dt = a.Pt + (chrow + ch * 32) * 64 + lane;
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const __nv_bfloat162 two = *reinterpret_cast<const __nv_bfloat162*>(&pk[jj]);
            dt[(2 * jj) * 64] = two.x;
            dt[(2 * jj + 1) * 64] = two.y;
          }
        }
      }
    }
    __syncthreads();
    if (warp < 4) {
      // ---- T = (I + A)^-1 of chunk `warp` by forward substitution; lane = column of T
      const float* Ab = sA + warp * 32 * 33;
      float tc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float acc0 = (i == lane) ? 1.f : 0.f, acc1 = 0.f;
#pragma unroll
        for (int m = 0; m < i; m += 2) {
          acc0 -= Ab[i * 33 + m] * tc[m];
          if (m + 1 < i) acc1 -= Ab[i * 33 + m + 1] * tc[m + 1];
        }
        tc[i] = acc0 + acc1;
      }
      // into the block-diagonal bf16 operand: row 32w + i, column 32w + lane
      const int col = warp * 32 + lane;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        *reinterpret_cast<__nv_bfloat16*>(sT + sw_off<TT>(warp * 32 + i, col)) = __float2bfloat16_rn(tc[i]);
    } else {
      // ---- beta e^gam k^ (a scaled copy of k^), q~ and K~ to global (warps 4-7: thread = row)
      const int t = threadIdx.x - 128;
      const float gi = sgam[t], bi = sbeta[t];
      const float Ei = __expf(gi), Fi = __expf(sgam[(t & ~31) + 31] - gi);
      __nv_bfloat16* qdst = a.Q + (chrow + t) * D;
      __nv_bfloat16* kdst = a.K + (chrow + t) * D;
#pragma unroll
      for (int jc = 0; jc < 16; ++jc) {
        const uint32_t off = sw_chunk<TT>(t, jc);
        const uint4 ku = *reinterpret_cast<const uint4*>(sK + off);
        const uint4 qu = *reinterpret_cast<const uint4*>(sQ + off);
        const __nv_bfloat162* kp = reinterpret_cast<const __nv_bfloat162*>(&ku);
        const __nv_bfloat162* qp = reinterpret_cast<const __nv_bfloat162*>(&qu);
        uint4 bk, qo, ko;
        uint32_t* bkw = reinterpret_cast<uint32_t*>(&bk);
        uint32_t* qow = reinterpret_cast<uint32_t*>(&qo);
        uint32_t* kow = reinterpret_cast<uint32_t*>(&ko);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kf = __bfloat1622float2(kp[e]), qf = __bfloat1622float2(qp[e]);
          bkw[e] = pack2(kf.x * bi * Ei, kf.y * bi * Ei);
          qow[e] = pack2(qf.x * Ei, qf.y * Ei);
          kow[e] = pack2(kf.x * Fi, kf.y * Fi);
        }
        *reinterpret_cast<uint4*>(sBK + off) = bk;
        *reinterpret_cast<uint4*>(qdst + jc * 8) = qo;
        if (s == 1) *reinterpret_cast<uint4*>(kdst + jc * 8) = ko;
      }
    }
    // ---- beta v (v tile scaled in place; threads 0-127 after the solve, one row each)
    ok = ok && mbar_wait(v_full, j & 1, a.err, ERR_GDN_WAIT, abort_flag);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (threadIdx.x < 128) {
      const int t = threadIdx.x;
      const float bi = sbeta[t];
#pragma unroll
      for (int jc = 0; jc < 16; ++jc) {
        const uint32_t off = sw_chunk<TT>(t, jc);
        uint4 u = *reinterpret_cast<const uint4*>(sV + off);
        __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(p[e]);
          p[e] = __floats2bfloat162_rn(f.x * bi, f.y * bi);
        }
        *reinterpret_cast<uint4*>(sV + off) = u;
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
      // ---- U = T (beta v), W = T (beta e^gam k^): A = T [t][t'] K-major, B [t'][d] N-contiguous
      tc_fence_after();
      const uint32_t t_addr = smem_u32(sT), v_addr = smem_u32(sV), bk_addr = smem_u32(sBK);
#pragma unroll
      for (int kk = 0; kk < TT / 16; ++kk) {
        const uint32_t offa = (kk >> 2) * (TT * 128) + (kk & 3) * 32;
        mma_bf16(tmem + U_COL, smem_desc(t_addr + offa, 16, 1024), smem_desc(v_addr + kk * 2048, TT * 128, 1024),
                 IDESC_128_BMN, kk > 0 ? 1u : 0u);
        mma_bf16(tmem + W_COL, smem_desc(t_addr + offa, 16, 1024), smem_desc(bk_addr + kk * 2048, TT * 128, 1024),
                 IDESC_128_BMN, kk > 0 ? 1u : 0u);
      }
      mma_commit(mma_b);
    }
    ok = warp_wait(mma_b, j & 1, a.err, abort_flag);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) break;
    // the v tile is free: start the next v-head's load while U and W are written out
    if (j + 1 < R) ++v_loads;
    if (threadIdx.x == 0 && j + 1 < R) {
      mbar_arrive_expect_tx(v_full, TILE_BYTES);
      for (int c = 0; c < 2; ++c) tma_load_2d(sV + c * TT * 128, &mv, v_full, (h + 1) * D + c * 64, (int)row0);
    }
    {
      // ---- U and W rows to global: warp w reads lanes of quadrant w % 4, columns half w / 4
      const int q = warp & 3, hf = warp >> 2, t = q * 32 + lane;
      const uint32_t lane_base = (uint32_t)(q * 32) << 16;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        if (which == 0 && a.U == nullptr) continue;  // the backward needs W only
        __nv_bfloat16* dst = (which == 0 ? a.U : a.W) + (chrow + t) * D + hf * 64;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t r[32];
          tmem_ld32r(tmem + lane_base + (which == 0 ? U_COL : W_COL) + hf * 64 + c2 * 32, r);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 u;
            u.x = pack2(__uint_as_float(r[8 * q4 + 0]), __uint_as_float(r[8 * q4 + 1]));
            u.y = pack2(__uint_as_float(r[8 * q4 + 2]), __uint_as_float(r[8 * q4 + 3]));
            u.z = pack2(__uint_as_float(r[8 * q4 + 4]), __uint_as_float(r[8 * q4 + 5]));
            u.w = pack2(__uint_as_float(r[8 * q4 + 6]), __uint_as_float(r[8 * q4 + 7]));
            *reinterpret_cast<uint4*>(dst + c2 * 32 + q4 * 8) = u;
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  // on an early exit: every load armed must land and every MMA issued must complete before the
  // CTA frees its TMEM and exits (bounded waits)
  if (threadIdx.x == 0 && !ok) {
    mbar_wait(qk_full, 0, a.err, ERR_GDN_WAIT, nullptr);
    mbar_wait(v_full, (v_loads - 1) & 1, a.err, ERR_GDN_WAIT, nullptr);
    mma_commit(drain);
    mbar_wait(drain, 0, a.err, ERR_GDN_WAIT, nullptr);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ============================================================================ kernel 2: recurrence
struct RArgs {
  const float* Ec;       // [NCH]
  const __nv_bfloat16* U;  // [NCH * 32, 128] (read by the epilogue through the TMA-staged tile)
  __nv_bfloat16* S_in;   // S^T per chunk entry: [B, nb, Hv, 128 (v), 128 (k)]
  __nv_bfloat16* o;      // [B, 2L, Hv, 128]
  int B, L, Hv, nb;
  int* err;
};

constexpr int R_THREADS = 320;  // warps 0-7 epilogue, 8 TMA, 9 MMA
constexpr int T8 = 32 * 128 * 2;  // one [32 x 128] bf16 tile: 8 KB (two boxes of [32][64])
struct RStage {
  // clean W, q~, K~, U; noised W, q~, U; clean P, noised P ([32][64] each)
  static constexpr int W = 0, Q = T8, K = 2 * T8, U = 3 * T8, WN = 4 * T8, QN = 5 * T8, UN = 6 * T8;
  static constexpr int P = 7 * T8, PN = 7 * T8 + 4096;
  static constexpr int BYTES = 7 * T8 + 2 * 4096;  // 64 KB
};
constexpr int NSTAGE = 2;
constexpr int R_SMEM = NSTAGE * RStage::BYTES + 1024 + 256;
// TMEM columns
constexpr uint32_t SA_COL = 0;     // S^T bf16 A operand (64 packed columns)
constexpr uint32_t VA_COL = 64;    // V'^T clean, bf16 A operand (16 packed columns)
constexpr uint32_t VNA_COL = 80;   // V'^T noised
constexpr uint32_t DW_COL = 128, DQ_COL = 160, DWN_COL = 192, DQN_COL = 224;
constexpr uint32_t DS_COL = 256;   // dS^T (128 columns)
constexpr uint32_t IDESC_N32 = idesc_bf16(128, 32, 0, 0);
constexpr uint32_t IDESC_N128_BMN = idesc_bf16(128, 128, 0, 1);

__global__ void __launch_bounds__(R_THREADS, 1)
    recur_kernel(const __grid_constant__ CUtensorMap mt, const __grid_constant__ CUtensorMap mp, RArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + NSTAGE * RStage::BYTES);
  uint64_t* full = bars;              // [NSTAGE]
  uint64_t* empty = bars + NSTAGE;    // [NSTAGE]
  uint64_t* d1_full = bars + 2 * NSTAGE;
  uint64_t* d2_full = d1_full + 1;
  uint64_t* va_ready = d1_full + 2;   // 8 arrivals (epilogue warps)
  uint64_t* sa_ready = d1_full + 3;   // 8 arrivals
  uint64_t* drain = d1_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d1_full + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / a.Hv, h = blockIdx.x % a.Hv;
  const int nb = a.nb;
  // chunk-head rows of the prep outputs: clean stream s = 1, noised s = 0
  const int64_t chc = (((int64_t)(b * 2 + 1) * a.Hv + h) * nb) * C;
  const int64_t chn = (((int64_t)(b * 2 + 0) * a.Hv + h) * nb) * C;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(d1_full, 1);
    mbar_init(d2_full, 1);
    mbar_init(va_ready, 8);
    mbar_init(sa_ready, 8);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mt);
    prefetch_tmap(&mp);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int last[NSTAGE];
      for (int s = 0; s < NSTAGE; ++s) last[s] = -1;
      for (int c = 0; c < nb; ++c) {
        const int s = c % NSTAGE;
        if (!mbar_wait(&empty[s], ((c / NSTAGE) & 1) ^ 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], RStage::BYTES);
        last[s] = c;
        uint8_t* st = sm + s * RStage::BYTES;
        const int yc = (int)(chc + (int64_t)c * C), yn = (int)(chn + (int64_t)c * C);
        // map mt spans the four [NCH * 32, 128] prep outputs stacked: U, W, Q, K (rows offset by
        // one array's rows each)
        const int nrow = a.B * 2 * a.Hv * nb * C;
        for (int x = 0; x < 2; ++x) {
          tma_load_2d(st + RStage::W + x * 4096, &mt, &full[s], x * 64, yc + 1 * nrow);
          tma_load_2d(st + RStage::Q + x * 4096, &mt, &full[s], x * 64, yc + 2 * nrow);
          tma_load_2d(st + RStage::K + x * 4096, &mt, &full[s], x * 64, yc + 3 * nrow);
          tma_load_2d(st + RStage::U + x * 4096, &mt, &full[s], x * 64, yc + 0 * nrow);
          tma_load_2d(st + RStage::WN + x * 4096, &mt, &full[s], x * 64, yn + 1 * nrow);
          tma_load_2d(st + RStage::QN + x * 4096, &mt, &full[s], x * 64, yn + 2 * nrow);
          tma_load_2d(st + RStage::UN + x * 4096, &mt, &full[s], x * 64, yn + 0 * nrow);
        }
        tma_load_2d(st + RStage::P, &mp, &full[s], 0, yc);
        tma_load_2d(st + RStage::PN, &mp, &full[s], 0, yn);
      }
      for (int s = 0; s < NSTAGE; ++s)
        if (last[s] >= 0) mbar_wait(&full[s], (last[s] / NSTAGE) & 1, a.err, ERR_GDN_WAIT, nullptr);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      bool ok = true;
      for (int c = 0; c < nb && ok; ++c) {
        const int s = c % NSTAGE;
        if (!mbar_wait(&full[s], (c / NSTAGE) & 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        if (!mbar_wait(sa_ready, c & 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(sm + s * RStage::BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // K = k (128)
          const uint32_t off = (kk >> 2) * 4096 + (kk & 3) * 32;
          const uint32_t acc = kk > 0 ? 1u : 0u;
          const uint32_t at = tmem + SA_COL + kk * 8;
          mma_ta(tmem + DW_COL, at, smem_desc(st + RStage::W + off, 16, 1024), IDESC_N32, acc);
          mma_ta(tmem + DQ_COL, at, smem_desc(st + RStage::Q + off, 16, 1024), IDESC_N32, acc);
          mma_ta(tmem + DWN_COL, at, smem_desc(st + RStage::WN + off, 16, 1024), IDESC_N32, acc);
          mma_ta(tmem + DQN_COL, at, smem_desc(st + RStage::QN + off, 16, 1024), IDESC_N32, acc);
        }
        mma_commit(d1_full);
        if (!mbar_wait(va_ready, c & 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {  // K = t (32)
          mma_ta(tmem + DS_COL, tmem + VA_COL + kk * 8, smem_desc(st + RStage::K + kk * 2048, 4096, 1024),
                 IDESC_N128_BMN, kk > 0 ? 1u : 0u);
          mma_ta(tmem + DQ_COL, tmem + VA_COL + kk * 8, smem_desc(st + RStage::P + kk * 32, 16, 1024), IDESC_N32, 1u);
          mma_ta(tmem + DQN_COL, tmem + VNA_COL + kk * 8, smem_desc(st + RStage::PN + kk * 32, 16, 1024), IDESC_N32,
                 1u);
        }
        mma_commit(d2_full);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_GDN_WAIT, nullptr);
    }
  } else {
    // -------------------------------------------------------------- epilogue (warps 0-7)
    const int q = warp & 3, hf = warp >> 2;
    const int v = q * 32 + lane;  // this thread's row of S^T (a v column of S)
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float S[64];  // S^T[v][64 hf + i]
#pragma unroll
    for (int i = 0; i < 64; ++i) S[i] = 0.f;
    // S_0 = 0: the bf16 operand and S_in[0]
    {
      uint32_t z[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = 0u;
      tmem_st32r(tmem + lane_base + SA_COL + hf * 32, z);
      uint4* dst = reinterpret_cast<uint4*>(a.S_in + ((((int64_t)b * nb + 0) * a.Hv + h) * D + v) * D + hf * 64);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sa_ready);
    }
    const int64_t tok_n = (int64_t)b * 2 * a.L, tok_c = tok_n + a.L;
    for (int c = 0; c < nb; ++c) {
      const int s = c % NSTAGE;
      const uint8_t* st = sm + s * RStage::BYTES;
      // ---- E1: V'^T = U^T - D_w for the clean chunk and the noised block, t in [16 hf, 16 hf + 16)
      // (the stage's own barrier makes the TMA-written U tiles visible to these generic loads)
      if (!warp_wait(&full[s], (c / NSTAGE) & 1, a.err, abort_flag)) break;
      if (!warp_wait(d1_full, c & 1, a.err, abort_flag)) break;
      tc_fence_after();
      {
        uint32_t dw[16], dwn[16];
        tmem_ld16r(tmem + lane_base + DW_COL + hf * 16, dw);
        tmem_ld16r(tmem + lane_base + DWN_COL + hf * 16, dwn);
        uint32_t pc[8], pn[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int t0 = hf * 16 + 2 * i, t1 = t0 + 1;
          const float u0 = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(st + RStage::U + sw_off<32>(t0, v)));
          const float u1 = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(st + RStage::U + sw_off<32>(t1, v)));
          const float n0 = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(st + RStage::UN + sw_off<32>(t0, v)));
          const float n1 = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(st + RStage::UN + sw_off<32>(t1, v)));
          pc[i] = pack2(u0 - __uint_as_float(dw[2 * i]), u1 - __uint_as_float(dw[2 * i + 1]));
          pn[i] = pack2(n0 - __uint_as_float(dwn[2 * i]), n1 - __uint_as_float(dwn[2 * i + 1]));
        }
        tmem_st8r(tmem + lane_base + VA_COL + hf * 8, pc);
        tmem_st8r(tmem + lane_base + VNA_COL + hf * 8, pn);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(va_ready);
      // ---- E2: state update, S_in[c + 1], bf16 S^T, outputs
      if (!warp_wait(d2_full, c & 1, a.err, abort_flag)) break;
      tc_fence_after();
      const float ec = a.Ec[(((int64_t)(b * 2 + 1) * a.Hv + h) * nb + c)];
      uint32_t spk[32];  // bf16 pairs of this thread's S^T row (k 64 hf + 2i, +1)
      {
        uint32_t r0[32], r1[32];
        tmem_ld32r(tmem + lane_base + DS_COL + hf * 64, r0);
        tmem_ld32r(tmem + lane_base + DS_COL + hf * 64 + 32, r1);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          S[i] = ec * S[i] + __uint_as_float(r0[i]);
          S[32 + i] = ec * S[32 + i] + __uint_as_float(r1[i]);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) spk[i] = pack2(S[2 * i], S[2 * i + 1]);
        tmem_st32r(tmem + lane_base + SA_COL + hf * 32, spk);
      }
      {
        uint32_t oc[16], on[16];
        tmem_ld16r(tmem + lane_base + DQ_COL + hf * 16, oc);
        tmem_ld16r(tmem + lane_base + DQN_COL + hf * 16, on);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sa_ready);  // the next chunk's state products may start
        if (warp == 0 && lane == 0) mbar_arrive(&empty[s]);  // every MMA reading the stage is done
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = hf * 16 + i;
          a.o[((tok_c + (int64_t)c * C + t) * a.Hv + h) * D + v] = __float2bfloat16_rn(__uint_as_float(oc[i]));
          a.o[((tok_n + (int64_t)c * C + t) * a.Hv + h) * D + v] = __float2bfloat16_rn(__uint_as_float(on[i]));
        }
      }
      if (c + 1 < nb) {
        // row v of S^T (this thread's 64 k values, already packed as bf16 pairs for TMEM)
        uint4* dst = reinterpret_cast<uint4*>(a.S_in + ((((int64_t)b * nb + c + 1) * a.Hv + h) * D + v) * D + hf * 64);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_uint4(spk[4 * i], spk[4 * i + 1], spk[4 * i + 2], spk[4 * i + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ============================================================================ kernel 3: reverse recurrence
// The backward's sequential part, one CTA per (batch, v-head), chunks in reverse order. The state
// gradient is kept transposed, dS^T [v = 128 TMEM lanes x k], as fp32 registers of 8 epilogue
// warps and as a bf16 copy in TMEM (the A operand). With dS = dS_{c+1} (the gradient of the state
// after clean chunk c) at step c:
//   MMA 1: dV'^T = dS^T K~^T + dO_c^T P_c   (clean, N 32)    dV'_n^T = dO_n^T P_n  (noised block c)
//   E1   : dV' of the clean chunk to global (fp32, for the chunk kernel); -dV'^T and -dV'_n^T as
//          bf16 A operands into TMEM
//   MMA 2: G^T = dO_c^T q~_c - dV'^T W_c + dO_n^T q~_n - dV'_n^T W_n   (N 128, K 32)
//   E2   : dS_c^T = e^gam_C dS^T + G^T; dS_out[c - 1] = dS_c (fp32, for the chunk kernel)
// The noised block's gradient of its starting state (q~_n^T dO_n - W_n^T dV'_n) is added here, so
// the noised chunk kernel need not store it. dO tiles are the M-contiguous A operands (dO^T) as
// TMA loads them; P enters transposed (K-major B).
struct BArgs {
  const float* Ec;  // [NCH]
  __nv_bfloat16* dS_out;  // dS_out^T per chunk: [B, nb, Hv, 128 (v), 128 (k)]
  float* dVp;       // [B, nb, Hv, 32, 128]
  int B, L, Hv, nb;
  int* err;
};
struct BStage {
  // clean dO, K~, q~, W, Pt; noised dO, q~, W, Pt
  static constexpr int DO = 0, K = T8, Q = 2 * T8, W = 3 * T8, DON = 4 * T8, QN = 5 * T8, WN = 6 * T8;
  static constexpr int PT = 7 * T8, PTN = 7 * T8 + 4096;
  static constexpr int BYTES = 7 * T8 + 2 * 4096;  // 64 KB
};
constexpr uint32_t IDESC_N32_AMN = idesc_bf16(128, 32, 1, 0);
constexpr uint32_t IDESC_N128_ABMN = idesc_bf16(128, 128, 1, 1);

__global__ void __launch_bounds__(R_THREADS, 1)
    bwd_recur_kernel(const __grid_constant__ CUtensorMap mt, const __grid_constant__ CUtensorMap mp,
                     const __grid_constant__ CUtensorMap mdo, BArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + NSTAGE * BStage::BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + NSTAGE;
  uint64_t* d1_full = bars + 2 * NSTAGE;
  uint64_t* d2_full = d1_full + 1;
  uint64_t* va_ready = d1_full + 2;
  uint64_t* sa_ready = d1_full + 3;
  uint64_t* drain = d1_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d1_full + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / a.Hv, h = blockIdx.x % a.Hv;
  const int nb = a.nb;
  const int64_t chc = (((int64_t)(b * 2 + 1) * a.Hv + h) * nb) * C;
  const int64_t chn = (((int64_t)(b * 2 + 0) * a.Hv + h) * nb) * C;
  const int64_t tok_n = (int64_t)b * 2 * a.L, tok_c = tok_n + a.L;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(d1_full, 1);
    mbar_init(d2_full, 1);
    mbar_init(va_ready, 8);
    mbar_init(sa_ready, 8);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mt);
    prefetch_tmap(&mp);
    prefetch_tmap(&mdo);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (reverse order)
      int last[NSTAGE];
      for (int s = 0; s < NSTAGE; ++s) last[s] = -1;
      const int nrow = a.B * 2 * a.Hv * nb * C;
      for (int i = 0; i < nb; ++i) {
        const int c = nb - 1 - i, s = i % NSTAGE;
        if (!mbar_wait(&empty[s], ((i / NSTAGE) & 1) ^ 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], BStage::BYTES);
        last[s] = i;
        uint8_t* st = sm + s * BStage::BYTES;
        const int yc = (int)(chc + (int64_t)c * C), yn = (int)(chn + (int64_t)c * C);
        for (int x = 0; x < 2; ++x) {
          tma_load_2d(st + BStage::DO + x * 4096, &mdo, &full[s], h * D + x * 64, (int)(tok_c + (int64_t)c * C));
          tma_load_2d(st + BStage::DON + x * 4096, &mdo, &full[s], h * D + x * 64, (int)(tok_n + (int64_t)c * C));
          tma_load_2d(st + BStage::K + x * 4096, &mt, &full[s], x * 64, yc + 3 * nrow);
          tma_load_2d(st + BStage::Q + x * 4096, &mt, &full[s], x * 64, yc + 2 * nrow);
          tma_load_2d(st + BStage::W + x * 4096, &mt, &full[s], x * 64, yc + 1 * nrow);
          tma_load_2d(st + BStage::QN + x * 4096, &mt, &full[s], x * 64, yn + 2 * nrow);
          tma_load_2d(st + BStage::WN + x * 4096, &mt, &full[s], x * 64, yn + 1 * nrow);
        }
        tma_load_2d(st + BStage::PT, &mp, &full[s], 0, yc);
        tma_load_2d(st + BStage::PTN, &mp, &full[s], 0, yn);
      }
      for (int s = 0; s < NSTAGE; ++s)
        if (last[s] >= 0) mbar_wait(&full[s], (last[s] / NSTAGE) & 1, a.err, ERR_GDN_WAIT, nullptr);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      for (int i = 0; i < nb; ++i) {
        const int s = i % NSTAGE;
        if (!mbar_wait(&full[s], (i / NSTAGE) & 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        if (!mbar_wait(sa_ready, i & 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(sm + s * BStage::BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)  // dS^T K~^T (K = k)
          mma_ta(tmem + DW_COL, tmem + SA_COL + kk * 8,
                 smem_desc(st + BStage::K + (kk >> 2) * 4096 + (kk & 3) * 32, 16, 1024), IDESC_N32, kk > 0);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {  // dO^T P (K = t')
          mma_bf16(tmem + DW_COL, smem_desc(st + BStage::DO + kk * 2048, 4096, 1024),
                   smem_desc(st + BStage::PT + kk * 32, 16, 1024), IDESC_N32_AMN, 1u);
          mma_bf16(tmem + DWN_COL, smem_desc(st + BStage::DON + kk * 2048, 4096, 1024),
                   smem_desc(st + BStage::PTN + kk * 32, 16, 1024), IDESC_N32_AMN, kk > 0);
        }
        mma_commit(d1_full);
        if (!mbar_wait(va_ready, i & 1, a.err, ERR_GDN_WAIT, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {  // K = t (32)
          const uint32_t acc = kk > 0;
          mma_bf16(tmem + DS_COL, smem_desc(st + BStage::DO + kk * 2048, 4096, 1024),
                   smem_desc(st + BStage::Q + kk * 2048, 4096, 1024), IDESC_N128_ABMN, acc);
          mma_ta(tmem + DS_COL, tmem + VA_COL + kk * 8, smem_desc(st + BStage::W + kk * 2048, 4096, 1024),
                 IDESC_N128_BMN, 1u);
          mma_bf16(tmem + DS_COL, smem_desc(st + BStage::DON + kk * 2048, 4096, 1024),
                   smem_desc(st + BStage::QN + kk * 2048, 4096, 1024), IDESC_N128_ABMN, 1u);
          mma_ta(tmem + DS_COL, tmem + VNA_COL + kk * 8, smem_desc(st + BStage::WN + kk * 2048, 4096, 1024),
                 IDESC_N128_BMN, 1u);
        }
        mma_commit(d2_full);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_GDN_WAIT, nullptr);
    }
  } else {
    // -------------------------------------------------------------- epilogue (warps 0-7)
    const int q = warp & 3, hf = warp >> 2;
    const int v = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float S[64];  // dS^T[v][64 hf + i]
#pragma unroll
    for (int i = 0; i < 64; ++i) S[i] = 0.f;
    {
      uint32_t z[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = 0u;
      tmem_st32r(tmem + lane_base + SA_COL + hf * 32, z);
      uint4* dst = reinterpret_cast<uint4*>(a.dS_out + ((((int64_t)b * nb + nb - 1) * a.Hv + h) * D + v) * D + hf * 64);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);  // nothing flows back after the last chunk
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sa_ready);
    }
    for (int i = 0; i < nb; ++i) {
      const int c = nb - 1 - i, s = i % NSTAGE;
      // ---- E1: dV' (clean) to global; -dV'^T, -dV'_n^T into TMEM; t in [16 hf, 16 hf + 16)
      if (!warp_wait(d1_full, i & 1, a.err, abort_flag)) break;
      tc_fence_after();
      {
        uint32_t dv[16], dvn[16];
        tmem_ld16r(tmem + lane_base + DW_COL + hf * 16, dv);
        tmem_ld16r(tmem + lane_base + DWN_COL + hf * 16, dvn);
        uint32_t pc[8], pn[8];
        float* g = a.dVp + ((((int64_t)b * nb + c) * a.Hv + h) * C) * D + v;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float x0 = __uint_as_float(dv[2 * j]), x1 = __uint_as_float(dv[2 * j + 1]);
          g[(hf * 16 + 2 * j) * D] = x0;
          g[(hf * 16 + 2 * j + 1) * D] = x1;
          pc[j] = pack2(-x0, -x1);
          pn[j] = pack2(-__uint_as_float(dvn[2 * j]), -__uint_as_float(dvn[2 * j + 1]));
        }
        tmem_st8r(tmem + lane_base + VA_COL + hf * 8, pc);
        tmem_st8r(tmem + lane_base + VNA_COL + hf * 8, pn);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(va_ready);
      // ---- E2: dS_c = e^gam_C dS_{c+1} + G
      if (!warp_wait(d2_full, i & 1, a.err, abort_flag)) break;
      tc_fence_after();
      const float ec = a.Ec[(((int64_t)(b * 2 + 1) * a.Hv + h) * nb + c)];
      uint32_t pk[32];  // bf16 pairs of this thread's dS^T row
      {
        uint32_t r0[32], r1[32];
        tmem_ld32r(tmem + lane_base + DS_COL + hf * 64, r0);
        tmem_ld32r(tmem + lane_base + DS_COL + hf * 64 + 32, r1);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          S[j] = ec * S[j] + __uint_as_float(r0[j]);
          S[32 + j] = ec * S[32 + j] + __uint_as_float(r1[j]);
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) pk[j] = pack2(S[2 * j], S[2 * j + 1]);
        tmem_st32r(tmem + lane_base + SA_COL + hf * 32, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sa_ready);
      if (warp == 0 && lane == 0) mbar_arrive(&empty[s]);
      if (c > 0) {
        uint4* dst = reinterpret_cast<uint4*>(a.dS_out + ((((int64_t)b * nb + c - 1) * a.Hv + h) * D + v) * D + hf * 64);
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------------------------- host
struct alignas(64) PrepLaunch {
  CUtensorMap mq, mk, mv;
  PArgs args;
};
struct alignas(64) RecurLaunch {
  CUtensorMap mt, mp;
  RArgs args;
};

}  // namespace gdn_tc

// Whether the tensor-core forward takes this problem: head dim 128 (k and v), chunk 32, the fork
// layout (no concat run), L a multiple of 128, TMA-compatible strides and bases, and not disabled
// by BDLLM_GDN_TC=0.
bool gdn_tc_eligible(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t L, int64_t C,
                     bool concat) {
  static const bool off = getenv("BDLLM_GDN_TC") != nullptr && getenv("BDLLM_GDN_TC")[0] == '0';
  if (off || concat || C != 32 || L % 128 != 0) return false;
  if (q.size(3) != 128 || v.size(3) != 128 || k.size(3) != 128) return false;
  const auto al = [](const at::Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; };
  if (!al(q) || !al(k) || !al(v) || q.stride(1) % 8 != 0 || v.stride(1) % 8 != 0) return false;
  if (q.size(1) != 2 * L) return false;
  return true;
}

// q, k [B, 2L, Hk, 128], v [B, 2L, Hv, 128] (strided token rows, heads packed), g, beta fp32
// contiguous [B, 2L, Hv]. Returns {o, S_in}.
std::vector<at::Tensor> gdn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                   const at::Tensor& beta, int64_t L) {
  using namespace gdn_tc;
  const int B = q.size(0), Hk = q.size(2), Hv = v.size(2);
  TORCH_CHECK(Hv % Hk == 0, "gdn_tc: Hv % Hk == 0");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16 &&
                  q.size(1) == 2 * L && k.sizes() == q.sizes() && v.size(0) == B && v.size(1) == q.size(1),
              "gdn_tc: bf16 q, k [B, 2L, Hk, 128] and v [B, 2L, Hv, 128]");
  TORCH_CHECK(g.numel() == (int64_t)B * 2 * L * Hv && beta.numel() == g.numel(), "gdn_tc: g, beta [B, 2L, Hv]");
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.stride(1) == k.stride(1) && q.stride(2) == 128 && k.stride(2) == 128 && v.stride(2) == 128 &&
                  q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1,
              "gdn_tc: heads packed within a token row, unit inner stride");
  TORCH_CHECK(B == 1 || (q.stride(0) == q.size(1) * q.stride(1) && k.stride(0) == k.size(1) * k.stride(1) &&
                         v.stride(0) == v.size(1) * v.stride(1)),
              "gdn_tc: batch and token dims must merge");
  TORCH_CHECK(g.is_contiguous() && beta.is_contiguous() && g.scalar_type() == at::kFloat &&
                  beta.scalar_type() == at::kFloat,
              "gdn_tc: g, beta fp32 contiguous [B, 2L, Hv]");
  const int nb = (int)(L / C);
  const int64_t nch = (int64_t)B * 2 * Hv * nb;
  TORCH_CHECK(nch * C * 4 < (int64_t)1 << 31, "gdn_tc: problem too large for 32-bit TMA row coordinates");
  auto bf = q.options().dtype(at::kBFloat16);
  auto f32 = q.options().dtype(at::kFloat);
  auto tiles = at::empty({4, nch * C, 128}, bf);  // U, W, q~, K~
  auto P = at::empty({nch * C, 64}, bf);
  auto Ec = at::empty({nch}, f32);
  auto S_in = at::empty({B, nb, Hv, 128, 128}, bf);  // S^T rows (v, k)
  auto o = at::empty({B, 2 * L, Hv, 128}, q.options());
  int* err = error_word_ptr();
  auto st = at::cuda::getCurrentCUDAStream();

  static thread_local PrepLaunch pl;
  make_map_bf16(&pl.mq, q.data_ptr(), (uint64_t)Hk * 128, (uint64_t)B * 2 * L, q.stride(1), 64, TT);
  make_map_bf16(&pl.mk, k.data_ptr(), (uint64_t)Hk * 128, (uint64_t)B * 2 * L, k.stride(1), 64, TT);
  make_map_bf16(&pl.mv, v.data_ptr(), (uint64_t)Hv * 128, (uint64_t)B * 2 * L, v.stride(1), 64, TT);
  auto* tb = reinterpret_cast<__nv_bfloat16*>(tiles.data_ptr());
  const int64_t tsz = nch * C * 128;
  pl.args = PArgs{g.data_ptr<float>(), beta.data_ptr<float>(), tb, tb + tsz, tb + 2 * tsz, tb + 3 * tsz,
                  reinterpret_cast<__nv_bfloat16*>(P.data_ptr()), Ec.data_ptr<float>(), nullptr, B, (int)L, Hk, Hv,
                  nb, 1.f / sqrtf(128.f), err};
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PSmem::BYTES));
    C10_CUDA_CHECK(cudaFuncSetAttribute(recur_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, R_SMEM));
    attr = true;
  }
  {
    void* kargs[4] = {&pl.mq, &pl.mk, &pl.mv, &pl.args};
    C10_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(prep_kernel), dim3(nb / 4, Hk, B * 2),
                                    dim3(P_THREADS), kargs, PSmem::BYTES, st));
  }
  static thread_local RecurLaunch rl;
  make_map_bf16(&rl.mt, tiles.data_ptr(), 128, (uint64_t)4 * nch * C, 128, 64, C);
  make_map_bf16(&rl.mp, P.data_ptr(), 64, (uint64_t)nch * C, 64, 64, C);
  rl.args = RArgs{Ec.data_ptr<float>(), tb, reinterpret_cast<__nv_bfloat16*>(S_in.data_ptr()),
                  reinterpret_cast<__nv_bfloat16*>(o.data_ptr()),
                  B, (int)L, Hv, nb, err};
  {
    void* kargs[3] = {&rl.mt, &rl.mp, &rl.args};
    C10_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(recur_kernel), dim3(B * Hv), dim3(R_THREADS), kargs,
                                    R_SMEM, st));
  }
  return {o, S_in};
}

// The backward's sequential part on tcgen05 for the fork layout (head dim 128, chunk 32): reruns the
// prep kernel (W, q~, K~, P^T, e^gam_C of both streams) and the reverse recurrence. dout is bf16
// contiguous [B, 2L, Hv, 128]; dS_out [B, nb, Hv, 128, 128] and dVp [B, nb, Hv, 32, 128] (fp32) are
// written: what the clean chunk kernel reads (dS_out as bf16 rows of dS_out^T, [v][k] per chunk).
// The noised blocks' state gradients are included.
void gdn_bwd_recurrence_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                           const at::Tensor& beta, const at::Tensor& dout, int64_t L, __nv_bfloat16* dS_out,
                           float* dVp) {
  using namespace gdn_tc;
  const int B = q.size(0), Hk = q.size(2), Hv = v.size(2);
  const int nb = (int)(L / C);
  const int64_t nch = (int64_t)B * 2 * Hv * nb;
  auto bf = q.options().dtype(at::kBFloat16);
  auto tiles = at::empty({4, nch * C, 128}, bf);  // (unused U slot), W, q~, K~
  auto Pt = at::empty({nch * C, 64}, bf);
  auto Ec = at::empty({nch}, q.options().dtype(at::kFloat));
  int* err = error_word_ptr();
  auto st = at::cuda::getCurrentCUDAStream();
  static thread_local PrepLaunch pl;
  make_map_bf16(&pl.mq, q.data_ptr(), (uint64_t)Hk * 128, (uint64_t)B * 2 * L, q.stride(1), 64, TT);
  make_map_bf16(&pl.mk, k.data_ptr(), (uint64_t)Hk * 128, (uint64_t)B * 2 * L, k.stride(1), 64, TT);
  make_map_bf16(&pl.mv, v.data_ptr(), (uint64_t)Hv * 128, (uint64_t)B * 2 * L, v.stride(1), 64, TT);
  auto* tb = reinterpret_cast<__nv_bfloat16*>(tiles.data_ptr());
  const int64_t tsz = nch * C * 128;
  pl.args = PArgs{g.data_ptr<float>(), beta.data_ptr<float>(), nullptr, tb + tsz, tb + 2 * tsz, tb + 3 * tsz, nullptr,
                  Ec.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(Pt.data_ptr()), B, (int)L, Hk, Hv, nb,
                  1.f / sqrtf(128.f), err};
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PSmem::BYTES));
    C10_CUDA_CHECK(cudaFuncSetAttribute(bwd_recur_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, R_SMEM));
    attr = true;
  }
  {
    void* kargs[4] = {&pl.mq, &pl.mk, &pl.mv, &pl.args};
    C10_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(prep_kernel), dim3(nb / 4, Hk, B * 2),
                                    dim3(P_THREADS), kargs, PSmem::BYTES, st));
  }
  struct alignas(64) BLaunch {
    CUtensorMap mt, mp, mdo;
    BArgs args;
  };
  static thread_local BLaunch bl;
  make_map_bf16(&bl.mt, tiles.data_ptr(), 128, (uint64_t)4 * nch * C, 128, 64, C);
  make_map_bf16(&bl.mp, Pt.data_ptr(), 64, (uint64_t)nch * C, 64, 64, C);
  make_map_bf16(&bl.mdo, dout.data_ptr(), (uint64_t)Hv * 128, (uint64_t)B * 2 * L, (uint64_t)Hv * 128, 64, C);
  bl.args = BArgs{Ec.data_ptr<float>(), dS_out, dVp, B, (int)L, Hv, nb, err};
  void* kargs[4] = {&bl.mt, &bl.mp, &bl.mdo, &bl.args};
  C10_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(bwd_recur_kernel), dim3(B * Hv), dim3(R_THREADS), kargs,
                                  R_SMEM, st));
}

}  // namespace bdllm
