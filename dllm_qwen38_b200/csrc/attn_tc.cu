// Complementary-mask attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Same contract as the mma.sync forward in attn.cu (O [B, T2, Hq, D] bf16 and the per-row
// log2-sum-exp of the scaled scores), same analytic mask and tile skipping, for head dims 128 and
// 256. One CTA = 128 query rows of one (batch, query head); 6 warps:
//   warp 4      TMA producer: the Q tile once, then K and V tiles of 64 keys into a 2-stage ring
//   warp 5      MMA issuer (one thread): S = Q K^T (M 128, N 64, K D) into one of two TMEM score
//               buffers, O += P V (M 128, N D, K 64) into the TMEM output accumulator
//   warps 0-3   softmax: thread = query row = TMEM lane; reads its 64 scores with tcgen05.ld,
//               masks, keeps a running max and sum, writes P (bf16) into a 128-byte-swizzled smem
//               tile that the next MMA reads as its K-major A operand
// The score MMA of tile j+1 is issued before the softmax of tile j, so the tensor pipe computes it
// while the softmax runs. O is rescaled lazily: a row's reference max moves only when a new score
// exceeds it by more than 2^8 (the probabilities stay <= 256, exact in fp32 / bf16 range), and the
// rescale reads O from TMEM, scales it and stores it back (tcgen05.st) after the previous O MMA
// has completed. Every mbarrier wait is bounded; on expiry the CTA records ERR_ATTN_WAIT, drains
// what it issued and frees its TMEM.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
void make_map_bf16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                   uint32_t box_outer);

namespace attn_tc {

constexpr int BQ = 128;   // query rows per CTA (MMA M)
constexpr int BKV = 64;   // keys per tile
constexpr int NTHR = 192;
constexpr float NEG_INF = -INFINITY;
constexpr float RESCALE_LOG2 = 8.f;

template <int D>
struct FCfg {
  static constexpr int Q_BYTES = BQ * D * 2;   // D/64 boxes of [128 rows][128 B]
  static constexpr int K_BYTES = BKV * D * 2;  // D/64 boxes of [64 rows][128 B]
  static constexpr int STAGE = 2 * K_BYTES;    // K then V
  static constexpr int P_BYTES = BQ * BKV * 2;  // [128 rows][128 B], one swizzle atom column
  static constexpr int SMEM = Q_BYTES + 2 * STAGE + 2 * P_BYTES + 1024 + 256;
  static constexpr int O_COL = (D == 256) ? 256 : 128;  // TMEM column of O; S buffers at 0 and 64
  static constexpr int TMEM_COLS = (D == 256) ? 512 : 256;
  static constexpr uint32_t IDESC_S = idesc_bf16(BQ, BKV, 0, 0);
  static constexpr uint32_t IDESC_O = idesc_bf16(BQ, D, 0, 1);  // V read N(=d)-contiguous
};

struct FArgs {
  __nv_bfloat16* o;
  float* lse2;
  int B, T2, L, Hq, Hk, block, leak;
  float scale_log2;
  int* err;
};

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

// does every row in [i0, i1] see every key in [j0, j1]? (then the tile needs no mask)
__device__ __forceinline__ bool tile_all(int i0, int i1, int j0, int j1, int T2, int L, int block, int leak) {
  if (i1 >= T2 || j1 >= T2) return false;
  if ((i0 < L) != (i1 < L) || (j0 < L) != (j1 < L)) return false;
  if (i1 < L) {
    const int qb0 = i0 / block, qb1 = i1 / block;
    if (j1 < L) {
      const int kb0 = j0 / block, kb1 = j1 / block;
      return leak ? (kb1 <= qb0) : (kb0 == kb1 && qb0 == qb1 && kb0 == qb0);
    }
    return (j1 - L) / block < qb0;
  }
  if (j1 < L) return false;
  return (j1 - L) / block <= (i0 - L) / block;
}

__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// wait for this thread's outstanding tcgen05.ld; the registers are operands so that no use of them
// is scheduled before the wait
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// a bounded wait whose outcome is the same in every lane of the warp (the tcgen05.ld / st that
// follow are warp-collective)
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, err, ERR_ATTN_WAIT, abort);
  return __all_sync(0xffffffffu, ok);
}

// next visible key tile at or after jt (nkt when none)
__device__ __forceinline__ int next_tile(int jt, int nkt, int i0, int i1, const FArgs& a) {
  for (; jt < nkt; ++jt)
    if (tile_may(i0, i1, jt * BKV, min(jt * BKV + BKV - 1, a.T2 - 1), a.L, a.block, a.leak)) return jt;
  return nkt;
}

template <int D>
__global__ void __launch_bounds__(NTHR, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                  const __grid_constant__ CUtensorMap mv, FArgs a) {
  using C = FCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + C::Q_BYTES;
  uint8_t* sP = sKV + 2 * C::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 7;
  uint64_t* o_done = bars + 9;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // heavy (late) query tiles first: x_0 rows see the most keys at the end of each stream
  const int nqt = gridDim.x;
  const int qt = nqt - 1 - blockIdx.x;
  const int i0 = qt * BQ, i1 = min(i0 + BQ - 1, a.T2 - 1);
  const int b = blockIdx.y / a.Hq, h = blockIdx.y % a.Hq, hk = h / (a.Hq / a.Hk);
  const int nkt = (a.T2 + BKV - 1) / BKV;
  const int row0 = b * a.T2;  // first row of this batch in the [B*T2, H*D] maps

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);  // one arrive per softmax warp
      mbar_init(&o_done[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mq);
    prefetch_tmap(&mk);
    prefetch_tmap(&mv);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_2d(sQ + c * BQ * 128, &mq, q_full, h * D + c * 64, row0 + i0);
      uint32_t armed = 0;
      int it = 0;
      bool ok = true;
      for (int jt = next_tile(0, nkt, i0, i1, a); jt < nkt; jt = next_tile(jt + 1, nkt, i0, i1, a), ++it) {
        const int s = it & 1;
        if (!mbar_wait(&kv_empty[s], ((it >> 1) & 1) ^ 1, a.err, ERR_ATTN_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], C::STAGE);
        armed |= 1u << s;
        uint8_t* dk = sKV + s * C::STAGE;
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(dk + c * BKV * 128, &mk, &kv_full[s], hk * D + c * 64, row0 + jt * BKV);
          tma_load_2d(dk + C::K_BYTES + c * BKV * 128, &mv, &kv_full[s], hk * D + c * 64, row0 + jt * BKV);
        }
      }
      // every load armed must land before the CTA exits (bounded): the last arming of each stage
      mbar_wait(q_full, 0, a.err, ERR_ATTN_WAIT, nullptr);
      for (int s = 0; s < 2; ++s)
        if (armed & (1u << s)) {
          const int last = ((it - 1) & 1) == s ? it - 1 : it - 2;
          if (last >= 0) mbar_wait(&kv_full[s], (last >> 1) & 1, a.err, ERR_ATTN_WAIT, nullptr);
        }
      (void)ok;
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      bool ok = mbar_wait(q_full, 0, a.err, ERR_ATTN_WAIT, abort_flag);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_s = [&](int it) {
        const int s = it & 1;
        const uint32_t k_addr = smem_u32(sKV + s * C::STAGE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off_q = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
          const uint32_t off_k = (kk >> 2) * (BKV * 128) + (kk & 3) * 32;
          mma_bf16(tmem + s * BKV, smem_desc(q_addr + off_q, 16, 1024), smem_desc(k_addr + off_k, 16, 1024),
                   C::IDESC_S, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[s]);
      };
      int jt = ok ? next_tile(0, nkt, i0, i1, a) : nkt;
      if (jt < nkt) {
        if (mbar_wait(&kv_full[0], 0, a.err, ERR_ATTN_WAIT, abort_flag)) {
          tc_fence_after();
          issue_s(0);
        } else {
          ok = false;
        }
      }
      for (int it = 0; ok && jt < nkt; ++it) {
        const int nxt = next_tile(jt + 1, nkt, i0, i1, a);
        if (nxt < nkt) {
          if (!mbar_wait(&kv_full[(it + 1) & 1], ((it + 1) >> 1) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(it + 1);
        }
        const int s = it & 1;
        if (!mbar_wait(&p_full[s], (it >> 1) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + s * C::P_BYTES);
        const uint32_t v_addr = smem_u32(sKV + s * C::STAGE + C::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          mma_bf16(tmem + C::O_COL, smem_desc(p_addr + kk * 32, 16, 1024), smem_desc(v_addr + kk * 2048, 8192, 1024),
                   C::IDESC_O, (it > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&o_done[s]);
        mma_commit(&kv_empty[s]);
        jt = nxt;
      }
      // every MMA issued must complete before TMEM is freed (bounded)
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_ATTN_WAIT, nullptr);
    }
  } else {
    // -------------------------------------------------------------- softmax (warps 0-3)
    const int r = warp * 32 + lane;
    const int row = i0 + r;
    const bool valid = row < a.T2;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float m_used = NEG_INF, l = 0.f;
    int it = 0;
    bool ok = true;
    for (int jt = next_tile(0, nkt, i0, i1, a); jt < nkt; jt = next_tile(jt + 1, nkt, i0, i1, a), ++it) {
      const int s = it & 1;
      const int j0 = jt * BKV;
      if (!warp_wait(&s_full[s], (it >> 1) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t ra[32], rb[32];
      tmem_ld32_async(tmem + lane_base + s * BKV, ra);
      tmem_ld32_async(tmem + lane_base + s * BKV + 32, rb);
      tmem_wait_ld(ra);
      tmem_wait_ld(rb);
      float x[64];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        x[c] = __uint_as_float(ra[c]) * a.scale_log2;
        x[32 + c] = __uint_as_float(rb[c]) * a.scale_log2;
      }
      if (!tile_all(i0, i0 + BQ - 1, j0, j0 + BKV - 1, a.T2, a.L, a.block, a.leak)) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int col = j0 + c;
          if (!valid || col >= a.T2 || !allowed(row, col, a.L, a.block, a.leak)) x[c] = NEG_INF;
        }
      }
      float mx = NEG_INF;
#pragma unroll
      for (int c = 0; c < 64; ++c) mx = fmaxf(mx, x[c]);
      float alpha = 1.f;
      if (mx > m_used + RESCALE_LOG2) {
        if (m_used != NEG_INF) alpha = exp2f(m_used - mx);
        m_used = mx;
      }
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        // O holds tiles < it: wait for the last O MMA, then rescale this warp's rows in TMEM
        if (!warp_wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ro[32];
          tmem_ld32_async(tmem + lane_base + C::O_COL + c * 32, ro);
          tmem_wait_ld(ro);
#pragma unroll
          for (int e = 0; e < 32; ++e) ro[e] = __float_as_uint(__uint_as_float(ro[e]) * alpha);
          tmem_st32(tmem + lane_base + C::O_COL + c * 32, ro);
        }
        tmem_wait_st();
      }
      l *= alpha;
      const float mu = (m_used == NEG_INF) ? 0.f : m_used;
      uint32_t pk[32];
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = exp2f(x[2 * c] - mu), p1 = exp2f(x[2 * c + 1] - mu);
        rs += p0 + p1;
        pk[c] = pack_bf16(p0, p1);
      }
      l += rs;
      // the P buffer s was read by the O MMA of tile it-2
      if (it >= 2 && !warp_wait(&o_done[s], ((it - 2) >> 1) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      uint8_t* prow = sP + s * C::P_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async();  // generic smem writes -> visible to the tensor core's async proxy
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    // epilogue: O / l (bf16) and the row's log2-sum-exp
    if (ok && it > 0 && !warp_wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1, a.err, abort_flag)) ok = false;
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __nv_bfloat16* orow = a.o + ((int64_t)b * a.T2 + row) * a.Hq * D + h * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t ro[32];
      if (ok && it > 0) {
        tmem_ld32_async(tmem + lane_base + C::O_COL + c * 32, ro);
        tmem_wait_ld(ro);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ro[e] = 0u;
      }
      if (valid) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = pack_bf16(__uint_as_float(ro[2 * e]) * inv, __uint_as_float(ro[2 * e + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
    }
    if (valid) a.lse2[((int64_t)b * a.Hq + h) * a.T2 + row] = m_used + log2f(fmaxf(l, 1e-30f));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

struct alignas(64) Maps {
  CUtensorMap q, k, v;
};

template <int D>
static void launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                   int64_t L, int64_t block, double scale, bool leak) {
  using C = FCfg<D>;
  const int B = q.size(0), T2 = q.size(1), Hq = q.size(2), Hk = k.size(2);
  Maps m;
  // [B*T2 rows, H*D cols] views with the tensors' token strides
  make_map_bf16(&m.q, q.data_ptr(), (uint64_t)Hq * D, (uint64_t)B * T2, q.stride(1), 64, BQ);
  make_map_bf16(&m.k, k.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, k.stride(1), 64, BKV);
  make_map_bf16(&m.v, v.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, v.stride(1), 64, BKV);
  FArgs a{};
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse2 = lse.data_ptr<float>();
  a.B = B, a.T2 = T2, a.L = (int)L, a.Hq = Hq, a.Hk = Hk, a.block = (int)block, a.leak = leak ? 1 : 0;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.err = error_word_ptr();
  auto kern = fwd_tc_kernel<D>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr = true;
  }
  const dim3 grid((T2 + BQ - 1) / BQ, B * Hq);
  kern<<<grid, NTHR, C::SMEM, at::cuda::getCurrentCUDAStream()>>>(m.q, m.k, m.v, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace attn_tc

// tcgen05 forward for head dims 128 / 256 (returns false when the shape is not covered)
bool attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                 int64_t L, int64_t block, double scale, bool leak) {
  const int64_t D = q.size(3);
  if (D != 128 && D != 256) return false;
  bind_context(q.get_device());
  if (D == 128)
    attn_tc::launch<128>(q, k, v, o, lse, L, block, scale, leak);
  else
    attn_tc::launch<256>(q, k, v, o, lse, L, block, scale, leak);
  return true;
}

}  // namespace bdllm
