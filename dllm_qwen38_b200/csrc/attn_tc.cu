// Complementary-mask attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
// (Reference path replaced: dense mask + HF eager / SDPA attention, `src/dllm_qwen38/blockdiff.py:50-66,178-182`.)
//
// Same contract as the mma.sync forward in attn.cu (O [B, T2, Hq, D] bf16 and the per-row
// log2-sum-exp of the scaled scores), same analytic mask and tile skipping, for head dims 128 and
// 256. One CTA = 128 query rows of one (batch, query head); 6 warps:
//   warp 4      TMA producers: the Q tile once, then K and V tiles of 64 (or 32) keys into two
//               rings (K released by its score MMA, V by the PV MMA; 3 K and 2 V stages at D 256)
//   warp 5      MMA issuer (one thread): S = Q K^T (M 128, N 64, K D) into one of three TMEM score
//               buffers, ahead of the softmax by as many tiles as the ring allows, and
//               O += P V (M 128, N D, K 64) into the TMEM output accumulator, with P read from TMEM
//               as the A operand
//   warps 0-3   softmax: thread = query row = TMEM lane; reads its scores with tcgen05.ld, masks,
//               keeps a running max and sum, and stores P (bf16, packed pairs) into TMEM
//               (tcgen05.st, double-buffered)
// Score MMAs run ahead of the softmax, so the tensor pipe computes the next tiles' scores while the
// softmax of this one runs. O is rescaled lazily: a row's reference max moves only when a new score
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
constexpr int NTHR = 192;
// backward kernels: warps 0-7 form dS (and P^T) from the score tiles (warp w: TMEM lane quadrant
// w % 4, half w / 4 of each 32-column tile), warp 8 loads, warp 9 issues the MMAs
constexpr int NTHR_K = 320;
constexpr float NEG_INF = -INFINITY;
constexpr float RESCALE_LOG2 = 8.f;

template <int D, int BKV_ = 64>
struct FCfg {
  static constexpr int BKV = BKV_;             // keys per tile
  static constexpr int Q_BYTES = BQ * D * 2;   // D/64 boxes of [128 rows][128 B]
  static constexpr int K_BYTES = BKV * D * 2;  // one K or V tile: D/64 boxes of [BKV rows][128 B]
  // separate K and V rings: a K stage is released as soon as its score MMA completes, a V stage
  // only after the PV MMA that follows the softmax, so K can run further ahead
  static constexpr int NTILE_FIT = (227 * 1024 - Q_BYTES - 1024 - 256) / K_BYTES;
  static constexpr int NV = NTILE_FIT >= 6 ? 3 : 2;
  static constexpr int NK_FIT = NTILE_FIT - NV;
  static constexpr int NK = NK_FIT > 4 ? 4 : NK_FIT;
  static constexpr int NS = 3;                 // TMEM score buffers
  static constexpr int AHEAD = (NS - 1) < (NK - 1) ? (NS - 1) : (NK - 1);  // score MMAs issued ahead
  static constexpr int SMEM = Q_BYTES + (NK + NV) * K_BYTES + 1024 + 256;
  // TMEM: NS score buffers of BKV columns, two bf16 P buffers of BKV/2 packed columns (the A
  // operand of the PV MMA), and O (D columns)
  static constexpr int S_COL = 0, P_COL = NS * BKV;
  static constexpr int O_COL = (P_COL + BKV <= 128 && D <= 128) ? 128 : 256;
  static constexpr int TMEM_COLS = (O_COL + D <= 256) ? 256 : 512;
  static constexpr uint32_t IDESC_S = idesc_bf16(BQ, BKV, 0, 0);
  static constexpr uint32_t IDESC_O = idesc_bf16(BQ, D, 0, 1);  // V read N(=d)-contiguous
  static_assert(NK >= 2 && NV >= 2 && P_COL + BKV <= O_COL && O_COL + D <= 512, "attention forward resources");
};

struct FArgs {
  __nv_bfloat16* o;
  float* lse2;
  int B, T2, L, Hq, Hk, block, leak;
  float scale_log2;
  int* err;
};

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
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A (M 128 x K 16, bf16) is read from TMEM, row i in lane i,
// consecutive K pairs packed in consecutive 32-bit columns (8 columns per instruction)
__device__ __forceinline__ void mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ex2 on the SFU (approximate, flush-to-zero): the softmax exponentials in base 2
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Dispatch rank r -> query tile, heaviest first. A query tile's work grows along each stream (x_t
// rows see the clean blocks before theirs, x_0 rows the clean prefix), so the two halves are
// walked down from their ends in turn: r = 0, 2, 4.. take the upper half [lo, n) from the top,
// r = 1, 3, 5.. the lower half [0, lo) from its top (a bijection on [0, n) for any n).
__host__ __device__ __forceinline__ int heavy_first(int r, int n) {
  const int lo = n / 2;
  return (r & 1) ? lo - 1 - (r >> 1) : n - 1 - (r >> 1);
}

// Up to two runs of tiles: [a0, a0 + na) then [b0, b0 + nb); k-th visible tile = at(k)
struct Span2 {
  int a0, na, b0, nb;
  __device__ __forceinline__ int n() const { return na + nb; }
  __device__ __forceinline__ int at(int k) const { return k < na ? a0 + k : b0 + (k - na); }
};

// tiles of W covering [lo1, hi1) and [lo2, hi2) (hi1 <= lo2 or an empty first range)
__device__ __forceinline__ Span2 span_of(int lo1, int hi1, int lo2, int hi2, int W) {
  Span2 s;
  s.a0 = lo1 / W;
  s.na = hi1 > lo1 ? (hi1 + W - 1) / W - s.a0 : 0;
  s.b0 = lo2 / W;
  int b1 = hi2 > lo2 ? (hi2 + W - 1) / W : s.b0;
  if (s.na > 0 && s.b0 < s.a0 + s.na) s.b0 = s.a0 + s.na;  // a tile straddling L is listed once
  s.nb = max(0, b1 - s.b0);
  return s;
}

// key tiles of width W that some row of the query rows [i0, i1] may see (exactly the tiles
// tile_may accepts): x_t keys of the rows' blocks (all earlier x_t blocks with the leak fault),
// and the clean keys before the last block of the x_t rows / up to the last x_0 row's block
__device__ __forceinline__ Span2 key_tiles(int i0, int i1, int L, int block, int leak, int W) {
  int k1lo = 0, k1hi = 0, c = 0;
  if (i0 < L) {
    const int qb0 = i0 / block, qb1 = min(i1, L - 1) / block;
    k1lo = leak ? 0 : qb0 * block;
    k1hi = min((qb1 + 1) * block, L);
    c = qb1 * block;
  }
  if (i1 >= L) c = max(c, min(((i1 - L) / block + 1) * block, L));
  return span_of(k1lo, k1hi, L, L + c, W);
}

// query-row tiles of width W that may see some key of [j0, j1] (a hull: tiles it adds are fully
// masked and contribute zeros)
__device__ __forceinline__ Span2 row_tiles(int j0, int j1, int L, int T2, int block, int leak, int W) {
  int r1lo = L, r1hi = 0, r2lo = T2;
  if (j0 < L) {
    const int kb0 = j0 / block, kb1 = min(j1, L - 1) / block;
    r1lo = kb0 * block;
    r1hi = leak ? L : min((kb1 + 1) * block, L);
  }
  if (j1 >= L) {
    const int kb0 = (max(j0, L) - L) / block;
    if ((kb0 + 1) * block < L) {
      r1lo = min(r1lo, (kb0 + 1) * block);
      r1hi = L;
    }
    r2lo = L + kb0 * block;
  }
  if (r1hi <= r1lo) r1lo = r1hi = 0;
  return span_of(r1lo, r1hi, r2lo, T2, W);
}

// keys visible to one query row i: x_t keys [lo_t, hi_t), x_0 keys [L, L + hi_0)
struct RowVis {
  int lo_t, hi_t, hi_0;
  __device__ __forceinline__ bool sees(int j, int L) const { return j < L ? (j >= lo_t && j < hi_t) : (j < L + hi_0); }
  // every key of [j0, j1] (one stream) visible?
  __device__ __forceinline__ bool sees_all(int j0, int j1, int L) const {
    return j1 < L ? (j0 >= lo_t && j1 < hi_t) : (j0 >= L && j1 < L + hi_0);
  }
};
__device__ __forceinline__ RowVis row_vis(int i, int L, int T2, int block, int leak) {
  RowVis r{0, 0, 0};
  if (i >= T2) return r;
  if (i < L) {
    const int bi = i / block;
    r.lo_t = leak ? 0 : bi * block;
    r.hi_t = min((bi + 1) * block, L);
    r.hi_0 = bi * block;
  } else {
    r.hi_0 = min(((i - L) / block + 1) * block, L);
  }
  return r;
}

// query rows that see one key j: x_t rows [lo_t, hi_t), x_0 rows [lo_0, T2)
struct KeyVis {
  int lo_t, hi_t, lo_0;
  __device__ __forceinline__ bool seen_by(int i, int L, int T2) const {
    return i < L ? (i >= lo_t && i < hi_t) : (i >= lo_0 && i < T2);
  }
  __device__ __forceinline__ bool seen_by_all(int i0, int i1, int L, int T2) const {
    return i1 < L ? (i0 >= lo_t && i1 < hi_t) : (i0 >= lo_0 && i0 >= L && i1 < T2);
  }
};
__device__ __forceinline__ KeyVis key_vis(int j, int L, int T2, int block, int leak) {
  KeyVis k{0, 0, T2};
  if (j >= T2) return k;
  if (j < L) {
    const int bj = j / block;
    k.lo_t = bj * block;
    k.hi_t = leak ? L : min((bj + 1) * block, L);
  } else {
    const int bj = (j - L) / block;
    k.lo_t = (bj + 1) * block;
    k.hi_t = L;
    k.lo_0 = L + bj * block;
  }
  return k;
}

// a bounded wait whose outcome is the same in every lane of the warp (the tcgen05.ld / st that
// follow are warp-collective)
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, err, ERR_ATTN_WAIT, abort);
  return __all_sync(0xffffffffu, ok);
}

template <int D, int BKV_>
__global__ void __launch_bounds__(NTHR, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                  const __grid_constant__ CUtensorMap mv, FArgs a) {
  using C = FCfg<D, BKV_>;
  constexpr int BKV = C::BKV, NK = C::NK, NV = C::NV, NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::Q_BYTES;
  uint8_t* sV = sK + NK * C::K_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NV * C::K_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + NK;
  uint64_t* v_full = k_empty + NK;
  uint64_t* v_empty = v_full + NV;
  uint64_t* s_full = v_empty + NV;
  uint64_t* p_full = s_full + NS;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // grid (B * Hq, query tiles): every head's tile of one work rank is dispatched before the next rank
  const int qt = heavy_first(blockIdx.y, gridDim.y);
  const int i0 = qt * BQ, i1 = min(i0 + BQ - 1, a.T2 - 1);
  const int b = blockIdx.x / a.Hq, h = blockIdx.x % a.Hq, hk = h / (a.Hq / a.Hk);
  const Span2 sp = key_tiles(i0, i1, a.L, a.block, a.leak, BKV);  // visible key tiles, in order
  const int nt = sp.n();
  const int row0 = b * a.T2;  // first row of this batch in the [B*T2, H*D] maps

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < NV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < NS; ++s) mbar_init(&s_full[s], 1);
    for (int s = 0; s < 2; ++s) {
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
    if (lane == 0 || lane == 1) {
      // ------------------------------------------------------------ TMA producers: lane 0 the Q
      // tile and the K ring, lane 1 the V ring (independent waits, so K runs ahead of V)
      const bool isk = lane == 0;
      const int nst = isk ? NK : NV;
      uint8_t* ring = isk ? sK : sV;
      uint64_t* full = isk ? k_full : v_full;
      uint64_t* empty = isk ? k_empty : v_empty;
      const CUtensorMap* map = isk ? &mk : &mv;
      if (isk) {
        mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) tma_load_2d(sQ + c * BQ * 128, &mq, q_full, h * D + c * 64, row0 + i0);
      }
      int last[4] = {-1, -1, -1, -1};
      for (int it = 0; it < nt; ++it) {
        const int jt = sp.at(it);
        const int s = it % nst;
        if (!mbar_wait(&empty[s], ((it / nst) & 1) ^ 1, a.err, ERR_ATTN_WAIT, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], C::K_BYTES);
        last[s] = it;
        uint8_t* dst = ring + s * C::K_BYTES;
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(dst + c * BKV * 128, map, &full[s], hk * D + c * 64, row0 + jt * BKV);
      }
      // every load armed must land before the CTA exits (bounded): the last arming of each stage
      if (isk) mbar_wait(q_full, 0, a.err, ERR_ATTN_WAIT, nullptr);
      for (int s = 0; s < nst; ++s)
        if (last[s] >= 0) mbar_wait(&full[s], (last[s] / nst) & 1, a.err, ERR_ATTN_WAIT, nullptr);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      bool ok = mbar_wait(q_full, 0, a.err, ERR_ATTN_WAIT, abort_flag);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      int issued = 0;  // score MMAs issued so far; up to AHEAD tiles ahead of the PV being waited
      for (int it = 0; ok && it < nt; ++it) {
        while (issued < nt && issued <= it + C::AHEAD) {
          if (!mbar_wait(&k_full[issued % NK], (issued / NK) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + (issued % NK) * C::K_BYTES);
          const uint32_t d_s = tmem + C::S_COL + (issued % NS) * BKV;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off_q = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
            const uint32_t off_k = (kk >> 2) * (BKV * 128) + (kk & 3) * 32;
            mma_bf16(d_s, smem_desc(q_addr + off_q, 16, 1024), smem_desc(k_addr + off_k, 16, 1024), C::IDESC_S,
                     kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[issued % NS]);
          mma_commit(&k_empty[issued % NK]);  // the K stage is free once these MMAs have read it
          ++issued;
        }
        if (!ok) break;
        const int pb = it & 1;
        if (!mbar_wait(&p_full[pb], (it >> 1) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) break;
        if (!mbar_wait(&v_full[it % NV], (it / NV) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (it % NV) * C::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          mma_bf16_ta(tmem + C::O_COL, tmem + C::P_COL + pb * (BKV / 2) + kk * 8,
                      smem_desc(v_addr + kk * 2048, BKV * 128, 1024), C::IDESC_O, (it > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&o_done[pb]);
        mma_commit(&v_empty[it % NV]);
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
    const RowVis vis = row_vis(row, a.L, a.T2, a.block, a.leak);
    const float c2 = a.scale_log2;
    float m_used = NEG_INF, l = 0.f;  // m_used in the scaled log2 domain
    int it = 0;
    bool ok = true;
    for (; it < nt; ++it) {
      const int sb = it % NS, pb = it & 1;
      const int j0 = sp.at(it) * BKV;
      if (!warp_wait(&s_full[sb], (it / NS) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[BKV];  // raw scores; masked ones -inf
#pragma unroll
      for (int h2 = 0; h2 < BKV / 32; ++h2) {
        uint32_t ra[32];
        tmem_ld32_async(tmem + lane_base + C::S_COL + sb * BKV + h2 * 32, ra);
        tmem_wait_ld(ra);
#pragma unroll
        for (int c = 0; c < 32; ++c) x[h2 * 32 + c] = __uint_as_float(ra[c]);
      }
      if (!__all_sync(0xffffffffu, vis.sees_all(j0, j0 + BKV - 1, a.L))) {
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (!vis.sees(j0 + c, a.L)) x[c] = NEG_INF;
      }
      float m8[8];  // eight independent chains, then a tree
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = x[e];
#pragma unroll
      for (int c = 8; c < BKV; ++c) m8[c & 7] = fmaxf(m8[c & 7], x[c]);
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * c2;
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
      const float nmu = (m_used == NEG_INF) ? 0.f : -m_used;
      uint32_t pk[BKV / 2];
      float r8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < BKV / 2; ++c) {
        const float p0 = ex2(fmaf(x[2 * c], c2, nmu)), p1 = ex2(fmaf(x[2 * c + 1], c2, nmu));
        r8[c & 7] += p0 + p1;
        pk[c] = pack_bf16(p0, p1);
      }
      l += ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
      // the P buffer pb was read by the O MMA of tile it-2
      if (it >= 2 && !warp_wait(&o_done[pb], ((it - 2) >> 1) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t q16[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) q16[e] = pk[c * 16 + e];
        tmem_st16(tmem + lane_base + C::P_COL + pb * (BKV / 2) + c * 16, q16);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[pb]);
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
        (void)BDLLM_CHECK(all_finite(reinterpret_cast<const float*>(ro), 32), row, a.T2);  // sentinel
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

// ================================================================== backward: dQ
// One CTA = 128 query rows of one (batch, query head), key tiles of 32:
//   S = Q K^T and dP = dO V^T (M 128, N 32, K D) into double-buffered TMEM;
//   warps 0-3 (thread = query row): P = 2^(S log2e scale - lse2), dS = P (dP - Delta), dS (bf16)
//   stored into TMEM (double-buffered), the A operand of the dQ MMA;
//   dQ += dS K (M 128, N D, K 32) in TMEM, with K read N(=d)-contiguous, from a 3-stage K/V ring.
// Delta = rowsum(dO * O) is computed by the row's thread at the start and stored for the dK/dV
// kernel.
constexpr int BK2 = 32;

template <int D>
struct QCfg {
  static constexpr int Q_BYTES = BQ * D * 2;    // Q, then dO: D/64 boxes of [128 rows][128 B]
  static constexpr int K_BYTES = BK2 * D * 2;   // D/64 boxes of [32 rows][128 B]
  static constexpr int STAGE = 2 * K_BYTES;     // K then V
  static constexpr int NST_FIT = (227 * 1024 - 2 * Q_BYTES - 1024 - 256) / STAGE;
  static constexpr int NST = NST_FIT > 4 ? 4 : NST_FIT;  // K / V ring stages
  // + 1 KB for the two half-row partial sums of Delta
  static constexpr int SMEM = 2 * Q_BYTES + NST * STAGE + 1024 + 256 + 1024;
  // TMEM: S and dP (NS buffers of 32 columns each), dS as the bf16 A operand of the dQ MMA (two
  // buffers of 16 packed columns), dQ (D columns)
  static constexpr int NS = 3;
  // S / dP MMAs issued ahead; the K/V stage they need must have been released two gradient MMAs
  // earlier (a stage released by the previous one is still loading)
  static constexpr int AHEAD_R = (NS - 1) < (NST - 2) ? (NS - 1) : (NST - 2);
  static constexpr int AHEAD = AHEAD_R < 1 ? 1 : AHEAD_R;
  static constexpr int S_COL = 0, DP_COL = NS * BK2, DS_COL = 2 * NS * BK2, DQ_COL = 256;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t IDESC_S = idesc_bf16(BQ, BK2, 0, 0);
  static constexpr uint32_t IDESC_DQ = idesc_bf16(BQ, D, 0, 1);
  static_assert(NST >= 2, "K / V ring needs two stages");
};

struct BArgs {
  const __nv_bfloat16* o;     // forward output [B, T2, Hq, D]
  const __nv_bfloat16* dout;  // [B, T2, Hq, D]
  const float* lse2;          // [B, Hq, T2]
  float* delta;               // [B, Hq, T2]
  __nv_bfloat16* dq;          // [B, T2, Hq, D]
  __nv_bfloat16* dk;          // [B, T2, Hk, D]
  __nv_bfloat16* dv;          // [B, T2, Hk, D]
  int B, T2, L, Hq, Hk, block, leak;
  float scale, scale_log2;
  int* err;
};


template <int D>
__global__ void __launch_bounds__(NTHR_K, 1)
    bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mdo,
                     const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv, BArgs a) {
  using C = QCfg<D>;
  constexpr int NST = C::NST, NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = smem + C::Q_BYTES;
  uint8_t* sKV = smem + 2 * C::Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + NST * C::STAGE);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NST;
  uint64_t* sd_full = kv_empty + NST;
  uint64_t* ds_full = sd_full + NS;
  uint64_t* dq_done = ds_full + 2;
  uint64_t* drain = dq_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* dpart = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);  // [2][128]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qt = heavy_first(blockIdx.y, gridDim.y);  // grid (B * Hq, query tiles), as the forward
  const int i0 = qt * BQ, i1 = min(i0 + BQ - 1, a.T2 - 1);
  const int b = blockIdx.x / a.Hq, h = blockIdx.x % a.Hq, hk = h / (a.Hq / a.Hk);
  const Span2 sp = key_tiles(i0, i1, a.L, a.block, a.leak, BK2);
  const int nt = sp.n();
  const int row0 = b * a.T2;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < NS; ++s) mbar_init(&sd_full[s], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ds_full[s], 8);  // the eight dS warps
      mbar_init(&dq_done[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mq);
    prefetch_tmap(&mdo);
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

  if (warp == 8) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sQ + c * BQ * 128, &mq, q_full, h * D + c * 64, row0 + i0);
        tma_load_2d(sdO + c * BQ * 128, &mdo, q_full, h * D + c * 64, row0 + i0);
      }
      int last[NST];
#pragma unroll
      for (int s = 0; s < NST; ++s) last[s] = -1;
      for (int it = 0; it < nt; ++it) {
        const int jt = sp.at(it);
        const int s = it % NST;
        if (!mbar_wait(&kv_empty[s], ((it / NST) & 1) ^ 1, a.err, ERR_ATTN_WAIT, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[s], C::STAGE);
        last[s] = it;
        uint8_t* dk = sKV + s * C::STAGE;
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(dk + c * BK2 * 128, &mk, &kv_full[s], hk * D + c * 64, row0 + jt * BK2);
          tma_load_2d(dk + C::K_BYTES + c * BK2 * 128, &mv, &kv_full[s], hk * D + c * 64, row0 + jt * BK2);
        }
      }
      mbar_wait(q_full, 0, a.err, ERR_ATTN_WAIT, nullptr);
#pragma unroll
      for (int s = 0; s < NST; ++s)
        if (last[s] >= 0) mbar_wait(&kv_full[s], (last[s] / NST) & 1, a.err, ERR_ATTN_WAIT, nullptr);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      bool ok = mbar_wait(q_full, 0, a.err, ERR_ATTN_WAIT, abort_flag);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sdO);
      int issued = 0;  // S / dP MMA pairs issued; up to AHEAD tiles ahead of the dQ MMA being waited
      for (int it = 0; ok && it < nt; ++it) {
        while (issued < nt && issued <= it + C::AHEAD) {
          if (!mbar_wait(&kv_full[issued % NST], (issued / NST) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sKV + (issued % NST) * C::STAGE), v_addr = k_addr + C::K_BYTES;
          const int sb = issued % NS;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oq = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
            const uint32_t ok_ = (kk >> 2) * (BK2 * 128) + (kk & 3) * 32;
            mma_bf16(tmem + C::S_COL + sb * BK2, smem_desc(q_addr + oq, 16, 1024), smem_desc(k_addr + ok_, 16, 1024),
                     C::IDESC_S, kk > 0 ? 1u : 0u);
            mma_bf16(tmem + C::DP_COL + sb * BK2, smem_desc(do_addr + oq, 16, 1024),
                     smem_desc(v_addr + ok_, 16, 1024), C::IDESC_S, kk > 0 ? 1u : 0u);
          }
          mma_commit(&sd_full[sb]);
          ++issued;
        }
        if (!ok) break;
        const int s = it & 1;
        if (!mbar_wait(&ds_full[s], (it >> 1) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sKV + (it % NST) * C::STAGE);
#pragma unroll
        for (int kk = 0; kk < BK2 / 16; ++kk)
          mma_bf16_ta(tmem + C::DQ_COL, tmem + C::DS_COL + s * 16 + kk * 8,
                      smem_desc(k_addr + kk * 2048, BK2 * 128, 1024), C::IDESC_DQ, (it > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&dq_done[s]);
        mma_commit(&kv_empty[it % NST]);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_ATTN_WAIT, nullptr);
    }
  } else {
    // -------------------------------------------------------------- dS (warps 0-7)
    // warp w: TMEM lane quadrant w % 4 (query row = thread), key columns [16 (w / 4), +16) of each
    // 32-key tile; Delta = rowsum(dO * O) is summed over half the head dim by each of a row's two
    // threads
    const int quad = warp & 3, hc = warp >> 2;
    const int r = quad * 32 + lane;
    const int row = i0 + r;
    const bool valid = row < a.T2;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int64_t otok = (int64_t)a.Hq * D;
    float lse = 0.f, dlt = 0.f;
    if (valid) {
      const uint4* po = reinterpret_cast<const uint4*>(a.o + ((int64_t)b * a.T2 + row) * otok + h * D) + hc * (D / 16);
      const uint4* pd =
          reinterpret_cast<const uint4*>(a.dout + ((int64_t)b * a.T2 + row) * otok + h * D) + hc * (D / 16);
#pragma unroll 4
      for (int c = 0; c < D / 16; ++c) {
        const uint4 x = po[c], y = pd[c];
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&x);
        const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 xf = __bfloat1622float2(x2[e]), yf = __bfloat1622float2(y2[e]);
          dlt += xf.x * yf.x + xf.y * yf.y;
        }
      }
      lse = a.lse2[((int64_t)b * a.Hq + h) * a.T2 + row];
    }
    dpart[hc * 128 + r] = dlt;
    asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight dS warps
    dlt = dpart[r] + dpart[128 + r];
    if (valid && hc == 0) {
      (void)BDLLM_CHECK(isfinite(dlt), row, a.T2);  // sentinel: non-finite O or dO row
      a.delta[((int64_t)b * a.Hq + h) * a.T2 + row] = dlt;
    }
    const bool live = valid && lse != NEG_INF;
    const RowVis vis = row_vis(live ? row : a.T2, a.L, a.T2, a.block, a.leak);  // nothing visible when dead
    const float c2 = a.scale_log2, nl = live ? -lse : 0.f;
    int it = 0;
    bool ok = true;
    for (; it < nt; ++it) {
      const int s = it & 1, sb = it % NS;
      const int j0 = sp.at(it) * BK2;
      if (!warp_wait(&sd_full[sb], (it / NS) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t rs[16], rp[16];
      tmem_ld16_async(tmem + lane_base + C::S_COL + sb * BK2 + 16 * hc, rs);
      tmem_ld16_async(tmem + lane_base + C::DP_COL + sb * BK2 + 16 * hc, rp);
      tmem_wait_ld16(rs);
      tmem_wait_ld16(rp);
      const bool full = __all_sync(0xffffffffu, vis.sees_all(j0, j0 + BK2 - 1, a.L));
      uint32_t pk[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float d2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int cl = 2 * c + e, cc = 16 * hc + cl;
          float p = ex2(fmaf(__uint_as_float(rs[cl]), c2, nl));
          if (!full && !vis.sees(j0 + cc, a.L)) p = 0.f;
          d2[e] = p * (__uint_as_float(rp[cl]) - dlt);
        }
        pk[c] = pack_bf16(d2[0], d2[1]);
      }
      if (it >= 2 && !warp_wait(&dq_done[s], ((it - 2) >> 1) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tmem_st8(tmem + lane_base + C::DS_COL + s * 16 + 8 * hc, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[s]);
    }
    if (ok && it > 0 && !warp_wait(&dq_done[(it - 1) & 1], ((it - 1) >> 1) & 1, a.err, abort_flag)) ok = false;
    tc_fence_after();
    __nv_bfloat16* qrow = a.dq + ((int64_t)b * a.T2 + row) * otok + h * D;
#pragma unroll 1
    for (int c = hc * (D / 64); c < (hc + 1) * (D / 64); ++c) {  // this warp's half of the head dim
      uint32_t ro[32];
      if (ok && it > 0) {
        tmem_ld32_async(tmem + lane_base + C::DQ_COL + c * 32, ro);
        tmem_wait_ld(ro);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) ro[e] = 0u;
      }
      if (valid) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = pack_bf16(__uint_as_float(ro[2 * e]) * a.scale, __uint_as_float(ro[2 * e + 1]) * a.scale);
        uint4* dst = reinterpret_cast<uint4*>(qrow + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ================================================================== backward: dK, dV
// One CTA = 128 keys of one (batch, kv head) and one 128-column slice z of dK / dV (D 256 runs
// two CTAs per key tile); it loops over the query heads of the GQA group and their 32-row query
// tiles that may see the key tile (Q / dO ring of up to 4 stages):
//   S^T = K Q^T and dP^T = V dO^T (M 128 keys, N 32, K D) into double-buffered TMEM;
//   warps 0-3 (thread = key): P^T = 2^(S^T log2e scale - lse2[q]), dS^T = P^T (dP^T - Delta[q]),
//   both (bf16) stored into TMEM (tcgen05.st, double-buffered), where the gradient MMAs read them
//   as their A operand (so the smem holds K, V and a 3-stage Q / dO ring);
//   dV += P^T dO[:, z] and dK += dS^T Q[:, z] (M 128, N 128, K 32) in TMEM.
constexpr int BQ2 = 32;

template <int D>
struct KCfg {
  static constexpr int KV_BYTES = BQ * D * 2;   // K, then V: D/64 boxes of [128 rows][128 B]
  static constexpr int T_BYTES = BQ2 * D * 2;   // Q tile, then dO tile: D/64 boxes of [32 rows][128 B]
  static constexpr int STAGE = 2 * T_BYTES;
  static constexpr int NST_FIT = (227 * 1024 - 2 * KV_BYTES - 1024 - 256) / STAGE;
  static constexpr int NST = NST_FIT > 4 ? 4 : NST_FIT;  // Q / dO ring stages
  static constexpr int SMEM = 2 * KV_BYTES + NST * STAGE + 1024 + 256;
  // TMEM: S^T and dP^T (NS buffers of 32 columns each), the bf16 P^T / dS^T operands of the
  // gradient MMAs (two buffers of 16 packed columns each), dV and dK slices (128 columns each)
  static constexpr int NS = 3;
  // S^T / dP^T MMAs issued ahead (same rule as the dQ kernel)
  static constexpr int AHEAD_R = (NS - 1) < (NST - 2) ? (NS - 1) : (NST - 2);
  static constexpr int AHEAD = AHEAD_R < 1 ? 1 : AHEAD_R;
  static constexpr int ST_COL = 0, DPT_COL = NS * BQ2, PT_COL = 2 * NS * BQ2, DST_COL = PT_COL + BQ2,
                       DV_COL = 256, DK_COL = 384;
  static constexpr int TMEM_COLS = 512;
  static_assert(DST_COL + BQ2 <= DV_COL, "TMEM layout");
  static constexpr uint32_t IDESC_S = idesc_bf16(BQ, BQ2, 0, 0);
  static constexpr uint32_t IDESC_G = idesc_bf16(BQ, 128, 0, 1);
  static_assert(NST >= 2, "Q / dO ring needs two stages");
};

template <int D>
__global__ void __launch_bounds__(NTHR_K, 1)
    bwd_dkv_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mdo,
                      const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv, BArgs a) {
  using C = KCfg<D>;
  constexpr int NST = C::NST, NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + C::KV_BYTES;
  uint8_t* sT = smem + 2 * C::KV_BYTES;  // stage s: Q tile at sT + s * STAGE, dO tile + T_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(sT + NST * C::STAGE);
  uint64_t* kv_full = bars;
  uint64_t* t_full = bars + 1;
  uint64_t* t_empty = t_full + NST;
  uint64_t* st_full = t_empty + NST;
  uint64_t* pt_full = st_full + NS;
  uint64_t* g_done = pt_full + 2;
  uint64_t* drain = g_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // grid (B * Hk * D/128 slices, key tiles): clean-stream key tiles (the most work, decreasing
  // along the stream) first, each for every (batch, kv head, slice) before the next tile
  const int nkt = gridDim.y;
  const int kt = (blockIdx.y + nkt / 2) % nkt;
  const int j0 = kt * BQ, j1 = min(j0 + BQ - 1, a.T2 - 1);
  constexpr int NZ = D / 128;
  const int z = blockIdx.x % NZ;
  const int b = (blockIdx.x / NZ) / a.Hk, hk = (blockIdx.x / NZ) % a.Hk;
  const int rep = a.Hq / a.Hk;
  const Span2 sp = row_tiles(j0, j1, a.L, a.T2, a.block, a.leak, BQ2);  // query tiles that may see a key
  const int nqv = sp.n();
  const int total = rep * nqv;  // (query head, query tile) pairs, head-major
  const int row0 = b * a.T2;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&t_full[s], 1);
      mbar_init(&t_empty[s], 1);
    }
    for (int s = 0; s < NS; ++s) mbar_init(&st_full[s], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&pt_full[s], 8);  // the eight P^T / dS^T warps
      mbar_init(&g_done[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mq);
    prefetch_tmap(&mdo);
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

  if (warp == 8) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      mbar_arrive_expect_tx(kv_full, 2 * C::KV_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sK + c * BQ * 128, &mk, kv_full, hk * D + c * 64, row0 + j0);
        tma_load_2d(sV + c * BQ * 128, &mv, kv_full, hk * D + c * 64, row0 + j0);
      }
      int last[NST];
#pragma unroll
      for (int s = 0; s < NST; ++s) last[s] = -1;
      for (int it = 0; it < total; ++it) {
        const int s = it % NST;
        if (!mbar_wait(&t_empty[s], ((it / NST) & 1) ^ 1, a.err, ERR_ATTN_WAIT, abort_flag)) break;
        mbar_arrive_expect_tx(&t_full[s], C::STAGE);
        last[s] = it;
        const int hq = hk * rep + it / nqv, i0 = sp.at(it % nqv) * BQ2;
        uint8_t* dst = sT + s * C::STAGE;
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(dst + c * BQ2 * 128, &mq, &t_full[s], hq * D + c * 64, row0 + i0);
          tma_load_2d(dst + C::T_BYTES + c * BQ2 * 128, &mdo, &t_full[s], hq * D + c * 64, row0 + i0);
        }
      }
      mbar_wait(kv_full, 0, a.err, ERR_ATTN_WAIT, nullptr);
#pragma unroll
      for (int s = 0; s < NST; ++s)
        if (last[s] >= 0) mbar_wait(&t_full[s], (last[s] / NST) & 1, a.err, ERR_ATTN_WAIT, nullptr);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      bool ok = mbar_wait(kv_full, 0, a.err, ERR_ATTN_WAIT, abort_flag);
      tc_fence_after();
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      int issued = 0;  // S^T / dP^T MMA pairs issued; up to AHEAD ahead of the gradient MMAs being waited
      for (int it = 0; ok && it < total; ++it) {
        while (issued < total && issued <= it + C::AHEAD) {
          if (!mbar_wait(&t_full[issued % NST], (issued / NST) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sT + (issued % NST) * C::STAGE), do_addr = q_addr + C::T_BYTES;
          const int sb = issued % NS;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t okv = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
            const uint32_t ot = (kk >> 2) * (BQ2 * 128) + (kk & 3) * 32;
            mma_bf16(tmem + C::ST_COL + sb * BQ2, smem_desc(k_addr + okv, 16, 1024),
                     smem_desc(q_addr + ot, 16, 1024), C::IDESC_S, kk > 0 ? 1u : 0u);
            mma_bf16(tmem + C::DPT_COL + sb * BQ2, smem_desc(v_addr + okv, 16, 1024),
                     smem_desc(do_addr + ot, 16, 1024), C::IDESC_S, kk > 0 ? 1u : 0u);
          }
          mma_commit(&st_full[sb]);
          ++issued;
        }
        if (!ok) break;
        const int pb = it & 1;
        if (!mbar_wait(&pt_full[pb], (it >> 1) & 1, a.err, ERR_ATTN_WAIT, abort_flag)) break;
        tc_fence_after();
        const int s = it % NST;
        const uint32_t q_addr = smem_u32(sT + s * C::STAGE) + z * 2 * (BQ2 * 128);
        const uint32_t do_addr = smem_u32(sT + s * C::STAGE + C::T_BYTES) + z * 2 * (BQ2 * 128);
#pragma unroll
        for (int kk = 0; kk < BQ2 / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          mma_bf16_ta(tmem + C::DV_COL, tmem + C::PT_COL + pb * 16 + kk * 8,
                      smem_desc(do_addr + kk * 2048, BQ2 * 128, 1024), C::IDESC_G, acc);
          mma_bf16_ta(tmem + C::DK_COL, tmem + C::DST_COL + pb * 16 + kk * 8,
                      smem_desc(q_addr + kk * 2048, BQ2 * 128, 1024), C::IDESC_G, acc);
        }
        mma_commit(&g_done[pb]);
        mma_commit(&t_empty[s]);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, a.err, ERR_ATTN_WAIT, nullptr);
    }
  } else {
    // -------------------------------------------------------------- P^T, dS^T (warps 0-7)
    const int quad = warp & 3, hc = warp >> 2;  // TMEM lane quadrant, half of the 32 query columns
    const int r = quad * 32 + lane;
    const int key = j0 + r;
    const bool kvalid = key < a.T2;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const KeyVis kv = key_vis(key, a.L, a.T2, a.block, a.leak);
    const float c2 = a.scale_log2;
    int it = 0;
    bool ok = true;
    for (; it < total; ++it) {
      const int sb = it % NS, pb = it & 1;
      const int hq = hk * rep + it / nqv, i0 = sp.at(it % nqv) * BQ2;
      // lane c holds lse2 / Delta of query row i0 + c
      const int qr = i0 + lane;
      const int64_t hoff = ((int64_t)b * a.Hq + hq) * a.T2;
      float lse_l = qr < a.T2 ? a.lse2[hoff + qr] : INFINITY;
      if (lse_l == NEG_INF) lse_l = INFINITY;  // a row that sees nothing: every p is 0
      const float dl_l = qr < a.T2 ? a.delta[hoff + qr] : 0.f;
      if (!warp_wait(&st_full[sb], (it / NS) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t rs[16], rp[16];
      tmem_ld16_async(tmem + lane_base + C::ST_COL + sb * BQ2 + 16 * hc, rs);
      tmem_ld16_async(tmem + lane_base + C::DPT_COL + sb * BQ2 + 16 * hc, rp);
      tmem_wait_ld16(rs);
      tmem_wait_ld16(rp);
      const bool full = __all_sync(0xffffffffu, kv.seen_by_all(i0, i0 + BQ2 - 1, a.L, a.T2));
      uint32_t pp[8], pd[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float p2[2], d2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int cl = 2 * c + e, cc = 16 * hc + cl;  // column within the half / within the tile
          const float lq = __shfl_sync(0xffffffffu, lse_l, cc);
          const float dq = __shfl_sync(0xffffffffu, dl_l, cc);
          float p = ex2(fmaf(__uint_as_float(rs[cl]), c2, -lq));
          if (!full && !kv.seen_by(i0 + cc, a.L, a.T2)) p = 0.f;
          p2[e] = p;
          d2[e] = p * (__uint_as_float(rp[cl]) - dq);
        }
        pp[c] = pack_bf16(p2[0], p2[1]);
        pd[c] = pack_bf16(d2[0], d2[1]);
      }
      // the TMEM operand buffers pb were read by the gradient MMAs of iteration it-2
      if (it >= 2 && !warp_wait(&g_done[pb], ((it - 2) >> 1) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tmem_st8(tmem + lane_base + C::PT_COL + pb * 16 + 8 * hc, pp);
      tmem_st8(tmem + lane_base + C::DST_COL + pb * 16 + 8 * hc, pd);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pt_full[pb]);
    }
    if (ok && it > 0 && !warp_wait(&g_done[(it - 1) & 1], ((it - 1) >> 1) & 1, a.err, abort_flag)) ok = false;
    tc_fence_after();
    const int64_t ktok = (int64_t)a.Hk * D;
    __nv_bfloat16* krow = a.dk + ((int64_t)b * a.T2 + key) * ktok + hk * D + z * 128;
    __nv_bfloat16* vrow = a.dv + ((int64_t)b * a.T2 + key) * ktok + hk * D + z * 128;
#pragma unroll 1
    for (int g = 0; g < 2; ++g) {
      const uint32_t col = g == 0 ? C::DV_COL : C::DK_COL;
      const float mul = g == 0 ? 1.f : a.scale;
      __nv_bfloat16* dst_row = g == 0 ? vrow : krow;
#pragma unroll 1
      for (int c = 2 * hc; c < 2 * hc + 2; ++c) {  // this warp's 64 of the slice's 128 columns
        uint32_t ro[32];
        if (ok && it > 0) {
          tmem_ld32_async(tmem + lane_base + col + c * 32, ro);
          tmem_wait_ld(ro);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) ro[e] = 0u;
        }
        if (kvalid) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = pack_bf16(__uint_as_float(ro[2 * e]) * mul, __uint_as_float(ro[2 * e + 1]) * mul);
          uint4* dst = reinterpret_cast<uint4*>(dst_row + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
    }
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

template <int D, int BKV>
static void launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                   int64_t L, int64_t block, double scale, bool leak) {
  using C = FCfg<D, BKV>;
  const int B = q.size(0), T2 = q.size(1), Hq = q.size(2), Hk = k.size(2);
  Maps m;
  // [B*T2 rows, H*D cols] views with the tensors' token strides
  make_map_bf16(&m.q, q.data_ptr(), (uint64_t)Hq * D, (uint64_t)B * T2, q.stride(1), 64, BQ);
  make_map_bf16(&m.k, k.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, k.stride(1), 64, C::BKV);
  make_map_bf16(&m.v, v.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, v.stride(1), 64, C::BKV);
  FArgs a{};
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse2 = lse.data_ptr<float>();
  a.B = B, a.T2 = T2, a.L = (int)L, a.Hq = Hq, a.Hk = Hk, a.block = (int)block, a.leak = leak ? 1 : 0;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.err = error_word_ptr();
  auto kern = fwd_tc_kernel<D, BKV>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr = true;
  }
  const dim3 grid(B * Hq, (T2 + BQ - 1) / BQ);
  kern<<<grid, NTHR, C::SMEM, at::cuda::getCurrentCUDAStream()>>>(m.q, m.k, m.v, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int D>
static void launch_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                       const at::Tensor& o, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
                       at::Tensor& dv, int64_t L, int64_t block, double scale, bool leak) {
  const int B = q.size(0), T2 = q.size(1), Hq = q.size(2), Hk = k.size(2);
  BArgs a{};
  a.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.lse2 = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  a.B = B, a.T2 = T2, a.L = (int)L, a.Hq = Hq, a.Hk = Hk, a.block = (int)block, a.leak = leak ? 1 : 0;
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.err = error_word_ptr();
  const int64_t otok = (int64_t)Hq * D;
  auto st = at::cuda::getCurrentCUDAStream();
  {  // dQ (and Delta)
    using C = QCfg<D>;
    Maps m;
    alignas(64) CUtensorMap mdo_al;
    make_map_bf16(&m.q, q.data_ptr(), (uint64_t)Hq * D, (uint64_t)B * T2, q.stride(1), 64, BQ);
    make_map_bf16(&mdo_al, dout.data_ptr(), (uint64_t)Hq * D, (uint64_t)B * T2, otok, 64, BQ);
    make_map_bf16(&m.k, k.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, k.stride(1), 64, BK2);
    make_map_bf16(&m.v, v.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, v.stride(1), 64, BK2);
    auto kern = bwd_dq_tc_kernel<D>;
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      attr = true;
    }
    kern<<<dim3(B * Hq, (T2 + BQ - 1) / BQ), NTHR_K, C::SMEM, st>>>(m.q, mdo_al, m.k, m.v, a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  {  // dK, dV
    using C = KCfg<D>;
    Maps m;
    alignas(64) CUtensorMap mdo_al;
    make_map_bf16(&m.q, q.data_ptr(), (uint64_t)Hq * D, (uint64_t)B * T2, q.stride(1), 64, BQ2);
    make_map_bf16(&mdo_al, dout.data_ptr(), (uint64_t)Hq * D, (uint64_t)B * T2, otok, 64, BQ2);
    make_map_bf16(&m.k, k.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, k.stride(1), 64, BQ);
    make_map_bf16(&m.v, v.data_ptr(), (uint64_t)Hk * D, (uint64_t)B * T2, v.stride(1), 64, BQ);
    auto kern = bwd_dkv_tc_kernel<D>;
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      attr = true;
    }
    kern<<<dim3(B * Hk * (D / 128), (T2 + BQ - 1) / BQ), NTHR_K, C::SMEM, st>>>(m.q, mdo_al, m.k, m.v, a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

}  // namespace attn_tc

// tcgen05 forward for head dims 128 / 256 (returns false when the shape is not covered)
bool attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                 int64_t L, int64_t block, double scale, bool leak) {
  const int64_t D = q.size(3);
  if (D != 128 && D != 256) return false;
  bind_context(q.get_device());
  static int bkv = -1;  // 64-key tiles (measured faster); BDLLM_ATTN_BKV=32 selects 32-key tiles
  if (bkv < 0) {
    const char* e = getenv("BDLLM_ATTN_BKV");
    bkv = (e != nullptr && atoi(e) == 32) ? 32 : 64;
  }
  if (D == 128)
    bkv == 32 ? attn_tc::launch<128, 32>(q, k, v, o, lse, L, block, scale, leak)
              : attn_tc::launch<128, 64>(q, k, v, o, lse, L, block, scale, leak);
  else
    bkv == 32 ? attn_tc::launch<256, 32>(q, k, v, o, lse, L, block, scale, leak)
              : attn_tc::launch<256, 64>(q, k, v, o, lse, L, block, scale, leak);
  return true;
}

// tcgen05 backward (dQ with Delta, then dK / dV) for head dims 128 / 256; dout and o contiguous
bool attn_bwd_tc(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                 const at::Tensor& o, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq, at::Tensor& dk,
                 at::Tensor& dv, int64_t L, int64_t block, double scale, bool leak) {
  const int64_t D = q.size(3);
  if (D != 128 && D != 256) return false;
  bind_context(q.get_device());
  if (D == 128)
    attn_tc::launch_bwd<128>(dout, q, k, v, o, lse, delta, dq, dk, dv, L, block, scale, leak);
  else
    attn_tc::launch_bwd<256>(dout, q, k, v, o, lse, delta, dq, dk, dv, L, block, scale, leak);
  return true;
}

}  // namespace bdllm
