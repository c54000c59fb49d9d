// State-fork GDN backward, chunk kernel, on tcgen05 / TMEM with TMA-staged tiles (head dim 128,
// chunk 32). Included by gdn.cu inside namespace bdllm::gdn: a drop-in for bwd_chunk_kernel<128,
// 128> for the fork layout in both modes (0: noised block, dV' = P^T dO; 1: clean chunk, dV' and
// dS_out from the reverse recurrence), used with the tensor-core recurrence, which adds the noised
// blocks' state gradients itself (so no dS_inj is stored here). The states come as bf16 S^T rows
// (the forward's S_in and the recurrence's dS_out, [v][k] per chunk) loaded by TMA; the dq, dk and
// dv rows of the chunk are staged in dead token tiles and written by TMA stores.
// (Reference: autograd through `src/dllm_qwen38/gdn.py:48-123`.)
//
// Per CTA = one chunk (32 tokens) of one v-head. Every product with a 128-wide operand (the state
// S, dS_out, or a feature dimension) runs as an M = 128 MMA with the feature dimension on the 128
// TMEM lanes and the 32 tokens as N: thread = feature row reads its row of 32 token values. The
// token x token products (k^k^T, q^k^T, dO V'^T, dV' R^T, dT T^T, T^T Z) run as M = 128 MMAs of
// which only lanes 0-31 are used (rows 32-127 of the A operand read whatever shared memory
// follows the tile: 4x the needed tensor work on 32 x 32 products, none of it waited on twice).
// Math, with R0 = V - diag(E) k^ S, R = diag(beta) R0, V' = T R (UT identities):
//   dR = T^T dV',  dV = diag(beta) dR,  dT = dV' R^T,  dA = strict_lower(-T^T dT T^T)
//   dq^ = diag(E) dO S^T + dPm k^                   (dP = dO V'^T, dPm = dP * Gam * incl)
//   dk^ = -diag(beta E) dR S^T + dPm^T q^ + diag(F) V' dS_out^T + (dKK + dKK^T) k^
//   dE = rowsum(q^S * dO) - beta rowsum(k^S * dR),  dF = rowsum(k^ dS_out * V'),  dEc = <S, dS_out>
//   dbeta = rowsum(dR * R0) + rowsum(dA * KK * Gam);  dKK = dA * beta_i * Gam
// Rounds (MMA batch -> bounded wait -> epilogue -> barrier):
//   R1  KK, QK (token x token); F1 = (k^S)^T, F2 = (q^S)^T [v x t]; F3 = (dO S^T)^T [k x t]
//   R2  V'^T = R^T T^T (A = R^T from TMEM); noised: dV'^T = dO^T P
//   R3  dR^T = dV'^T T; dP; clean: F6 = (V' dS_out^T)^T [k x t], F7 = (k^ dS_out)^T [v x t]
//   R4  dT; F4 = (dR S^T)^T; dQb = (dPm k^)^T; dKb = (dPm^T q^)^T
//   R5  Z = dT T^T     R6  dA' = T^T Z     R7  dKc = ((dKK + dKK^T) k^)^T
// Bounded waits as everywhere (ERR_GDN_WAIT); no multicast.

namespace btc {

// warps 0-7 features (warp w: TMEM lane quadrant w % 4, tokens [16 (w / 4), +16) of the chunk),
// warp 8 tokens, warp 9 control (TMA + MMA)
constexpr int NTH = 320;
constexpr int TOKW = 8;    // the token warp (reads TMEM lanes 0-31, where token x token products land)
constexpr int CTL = 288;   // the control thread
constexpr int TOK = 32 * 128 * 2;  // token tile [32 x 128] bf16, two [32][64] boxes (8 KB)
constexpr int TT = 4096;           // token x token tile [32 x 64] bf16 (32 columns used)
constexpr int ST = 128 * 128 * 2;  // state tile [128 x 128] bf16, two [128][64] boxes (32 KB)
struct L {
  // token tiles (order matters: a token tile used as a padded A operand needs 12 KB of shared memory
  // after each of its boxes)
  static constexpr int Q = 0, K = TOK, DO = 2 * TOK, V = 3 * TOK, VP = 4 * TOK, DV = 5 * TOK, R = 6 * TOK,
                       DR = 7 * TOK;
  static constexpr int TTB = 8 * TOK;  // token x token tiles
  static constexpr int T_ = TTB, TT_ = TTB + TT, PT = TTB + 2 * TT, DPM = TTB + 3 * TT, DPMT = TTB + 4 * TT,
                       DT = TTB + 5 * TT, ZT = TTB + 6 * TT, SYM = TTB + 7 * TT;
  static constexpr int S = TTB + 8 * TT;  // state tiles
  static constexpr int DS = S + ST;
  static constexpr int RED = DS + ST;         // fp32 [128][33] reduction buffer
  static constexpr int TB = RED + 128 * 33 * 4;   // fp32 [96][33]: KK rows, P rows, dKK rows (token warp)
  static constexpr int SC = TB + 96 * 33 * 4;     // fp32 scalars per token: gam, beta, E, F, rq, rk, dE, dF, ...
  static constexpr int PART = SC + 16 * 32 * 4;   // fp32 [3][4 warps][32]: per-warp partials of token sums
  static constexpr int BAR = PART + 3 * 128 * 4;
  static constexpr int BYTES = BAR + 128 + 1024;
};
static_assert(L::BYTES <= 227 * 1024, "gdn bwd tc smem");
// TMEM columns
constexpr uint32_t F1 = 0, F2 = 32, F3 = 64, KK = 96, QK = 128, VPT = 160, DVT = 192, RA = 224, DVA = 240,
                   DRT = 256, DP = 288, F6 = 320, F7 = 352, F4 = 384, DQB = 416, DKB = 448, DA = 480;
constexpr uint32_t DT_C = 160, Z_C = 192, DKC = 224;  // reuse after consumption
constexpr uint32_t ID_TT = idesc_bf16(128, 32, 0, 0);        // K-major A and B, N 32
constexpr uint32_t ID_A_MN = idesc_bf16(128, 32, 1, 0);      // A M-contiguous, B K-major, N 32

// element (r, c) of a [R x 128] tile held as two 128-byte-swizzled boxes [R][64]
template <int R>
__device__ __forceinline__ uint32_t off2(int r, int c) {
  return (uint32_t)((c >> 6) * (R * 128) + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + ((c & 7) << 1));
}
// element (r, c) of a token x token tile (one box [32][64])
__device__ __forceinline__ uint32_t off1(int r, int c) {
  return (uint32_t)(r * 128 + (((c >> 3) ^ (r & 7)) << 4) + ((c & 7) << 1));
}
__device__ __forceinline__ void put(uint8_t* base, uint32_t off, float x) {
  *reinterpret_cast<__nv_bfloat16*>(base + off) = __float2bfloat16_rn(x);
}
__device__ __forceinline__ float get(const uint8_t* base, uint32_t off) {
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(base + off));
}
// descriptors: token tile K-major (rows = M or N, K = 128 features)
__device__ __forceinline__ uint64_t d_tok_k(uint32_t a, int kk) { return smem_desc(a + (kk >> 2) * 4096 + (kk & 3) * 32, 16, 1024); }
// token tile as an M- or N-contiguous operand (features = M or N, K = 32 tokens)
__device__ __forceinline__ uint64_t d_tok_mn(uint32_t a, int kk) { return smem_desc(a + kk * 2048, 4096, 1024); }
// state tile K-major (M = k rows, K = v) / M-contiguous (M = v, K = k)
__device__ __forceinline__ uint64_t d_st_k(uint32_t a, int kk) { return smem_desc(a + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024); }
__device__ __forceinline__ uint64_t d_st_mn(uint32_t a, int kk) { return smem_desc(a + kk * 2048, 16384, 1024); }
// token x token tile K-major (rows = M or N, K = 32 columns) / M-contiguous (M = columns, K = rows)
__device__ __forceinline__ uint64_t d_tt_k(uint32_t a, int kk) { return smem_desc(a + kk * 32, 16, 1024); }
__device__ __forceinline__ uint64_t d_tt_mn(uint32_t a, int kk) { return smem_desc(a + kk * 2048, 4096, 1024); }

__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[32]) {
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
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// Half-width transpose-reduce: every lane holds 16 per-token values; after 31 shuffles lane l
// holds the sum over all 32 lanes of value l % 16.
__device__ __forceinline__ float fold16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], 16);
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = hi ? v[i] : v[i + o];
      const float keep = hi ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}
// Warp transpose-reduce: every lane holds 32 per-token values; after 31 shuffles lane l holds the
// sum over the warp's lanes of value l.
__device__ __forceinline__ float fold32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = hi ? v[i] : v[i + o];
      const float keep = hi ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}
__device__ __forceinline__ uint32_t pk2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void mma_s(uint32_t d, uint64_t ad, uint64_t bd, uint32_t id, uint32_t acc) {
  mma_bf16(d, ad, bd, id, acc);
}
__device__ __forceinline__ void mma_t(uint32_t d, uint32_t a_tmem, uint64_t bd, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(bd), "r"(id), "r"(acc)
      : "memory");
}

}  // namespace btc

__device__ __forceinline__ void tma_store_tile(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}

__global__ void __launch_bounds__(btc::NTH, 1)
    bwd_chunk_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                        const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
                        const __grid_constant__ CUtensorMap ms, const __grid_constant__ CUtensorMap mds,
                        const __grid_constant__ CUtensorMap mdq, const __grid_constant__ CUtensorMap mdk,
                        const __grid_constant__ CUtensorMap mdv, Args a, int mode, int* err) {
  using namespace btc;
  constexpr int D = 128, C = 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(sm + L::RED);
  float* tb = reinterpret_cast<float*>(sm + L::TB);  // rows 0-31 KK, 32-63 P, 64-95 dKK
  float* part = reinterpret_cast<float*>(sm + L::PART);  // [3][4][32]
  float* sc = reinterpret_cast<float*>(sm + L::SC);
  float *sgam = sc, *sbeta = sc + 32, *sE = sc + 64, *sF = sc + 96, *srq = sc + 128, *srk = sc + 160, *sdE = sc + 192,
        *sdF = sc + 224, *sdgam = sc + 256, *sdb = sc + 288, *sdEc = sc + 320;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* ld_bar = bars;      // TMA tiles landed
  uint64_t* mma_bar = bars + 1;  // one phase per round
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stream = mode == 0 ? 0 : 1;
  const int c = blockIdx.x, bh = blockIdx.y, b = bh / a.Hv, h = bh % a.Hv;
  const int hk = h / (a.Hv / a.Hk);
  const int64_t base = (((int64_t)b * a.nb + c) * a.Hv + h);
  const int64_t tok0 = (int64_t)b * 2 * a.L + (stream ? a.L : 0) + (int64_t)c * C;  // first token row
  const bool clean = mode == 1;
  mark(a, 0);

  if (threadIdx.x == 0) {
    mbar_init(ld_bar, 1);
    mbar_init(mma_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sb = smem_u32(sm);
  if (threadIdx.x == CTL) {  // TMA: raw q, k, v rows and dO of this chunk; S^T (and dS_out^T) tiles
    mbar_arrive_expect_tx(ld_bar, 4 * TOK + (clean ? 2 : 1) * ST);
    for (int x = 0; x < 2; ++x) {
      tma_load_2d(sm + L::Q + x * 4096, &mq, ld_bar, hk * D + x * 64, (int)tok0);
      tma_load_2d(sm + L::K + x * 4096, &mk, ld_bar, hk * D + x * 64, (int)tok0);
      tma_load_2d(sm + L::V + x * 4096, &mv, ld_bar, h * D + x * 64, (int)tok0);
      tma_load_2d(sm + L::DO + x * 4096, &mdo, ld_bar, h * D + x * 64, (int)tok0);
      tma_load_2d(sm + L::S + x * 16384, &ms, ld_bar, x * 64, (int)(base * D));
      if (clean) tma_load_2d(sm + L::DS + x * 16384, &mds, ld_bar, x * 64, (int)(base * D));
    }
  }
  // ---- gates (token warp): gam = cumsum g, beta, E, F
  if (warp == TOKW) {
    const int64_t t = tok0 + lane;
    float gv = a.g[t * a.Hv + h];
    const float bv = a.beta[t * a.Hv + h];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, gv, o);
      if (lane >= o) gv += y;
    }
    const float gl = __shfl_sync(0xffffffffu, gv, 31);
    sgam[lane] = gv, sbeta[lane] = bv, sE[lane] = __expf(gv), sF[lane] = __expf(gl - gv);
    sdE[lane] = 0.f, sdF[lane] = 0.f, sdgam[lane] = 0.f, sdb[lane] = 0.f;
  }
  bool ok = mbar_wait(ld_bar, 0, err, ERR_GDN_WAIT, abort_flag);
  ok = __syncthreads_and(ok);
  if (ok && clean && threadIdx.x < 128) {  // <S, dS_out> partial of row v = thread
    const int v = threadIdx.x;
    float dot = 0.f;
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
      const uint32_t o = (j >> 3) * 16384 + v * 128 + (((j & 7) ^ (v & 7)) << 4);
      const uint4 x = *reinterpret_cast<const uint4*>(sm + L::S + o), y = *reinterpret_cast<const uint4*>(sm + L::DS + o);
      const __nv_bfloat162* px = reinterpret_cast<const __nv_bfloat162*>(&x);
      const __nv_bfloat162* py = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fx = __bfloat1622float2(px[e]), fy = __bfloat1622float2(py[e]);
        dot += fx.x * fy.x + fx.y * fy.y;
      }
    }
    red[v * 33] = dot;
  }
  // <S, dS_out> and the l2 normalisation of q, k rows (threads 0-63: k rows 0-31 then q rows)
  if (ok && threadIdx.x < 64) {
    const int r = threadIdx.x & 31;
    const bool isq = threadIdx.x >= 32;
    uint8_t* tile = sm + (isq ? L::Q : L::K);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint4 u = *reinterpret_cast<const uint4*>(tile + (j >> 3) * 4096 + r * 128 + (((j & 7) ^ (r & 7)) << 4));
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p[e]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    const float rr = rsqrtf(ss + 1e-6f);
    const float mul = rr * (isq ? a.scale : 1.f);
    (isq ? srq : srk)[r] = rr;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      uint8_t* pp = tile + (j >> 3) * 4096 + r * 128 + (((j & 7) ^ (r & 7)) << 4);
      uint4 u = *reinterpret_cast<const uint4*>(pp);
      __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p[e]);
        p[e] = __floats2bfloat162_rn(f.x * mul, f.y * mul);
      }
      *reinterpret_cast<uint4*>(pp) = u;
    }
  }
  __syncthreads();
  if (ok && warp == TOKW && clean) {  // dEc = <S, dS_out>: sum the 128 row partials
    float s = 0.f;
    for (int k = lane; k < 128; k += 32) s += red[k * 33];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) sdEc[0] = s;
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  mark(a, 1);  // state tiles converted, q / k normalised, gates
  uint32_t rnd = 0;  // completed MMA rounds (mma_bar phase)
  auto round_wait = [&]() -> bool {
    bool w = mbar_wait(mma_bar, rnd & 1, err, ERR_GDN_WAIT, abort_flag);
    ++rnd;
    w = __syncthreads_and(w);
    tc_fence_after();
    return w;
  };
  auto round_end = [&]() {
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  const bool ctl = threadIdx.x == CTL;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
  const int f = (warp & 3) * 32 + lane;  // feature row of the feature warps
  const int q4 = warp & 3, hh = (warp >> 2) & 1, tb0 = 16 * hh;  // lane quadrant, token half

  // ================================================================ R1
  if (ok && ctl) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t acc = kk > 0;
      mma_s(tmem + KK, d_tok_k(sb + L::K, kk), d_tok_k(sb + L::K, kk), ID_TT, acc);
      mma_s(tmem + QK, d_tok_k(sb + L::Q, kk), d_tok_k(sb + L::K, kk), ID_TT, acc);
      mma_s(tmem + F1, d_st_k(sb + L::S, kk), d_tok_k(sb + L::K, kk), ID_TT, acc);
      mma_s(tmem + F2, d_st_k(sb + L::S, kk), d_tok_k(sb + L::Q, kk), ID_TT, acc);
      mma_s(tmem + F3, d_st_mn(sb + L::S, kk), d_tok_k(sb + L::DO, kk), ID_A_MN, acc);
    }
    mma_commit(mma_bar);
  }
  ok = ok && round_wait();
  float f1[16];  // (k^ S)^T row v of this thread, its 16 tokens (kept for dE)
  if (ok && warp < 8) {
    // R0^T = V^T - E * F1 (v = f); R = beta R0 -> tile and TMEM A; dE_a = sum_v F2 * dO
    float f2[16];
    ld16(tmem + lane_base + F1 + tb0, f1);
    ld16(tmem + lane_base + F2 + tb0, f2);
    uint32_t ra[8];
#pragma unroll
    for (int u = 0; u < 16; u += 2) {
      const int t = tb0 + u;
      const float r00 = get(sm + L::V, off2<32>(t, f)) - sE[t] * f1[u];
      const float r01 = get(sm + L::V, off2<32>(t + 1, f)) - sE[t + 1] * f1[u + 1];
      f2[u] *= get(sm + L::DO, off2<32>(t, f));
      f2[u + 1] *= get(sm + L::DO, off2<32>(t + 1, f));
      const float rb0 = sbeta[t] * r00, rb1 = sbeta[t + 1] * r01;
      put(sm + L::R, off2<32>(t, f), rb0);
      put(sm + L::R, off2<32>(t + 1, f), rb1);
      ra[u >> 1] = pk2(rb0, rb1);
    }
    st8(tmem + lane_base + RA + 8 * hh, ra);
    const float s0 = fold16(f2, lane);  // dE_a partial of token tb0 + lane % 16 over this warp's features
    if (lane < 16) part[q4 * 32 + tb0 + lane] = s0;
  }
  __syncthreads();
  if (ok && warp == TOKW) sdE[lane] = part[lane] + part[32 + lane] + part[64 + lane] + part[96 + lane];
  if (ok && warp == TOKW) {
    float kk[32], qk[32];
    ld32(tmem + KK, kk);
    ld32(tmem + QK, qk);
    const float gi = sgam[lane], bi = sbeta[lane];
    float* Arow = red + lane * 33;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float gm = __expf(gi - sgam[j]);
      Arow[j] = j < lane ? bi * kk[j] * gm : 0.f;
      const float p = j <= lane ? qk[j] * gm : 0.f;
      put(sm + L::PT, off1(j, lane), p);    // P^T[j][lane] = P[lane][j]
      tb[lane * 33 + j] = kk[j];         // KK row kept for dbeta / dgam
      tb[(32 + lane) * 33 + j] = p;      // P row kept for dgam
    }
    __syncwarp();
    // T = (I + A)^-1, lane = column
    float tc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float acc0 = (i == lane) ? 1.f : 0.f, acc1 = 0.f;
#pragma unroll
      for (int m = 0; m < i; m += 2) {
        acc0 -= red[i * 33 + m] * tc[m];
        if (m + 1 < i) acc1 -= red[i * 33 + m + 1] * tc[m + 1];
      }
      tc[i] = acc0 + acc1;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      put(sm + L::T_, off1(i, lane), tc[i]);   // T[i][lane]
      put(sm + L::TT_, off1(lane, i), tc[i]);  // T^T[lane][i]
    }
  }
  round_end();
  mark(a, 2);

  // ================================================================ R2
  if (ok && ctl) {
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      mma_t(tmem + VPT, tmem + RA + kk * 8, d_tt_k(sb + L::T_, kk), ID_TT, kk > 0);
      if (!clean) mma_s(tmem + DVT, d_tok_mn(sb + L::DO, kk), d_tt_k(sb + L::PT, kk), ID_A_MN, kk > 0);
    }
    mma_commit(mma_bar);
  }
  ok = ok && round_wait();
  if (ok && warp < 8) {
    float vp[16], dv[16];
    ld16(tmem + lane_base + VPT + tb0, vp);
    if (clean) {
      const float* g = a.dVp + base * C * D + (int64_t)tb0 * D + f;
#pragma unroll
      for (int u = 0; u < 16; ++u) dv[u] = g[u * D];
    } else {
      ld16(tmem + lane_base + DVT + tb0, dv);
    }
    uint32_t da[8];
#pragma unroll
    for (int u = 0; u < 16; u += 2) {
      const int t = tb0 + u;
      put(sm + L::VP, off2<32>(t, f), vp[u]);
      put(sm + L::VP, off2<32>(t + 1, f), vp[u + 1]);
      put(sm + L::DV, off2<32>(t, f), dv[u]);
      put(sm + L::DV, off2<32>(t + 1, f), dv[u + 1]);
      da[u >> 1] = pk2(dv[u], dv[u + 1]);
    }
    st8(tmem + lane_base + DVA + 8 * hh, da);
  }
  round_end();
  mark(a, 3);

  // ================================================================ R3
  if (ok && ctl) {
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) mma_t(tmem + DRT, tmem + DVA + kk * 8, d_tt_k(sb + L::TT_, kk), ID_TT, kk > 0);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t acc = kk > 0;
      mma_s(tmem + DP, d_tok_k(sb + L::DO, kk), d_tok_k(sb + L::VP, kk), ID_TT, acc);
      if (clean) {
        mma_s(tmem + F6, d_st_mn(sb + L::DS, kk), d_tok_k(sb + L::VP, kk), ID_A_MN, acc);
        mma_s(tmem + F7, d_st_k(sb + L::DS, kk), d_tok_k(sb + L::K, kk), ID_TT, acc);
      }
    }
    mma_commit(mma_bar);
  }
  ok = ok && round_wait();
  float dK[16];  // dk^ row k = f, this warp's 16 tokens (accumulated over the rounds), dQ likewise
  float dQ[16];
  if (ok && warp < 8) {
    float dr[16];
    ld16(tmem + lane_base + DRT + tb0, dr);
    float vp[16];
    ld16(tmem + lane_base + VPT + tb0, vp);  // V'^T row v (still in TMEM)
    // dv = beta dR (global), dR tile, -beta E dR tile (noised); per-token sums over the features:
    // dbeta_a = sum_v dR R0, dE_b = -beta sum_v F1 dR, dF = sum_v F7 V'
    // (dv is staged in the V' tile, whose last reader was this round's MMAs, and TMA-stored)
    float f7[16], pb[16];
    if (clean) ld16(tmem + lane_base + F7 + tb0, f7);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int t = tb0 + u;
      const float r0 = get(sm + L::V, off2<32>(t, f)) - sE[t] * f1[u];
      put(sm + L::VP, off2<32>(t, f), sbeta[t] * dr[u]);
      put(sm + L::DR, off2<32>(t, f), dr[u]);
      pb[u] = dr[u] * r0;
      f1[u] *= dr[u];
      f7[u] = clean ? f7[u] * vp[u] : 0.f;
    }
    {
      const float s0 = fold16(pb, lane), s1 = fold16(f1, lane), s2 = fold16(f7, lane);
      if (lane < 16) {
        part[q4 * 32 + tb0 + lane] = s0;
        part[128 + q4 * 32 + tb0 + lane] = s1;
        part[256 + q4 * 32 + tb0 + lane] = s2;
      }
    }
    // dK^T (row k = f): clean F * (V' dS_out^T)^T ; dQ^T = E * F3
    float f3[16];
    ld16(tmem + lane_base + F3 + tb0, f3);
    if (clean) {
      float f6[16];
      ld16(tmem + lane_base + F6 + tb0, f6);
#pragma unroll
      for (int u = 0; u < 16; ++u) dK[u] = sF[tb0 + u] * f6[u];
    } else {
#pragma unroll
      for (int u = 0; u < 16; ++u) dK[u] = 0.f;
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) dQ[u] = sE[tb0 + u] * f3[u];
    fence_proxy_async();  // the staged dv tile -> the TMA store below
  }
  // dP -> dPm = dP Gam incl (tile, and transposed), G1 = dP * P -> dgam, on the token and the
  // control warp (free after issuing this round): the token warp moves the dP rows out of TMEM
  // lanes 0-31, then warp 8 + w takes rows [16 w, 16 w + 16) with lane = column.
  float* dpr = red;                 // dP rows [32][33]
  float* g1sum = red + 32 * 33;     // row sums of G1 [32], then the two column partials [2][32]
  if (ok && warp == TOKW) {
    float dp[32];
    ld32(tmem + DP, dp);
#pragma unroll
    for (int j = 0; j < 32; ++j) dpr[lane * 33 + j] = dp[j];
  }
  if (ok && warp >= TOKW) {
    asm volatile("bar.sync 2, 64;" ::: "memory");  // warps 8 and 9
    const int j = lane, w = warp - TOKW;
    const float gj = sgam[j];
    float cs = 0.f;
#pragma unroll 4
    for (int r = 0; r < 16; ++r) {
      const int i = 16 * w + r;
      const float dpv = dpr[i * 33 + j];
      const float x = j <= i ? dpv * __expf(sgam[i] - gj) : 0.f;
      put(sm + L::DPM, off1(i, j), x);
      put(sm + L::DPMT, off1(j, i), x);
      const float g1 = dpv * tb[(32 + i) * 33 + j];
      float rs = g1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
      if (lane == 0) g1sum[i] = rs;
      cs += g1;
    }
    g1sum[32 + 32 * w + j] = cs;
    asm volatile("bar.sync 2, 64;" ::: "memory");
    if (w == 0) sdgam[j] += g1sum[j] - (g1sum[32 + j] + g1sum[64 + j]);  // row total - column total
  }
  __syncthreads();
  if (ok && ctl) {  // dv rows of this chunk: two [32][64] boxes
    tma_store_tile(&mdv, sm + L::VP, h * D, (int)tok0);
    tma_store_tile(&mdv, sm + L::VP + 4096, h * D + 64, (int)tok0);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  if (ok && warp == TOKW) {  // combine the four lane quadrants' partials
    float sb_ = 0.f, se = 0.f, sf = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      sb_ += part[w * 32 + lane];
      se += part[128 + w * 32 + lane];
      sf += part[256 + w * 32 + lane];
    }
    sdb[lane] += sb_;
    sdE[lane] -= sbeta[lane] * se;
    sdF[lane] = sf;
  }
  round_end();
  mark(a, 4);

  // ================================================================ R4
  if (ok && ctl) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t acc = kk > 0;
      mma_s(tmem + DT_C, d_tok_k(sb + L::DV, kk), d_tok_k(sb + L::R, kk), ID_TT, acc);
      mma_s(tmem + F4, d_st_mn(sb + L::S, kk), d_tok_k(sb + L::DR, kk), ID_A_MN, acc);
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      mma_s(tmem + DQB, d_tok_mn(sb + L::K, kk), d_tt_k(sb + L::DPM, kk), ID_A_MN, kk > 0);
      mma_s(tmem + DKB, d_tok_mn(sb + L::Q, kk), d_tt_k(sb + L::DPMT, kk), ID_A_MN, kk > 0);
    }
    mma_commit(mma_bar);
  }
  ok = ok && round_wait();
  if (ok && warp < 8) {
    float x[16];
    ld16(tmem + lane_base + F4 + tb0, x);
#pragma unroll
    for (int u = 0; u < 16; ++u) dK[u] -= sbeta[tb0 + u] * sE[tb0 + u] * x[u];
    ld16(tmem + lane_base + DQB + tb0, x);
#pragma unroll
    for (int u = 0; u < 16; ++u) dQ[u] += x[u];
    ld16(tmem + lane_base + DKB + tb0, x);
#pragma unroll
    for (int u = 0; u < 16; ++u) dK[u] += x[u];
  }
  if (ok && warp == TOKW) {  // dT -> tile (A operand of Z = dT T^T)
    float dt[32];
    ld32(tmem + DT_C, dt);
#pragma unroll
    for (int j = 0; j < 32; ++j) put(sm + L::DT, off1(lane, j), dt[j]);  // dT = dV' R^T (R = beta R0)
  }
  round_end();
  mark(a, 5);

  // ================================================================ R5: Z = dT T^T
  if (ok && ctl) {
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) mma_s(tmem + Z_C, d_tt_k(sb + L::DT, kk), d_tt_k(sb + L::T_, kk), ID_TT, kk > 0);
    mma_commit(mma_bar);
  }
  ok = ok && round_wait();
  if (ok && warp == TOKW) {
    float z[32];
    ld32(tmem + Z_C, z);
#pragma unroll
    for (int j = 0; j < 32; ++j) put(sm + L::ZT, off1(j, lane), z[j]);  // Z^T[j][lane] = Z[lane][j]
  }
  round_end();
  mark(a, 6);

  // ================================================================ R6: dA' = T^T Z
  if (ok && ctl) {
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) mma_s(tmem + DA, d_tt_mn(sb + L::T_, kk), d_tt_k(sb + L::ZT, kk), ID_A_MN, kk > 0);
    mma_commit(mma_bar);
  }
  ok = ok && round_wait();
  // dA = strict_lower(-dA'); dKK = dA beta_i Gam; H2 = dA beta KK Gam -> dgam, dbeta; sym tile.
  // Spread over the four feature warps (idle in this round): warp 0 moves the dA' rows out of
  // TMEM lanes 0-31, then warp w takes rows [8 w, 8 w + 8) with lane = column.
  if (ok && warp == 0) {
    float da[32];
    ld32(tmem + DA, da);
#pragma unroll
    for (int j = 0; j < 32; ++j) red[lane * 33 + j] = da[j];
  }
  if (ok && warp < 4) {
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four feature warps
    const int j = lane;
    const float gj = sgam[j];
    float csH = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int i = 8 * warp + r;
      const float gm = j < i ? __expf(sgam[i] - gj) : 0.f;
      const float dA = j < i ? -red[i * 33 + j] : 0.f;
      const float kkv = tb[i * 33 + j];
      const float dkk = dA * sbeta[i] * gm;
      const float h2 = dkk * kkv;
      float rb = dA * kkv * gm, rh = h2;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        rb += __shfl_xor_sync(0xffffffffu, rb, o);
        rh += __shfl_xor_sync(0xffffffffu, rh, o);
      }
      if (lane == 0) part[128 + i] = rh, part[160 + i] = rb;  // row sums of H2 and dA KK Gam
      csH += h2;
      tb[(64 + i) * 33 + j] = dkk;
    }
    part[warp * 32 + j] = csH;  // column partial of H2 over this warp's rows
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (warp == 0) {
      const float cs = part[j] + part[32 + j] + part[64 + j] + part[96 + j];
      sdgam[j] += part[128 + j] - cs;
      sdb[j] += part[160 + j];
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {  // sym = dKK + dKK^T
      const int i = 8 * warp + r;
      put(sm + L::SYM, off1(i, j), tb[(64 + i) * 33 + j] + tb[(64 + j) * 33 + i]);
    }
  }
  round_end();
  mark(a, 7);

  // ================================================================ R7: dKc = (sym k^)^T
  if (ok && ctl) {
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) mma_s(tmem + DKC, d_tok_mn(sb + L::K, kk), d_tt_k(sb + L::SYM, kk), ID_A_MN, kk > 0);
    mma_commit(mma_bar);
  }
  ok = ok && round_wait();
  mark(a, 8);  // R7 MMA
  if (ok && warp < 8) {
    float x[16];
    ld16(tmem + lane_base + DKC + tb0, x);
#pragma unroll
    for (int u = 0; u < 16; ++u) dK[u] += x[u];
    // l2norm backward needs per-token dots <k^, dk^> and <q^, dq^> over the 128 features
    float xk[16], xq[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      xk[u] = get(sm + L::K, off2<32>(tb0 + u, f)) * dK[u];
      xq[u] = get(sm + L::Q, off2<32>(tb0 + u, f)) * dQ[u];
    }
    const float s0 = fold16(xk, lane), s1 = fold16(xq, lane);
    if (lane < 16) {
      part[q4 * 32 + tb0 + lane] = s0;
      part[128 + q4 * 32 + tb0 + lane] = s1;
    }
  }
  __syncthreads();
  if (ok && warp == TOKW) {
    sc[352 + lane] = part[lane] + part[32 + lane] + part[64 + lane] + part[96 + lane];  // <k^, dk^>
    sc[384 + lane] = part[128 + lane] + part[160 + lane] + part[192 + lane] + part[224 + lane];  // <q^, dq^>
  }
  __syncthreads();
  mark(a, 9);  // R7 and the l2 folds
  if (ok && warp < 8) {
    // dk = rk (dk^ - k^ <k^, dk^>); dq = rq scale (dq^ - q^n <q^n, dq^>) with q^ = q^n scale,
    // staged in the V and dO tiles (no reader left) and TMA-stored
    const float inv_s2 = 1.f / (a.scale * a.scale);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int t = tb0 + u;
      const float kn = get(sm + L::K, off2<32>(t, f));
      const float qh = get(sm + L::Q, off2<32>(t, f));
      put(sm + L::V, off2<32>(t, f), srk[t] * (dK[u] - kn * sc[352 + t]));
      // q^ = s qn: dq = r (s dq^ - qn <qn, s dq^>) = r s (dq^ - q^ <q^, dq^> / s^2)
      put(sm + L::DO, off2<32>(t, f), srq[t] * a.scale * (dQ[u] - qh * sc[384 + t] * inv_s2));
    }
    fence_proxy_async();
  }
  if (ok && warp == TOKW) {
    // gates: dgam += dE E - dF F; last += sum dF F + dEc Ec; dg = reverse cumsum; dbeta
    const int i = lane;
    float dgi = sdgam[i] + sdE[i] * sE[i] - sdF[i] * sF[i];
    float fsum = sdF[i] * sF[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) fsum += __shfl_xor_sync(0xffffffffu, fsum, o);
    if (i == 31) dgi += fsum + (clean ? sdEc[0] * sE[31] : 0.f);
    float v = dgi;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_down_sync(0xffffffffu, v, o);
      if (i + o < 32) v += y;
    }
    const int64_t t = tok0 + i;
    a.dg[t * a.Hv + h] = v;
    a.dbeta[t * a.Hv + h] = sdb[i];
  }
  __syncthreads();
  if (ctl) {
    if (ok) {
      tma_store_tile(&mdk, sm + L::V, h * D, (int)tok0);
      tma_store_tile(&mdk, sm + L::V + 4096, h * D + 64, (int)tok0);
      tma_store_tile(&mdq, sm + L::DO, h * D, (int)tok0);
      tma_store_tile(&mdq, sm + L::DO + 4096, h * D + 64, (int)tok0);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the staged tiles have been read
  }
  mark(a, 10);
  mark(a, 11);
  tc_fence_before();
  __syncthreads();
  mark(a, 12);
  if (warp == 0) tmem_dealloc(tmem, 512);
}
