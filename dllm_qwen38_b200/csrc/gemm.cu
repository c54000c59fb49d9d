// Persistent warp-specialised bf16 GEMM for sm_100a: TMA -> shared memory -> tcgen05.mma with
// the fp32 accumulator in TMEM -> tcgen05.ld epilogue with fused element-wise ops.
// (Reference: nn.Linear / cuBLAS for every projection, `src/dllm_qwen38/gdn.py:212-215,233`,
// `blockdiff.py:179-187`, and the masked-row lm_head, `objective.py:79-84`.)
//
//   C[m, n] = sum_k A(m, k) * B(n, k)
//
// Operands are either K-major (A stored [M, K], B stored [N, K]) or MN-major (A stored [K, M],
// B stored [K, N]); that covers y = x W^T (K,K), dx = dy W (K,MN) and dW = dy^T x (MN,MN)
// without transposing anything in memory.
//
// CTA = 6 warps: warp 0 issues TMA loads, warp 1 allocates TMEM and issues MMAs (one elected
// lane), warps 2..5 drain TMEM (warp w owns TMEM lanes 32*(w%4)..+31). Tiles 128 x BN x 64,
// STAGES-deep smem ring, two TMEM accumulators so the epilogue of tile i overlaps the MMAs of
// tile i+1. One CTA per SM, grid = min(#tiles, #SMs), grouped tile raster for L2 reuse.
// Every TMA load copies into the issuing CTA only.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <string>
#include <tuple>
#include <vector>

#include "common.cuh"

namespace bdllm {

enum Epi : int {
  EPI_BF16 = 0,      // C (bf16) = acc
  EPI_F32 = 1,       // C (fp32) = acc
  EPI_ADD_BF16 = 2,  // C (bf16) = acc + R (bf16; R may alias C)
  EPI_ACC_F32 = 3,   // C (fp32) += acc
  EPI_SWIGLU = 4,    // B rows [j, F + j] interleaved per tile; C = silu(gate) * up, optional GU store
  EPI_PEER_F32 = 5,  // tensor parallel: fp32 partial rows stored into the owner rank's slot (peer memory)
};

// Tensor-parallel hooks (peer memory; see csrc/tp.cu for the other half of each collective).
// Counters in `ctr` (this rank's device memory): sequence numbers advanced on the device so that
// a captured CUDA graph replays with fresh values.
enum TpCtr : int { CTR_RS = 0, CTR_RS_ARRIVE = 1, CTR_AGC = 2, CTR_AGC_ARRIVE = 3 };
enum TpSlot : int { TP_SLOT_RS = 8, TP_SLOT_AG = 9, TP_SLOT_CONF = 10 };
constexpr int TP_MAX = 8;

constexpr int BM = 128;
constexpr int BK = 64;
// warps 0..5 as described above; warps 6..7 copy the weight shards from the peers in the fused
// all-gather variant (idle otherwise)
constexpr int NUM_THREADS = 256;

struct GemmArgs {
  int M, N, K;       // N = output columns (for SWIGLU: F, the activation width)
  void* C;           // output
  int ldc;           // elements
  const void* R;     // residual (EPI_ADD_BF16)
  int ldr;
  __nv_bfloat16* GU;  // SWIGLU: optional [M, 2F] store of (gate | up)
  int ldgu;
  int* err;     // device error word
  float alpha;  // accumulator scale applied before the epilogue op
  // tensor parallel (EPI_PEER_F32 and/or wait_ag)
  int64_t peers[TP_MAX];  // symmetric heap bases of the TP ranks
  int world, rank;
  int rows_per_rank;      // EPI_PEER_F32: output row r belongs to rank r / rows_per_rank
  int64_t part_off;       // EPI_PEER_F32: byte offset of the owners' fp32 partial slots [world][rows][ldc]
  int64_t flag_off;       // byte offset of the flag rows (u32 [16 slots][16 ranks]) in every heap
  unsigned* ctr;          // this rank's TP counters
  int wait_ag;            // the producer waits until every rank pushed the gathered A rows
  uint64_t timeout_ns;
  // split-K (EPI_F32 only): work item = (tile, split); split s covers k-blocks [s*kbs, (s+1)*kbs)
  // and writes its fp32 partial at C + s * split_stride
  int ksplit, kbs;
  int64_t split_stride;
  // fused FSDP all-gather (ag_nchunks > 0): the B operand lives in `ag_dst`, the gathered buffer of a
  // unit whose rank-p shard is at peers[p] + ag_src_off (ag_shard_bytes each). Warps 6-7 of every
  // CTA claim 16-byte-aligned chunks of ag_chunk bytes (chunk k = shard k / cps, piece k % cps) in
  // priority order starting at ag_first, copy them from the owning peer and publish ready[k] = seq;
  // the TMA producer waits for the chunks under each B tile before loading it.
  int ag_nchunks, ag_first, ag_world, ag_rank;  // ag_nchunks: chunks this launch copies, from ag_first
  int64_t ag_src_off, ag_shard_bytes, ag_chunk, ag_b_off;
  char* ag_dst;
  unsigned* ag_ready;
  unsigned* ag_claim;
  unsigned ag_seq, ag_epoch;
  // tile raster: groups of raster_g tile rows along M (raster_n = 0) or tile columns along N
  // (raster_n = 1); 0 = 8 along M
  int raster_g, raster_n;
  const float* alpha_dev;  // optional device scalar multiplying alpha (read once per tile)
};

__device__ __forceinline__ void tp_st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned tp_ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned* tp_flag(int64_t base, int64_t flag_off, int slot, int src) {
  return reinterpret_cast<unsigned*>(base + flag_off) + slot * 16 + src;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
struct Cfg {
  static constexpr int BN_OUT = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr uint32_t IDESC = idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
};

// Tile t -> (tm, tn). Tiles run in groups of G tile rows (or, along N, G tile columns); within a
// group the short side varies fastest, so the CTAs resident at one time share the group's
// operand tiles through L2 and the other operand streams once per group.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int G, int along_n, int& tm, int& tn) {
  if (G <= 0) G = 8;
  if (!along_n) {
    const int group_size = G * tiles_n;
    const int first_m = (t / group_size) * G;
    const int rows = min(G, tiles_m - first_m);
    const int r = t % group_size;
    tm = first_m + r % rows;
    tn = r / rows;
  } else {
    const int group_size = G * tiles_m;
    const int first_n = (t / group_size) * G;
    const int cols = min(G, tiles_n - first_n);
    const int r = t % group_size;
    tn = first_n + r % cols;
    tm = r / cols;
  }
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// fused all-gather, copy side (one warp): wait for the peers' parameter epoch, then claim and copy
// chunks until none is left
__device__ void ag_copy_warp(const GemmArgs& a, int lane, volatile int* abort_flag) {
  int ok = 1;
  if (lane == 0) {
    const uint64_t t0 = globaltimer();
    for (int p = 0; p < a.ag_world && ok; ++p) {
      const unsigned* f = reinterpret_cast<const unsigned*>(a.peers[a.ag_rank] + a.flag_off) + p;  // slot 0: epoch
      while (static_cast<int>(tp_ld_acquire(f) - a.ag_epoch) < 0) {
        if (globaltimer() - t0 > a.timeout_ns || *abort_flag) {
          record_error(a.err, ERR_COMM_WAIT);
          *abort_flag = 1;
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return;
  const int64_t cps = (a.ag_shard_bytes + a.ag_chunk - 1) / a.ag_chunk;
  for (;;) {
    unsigned c = 0;
    if (lane == 0) c = atomicAdd(a.ag_claim, 1u);
    c = __shfl_sync(0xffffffffu, c, 0);
    if (c >= (unsigned)a.ag_nchunks || *abort_flag) break;
    const int64_t k = a.ag_first + (int64_t)c;
    const int p = (int)(k / cps);
    const int64_t lo = (k % cps) * a.ag_chunk, n = min(a.ag_chunk, a.ag_shard_bytes - lo);
    const char* src = reinterpret_cast<const char*>(a.peers[p] + a.ag_src_off) + lo;
    char* dst = a.ag_dst + (int64_t)p * a.ag_shard_bytes + lo;
    constexpr int U = 8;
    for (int64_t o = (int64_t)lane * 16; o < n; o += 32 * 16 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (o + u * 512 < n) v[u] = __ldcg(reinterpret_cast<const uint4*>(src + o + u * 512));
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (o + u * 512 < n) *reinterpret_cast<uint4*>(dst + o + u * 512) = v[u];
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");  // our generic stores -> later TMA reads
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release_gpu(a.ag_ready + k, a.ag_seq);
  }
}

// fused all-gather, consumer side (TMA producer thread): wait until every chunk overlapping the
// gathered-buffer byte range [lo, hi) is published
__device__ bool ag_wait_range(const GemmArgs& a, int64_t lo, int64_t hi, volatile int* abort_flag) {
  const int64_t cps = (a.ag_shard_bytes + a.ag_chunk - 1) / a.ag_chunk;
  auto chunk_of = [&](int64_t x) { return (x / a.ag_shard_bytes) * cps + (x % a.ag_shard_bytes) / a.ag_chunk; };
  const int64_t k0 = chunk_of(lo), k1 = chunk_of(hi - 1);
  const uint64_t t0 = globaltimer();
  for (int64_t k = k0; k <= k1; ++k) {
    while (static_cast<int>(ld_acquire_gpu(a.ag_ready + k) - a.ag_seq) < 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > a.timeout_ns) {
        record_error(a.err, ERR_COMM_WAIT);
        *abort_flag = 1;
        return false;
      }
      __nanosleep(32);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// Epilogue of one accumulator tile for the thread's row: TMEM columns -> the epilogue op -> global.
// t_row: this warp's TMEM lane quadrant at the accumulator's first column; n0: first output
// column; split_off / t / mn_tiles / ksplit: the k-split bookkeeping of the tile.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& args, uint32_t t_row, int row, bool row_ok, int n0,
                                              int64_t split_off, int t, int mn_tiles, int ksplit, int lane) {
  constexpr int BN_OUT = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  (void)lane;
  const float alpha = args.alpha_dev != nullptr ? args.alpha * __ldg(args.alpha_dev) : args.alpha;
#pragma unroll 1
  for (int c = 0; c < BN_OUT / 32; ++c) {
    float v[32];
    tmem_ld32(t_row + c * 32, v);
    if (alpha != 1.f) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= alpha;
    }
    const int col0 = n0 + c * 32;
    if (row_ok) (void)BDLLM_CHECK(all_finite(v, 32), row, col0);  // sentinel: non-finite accumulator
    if constexpr (EPI == EPI_SWIGLU) {
      float u[32];
      tmem_ld32(t_row + BN / 2 + c * 32, u);
      if (row_ok) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + col0;
        __nv_bfloat16* gu = args.GU ? args.GU + (size_t)row * args.ldgu + col0 : nullptr;
        if (col0 + 32 <= args.N && BDLLM_CHECK(((uintptr_t)out & 15) == 0, row, col0)) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk, pg, pu;
            __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
            __nv_bfloat162* g2 = reinterpret_cast<__nv_bfloat162*>(&pg);
            __nv_bfloat162* u2 = reinterpret_cast<__nv_bfloat162*>(&pu);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // the activation uses the bf16-rounded gate/up so that backward (which reads the
              // stored bf16 gate/up) differentiates exactly the function forward computed
              __nv_bfloat162 gb = __floats2bfloat162_rn(v[j + 2 * e], v[j + 2 * e + 1]);
              __nv_bfloat162 ub = __floats2bfloat162_rn(u[j + 2 * e], u[j + 2 * e + 1]);
              float2 gf = __bfloat1622float2(gb), uf = __bfloat1622float2(ub);
              p2[e] = __floats2bfloat162_rn(silu_f(gf.x) * uf.x, silu_f(gf.y) * uf.y);
              g2[e] = gb;
              u2[e] = ub;
            }
            *reinterpret_cast<uint4*>(out + j) = pk;
            if (gu) {
              *reinterpret_cast<uint4*>(gu + j) = pg;
              *reinterpret_cast<uint4*>(gu + args.N + j) = pu;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (col0 + j < args.N) {
              float g = __bfloat162float(__float2bfloat16(v[j])), uu = __bfloat162float(__float2bfloat16(u[j]));
              out[j] = __float2bfloat16(silu_f(g) * uu);
              if (gu) {
                gu[j] = __float2bfloat16(g);
                gu[args.N + j] = __float2bfloat16(uu);
              }
            }
          }
        }
      }
    } else if constexpr (EPI == EPI_PEER_F32) {
      // lane = row: 16-byte stores of this row's 32 columns into the owner's slot (a transposed,
      // row-contiguous variant measured slower over NVLink)
      if (row_ok) {
        const int owner = row / args.rows_per_rank, lr = row - owner * args.rows_per_rank;
        const int64_t slot = (int64_t)args.rank * ksplit + t / mn_tiles;  // [src rank][k split]
        float* out = reinterpret_cast<float*>(args.peers[owner] + args.part_off) +
                     (slot * args.rows_per_rank + lr) * args.ldc + col0;
        if (col0 + 32 <= args.N && BDLLM_CHECK(((uintptr_t)out & 15) == 0, row, col0)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(out + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < args.N) out[j] = v[j];
        }
      }
    } else if constexpr (EPI == EPI_F32 || EPI == EPI_ACC_F32) {
      if (row_ok) {
        float* out = reinterpret_cast<float*>(args.C) + split_off + (size_t)row * args.ldc + col0;
        if (col0 + 32 <= args.N && BDLLM_CHECK(((uintptr_t)out & 15) == 0, row, col0)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            if constexpr (EPI == EPI_ACC_F32) {
              float4 p = *reinterpret_cast<float4*>(out + j);
              o.x += p.x, o.y += p.y, o.z += p.z, o.w += p.w;
            }
            *reinterpret_cast<float4*>(out + j) = o;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < args.N) out[j] = (EPI == EPI_ACC_F32 ? out[j] : 0.f) + v[j];
        }
      }
    } else {  // EPI_BF16 / EPI_ADD_BF16
      if (row_ok) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + col0;
        const __nv_bfloat16* res =
            (EPI == EPI_ADD_BF16) ? reinterpret_cast<const __nv_bfloat16*>(args.R) + (size_t)row * args.ldr + col0
                                  : nullptr;
        if (col0 + 32 <= args.N && BDLLM_CHECK(((uintptr_t)out & 15) == 0, row, col0)) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
            if constexpr (EPI == EPI_ADD_BF16) {
              uint4 rr = *reinterpret_cast<const uint4*>(res + j);
              const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float2 rf = __bfloat1622float2(r2[e]);
                p2[e] = __floats2bfloat162_rn(v[j + 2 * e] + rf.x, v[j + 2 * e + 1] + rf.y);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(v[j + 2 * e], v[j + 2 * e + 1]);
            }
            *reinterpret_cast<uint4*>(out + j) = pk;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (col0 + j < args.N) {
              float r = (EPI == EPI_ADD_BF16) ? __bfloat162float(res[j]) : 0.f;
              out[j] = __float2bfloat16(v[j] + r);
            }
          }
        }
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, GemmArgs args) {
  using C_ = Cfg<BN, A_MN, B_MN, EPI>;
  constexpr int STAGES = C_::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * C_::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C_::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tiles_m = (args.M + BM - 1) / BM;
  const int tiles_n = (args.N + C_::BN_OUT - 1) / C_::BN_OUT;
  const int mn_tiles = tiles_m * tiles_n;
  const int ksplit = args.ksplit > 1 ? args.ksplit : 1;
  const int num_tiles = mn_tiles * ksplit;
  const int kblocks_all = (args.K + BK - 1) / BK;
  const int kbs = ksplit > 1 ? args.kbs : kblocks_all;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer
    int stage = 0;
    uint32_t round = 0;
    uint32_t armed_mask = 0;  // stages with a load in flight or landed (bit s)
    bool ok = true;
    if (args.wait_ag) {  // fused all-gather: A's rows are pushed by every rank; wait for all of them
      const unsigned target = args.ctr[CTR_AGC] + 1u;
      const uint64_t t0 = globaltimer();
      for (int p = 0; p < args.world && ok; ++p) {
        const unsigned* f = tp_flag(args.peers[args.rank], args.flag_off, TP_SLOT_AG, p);
        while (static_cast<int>(tp_ld_acquire(f) - target) < 0) {
          if (globaltimer() - t0 > args.timeout_ns || *reinterpret_cast<volatile int*>(args.err) != 0) {
            record_error(args.err, ERR_COMM_WAIT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          __nanosleep(64);
        }
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");  // peers' generic writes -> our TMA reads
    }
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      int tm, tn;
      tile_coords(t % mn_tiles, tiles_m, tiles_n, args.raster_g, args.raster_n, tm, tn);
      const int m0 = tm * BM, n0 = tn * C_::BN_OUT;
      const int kb0 = (t / mn_tiles) * kbs, kb1 = min(kblocks_all, kb0 + kbs);
      if constexpr (!B_MN) {
        if (args.ag_nchunks > 0) {  // the weight rows of this tile must have landed
          const int64_t rb = (int64_t)args.K * 2;
          const int rows = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
          const int n_rows = args.N;
          bool got = ag_wait_range(args, args.ag_b_off + n0 * rb, args.ag_b_off + min(n0 + rows, n_rows) * rb,
                                   abort_flag);
          if (got && EPI == EPI_SWIGLU)
            got = ag_wait_range(args, args.ag_b_off + (int64_t)(n_rows + n0) * rb,
                                args.ag_b_off + (int64_t)(n_rows + min(n0 + rows, n_rows)) * rb, abort_flag);
          if (!got) {
            ok = false;
            break;
          }
        }
      }
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], (round & 1) ^ 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], C_::STAGE_BYTES);
        armed_mask |= 1u << stage;
        const int k0 = kb * BK;
        uint8_t* a_dst = sa + stage * C_::A_BYTES;
        uint8_t* b_dst = sb + stage * C_::B_BYTES;
        if constexpr (!A_MN) {
          tma_load_2d(a_dst, &map_a, &full[stage], k0, m0);
        } else {
          tma_load_2d(a_dst, &map_a, &full[stage], m0, k0);
          tma_load_2d(a_dst + 8192, &map_a, &full[stage], m0 + 64, k0);
        }
        if constexpr (EPI == EPI_SWIGLU) {
          tma_load_2d(b_dst, &map_b, &full[stage], k0, n0);
          tma_load_2d(b_dst + (BN / 2) * 128, &map_b, &full[stage], k0, args.N + n0);
        } else if constexpr (!B_MN) {
          tma_load_2d(b_dst, &map_b, &full[stage], k0, n0);
        } else {
#pragma unroll
          for (int i = 0; i < BN / 64; ++i) tma_load_2d(b_dst + i * 8192, &map_b, &full[stage], n0 + i * 64, k0);
        }
        if (++stage == STAGES) {
          stage = 0;
          ++round;
        }
      }
    }
    if (!ok) {
      // drain: every load this thread armed must land before the CTA's smem is released. Stage s
      // was last armed in round (round - 1) if s >= stage, else in the current round.
      for (int s = 0; s < STAGES; ++s)
        if (armed_mask & (1u << s))
          mbar_wait(&full[s], (s < stage ? round : round - 1) & 1, args.err, ERR_GEMM_WAIT, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA issuer
    int stage = 0;
    uint32_t round = 0;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t use = it >> 1;
      if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      const int kb0 = (t / mn_tiles) * kbs, kb1 = min(kblocks_all, kb0 + kbs);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], round & 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sa + stage * C_::A_BYTES);
        const uint32_t b_addr = smem_u32(sb + stage * C_::B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          uint64_t ad, bd;
          if constexpr (!A_MN)
            ad = smem_desc(a_addr + k * 32, 16, 1024);
          else
            ad = smem_desc(a_addr + k * 2048, 8192, 1024);
          if constexpr (!B_MN || EPI == EPI_SWIGLU)
            bd = smem_desc(b_addr + k * 32, 16, 1024);
          else
            bd = smem_desc(b_addr + k * 2048, 8192, 1024);
          mma_bf16(d_tmem, ad, bd, C_::IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&empty[stage]);  // frees this smem stage once these MMAs have read it
        if (++stage == STAGES) {
          stage = 0;
          ++round;
        }
      }
      if (ok) mma_commit(&tfull[acc]);  // accumulator ready for the epilogue
    }
    if (!ok) {
      // aborted: wait (bounded) until every MMA already issued has finished reading smem and
      // writing TMEM, so the dealloc below never races an in-flight MMA
      mma_commit(drain);
      mbar_wait(drain, 0, args.err, ERR_GEMM_WAIT, nullptr);
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- fused all-gather copies
    if (args.ag_nchunks > 0) ag_copy_warp(args, lane, abort_flag);
  } else if (warp >= 2) {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t use = it >> 1;
      if (!mbar_wait(&tfull[acc], use & 1, args.err, ERR_GEMM_WAIT, abort_flag)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(t % mn_tiles, tiles_m, tiles_n, args.raster_g, args.raster_n, tm, tn);
      const int64_t split_off = (int64_t)(t / mn_tiles) * args.split_stride;
      const int row = tm * BM + row_in_tile;
      const int n0 = tn * C_::BN_OUT;
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      const bool row_ok = row < args.M;
      epilogue_tile<BN, EPI>(args, t_row, row, row_ok, n0, split_off, t, mn_tiles, ksplit, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  if constexpr (EPI == EPI_PEER_F32) __threadfence_system();  // this thread's peer stores
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::TMEM_COLS);
  }
  if ((EPI == EPI_PEER_F32 || args.wait_ag) && threadIdx.x == 0) {
    // the last CTA to finish advances the device counters and, for EPI_PEER_F32, tells every
    // owner that this rank's partial rows have landed
    __threadfence_system();
    const int arrive = EPI == EPI_PEER_F32 ? CTR_RS_ARRIVE : CTR_AGC_ARRIVE;
    const unsigned prev = atomicAdd(&args.ctr[arrive], 1u);
    if (prev == gridDim.x - 1) {
      args.ctr[arrive] = 0u;
      if (args.wait_ag) args.ctr[CTR_AGC] += 1u;
      if constexpr (EPI == EPI_PEER_F32) {
        const unsigned seq = args.ctr[CTR_RS] + 1u;
        args.ctr[CTR_RS] = seq;
        __threadfence_system();
        for (int p = 0; p < args.world; ++p)
          tp_st_release(tp_flag(args.peers[p], args.flag_off, TP_SLOT_RS, args.rank), seq);
      }
    }
  }
}

// ============================================================================== 2-CTA variant
// A CTA pair (cluster of 2, cta_group::2) computes 256 x NP tiles (NP = 256 or 512): CTA rank r
// of the pair loads A rows [m0 + 128 r, +128) into its own smem, and for each of the NP / 256
// MMAs h of a k step the B rows [n0 + 256 h + 128 r, +128) (for SwiGLU: rank 0 the gate rows,
// rank 1 the up rows of activation columns [n0 + 128 h, +128)). The leader (rank 0) issues
// M = 256, N = 256 MMAs that read both CTAs' tiles; each CTA's TMEM receives its 128 rows.
//   NP = 256: 32 KB per stage, 6 stages, two TMEM accumulators (the epilogue of one tile overlaps
//             the next tile's MMAs), 4 epilogue warps.
//   NP = 512: 48 KB per stage (A 16 KB + B 2 x 16 KB), 4 stages, one 512-column accumulator,
//             8 epilogue warps (warp 2 + e drains lane quadrant (2 + e) % 4 of MMA half e / 4).
//             Each SM streams 48 instead of 64 bytes per 4096 MACs, a quarter less L2 -> SM
//             traffic, which under the 1 kW power cap turns into clock. A last partial wave of
//             tiles is split into half-tiles (one MMA half each) so that the tail takes half as
//             long, and a tile whose second half lies beyond N skips it.
// Both CTAs' TMA loads complete on the leader's full barriers; the leader's MMA commits arrive on
// both CTAs' empty / tfull barriers; both CTAs' epilogue warps arrive on the leader's tempty
// barriers. Every wait is bounded as in gemm_kernel; all paths reach the final cluster barrier.
constexpr int STAGES2 = 6;
template <int EPI, bool A_MN, bool B_MN, int NP = 256>
struct Cfg2 {
  static_assert(NP == 256 || EPI == EPI_BF16 || EPI == EPI_ADD_BF16 || EPI == EPI_SWIGLU,
                "256 x 512 tiles: bf16 epilogues only");
  static constexpr int NH = NP / 256;                           // N = 256 MMAs per k step
  static constexpr int BN = 256;                                // MMA N (both CTAs' B halves)
  static constexpr int BN_OUT = (EPI == EPI_SWIGLU) ? NP / 2 : NP;  // output columns per tile
  static constexpr int HALF_OUT = BN_OUT / NH;                  // output columns per MMA half
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_HALF = 128 * BK * 2;                   // this CTA's rows of one MMA's B
  static constexpr int B_BYTES = NH * B_HALF;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int ST = (NP == 256) ? STAGES2 : 3;
  // NP = 512: one MMA half of the output (128 rows x 256 bf16 columns) staged for TMA stores, as
  // four 128-byte-swizzled blocks of 64 columns
  static constexpr int STAGING = (NP == 256) ? 0 : 128 * 256 * 2;
  static constexpr int SMEM = ST * STAGE_BYTES + STAGING + 1024 + 256;
  static constexpr int NACC = (NP == 256) ? 2 : 1;
  static constexpr int TMEM_COLS = 512;
  static constexpr int EPI_WARPS = 4 * NH;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS + 64;  // TMA, MMA, epilogue, 2 all-gather copy warps
  static constexpr uint32_t IDESC = idesc_bf16(256, 256, A_MN ? 1 : 0, B_MN ? 1 : 0);
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void commit2(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t leader_bar, int x,
                                                 int y) {
  if (!BDLLM_CHECK((x & 7) == 0, x, 8)) return;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// TMA store (or, with ADD, an element-wise bf16 add in L2) of a 2-D box from this CTA's smem
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  if (!BDLLM_CHECK((x & 7) == 0 && x >= 0 && y >= 0, x, 8)) return;
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  if (!BDLLM_CHECK((x & 7) == 0 && x >= 0 && y >= 0, x, 8)) return;
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void epi_bar_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Work unit u of the pair kernel -> tile (tm, tn) and the MMA halves [h0, h1) it computes. Units
// below `full` are whole tiles; the tiles of the last partial wave come as one unit per half.
// Returns false for a unit with nothing inside N (every role skips it alike).
template <class C_>
__device__ __forceinline__ bool pair_unit(int u, int full, int tiles_m, int tiles_n, const GemmArgs& args, int& t,
                                          int& tm, int& tn, int& h0, int& h1) {
  if (u < full) {
    t = u, h0 = 0, h1 = C_::NH;
  } else {
    const int v = u - full;
    t = full + v / C_::NH, h0 = v % C_::NH, h1 = h0 + 1;
  }
  tile_coords(t, tiles_m, tiles_n, args.raster_g, args.raster_n, tm, tn);
  const int left = args.N - tn * C_::BN_OUT;  // output columns of this tile inside N
  const int nvalid = min(C_::NH, (left + C_::HALF_OUT - 1) / C_::HALF_OUT);
  h1 = min(h1, nvalid);
  return h0 < h1;
}

template <int EPI, bool A_MN, bool B_MN, int NP>
__global__ void __launch_bounds__(Cfg2<EPI, A_MN, B_MN, NP>::THREADS, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_g,
                 const __grid_constant__ CUtensorMap map_u, GemmArgs args) {
  using C_ = Cfg2<EPI, A_MN, B_MN, NP>;
  constexpr int STAGES = C_::ST;
  constexpr bool WIDE = (NP == 512);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * C_::A_BYTES;
  uint8_t* stg = smem + STAGES * C_::STAGE_BYTES;  // output staging (wide tiles), 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(stg + C_::STAGING);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;  // per accumulator (256 x 256 tiles) or per MMA half (256 x 512)
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t crank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_m = (args.M + 255) / 256;
  const int tiles_n = (args.N + C_::BN_OUT - 1) / C_::BN_OUT;
  const int num_tiles = tiles_m * tiles_n;
  const int full_units = (C_::NH == 2) ? (num_tiles / npairs) * npairs : num_tiles;
  const int num_units = full_units + (num_tiles - full_units) * C_::NH;
  const int kblocks = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s2 = 0; s2 < STAGES; ++s2) {
      mbar_init(&full[s2], 1);
      mbar_init(&empty[s2], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * C_::EPI_WARPS);  // the epilogue warps of both CTAs of the pair
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
    if constexpr (WIDE) prefetch_tmap(&map_c);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C_::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full0 = map_to(smem_u32(full), 0);     // the leader's full barriers
  const uint32_t tempty0 = map_to(smem_u32(tempty), 0);  // the leader's tempty barriers

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    int stage = 0;
    uint32_t round = 0;
    uint32_t armed_mask = 0;
    bool ok = true;
    for (int u = pair; u < num_units && ok; u += npairs) {
      int t, tm, tn, h0, h1;
      if (!pair_unit<C_>(u, full_units, tiles_m, tiles_n, args, t, tm, tn, h0, h1)) continue;
      const int m0 = tm * 256 + (int)crank * 128;
      const int n0 = tn * C_::BN_OUT;
      // this CTA's B rows of MMA half h
      auto brow = [&](int h) {
        return (EPI == EPI_SWIGLU) ? (crank ? args.N : 0) + n0 + h * 128 : n0 + h * 256 + (int)crank * 128;
      };
      if constexpr (!B_MN) {
        if (args.ag_nchunks > 0) {  // fused all-gather: this CTA's weight rows must have landed
          const int64_t rb = (int64_t)args.K * 2;
          const int64_t rows_total = (EPI == EPI_SWIGLU) ? 2 * (int64_t)args.N : (int64_t)args.N;
          for (int h = h0; h < h1 && ok; ++h) {
            const int64_t r0 = brow(h), r1 = min(r0 + 128, rows_total);
            if (r1 > r0 && !ag_wait_range(args, args.ag_b_off + r0 * rb, args.ag_b_off + r1 * rb, abort_flag))
              ok = false;
          }
          if (!ok) break;
        }
      }
      const uint32_t tx = 2u * (uint32_t)(C_::A_BYTES + (h1 - h0) * C_::B_HALF);  // both CTAs' bytes
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&empty[stage], (round & 1) ^ 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        if (crank == 0) mbar_arrive_expect_tx(&full[stage], tx);
        armed_mask |= 1u << stage;
        const int k0 = kb * BK;
        const uint32_t bar = full0 + stage * 8;
        uint8_t* a_dst = sa + stage * C_::A_BYTES;
        uint8_t* b_dst = sb + stage * C_::B_BYTES;
        if constexpr (!A_MN) {
          tma_load_2d_pair(a_dst, &map_a, bar, k0, m0);
        } else {  // [K, M] operand: two 64-row (128-byte) swizzle atoms along M
          tma_load_2d_pair(a_dst, &map_a, bar, m0, k0);
          tma_load_2d_pair(a_dst + 8192, &map_a, bar, m0 + 64, k0);
        }
        for (int h = h0; h < h1; ++h) {
          uint8_t* bh = b_dst + h * C_::B_HALF;
          if constexpr (!B_MN) {
            tma_load_2d_pair(bh, &map_b, bar, k0, brow(h));
          } else {
            tma_load_2d_pair(bh, &map_b, bar, brow(h), k0);
            tma_load_2d_pair(bh + 8192, &map_b, bar, brow(h) + 64, k0);
          }
        }
        if (++stage == STAGES) {
          stage = 0;
          ++round;
        }
      }
    }
    if (!ok && crank == 0) {  // drain the leader's in-flight stages (bounded)
      for (int s2 = 0; s2 < STAGES; ++s2)
        if (armed_mask & (1u << s2))
          mbar_wait(&full[s2], (s2 < stage ? round : round - 1) & 1, args.err, ERR_GEMM_WAIT, nullptr);
    }
  } else if (warp == 1 && lane == 0 && crank == 0) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    int stage = 0;
    uint32_t round = 0;
    int it = 0;
    uint32_t hal_use0 = 0, hal_use1 = 0;  // wide tiles: units that used MMA half 0 / 1 so far
    bool ok = true;
    // the 4 k16 MMAs of one stage for MMA half h
    auto mma_stage = [&](int s2, int h, uint32_t d_tmem, bool first) {
      const uint32_t a_addr = smem_u32(sa + s2 * C_::A_BYTES);
      const uint32_t bh = smem_u32(sb + s2 * C_::B_BYTES) + h * C_::B_HALF;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        const uint64_t ad = A_MN ? smem_desc(a_addr + k * 2048, 8192, 1024) : smem_desc(a_addr + k * 32, 16, 1024);
        const uint64_t bd = B_MN ? smem_desc(bh + k * 2048, 8192, 1024) : smem_desc(bh + k * 32, 16, 1024);
        mma_bf16_pair(d_tmem + h * C_::BN, ad, bd, C_::IDESC, (!first || k > 0) ? 1u : 0u);
      }
    };
    auto free_stage = [&](int s2) {
      const uint32_t e = smem_u32(&empty[s2]);
      commit2(map_to(e, 0));  // frees this stage in both CTAs once the MMAs have read it
      commit2(map_to(e, 1));
    };
    for (int u = pair; u < num_units && ok; u += npairs) {
      int t, tm, tn, h0, h1;
      if (!pair_unit<C_>(u, full_units, tiles_m, tiles_n, args, t, tm, tn, h0, h1)) continue;
      const int acc = (C_::NACC == 2) ? (it & 1) : 0;
      const uint32_t use = (C_::NACC == 2) ? (uint32_t)(it >> 1) : (uint32_t)it;
      ++it;
      const uint32_t d_tmem = tmem_base + acc * C_::BN;
      int kb = 0;
      if constexpr (WIDE) {
        // Each MMA half is released by the epilogue on its own. A whole tile runs half 0 over the
        // first stages while half 1 of the previous tile drains, then half 1 over the same stages
        // (still resident), then both halves per stage.
        if (!mbar_wait(&tempty[h0], ((h0 ? hal_use1 : hal_use0) & 1) ^ 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (h1 - h0 == 2) {
          const int P = min(STAGES, kblocks);
          int s2 = stage;
          uint32_t r2 = round;
          for (int j = 0; j < P && ok; ++j) {
            if (!mbar_wait(&full[s2], r2 & 1, args.err, ERR_GEMM_WAIT, abort_flag)) ok = false;
            if (!ok) break;
            tc_fence_after();
            mma_stage(s2, 0, d_tmem, j == 0);
            if (++s2 == STAGES) {
              s2 = 0;
              ++r2;
            }
          }
          if (!ok) break;
          if (!mbar_wait(&tempty[1], (hal_use1 & 1) ^ 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int j = 0; j < P; ++j) {
            mma_stage(stage, 1, d_tmem, j == 0);
            free_stage(stage);
            if (++stage == STAGES) {
              stage = 0;
              ++round;
            }
          }
          kb = P;
        }
        hal_use0 += (h0 == 0);
        hal_use1 += (h1 == 2);
      } else {
        if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      for (; kb < kblocks; ++kb) {
        if (!mbar_wait(&full[stage], round & 1, args.err, ERR_GEMM_WAIT, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int h = h0; h < h1; ++h) mma_stage(stage, h, d_tmem, kb == 0);
        free_stage(stage);
        if (++stage == STAGES) {
          stage = 0;
          ++round;
        }
      }
      if (ok) {
        const uint32_t f = smem_u32(&tfull[acc]);
        commit2(map_to(f, 0));
        commit2(map_to(f, 1));
      }
    }
    if (!ok) {
      commit2(map_to(smem_u32(drain), 0));
      mbar_wait(drain, 0, args.err, ERR_GEMM_WAIT, nullptr);
    }
  } else if (warp >= 2 && warp < 2 + C_::EPI_WARPS) {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int it = 0;
    if constexpr (WIDE) {
      // Per MMA half: TMEM -> registers -> bf16 -> the swizzled staging blocks (warp 2 + e takes
      // lane quadrant quad and columns [128 (e / 4), +128) of the half), release the half's TMEM,
      // then one thread stores (or adds) the staged half with four TMA box copies of 64 x 128.
      const int cbase = ((warp - 2) / 4) * 128;
      const bool leader_thread = (warp == 2 && lane == 0);
      const float alpha_h = args.alpha;
      for (int u = pair; u < num_units; u += npairs) {
        int t, tm, tn, h0, h1;
        if (!pair_unit<C_>(u, full_units, tiles_m, tiles_n, args, t, tm, tn, h0, h1)) continue;
        const uint32_t use = (uint32_t)it;
        ++it;
        // every epilogue warp runs every unit and both named barriers, whatever its wait returned
        // (a warp leaving the loop early would strand the others at a barrier); after a failed
        // wait (the abort flag is set) the work is skipped and later waits return at once
        const bool live = mbar_wait(&tfull[0], use & 1, args.err, ERR_GEMM_WAIT, abort_flag);
        tc_fence_after();
        const float alpha = args.alpha_dev != nullptr ? alpha_h * __ldg(args.alpha_dev) : alpha_h;
        const int row0 = tm * 256 + (int)crank * 128;
        for (int h = h0; h < h1; ++h) {
          if (leader_thread) bulk_wait_read0();  // the previous half's stores have read the staging
          epi_bar_sync(32 * C_::EPI_WARPS);
          if (!live) {
            epi_bar_sync(32 * C_::EPI_WARPS);
            if (EPI == EPI_SWIGLU && args.GU != nullptr) {  // round B's two barriers
              epi_bar_sync(32 * C_::EPI_WARPS);
              epi_bar_sync(32 * C_::EPI_WARPS);
            }
            continue;
          }
          if constexpr (EPI == EPI_SWIGLU) {
            // half h holds gate (columns [0, 128)) and up ([128, 256)) of activation columns
            // [a0, a0 + 128); warp 2 + e takes activation columns [64 (e / 4), +64). Round A stages
            // act (blocks 0-1) and, with the gate / up store, gate (blocks 2-3); round B stages up.
            const bool gu = args.GU != nullptr;
            const int ab = ((warp - 2) / 4) * 64;
            const uint32_t t_g = tmem_base + ((uint32_t)(quad * 32) << 16) + h * C_::BN + ab;
            auto stage = [&](int blk, int c, const float (&f)[32]) {
              uint8_t* bp = stg + blk * 16384 + row_in_tile * 128;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 pk;
                __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(f[8 * q + 2 * e], f[8 * q + 2 * e + 1]);
                *reinterpret_cast<uint4*>(bp + (((4 * c + q) ^ (row_in_tile & 7)) << 4)) = pk;
              }
            };
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              float g[32], u[32], act[32];
              tmem_ld32(t_g + c * 32, g);
              tmem_ld32(t_g + 128 + c * 32, u);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                // the activation uses the bf16-rounded gate / up, which the backward reads back
                g[j] = __bfloat162float(__float2bfloat16(g[j] * alpha));
                u[j] = __bfloat162float(__float2bfloat16(u[j] * alpha));
                act[j] = silu_f(g[j]) * u[j];
              }
              stage(ab / 64, c, act);
              if (gu) stage(2 + ab / 64, c, g);
            }
            if (!gu) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) arrive_remote(tempty0 + h * 8);
            }
            fence_proxy_async_smem();
            epi_bar_sync(32 * C_::EPI_WARPS);
            const int a0 = tn * C_::BN_OUT + h * C_::HALF_OUT;
            if (leader_thread && row0 < args.M) {
              for (int b = 0; b < 2; ++b) {
                if (a0 + b * 64 >= args.N) break;
                tma_store_2d(&map_c, stg + b * 16384, a0 + b * 64, row0);
                if (gu) tma_store_2d(&map_g, stg + (2 + b) * 16384, a0 + b * 64, row0);
              }
              bulk_commit();
            }
            if (gu) {  // round B: up
              if (leader_thread) bulk_wait_read0();
              epi_bar_sync(32 * C_::EPI_WARPS);
#pragma unroll 1
              for (int c = 0; c < 2; ++c) {
                float u[32];
                tmem_ld32(t_g + 128 + c * 32, u);
#pragma unroll
                for (int j = 0; j < 32; ++j) u[j] *= alpha;
                stage(ab / 64, c, u);
              }
              tc_fence_before();
              __syncwarp();
              if (lane == 0) arrive_remote(tempty0 + h * 8);
              fence_proxy_async_smem();
              epi_bar_sync(32 * C_::EPI_WARPS);
              if (leader_thread && row0 < args.M) {
                for (int b = 0; b < 2; ++b) {
                  if (a0 + b * 64 >= args.N) break;
                  tma_store_2d(&map_u, stg + b * 16384, a0 + b * 64, row0);
                }
                bulk_commit();
              }
            }
            continue;
          }
          const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + h * C_::BN + cbase;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(t_row + c * 32, v);
            const int col = cbase + c * 32;  // column within the half
            uint8_t* blk = stg + (col / 64) * 16384 + row_in_tile * 128;
            const int ch0 = (col % 64) / 8;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 pk;
              __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
              for (int e = 0; e < 4; ++e) p2[e] = __floats2bfloat162_rn(v[8 * q + 2 * e] * alpha, v[8 * q + 2 * e + 1] * alpha);
              *reinterpret_cast<uint4*>(blk + (((ch0 + q) ^ (row_in_tile & 7)) << 4)) = pk;
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_remote(tempty0 + h * 8);  // this half's TMEM may be overwritten
          fence_proxy_async_smem();
          epi_bar_sync(32 * C_::EPI_WARPS);
          if (leader_thread && row0 < args.M) {
            const int x0 = tn * C_::BN_OUT + h * C_::HALF_OUT;
#pragma unroll 1
            for (int b = 0; b < 4; ++b) {
              if (x0 + b * 64 >= args.N) break;
              if constexpr (EPI == EPI_ADD_BF16)
                tma_reduce_add_2d(&map_c, stg + b * 16384, x0 + b * 64, row0);
              else
                tma_store_2d(&map_c, stg + b * 16384, x0 + b * 64, row0);
            }
            bulk_commit();
          }
        }
      }
      if (leader_thread) bulk_wait0();  // every store has landed before the CTA exits
    } else {
      for (int u = pair; u < num_units; u += npairs) {
        int t, tm, tn, h0, h1;
        if (!pair_unit<C_>(u, full_units, tiles_m, tiles_n, args, t, tm, tn, h0, h1)) continue;
        const int acc = (C_::NACC == 2) ? (it & 1) : 0;
        const uint32_t use = (C_::NACC == 2) ? (uint32_t)(it >> 1) : (uint32_t)it;
        ++it;
        if (!mbar_wait(&tfull[acc], use & 1, args.err, ERR_GEMM_WAIT, abort_flag)) break;
        tc_fence_after();
        const int row = tm * 256 + (int)crank * 128 + row_in_tile;
        const int n0 = tn * C_::BN_OUT;
        const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * C_::BN;
        epilogue_tile<256, EPI>(args, t_row, row, row < args.M, n0, 0, t, num_tiles, 1, lane);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_remote(tempty0 + acc * 8);
      }
    }
  } else if (warp >= 2 + C_::EPI_WARPS) {
    // ---------------------------------------------------------------- fused all-gather copies
    if (args.ag_nchunks > 0) ag_copy_warp(args, lane, abort_flag);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still read its smem or signal its barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C_::TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------------------------- host

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map: `inner` contiguous elements per row, `outer` rows, `ld` elements between rows,
// box {box_inner, box_outer}, 128-byte swizzle, zero fill out of bounds. Written through a pointer:
// CUtensorMap is a 64-byte-aligned type and is never passed or returned by value on the host
// (a by-value copy made the host code depend on the calling thread's stack alignment).
void make_map_bf16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                   uint32_t box_outer) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(m) % 64 == 0, "tensor map storage must be 64-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes (ld % 8 == 0)");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
}

// Kernel parameters assembled in 64-byte-aligned thread-local storage and handed to
// cudaLaunchKernel by pointer (the runtime copies them at launch).
struct alignas(64) GemmLaunch {
  CUtensorMap ma;
  CUtensorMap mb;
  CUtensorMap mc;  // the output, for the TMA-store epilogue of the 256 x 512 pair kernel
  CUtensorMap mg;  // SwiGLU gate / up store: the gate half and the up half of [M, 2F]
  CUtensorMap mu;
  GemmArgs args;
};
static thread_local GemmLaunch tls_launch;

// cuTensorMapEncodeTiled is a driver-API call and needs a current context in the calling thread.
// A thread that has only touched cached allocations (autograd's worker threads do exactly that)
// may have none: torch skips cudaSetDevice when the device index is unchanged. Bind the device's
// primary context once per thread before the first encode.
void bind_context(int dev) {
  static thread_local int bound = -1;
  if (bound != dev) {
    C10_CUDA_CHECK(cudaSetDevice(dev));
    C10_CUDA_CHECK(cudaFree(nullptr));
    bound = dev;
  }
}

// BDLLM_GEMM_TRACE=1 prints host-side checkpoints of every GEMM call to stderr (diagnostics).
static bool trace_on() {
  static int on = -1;
  if (on < 0) on = getenv("BDLLM_GEMM_TRACE") != nullptr;
  return on == 1;
}
#define GTRACE(msg)                                                    \
  do {                                                                 \
    if (trace_on()) {                                                  \
      fprintf(stderr, "[gemm] %s\n", msg);                            \
      fflush(stderr);                                                  \
    }                                                                  \
  } while (0)

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

// CTA pairs: for GEMMs large enough to give every pair a few 256 x 256 tiles, any operand majors
// (SwiGLU: K-major only), with or without the fused all-gather (the last two warps of both CTAs
// copy the weight's chunks; each CTA's producer waits for its own weight rows) (BDLLM_GEMM_PAIR=0
// keeps the one-CTA kernel)
static bool use_pair(bool a_mn, bool b_mn, int64_t M, int64_t N, int64_t epi, const void* tp, const void* ag) {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("BDLLM_GEMM_PAIR");
    env = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  if (!env || tp != nullptr) return false;
  if (ag != nullptr && b_mn) return false;  // the fused all-gather waits on K-major weight rows
  if (epi == EPI_SWIGLU && (a_mn || b_mn)) return false;
  if (!(epi == EPI_BF16 || epi == EPI_F32 || epi == EPI_ADD_BF16 || epi == EPI_SWIGLU)) return false;
  const int64_t tiles = ((M + 255) / 256) * ((N + (epi == EPI_SWIGLU ? 127 : 255)) / (epi == EPI_SWIGLU ? 128 : 256));
  return M >= 512 && tiles >= 148;
}

// Tile width of the pair kernel: 256 x 512 (BDLLM_GEMM_WIDE unset or not "0") or 256 x 256.
// Read at every call, so that a test can compare both in one process.
static bool pair_wide() {
  const char* e = getenv("BDLLM_GEMM_WIDE");
  return e == nullptr || e[0] != '0';
}

// Tile raster of the pair kernel. BDLLM_GEMM_RASTER: "m<G>" / "n<G>" fixes G tile rows along M /
// tile columns along N; "auto" picks, from a DRAM-traffic model, the orientation and G for which
// the grouped operand (G tiles x K, bf16) fits in 48 MB of L2 and (operand read once) + (other
// operand x number of groups) is smallest; unset = "m8".
static void choose_raster(GemmArgs& g, int64_t M, int64_t NB, int64_t K, int tiles_m, int tiles_n) {
  static int mode = -1, fixed_g = 8;  // 0: fixed along M, 1: fixed along N, 2: auto
  if (mode < 0) {
    const char* e = getenv("BDLLM_GEMM_RASTER");
    mode = 0;
    if (e != nullptr && strcmp(e, "auto") == 0) {
      mode = 2;
    } else if (e != nullptr && (e[0] == 'm' || e[0] == 'n') && atoi(e + 1) > 0) {
      mode = e[0] == 'n' ? 1 : 0;
      fixed_g = atoi(e + 1);
    }
  }
  if (mode < 2) {
    g.raster_g = fixed_g;
    g.raster_n = mode;
    return;
  }
  const double tile_bytes = 256.0 * (double)K * 2.0;
  const int gmax = std::max(1, (int)(48e6 / tile_bytes));
  const double a = (double)M * K * 2.0, b = (double)NB * K * 2.0;
  const int gm = std::min(gmax, tiles_m), gn = std::min(gmax, tiles_n);
  const double tm = a + b * (double)((tiles_m + gm - 1) / gm);
  const double tn = b + a * (double)((tiles_n + gn - 1) / gn);
  g.raster_n = tn < tm ? 1 : 0;
  g.raster_g = tn < tm ? gn : gm;
}

template <int EPI, bool A_MN, bool B_MN, int NP>
static void launch_pair(GemmLaunch* L, cudaStream_t st) {
  using C_ = Cfg2<EPI, A_MN, B_MN, NP>;
  auto kern = gemm2_kernel<EPI, A_MN, B_MN, NP>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM));
    attr = true;
  }
  const GemmArgs& args = L->args;
  // at most one pair per work unit (a tile, or each half of a tile when there are fewer tiles
  // than pairs)
  const int tiles = (int)(((args.M + 255) / 256) * ((args.N + C_::BN_OUT - 1) / C_::BN_OUT));
  const int pairs = std::max(1, std::min(tiles * C_::NH, num_sms() / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(C_::THREADS);
  cfg.dynamicSmemBytes = C_::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  void* kargs[6] = {&L->ma, &L->mb, &L->mc, &L->mg, &L->mu, &L->args};
  C10_CUDA_CHECK(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kern), kargs));
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static void launch(GemmLaunch* L, cudaStream_t st) {
  using C_ = Cfg<BN, A_MN, B_MN, EPI>;
  auto kern = gemm_kernel<BN, A_MN, B_MN, EPI>;
  GTRACE("maps ok");
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM));
    attr = true;
  }
  GTRACE("attr ok");
  const GemmArgs& args = L->args;
  const int tiles = ((args.M + BM - 1) / BM) * ((args.N + C_::BN_OUT - 1) / C_::BN_OUT);
  const int grid = std::max(1, std::min(tiles, num_sms()));
  void* kargs[3] = {&L->ma, &L->mb, &L->args};
  C10_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(NUM_THREADS), kargs,
                                  C_::SMEM, st));
  GTRACE("launched");
}

// C = A B^T-style contraction with operand majors; see the file header for the conventions.
// a: K-major -> [M, K] (lda); MN-major -> [K, M] (lda). b: K-major -> [N, K]; MN-major -> [K, N].
// out (bf16) = sum_s ws[s] (+ residual), ws [S, M, N] fp32 contiguous
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int S, int64_t M, int N,
                                     __nv_bfloat16* __restrict__ out, int64_t ldo,
                                     const __nv_bfloat16* __restrict__ res, int64_t ldr) {
  const int64_t nv = M * (N / 4);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / (N / 4);
    const int n = (int)(i - m * (N / 4)) * 4;
    float4 a = *reinterpret_cast<const float4*>(ws + m * N + n);
    for (int s2 = 1; s2 < S; ++s2) {
      const float4 b = *reinterpret_cast<const float4*>(ws + (int64_t)s2 * M * N + m * N + n);
      a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
    }
    if (res != nullptr) {
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(res + m * ldr + n);
      const float2 r0 = __bfloat1622float2(r2[0]), r1 = __bfloat1622float2(r2[1]);
      a.x += r0.x, a.y += r0.y, a.z += r1.x, a.w += r1.y;
    }
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(out + m * ldo + n);
    o2[0] = __floats2bfloat162_rn(a.x, a.y);
    o2[1] = __floats2bfloat162_rn(a.z, a.w);
  }
}

struct TpHook {
  const std::vector<int64_t>* peers;
  int rank, rows_per_rank, wait_ag;
  int64_t part_off, flag_off;
  unsigned* ctr;
  double timeout_s;
  int ksplit, kbs;
  int64_t split_stride;
  // fused FSDP all-gather (ag_nchunks > 0): the B operand lives in `ag_dst`, the gathered buffer of a
  // unit whose rank-p shard is at peers[p] + ag_src_off (ag_shard_bytes each). Warps 6-7 of every
  // CTA claim 16-byte-aligned chunks of ag_chunk bytes (chunk k = shard k / cps, piece k % cps) in
  // priority order starting at ag_first, copy them from the owning peer and publish ready[k] = seq;
  // the TMA producer waits for the chunks under each B tile before loading it.
  int ag_nchunks, ag_first, ag_world, ag_rank;  // ag_nchunks: chunks this launch copies, from ag_first
  int64_t ag_src_off, ag_shard_bytes, ag_chunk, ag_b_off;
  char* ag_dst;
  unsigned* ag_ready;
  unsigned* ag_claim;
  unsigned ag_seq, ag_epoch;
};

// k-split that gives every split >= 1 k-block: returns {splits, k-blocks per split}
static std::pair<int, int> split_plan(int64_t K, int64_t S) {
  const int64_t kblocks = (K + BK - 1) / BK;
  S = std::max<int64_t>(1, std::min<int64_t>(S, kblocks));
  const int64_t kbs = (kblocks + S - 1) / S;
  return {(int)((kblocks + kbs - 1) / kbs), (int)kbs};
}

struct AgHook {
  const std::vector<int64_t>* peers;
  int rank, nchunks, first;
  int64_t src_off, shard_bytes, chunk, b_off, flag_off;
  char* dst;
  unsigned* ready;
  unsigned* claim;
  unsigned seq, epoch;
  double timeout_s;
};

static void gemm_impl(const at::Tensor& a, bool a_mn, int64_t lda, const at::Tensor& b, bool b_mn, int64_t ldb,
                      int64_t M, int64_t N, int64_t K, at::Tensor& c, int64_t ldc, int64_t epi,
                      const c10::optional<at::Tensor>& r, int64_t ldr, const c10::optional<at::Tensor>& gu, int64_t bn,
                      double alpha, const TpHook* tp, const AgHook* ag = nullptr, const float* alpha_dev = nullptr);

void gemm(const at::Tensor& a, bool a_mn, int64_t lda, const at::Tensor& b, bool b_mn, int64_t ldb, int64_t M,
          int64_t N, int64_t K, at::Tensor& c, int64_t ldc, int64_t epi, const c10::optional<at::Tensor>& r,
          int64_t ldr, const c10::optional<at::Tensor>& gu, int64_t bn, double alpha,
          const c10::optional<at::Tensor>& alpha_t) {
  TORCH_CHECK(epi != EPI_PEER_F32, "gemm: the peer epilogue goes through gemm_tp");
  const float* ad = nullptr;
  if (alpha_t.has_value()) {
    TORCH_CHECK(alpha_t->is_cuda() && alpha_t->scalar_type() == at::kFloat && alpha_t->numel() == 1,
                "gemm: alpha_t must be one fp32 element on the device");
    ad = alpha_t->data_ptr<float>();
  }
  gemm_impl(a, a_mn, lda, b, b_mn, ldb, M, N, K, c, ldc, epi, r, ldr, gu, bn, alpha, nullptr, nullptr, ad);
}

// Split-K GEMM for skinny problems (few output tiles): out[M, N] (bf16) = a b^T (+ residual), both
// K-major. `ws` is an fp32 workspace of >= S * M * N elements.
void gemm_splitk(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, at::Tensor& ws, int64_t S,
                 const c10::optional<at::Tensor>& residual) {
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "gemm_splitk: K-major 2-D");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(N % 4 == 0 && ws.is_contiguous() && ws.scalar_type() == at::kFloat && ws.numel() >= S * M * N,
              "gemm_splitk: N % 4 == 0 and an fp32 workspace of S*M*N");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.stride(0) % 8 == 0, "gemm_splitk: out");
  const int64_t kblocks = (K + BK - 1) / BK;
  const int64_t kbs = (kblocks + S - 1) / S;
  const int64_t splits = (kblocks + kbs - 1) / kbs;  // every split gets >= 1 k-block
  at::Tensor w2 = ws.view({-1}).narrow(0, 0, splits * M * N).view({splits * M, N});
  {
    // reuse the plain path with the split fields set (EPI_F32, 256-wide tiles)
    c10::cuda::CUDAGuard guard(a.device());
    bind_context(a.get_device());
    cudaStream_t st = at::cuda::getCurrentCUDAStream();
    GemmLaunch* L = &tls_launch;
    L->args = GemmArgs{};
    GemmArgs& g = L->args;
    g.M = (int)M, g.N = (int)N, g.K = (int)K, g.C = w2.data_ptr(), g.ldc = (int)N, g.err = error_word_ptr();
    g.alpha = 1.f, g.ksplit = (int)splits, g.kbs = (int)kbs, g.split_stride = M * N;
    make_map_bf16(&L->ma, a.data_ptr(), K, M, a.stride(0), 64, 128);
    make_map_bf16(&L->mb, b.data_ptr(), K, N, b.stride(0), 64, 256);
    using C_ = Cfg<256, false, false, EPI_F32>;
    auto kern = gemm_kernel<256, false, false, EPI_F32>;
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM));
      attr = true;
    }
    const int tiles = (int)(((M + BM - 1) / BM) * ((N + 255) / 256) * splits);
    const int grid = std::max(1, std::min(tiles, num_sms()));
    void* kargs[3] = {&L->ma, &L->mb, &L->args};
    C10_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(NUM_THREADS), kargs,
                                    C_::SMEM, st));
    const __nv_bfloat16* res = nullptr;
    int64_t ldr = 0;
    if (residual.has_value()) {
      TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1, "gemm_splitk: residual");
      res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
      ldr = residual->stride(0);
    }
    const int64_t nv = M * (N / 4);
    const int rgrid = (int)std::min<int64_t>((nv + 255) / 256, 148 * 8);
    splitk_reduce_kernel<<<rgrid, 256, 0, st>>>(w2.data_ptr<float>(), (int)splits, M, (int)N,
                                                reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), res,
                                                ldr);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// Tensor-parallel GEMM: y = a b^T (K-major operands) with the collective hooks. epi EPI_PEER_F32:
// output rows go to their owner's fp32 partial slot in peer memory (c is only the shape/stride
// template, [M, N] fp32); other epilogues write c locally. wait_ag: wait for every rank's pushed
// A rows first (the gathered A lives in this rank's heap).
// ksplit > 1 (skinny problems): EPI_F32 writes split s at c + s * M * N (c is [S * M, N] fp32);
// EPI_PEER_F32 writes split s of source rank r into the owner's slot r * S + s. Returns the number of
// splits used (the consumer sums that many slots).
int64_t gemm_tp(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, int64_t epi,
                const c10::optional<at::Tensor>& gu, const std::vector<int64_t>& peers, int64_t rank,
                int64_t rows_per_rank, int64_t part_off, int64_t flag_off, const at::Tensor& ctr, bool wait_ag,
                double timeout_s, int64_t bn, int64_t ksplit) {
  TORCH_CHECK(peers.size() >= 1 && peers.size() <= (size_t)TP_MAX, "gemm_tp: 1..8 ranks");
  TORCH_CHECK(ctr.is_cuda() && ctr.scalar_type() == at::kInt && ctr.numel() >= 4, "gemm_tp: int32 counters [>= 4]");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "gemm_tp: 2-D K-major operands");
  const int64_t M = a.size(0), K = a.size(1), N = (epi == EPI_SWIGLU) ? b.size(0) / 2 : b.size(0);
  if (epi == EPI_PEER_F32)
    TORCH_CHECK(rows_per_rank > 0 && M % rows_per_rank == 0 && M / rows_per_rank == (int64_t)peers.size() &&
                    c.scalar_type() == at::kFloat && c.size(1) == N && (c.stride(0) * 4) % 16 == 0,
                "gemm_tp: peer epilogue needs M = world * rows_per_rank and an fp32 [M, N] template");
  TpHook h{&peers, (int)rank, (int)rows_per_rank, wait_ag ? 1 : 0, part_off, flag_off,
           reinterpret_cast<unsigned*>(ctr.data_ptr<int>()), timeout_s, 1, 0, 0};
  if (ksplit > 1) {
    TORCH_CHECK(epi == EPI_F32 || epi == EPI_PEER_F32, "gemm_tp: k-split with the fp32 or peer epilogue only");
    auto [S, kbs] = split_plan(K, ksplit);
    h.ksplit = S, h.kbs = kbs, h.split_stride = (epi == EPI_F32) ? M * N : 0;
    if (epi == EPI_F32)
      TORCH_CHECK(c.is_contiguous() && c.numel() >= (int64_t)S * M * N, "gemm_tp: fp32 workspace [S*M, N]");
  }
  gemm_impl(a, false, a.stride(0), b, false, b.stride(0), M, N, K, c, c.stride(0), epi, c10::nullopt, 0, gu, bn, 1.0,
            &h);
  return h.ksplit;
}

// Reductions of k-split partials: out (bf16) = sum_s ws[s] (+ residual); or, for the gate|up GEMM,
// act = silu(sum_s gate) * (sum_s up) with ws [S, M, 2F].
__global__ void splitk_swiglu_kernel(const float* __restrict__ ws, int S, int64_t M, int F,
                                     __nv_bfloat16* __restrict__ act) {
  const int64_t n = M * F;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / F;
    const int j = (int)(i - m * F);
    float g = 0.f, u = 0.f;
    for (int s2 = 0; s2 < S; ++s2) {
      const float* row = ws + ((int64_t)s2 * M + m) * 2 * F;
      g += row[j];
      u += row[F + j];
    }
    // same rounding as the SwiGLU epilogue: bf16 gate and up first
    g = __bfloat162float(__float2bfloat16(g));
    u = __bfloat162float(__float2bfloat16(u));
    act[i] = __float2bfloat16(silu_f(g) * u);
  }
}

void splitk_reduce(const at::Tensor& ws, int64_t S, at::Tensor& out, const c10::optional<at::Tensor>& residual,
                   bool swiglu) {
  TORCH_CHECK(ws.is_contiguous() && ws.scalar_type() == at::kFloat, "splitk_reduce: fp32 workspace");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1, "splitk_reduce: bf16 out");
  const int64_t M = out.size(0), N = out.size(1);
  c10::cuda::CUDAGuard g(ws.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (swiglu) {
    TORCH_CHECK(out.is_contiguous() && ws.numel() >= S * M * 2 * N, "splitk_reduce: swiglu shapes");
    const int grid = (int)std::min<int64_t>((M * N + 255) / 256, 148 * 8);
    splitk_swiglu_kernel<<<grid, 256, 0, st>>>(ws.data_ptr<float>(), (int)S, M, (int)N,
                                               reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  } else {
    TORCH_CHECK(N % 4 == 0 && ws.numel() >= S * M * N && out.stride(0) % 4 == 0, "splitk_reduce: shapes");
    const __nv_bfloat16* res = nullptr;
    int64_t ldr = 0;
    if (residual.has_value()) {
      res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
      ldr = residual->stride(0);
    }
    const int grid = (int)std::min<int64_t>((M * (N / 4) + 255) / 256, 148 * 8);
    splitk_reduce_kernel<<<grid, 256, 0, st>>>(ws.data_ptr<float>(), (int)S, M, (int)N,
                                               reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), res, ldr);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fused FSDP all-gather -> GEMM: y = a W^T where W ([N, K], or [2F, K] for the SwiGLU epilogue) is a
// view into `gathered`, the unit's full buffer that this launch fills from the peers' shards while
// it computes (see GemmArgs::ag_*). Every chunk of the unit is copied, not only W's, so the buffer
// is complete when the kernel ends. `ready` (int32, >= chunks) holds per-chunk sequence numbers,
// `claim` (int32) is the chunk claim counter (zeroed here).
void gemm_ag(const at::Tensor& a, const at::Tensor& w, at::Tensor& c, int64_t epi, const c10::optional<at::Tensor>& gu,
             const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard_bytes,
             at::Tensor& gathered, at::Tensor& ready, at::Tensor& claim, int64_t seq, int64_t epoch, int64_t flag_off,
             double timeout_s, int64_t lo, int64_t hi) {
  const int world = (int)peers.size();
  TORCH_CHECK(world >= 1 && world <= TP_MAX, "gemm_ag: 1..8 ranks");
  TORCH_CHECK(a.dim() == 2 && w.dim() == 2 && a.stride(1) == 1 && w.stride(1) == 1, "gemm_ag: K-major 2-D operands");
  TORCH_CHECK(shard_bytes % 16 == 0 && src_off % 16 == 0, "gemm_ag: 16-byte shards");
  TORCH_CHECK(gathered.is_cuda() && gathered.numel() * gathered.element_size() >= shard_bytes * world,
              "gemm_ag: gathered buffer too small");
  char* base = reinterpret_cast<char*>(gathered.data_ptr());
  const int64_t b_off = reinterpret_cast<char*>(w.data_ptr()) - base;
  TORCH_CHECK(b_off >= 0 && b_off + w.numel() * 2 <= shard_bytes * world, "gemm_ag: W must lie in the gathered buffer");
  int64_t chunk = std::max<int64_t>(256 * 1024, (shard_bytes * world + 8191) / 8192);
  chunk = (chunk + 15) / 16 * 16;
  const int64_t cps = (shard_bytes + chunk - 1) / chunk;
  const int64_t nchunks = cps * world;
  TORCH_CHECK(ready.is_cuda() && ready.scalar_type() == at::kInt && ready.numel() >= nchunks, "gemm_ag: ready flags");
  (void)nchunks;
  TORCH_CHECK(claim.is_cuda() && claim.scalar_type() == at::kInt && claim.numel() >= 1, "gemm_ag: claim counter");
  C10_CUDA_CHECK(cudaMemsetAsync(claim.data_ptr(), 0, sizeof(int), at::cuda::getCurrentCUDAStream()));
  // chunks to copy: those overlapping gathered bytes [lo, hi) (default: the whole unit)
  if (hi <= lo) lo = 0, hi = shard_bytes * world;
  TORCH_CHECK(lo >= 0 && hi <= shard_bytes * world && lo <= b_off && b_off + w.numel() * 2 <= hi,
              "gemm_ag: the copied range must cover W");
  auto chunk_of = [&](int64_t x) { return (x / shard_bytes) * cps + (x % shard_bytes) / chunk; };
  const int64_t k_lo = chunk_of(lo), k_hi = chunk_of(hi - 1);
  AgHook h{&peers, (int)rank, (int)(k_hi - k_lo + 1), (int)k_lo,
           src_off, shard_bytes, chunk, b_off, flag_off, base, reinterpret_cast<unsigned*>(ready.data_ptr<int>()),
           reinterpret_cast<unsigned*>(claim.data_ptr<int>()), (unsigned)seq, (unsigned)epoch, timeout_s};
  const int64_t M = a.size(0), K = a.size(1), N = (epi == EPI_SWIGLU) ? w.size(0) / 2 : w.size(0);
  gemm_impl(a, false, a.stride(0), w, false, w.stride(0), M, N, K, c, c.stride(0), epi, c10::nullopt, 0, gu, 256, 1.0,
            nullptr, &h);
}

static void gemm_impl(const at::Tensor& a, bool a_mn, int64_t lda, const at::Tensor& b, bool b_mn, int64_t ldb,
                      int64_t M, int64_t N, int64_t K, at::Tensor& c, int64_t ldc, int64_t epi,
                      const c10::optional<at::Tensor>& r, int64_t ldr, const c10::optional<at::Tensor>& gu, int64_t bn,
                      double alpha, const TpHook* tp, const AgHook* ag, const float* alpha_dev) {
  GTRACE("enter");
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm: CUDA tensors expected");
  bind_context(a.get_device());
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  GTRACE("stream ok");
  GemmLaunch* L = &tls_launch;
  L->args = GemmArgs{(int)M, (int)N, (int)K, c.data_ptr(), (int)ldc, nullptr, (int)ldr, nullptr, 0, error_word_ptr(),
                     (float)alpha};
  GemmArgs& args = L->args;
  args.alpha_dev = alpha_dev;
  if (epi == EPI_ADD_BF16) {
    TORCH_CHECK(r.has_value(), "EPI_ADD_BF16 needs a residual");
    args.R = r->data_ptr();
  }
  if (epi == EPI_SWIGLU && gu.has_value()) {
    args.GU = reinterpret_cast<__nv_bfloat16*>(gu->data_ptr());
    args.ldgu = (int)(2 * N);
  }
  if (tp != nullptr) {
    const int w = (int)tp->peers->size();
    for (int i = 0; i < w; ++i) args.peers[i] = (*tp->peers)[i];
    args.world = w;
    args.rank = tp->rank;
    args.rows_per_rank = tp->rows_per_rank;
    args.part_off = tp->part_off;
    args.flag_off = tp->flag_off;
    args.ctr = tp->ctr;
    args.wait_ag = tp->wait_ag;
    args.timeout_ns = (uint64_t)(tp->timeout_s * 1e9);
    args.ksplit = tp->ksplit;
    args.kbs = tp->kbs;
    args.split_stride = tp->split_stride;
  }
  if (ag != nullptr) {
    const int w = (int)ag->peers->size();
    for (int i = 0; i < w; ++i) args.peers[i] = (*ag->peers)[i];
    args.flag_off = ag->flag_off;
    args.timeout_ns = (uint64_t)(ag->timeout_s * 1e9);
    args.ag_nchunks = ag->nchunks;
    args.ag_first = ag->first;
    args.ag_world = w;
    args.ag_rank = ag->rank;
    args.ag_src_off = ag->src_off;
    args.ag_shard_bytes = ag->shard_bytes;
    args.ag_chunk = ag->chunk;
    args.ag_b_off = ag->b_off;
    args.ag_dst = ag->dst;
    args.ag_ready = ag->ready;
    args.ag_claim = ag->claim;
    args.ag_seq = ag->seq;
    args.ag_epoch = ag->epoch;
  }
  const bool f32_out = (epi == EPI_F32 || epi == EPI_ACC_F32 || epi == EPI_PEER_F32);
  TORCH_CHECK(c.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm: output dtype does not match the epilogue");
  // the epilogue stores (and reads the residual) in 16-byte vectors: rows must stay 16-byte aligned
  const int64_t esz = f32_out ? 4 : 2;
  // (an output narrower than 32 columns only ever takes the scalar tail path)
  const bool vec = N >= 32;
  TORCH_CHECK(!vec || ((ldc * esz) % 16 == 0 && reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0),
              "gemm: output rows must be 16-byte aligned");
  if (args.R)
    TORCH_CHECK(!vec || ((ldr * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(args.R) % 16 == 0),
                "gemm: residual rows must be 16-byte aligned");
  if (args.GU)
    TORCH_CHECK((N % 8) == 0 && reinterpret_cast<uintptr_t>(args.GU) % 16 == 0, "gemm: gate/up store misaligned");
  TORCH_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm: dims exceed int32");

  GTRACE("args ok");
  // the CTA-pair kernel for large forward (K-major) GEMMs
  if (use_pair(a_mn, b_mn, M, N, epi, tp, ag)) {
    // 256 x 512 tiles for bf16 outputs (an add only in place: the TMA reduce adds into C itself)
    const bool wide = pair_wide() && (epi == EPI_BF16 || epi == EPI_SWIGLU ||
                                      (epi == EPI_ADD_BF16 && args.R == c.data_ptr() && ldr == ldc));
    const int64_t tile_out = (epi == EPI_SWIGLU ? 128 : 256) * (wide ? 2 : 1);
    choose_raster(args, M, epi == EPI_SWIGLU ? 2 * N : N, K, (int)((M + 255) / 256), (int)((N + tile_out - 1) / tile_out));
    if (a_mn)
      make_map_bf16(&L->ma, a.data_ptr(), M, K, lda, 64, 64);
    else
      make_map_bf16(&L->ma, a.data_ptr(), K, M, lda, 64, 128);
    if (b_mn)
      make_map_bf16(&L->mb, b.data_ptr(), N, K, ldb, 64, 64);
    else
      make_map_bf16(&L->mb, b.data_ptr(), K, epi == EPI_SWIGLU ? 2 * N : N, ldb, 64, 128);
    if (wide) {
      TORCH_CHECK(reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0 && (ldc * 2) % 16 == 0,
                  "gemm: TMA-store output must have 16-byte aligned rows");
      make_map_bf16(&L->mc, c.data_ptr(), N, M, ldc, 64, 128);
      if (epi == EPI_SWIGLU && args.GU != nullptr) {
        make_map_bf16(&L->mg, args.GU, N, M, 2 * N, 64, 128);
        make_map_bf16(&L->mu, args.GU + N, N, M, 2 * N, 64, 128);
      }
    }
#define BDLLM_PAIR_CASE(E, AM, BMN)                   \
  if (epi == E && a_mn == AM && b_mn == BMN) {        \
    launch_pair<E, AM, BMN, 256>(L, st);              \
    return;                                           \
  }
#define BDLLM_WIDE_CASE(E, AM, BMN)                   \
  if (wide && epi == E && a_mn == AM && b_mn == BMN) { \
    launch_pair<E, AM, BMN, 512>(L, st);              \
    return;                                           \
  }
    BDLLM_WIDE_CASE(EPI_BF16, false, false)
    BDLLM_WIDE_CASE(EPI_SWIGLU, false, false)
    BDLLM_WIDE_CASE(EPI_ADD_BF16, false, false)
    BDLLM_WIDE_CASE(EPI_BF16, false, true)
    BDLLM_WIDE_CASE(EPI_ADD_BF16, false, true)
    BDLLM_WIDE_CASE(EPI_BF16, true, true)
    BDLLM_WIDE_CASE(EPI_ADD_BF16, true, true)
#undef BDLLM_WIDE_CASE
    BDLLM_PAIR_CASE(EPI_BF16, false, false)
    BDLLM_PAIR_CASE(EPI_F32, false, false)
    BDLLM_PAIR_CASE(EPI_ADD_BF16, false, false)
    BDLLM_PAIR_CASE(EPI_SWIGLU, false, false)
    BDLLM_PAIR_CASE(EPI_BF16, false, true)
    BDLLM_PAIR_CASE(EPI_F32, false, true)
    BDLLM_PAIR_CASE(EPI_ADD_BF16, false, true)
    BDLLM_PAIR_CASE(EPI_BF16, true, true)
    BDLLM_PAIR_CASE(EPI_F32, true, true)
    BDLLM_PAIR_CASE(EPI_ADD_BF16, true, true)
#undef BDLLM_PAIR_CASE
  }
  if (a_mn)
    make_map_bf16(&L->ma, a.data_ptr(), M, K, lda, 64, 64);
  else
    make_map_bf16(&L->ma, a.data_ptr(), K, M, lda, 64, 128);
  const int BN = (bn == 128) ? 128 : 256;
  if (epi == EPI_SWIGLU) {
    TORCH_CHECK(!a_mn && !b_mn, "swiglu epilogue: K-major operands only");
    make_map_bf16(&L->mb, b.data_ptr(), K, 2 * N, ldb, 64, BN / 2);
  } else if (b_mn) {
    make_map_bf16(&L->mb, b.data_ptr(), N, K, ldb, 64, 64);
  } else {
    make_map_bf16(&L->mb, b.data_ptr(), K, N, ldb, 64, BN);
  }

#define BDLLM_GEMM_CASE(BN_, AM, BMN, E)                                       \
  if (BN == BN_ && a_mn == AM && b_mn == BMN && epi == E) {                     \
    launch<BN_, AM, BMN, E>(L, st);                                             \
    return;                                                                     \
  }
  BDLLM_GEMM_CASE(256, false, false, EPI_BF16)
  BDLLM_GEMM_CASE(256, false, false, EPI_F32)
  BDLLM_GEMM_CASE(256, false, false, EPI_ADD_BF16)
  BDLLM_GEMM_CASE(256, false, false, EPI_SWIGLU)
  BDLLM_GEMM_CASE(256, false, false, EPI_PEER_F32)
  BDLLM_GEMM_CASE(128, false, false, EPI_PEER_F32)
  BDLLM_GEMM_CASE(128, false, false, EPI_SWIGLU)
  BDLLM_GEMM_CASE(256, false, true, EPI_BF16)
  BDLLM_GEMM_CASE(256, false, true, EPI_ADD_BF16)
  BDLLM_GEMM_CASE(256, false, true, EPI_F32)
  BDLLM_GEMM_CASE(256, true, true, EPI_F32)
  BDLLM_GEMM_CASE(256, true, true, EPI_ACC_F32)
  BDLLM_GEMM_CASE(256, true, true, EPI_BF16)
  BDLLM_GEMM_CASE(256, true, true, EPI_ADD_BF16)
  BDLLM_GEMM_CASE(128, false, false, EPI_BF16)
  BDLLM_GEMM_CASE(128, false, false, EPI_F32)
  BDLLM_GEMM_CASE(128, false, true, EPI_BF16)
  BDLLM_GEMM_CASE(128, true, true, EPI_F32)
  BDLLM_GEMM_CASE(128, true, true, EPI_ACC_F32)
#undef BDLLM_GEMM_CASE
  TORCH_CHECK(false, "gemm: unsupported combination bn=", BN, " a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

int* error_word_ptr() {
  static int* ptrs[64] = {nullptr};
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (!ptrs[dev]) {
    C10_CUDA_CHECK(cudaMalloc(&ptrs[dev], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(ptrs[dev], 0, sizeof(int)));
  }
  return ptrs[dev];
}

// (file, line, index, limit, failures) of every translation unit whose bounds record is set; empty
// in the normal build (no unit registers a record there).
std::vector<std::tuple<std::string, int64_t, int64_t, int64_t, int64_t>> bounds_report(bool reset) {
  std::vector<std::tuple<std::string, int64_t, int64_t, int64_t, int64_t>> out;
  int n = 0;
  BoundsUnit* units = bounds_units(&n);
  for (int i = 0; i < n; ++i) {
    BoundsRec r{};
    units[i].read(&r, reset);
    if (r.count)
      out.emplace_back(units[i].file, (int64_t)r.line, (int64_t)r.idx, (int64_t)r.lim, (int64_t)r.count);
  }
  C10_CUDA_CHECK(cudaGetLastError());
  return out;
}

bool debug_bounds_build() { return BDLLM_DEBUG_BUILD != 0; }

int64_t read_error_word(bool reset) {
  int v = 0;
  int* p = error_word_ptr();
  C10_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return v;
}

}  // namespace bdllm
