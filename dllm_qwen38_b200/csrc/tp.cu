// Tensor-parallel decode collectives over peer memory (the halves that are not inside the GEMM).
// (The reference decodes on one device, `src/dllm_qwen38/decode.py:35-99`; tensor parallelism is new here.)
//
// The residual stream is sharded by rows: rank r owns rows [r*R, (r+1)*R) of the M = world*R
// rows of a step. A row-parallel GEMM (csrc/gemm.cu, EPI_PEER_F32) stores each rank's fp32
// partial of every output row into the owner's slot part[src][row]; then
//
//   reduce_norm_push   owner: wait for every rank's partials, h = bf16(h + sum_src part[src])
//                      (rank order), y = RMSNorm(1+w)(h), push y into every rank's gathered
//                      buffer at rows [r*R, (r+1)*R) and publish the all-gather flag. The next
//                      column-parallel GEMM waits for that flag inside its producer warp (fused
//                      all-gather -> GEMM), so the gather costs no launch of its own.
//   conf_push          per logits row of this rank's vocab slice: (max, sum exp, argmax) pushed to
//                      every rank
//   conf_merge         every rank merges the slices in rank order: identical confidence and pick
//                      on all ranks, so the device commit rule runs replicated
//
// Sequence numbers live in device counters advanced by the kernels themselves, so a captured
// CUDA graph replays with fresh values. Every wait is bounded (ERR_COMM_WAIT, then return).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
namespace tp {

constexpr int MAXW = 8;
enum Ctr : int { CTR_RS = 0, CTR_AGC = 2, CTR_RED = 4, CTR_RED_ARRIVE = 5, CTR_AGP = 6, CTR_CONF_P = 7,
                 CTR_CONF_ARRIVE = 8, CTR_CONF_M = 9 };
enum Slot : int { SLOT_RS = 8, SLOT_AG = 9, SLOT_CONF = 10 };

struct Peers {
  int64_t p[MAXW];
};

__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned* flag(int64_t base, int64_t flag_off, int slot, int src) {
  return reinterpret_cast<unsigned*>(base + flag_off) + slot * 16 + src;
}

__device__ bool wait_slot(const Peers& P, int world, int rank, int64_t flag_off, int slot, unsigned target, int* err,
                          uint64_t tmo) {
  const uint64_t t0 = globaltimer();
  for (int p = 0; p < world; ++p) {
    const unsigned* f = flag(P.p[rank], flag_off, slot, p);
    while (static_cast<int>(ld_acquire(f) - target) < 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (globaltimer() - t0 > tmo) {
        record_error(err, ERR_COMM_WAIT);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// last-block bookkeeping: returns true in exactly one thread of the last block to arrive
__device__ bool last_block(unsigned* arrive) {
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(arrive, 1u);
    last = prev == gridDim.x - 1;
    if (last) *arrive = 0u;
  }
  __syncthreads();
  return last && threadIdx.x == 0;
}

// One block per owned row. D % 8 == 0, D <= 8 * blockDim.x * 4.
__global__ void __launch_bounds__(256) reduce_norm_push_kernel(
    Peers P, int world, int rank, int R, int D, int64_t part_off, __nv_bfloat16* __restrict__ h, int has_partials,
    const float* __restrict__ w1, float eps, int64_t gather_off, int64_t flag_off, unsigned* ctr, int* err,
    uint64_t tmo, int do_push, int nslots) {
  __shared__ int ok;
  __shared__ float red[8];
  const int row = blockIdx.x;
  if (threadIdx.x == 0) {
    ok = *reinterpret_cast<volatile int*>(err) == 0;
    if (ok && has_partials) ok = wait_slot(P, world, rank, flag_off, SLOT_RS, ctr[CTR_RED] + 1u, err, tmo);
  }
  __syncthreads();
  float x[4][8];
  float ss = 0.f;
  const int nv = D / 8;
  if (ok) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = threadIdx.x + u * blockDim.x;
      if (v >= nv) continue;
      uint4 hv = *reinterpret_cast<const uint4*>(h + (int64_t)row * D + v * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&hv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        x[u][2 * e] = f.x;
        x[u][2 * e + 1] = f.y;
      }
      if (has_partials) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int p = 0; p < nslots; ++p) {  // [source rank][k split], summed in that order
          const float* src = reinterpret_cast<const float*>(P.p[rank] + part_off) + ((int64_t)p * R + row) * D + v * 8;
          const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
          const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
          acc[0] += a.x, acc[1] += a.y, acc[2] += a.z, acc[3] += a.w;
          acc[4] += b.x, acc[5] += b.y, acc[6] += b.z, acc[7] += b.w;
        }
        uint4 o;
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // same rounding as the single-GPU residual epilogue: bf16(acc + h)
          o2[e] = __floats2bfloat162_rn(acc[2 * e] + x[u][2 * e], acc[2 * e + 1] + x[u][2 * e + 1]);
          const float2 f = __bfloat1622float2(o2[e]);
          x[u][2 * e] = f.x;
          x[u][2 * e + 1] = f.y;
        }
        *reinterpret_cast<uint4*>(h + (int64_t)row * D + v * 8) = o;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += x[u][e] * x[u][e];
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / D + eps);
  if (ok && do_push) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = threadIdx.x + u * blockDim.x;
      if (v >= nv) continue;
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o2[e] = __floats2bfloat162_rn(x[u][2 * e] * inv * w1[v * 8 + 2 * e],
                                      x[u][2 * e + 1] * inv * w1[v * 8 + 2 * e + 1]);
      for (int p = 0; p < world; ++p)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(P.p[p] + gather_off) +
                                  ((int64_t)rank * R + row) * D + v * 8) = o;
    }
  }
  if (last_block(&ctr[CTR_RED_ARRIVE])) {
    if (has_partials) ctr[CTR_RED] += 1u;
    if (!do_push) return;
    const unsigned seq = ctr[CTR_AGP] + 1u;
    ctr[CTR_AGP] = seq;
    __threadfence_system();
    for (int p = 0; p < world; ++p) st_release(flag(P.p[p], flag_off, SLOT_AG, rank), seq);
  }
}

// ------------------------------------------------------------------------------- confidence
struct Best {
  float m, s;
  int idx;
};
__device__ __forceinline__ Best merge(Best a, Best b) {
  if (b.m > a.m || (b.m == a.m && b.idx < a.idx)) {
    const Best t = a;
    a = b;
    b = t;
  }
  return Best{a.m, a.s + (b.m == -INFINITY ? 0.f : b.s * __expf(b.m - a.m)), a.idx};
}

// one block per logits row (all M rows, this rank's vocab slice starting at v0)
__global__ void __launch_bounds__(512) conf_push_kernel(Peers P, int world, int rank, const __nv_bfloat16* logits,
                                                        int64_t ld, int V, int v0, int64_t conf_off, int64_t flag_off,
                                                        unsigned* ctr) {
  const __nv_bfloat16* row = logits + (int64_t)blockIdx.x * ld;
  Best b{-INFINITY, 0.f, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = __bfloat162float(row[i]);
    if (x > b.m) {
      b.s = (b.m == -INFINITY ? 0.f : b.s * __expf(b.m - x)) + 1.f;
      b.m = x;
      b.idx = v0 + i;
    } else {
      b.s += __expf(x - b.m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    b = merge(b, Best{__shfl_xor_sync(0xffffffffu, b.m, o), __shfl_xor_sync(0xffffffffu, b.s, o),
                      __shfl_xor_sync(0xffffffffu, b.idx, o)});
  __shared__ Best red[16];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) b = merge(b, red[i]);
    const float4 rec = make_float4(b.m, b.s, __int_as_float(b.idx), 0.f);
    for (int p = 0; p < world; ++p)
      reinterpret_cast<float4*>(P.p[p] + conf_off)[(int64_t)rank * gridDim.x + blockIdx.x] = rec;
  }
  if (last_block(&ctr[CTR_CONF_ARRIVE])) {
    const unsigned seq = ctr[CTR_CONF_P] + 1u;
    ctr[CTR_CONF_P] = seq;
    __threadfence_system();
    for (int p = 0; p < world; ++p) st_release(flag(P.p[p], flag_off, SLOT_CONF, rank), seq);
  }
}

// one thread per row; merges the world slices in rank order
__global__ void conf_merge_kernel(Peers P, int world, int rank, int M, int64_t conf_off, int64_t flag_off,
                                  unsigned* ctr, float* conf, int64_t* pick, int* err, uint64_t tmo) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_slot(P, world, rank, flag_off, SLOT_CONF, ctr[CTR_CONF_M] + 1u, err, tmo);
  __syncthreads();
  if (ok) {
    for (int r = threadIdx.x; r < M; r += blockDim.x) {
      Best b{-INFINITY, 0.f, 0x7fffffff};
      for (int p = 0; p < world; ++p) {
        const float4 rec = __ldcg(reinterpret_cast<const float4*>(P.p[rank] + conf_off) + (int64_t)p * M + r);
        b = merge(b, Best{rec.x, rec.y, __float_as_int(rec.z)});
      }
      conf[r] = 1.f / b.s;
      pick[r] = b.idx;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) ctr[CTR_CONF_M] += 1u;
}

static Peers to_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(!v.empty() && v.size() <= (size_t)MAXW, "tp: 1..8 ranks");
  Peers p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = v[i];
  return p;
}

}  // namespace tp

void tp_reduce_norm_push(const std::vector<int64_t>& peers, int64_t rank, int64_t R, int64_t D, int64_t part_off,
                         at::Tensor& h, bool has_partials, const at::Tensor& w1, double eps, int64_t gather_off,
                         int64_t flag_off, at::Tensor& ctr, double timeout_s, bool do_push, int64_t nslots) {
  TORCH_CHECK(h.is_contiguous() && h.scalar_type() == at::kBFloat16 && h.numel() == R * D, "tp: h [R, D] bf16");
  TORCH_CHECK(w1.is_contiguous() && w1.scalar_type() == at::kFloat && w1.numel() == D, "tp: w1 fp32 [D]");
  TORCH_CHECK(D % 8 == 0 && D <= 8 * 256 * 4, "tp: D % 8 == 0 and D <= 8192");
  TORCH_CHECK(ctr.scalar_type() == at::kInt && ctr.numel() >= 16, "tp: int32 counters [16]");
  c10::cuda::CUDAGuard g(h.device());
  tp::reduce_norm_push_kernel<<<(int)R, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tp::to_peers(peers), (int)peers.size(), (int)rank, (int)R, (int)D, part_off,
      reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), has_partials ? 1 : 0, w1.data_ptr<float>(), (float)eps,
      gather_off, flag_off, reinterpret_cast<unsigned*>(ctr.data_ptr<int>()), error_word_ptr(),
      (uint64_t)(timeout_s * 1e9), do_push ? 1 : 0, (int)(nslots > 0 ? nslots : (int64_t)peers.size()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_confidence(const std::vector<int64_t>& peers, int64_t rank, const at::Tensor& logits, int64_t v0,
                   int64_t conf_off, int64_t flag_off, at::Tensor& ctr, at::Tensor& conf, at::Tensor& pick,
                   double timeout_s) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16,
              "tp_confidence: bf16 logits [M, Vslice]");
  const int M = logits.size(0);
  TORCH_CHECK(conf.numel() >= M && pick.numel() >= M && conf.scalar_type() == at::kFloat &&
                  pick.scalar_type() == at::kLong,
              "tp_confidence: outputs");
  c10::cuda::CUDAGuard g(logits.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const tp::Peers P = tp::to_peers(peers);
  unsigned* c = reinterpret_cast<unsigned*>(ctr.data_ptr<int>());
  tp::conf_push_kernel<<<M, 512, 0, st>>>(P, (int)peers.size(), (int)rank,
                                          reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
                                          (int)logits.size(1), (int)v0, conf_off, flag_off, c);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  tp::conf_merge_kernel<<<1, 256, 0, st>>>(P, (int)peers.size(), (int)rank, M, conf_off, flag_off, c,
                                           conf.data_ptr<float>(), pick.data_ptr<int64_t>(), error_word_ptr(),
                                           (uint64_t)(timeout_s * 1e9));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bdllm
