// Symmetric peer memory over NVLink / NVSwitch and the collectives built on it.
// (Reference: FSDP2's NCCL all-gather / fp32 reduce-scatter per unit, `src/dllm_qwen38/fsdp_train.py:133-171`,
// and the all_reduce of replicated gradients, `fsdp_train.py:207-221`.)
//
// A symmetric heap is one cudaMalloc region of the same size on every rank of a node, exported
// with a CUDA IPC handle and opened by every other rank; the ranks carve it up with identical
// allocation sequences, so an object at byte offset `o` of rank r's heap is at `peers[r] + o` from
// anywhere. Kernels here read peers' memory with plain 16-byte loads (L1 bypassed) and publish
// progress with release stores of 32-bit sequence numbers into the peers' flag rows; every wait
// for a peer is bounded by %globaltimer and the host-given timeout, after which the kernel records
// ERR_COMM_WAIT in the error word and returns (a kernel that finds the error word already set
// skips its work). No TMA is used here, and no multicast of any kind.
//
// Heap header (first 64 KiB of every heap):
//   flags[slot][src]     u32, slot < 16, src < 16   written by rank `src` into this rank's heap
//   counters[16]         u32                          this rank's own block-arrival counters
//   xchg[2][16][64]      f32                          small all-reduce exchange, double buffered
//
// Collectives (used by the sharded training engine, one launch each):
//   all_gather      out[p*S : (p+1)*S] = shard of rank p     (waits for every peer's param epoch)
//   reduce_scatter  out = scale * sum_p grad_p[r*S : (r+1)*S] in fp32, bf16 or fp32 input, with the
//                   sum of squares of `out` added to a device scalar (the global-norm clip input);
//                   ends when every peer has finished reading this rank's buffer
//   allreduce_f32   a few floats summed over ranks in rank order (identical on every rank)
//   signal          publish a value in one slot of every peer's flag row
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
namespace peer {

constexpr int kSlots = 16;
constexpr int kMaxWorld = 16;
constexpr int64_t kFlagsOff = 0;
constexpr int64_t kCountersOff = kSlots * kMaxWorld * 4;             // 1024
constexpr int64_t kXchgOff = kCountersOff + 16 * 4 + 960;            // 2048
constexpr int kXchgN = 64;
constexpr int64_t kHeaderBytes = 64 * 1024;

enum Slot : int { SLOT_EPOCH = 0, SLOT_RS_READY = 1, SLOT_RS_DONE = 2, SLOT_AR = 3 };
enum Counter : int { CTR_RS = 0 };

struct Ptrs {
  int64_t p[kMaxWorld];
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned* flag_row(int64_t base, int slot) {
  return reinterpret_cast<unsigned*>(base + kFlagsOff) + slot * kMaxWorld;
}

// Wait until flags[0..world) of `row` (this rank's memory) all reach `target` (wrap-safe).
__device__ bool wait_all(const unsigned* row, int world, unsigned target, int* err, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer();
  for (int p = 0; p < world; ++p) {
    while (static_cast<int>(ld_acquire_sys(row + p) - target) < 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (globaltimer() - t0 > timeout_ns) {
        record_error(err, ERR_COMM_WAIT);
        return false;
      }
      __nanosleep(100);
    }
  }
  return true;
}

// Every peer's flag row `slot`, entry [rank] := v, after all of this thread's (and, through a
// preceding __syncthreads, this block's) prior writes are visible system-wide.
__device__ void signal_all(const Ptrs& peers, int world, int rank, int slot, unsigned v) {
  __threadfence_system();
  for (int p = 0; p < world; ++p) st_release_sys(flag_row(peers.p[p], slot) + rank, v);
}

__device__ __forceinline__ uint4 ldcg16(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void bf16x8_to_f(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// ---------------------------------------------------------------------------------- kernels

__global__ void signal_kernel(Ptrs peers, int world, int rank, int slot, unsigned v) {
  if (threadIdx.x == 0 && blockIdx.x == 0) signal_all(peers, world, rank, slot, v);
}

// out[p * nvec + j] = peer p's shard vector j (16-byte vectors), after every peer's SLOT_EPOCH
// flag (in this rank's row) reached `epoch`.
__global__ void __launch_bounds__(512) all_gather_kernel(Ptrs peers, int world, int rank, int64_t src_off,
                                                         int64_t nvec, uint4* __restrict__ out, unsigned epoch,
                                                         int* err, uint64_t timeout_ns) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = (*reinterpret_cast<volatile int*>(err) == 0) &&
                             wait_all(flag_row(peers.p[rank], SLOT_EPOCH), world, epoch, err, timeout_ns);
  __syncthreads();
  if (!ok) return;
  const int64_t total = nvec * world;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  constexpr int U = 4;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; base < total;
       base += stride * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + u * stride;
      if (i < total) {
        // rotate the peer order by rank so that the ranks start on different peers
        const int q = static_cast<int>(i / nvec);
        const int p = (q + rank) % world;
        const int64_t j = i - static_cast<int64_t>(q) * nvec;
        v[u] = ldcg16(reinterpret_cast<const char*>(peers.p[p] + src_off) + j * 16);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + u * stride;
      if (i < total) {
        const int q = static_cast<int>(i / nvec);
        const int p = (q + rank) % world;
        out[static_cast<int64_t>(p) * nvec + (i - static_cast<int64_t>(q) * nvec)] = v[u];
      }
    }
  }
}

// Bytes [lo, hi) (16-byte aligned) of the gathered buffer: byte x comes from rank x / shard_bytes.
__global__ void gather_range_kernel(Ptrs peers, int world, int rank, int64_t src_off, int64_t shard_bytes, int64_t lo,
                                    int64_t hi, char* __restrict__ out, unsigned epoch, int* err,
                                    uint64_t timeout_ns) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = (*reinterpret_cast<volatile int*>(err) == 0) &&
                             wait_all(flag_row(peers.p[rank], SLOT_EPOCH), world, epoch, err, timeout_ns);
  __syncthreads();
  if (!ok) return;
  for (int64_t x = lo + ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 16; x < hi;
       x += (int64_t)gridDim.x * blockDim.x * 16) {
    const int p = (int)(x / shard_bytes);
    *reinterpret_cast<uint4*>(out + x) = ldcg16(reinterpret_cast<const char*>(peers.p[p] + src_off) + x % shard_bytes);
  }
}

// AdamW fused into the reduce-scatter (runs without gradient clipping): the averaged gradient
// never leaves registers; master/moments are fp32 shards, p the bf16 parameter shard.
struct Adam {
  float* w;
  float* m;
  float* v;
  __nv_bfloat16* p;
  float lr, b1, b2, eps, wd, bc1, bc2;
};


// out[i] = scale * sum_p in_p[rank * shard + i] (fp32), sq += sum_i out[i]^2; with A.w set, the
// AdamW update of element i is applied right away instead (out may then be null).
template <typename TIn>
__global__ void __launch_bounds__(512) reduce_scatter_kernel(Ptrs peers, int world, int rank, int64_t src_off,
                                                             int64_t shard, float* __restrict__ out, float scale,
                                                             float* __restrict__ sq, unsigned seq, int* err,
                                                             uint64_t timeout_ns, Adam A) {
  constexpr int EPV = 16 / sizeof(TIn);  // elements per 16-byte vector
  __shared__ int ok;
  __shared__ float red[16];
  if (threadIdx.x == 0) {
    ok = *reinterpret_cast<volatile int*>(err) == 0;
    if (ok) {
      signal_all(peers, world, rank, SLOT_RS_READY, seq);
      ok = wait_all(flag_row(peers.p[rank], SLOT_RS_READY), world, seq, err, timeout_ns);
    }
  }
  __syncthreads();
  float acc2 = 0.f;
  if (ok) {
    const int64_t nvec = shard / EPV;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t off = src_off + static_cast<int64_t>(rank) * shard * sizeof(TIn);
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint4 raw[kMaxWorld];
#pragma unroll
      for (int p = 0; p < kMaxWorld; ++p)
        if (p < world) raw[p] = ldcg16(reinterpret_cast<const char*>(peers.p[p] + off) + v * 16);
#pragma unroll
      for (int p = 0; p < kMaxWorld; ++p) {
        if (p < world) {
          if constexpr (sizeof(TIn) == 2) {
            float f[8];
            bf16x8_to_f(raw[p], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) s[e] += f[e];
          } else {
            const float* f = reinterpret_cast<const float*>(&raw[p]);
#pragma unroll
            for (int e = 0; e < 4; ++e) s[e] += f[e];
          }
        }
      }
#pragma unroll
      for (int e = 0; e < EPV; ++e) {
        s[e] *= scale;
        acc2 += s[e] * s[e];
      }
      if (A.w != nullptr) {  // vectorised AdamW on EPV consecutive elements
        const int64_t i0 = v * EPV;
        float w[8], m[8], vv[8];
#pragma unroll
        for (int q = 0; q < EPV / 4; ++q) {
          const float4 a4 = reinterpret_cast<const float4*>(A.w + i0)[q];
          const float4 m4 = reinterpret_cast<const float4*>(A.m + i0)[q];
          const float4 v4 = reinterpret_cast<const float4*>(A.v + i0)[q];
          w[4 * q] = a4.x, w[4 * q + 1] = a4.y, w[4 * q + 2] = a4.z, w[4 * q + 3] = a4.w;
          m[4 * q] = m4.x, m[4 * q + 1] = m4.y, m[4 * q + 2] = m4.z, m[4 * q + 3] = m4.w;
          vv[4 * q] = v4.x, vv[4 * q + 1] = v4.y, vv[4 * q + 2] = v4.z, vv[4 * q + 3] = v4.w;
        }
        __nv_bfloat16 pb[8];
#pragma unroll
        for (int e = 0; e < EPV; ++e) {
          float wi = w[e];
          if (A.wd != 0.f) wi *= 1.f - A.lr * A.wd;
          m[e] = A.b1 * m[e] + (1.f - A.b1) * s[e];
          vv[e] = A.b2 * vv[e] + (1.f - A.b2) * s[e] * s[e];
          wi -= A.lr * (m[e] / A.bc1) / (sqrtf(vv[e] / A.bc2) + A.eps);
          w[e] = wi;
          pb[e] = __float2bfloat16(wi);
        }
#pragma unroll
        for (int q = 0; q < EPV / 4; ++q) {
          reinterpret_cast<float4*>(A.w + i0)[q] = make_float4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          reinterpret_cast<float4*>(A.m + i0)[q] = make_float4(m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3]);
          reinterpret_cast<float4*>(A.v + i0)[q] =
              make_float4(vv[4 * q], vv[4 * q + 1], vv[4 * q + 2], vv[4 * q + 3]);
        }
        if constexpr (EPV == 8)
          *reinterpret_cast<uint4*>(A.p + i0) = *reinterpret_cast<const uint4*>(pb);
        else
          *reinterpret_cast<uint2*>(A.p + i0) = *reinterpret_cast<const uint2*>(pb);
      } else {
        float4* o = reinterpret_cast<float4*>(out + v * EPV);
        o[0] = make_float4(s[0], s[1], s[2], s[3]);
        if constexpr (EPV == 8) o[1] = make_float4(s[4], s[5], s[6], s[7]);
      }
    }
  }
  // block sum of squares
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) acc2 += __shfl_xor_sync(0xffffffffu, acc2, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc2;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    if (sq != nullptr && ok) atomicAdd(sq, t);
    // the last block to finish tells the peers that this rank is done reading their buffers, then
    // waits until every peer is done reading this rank's buffer (the caller may then reuse it)
    __threadfence();
    unsigned* ctr = reinterpret_cast<unsigned*>(peers.p[rank] + kCountersOff) + CTR_RS;
    const unsigned prev = atomicAdd(ctr, 1u);
    if (prev == gridDim.x - 1) {
      *ctr = 0u;
      if (*reinterpret_cast<volatile int*>(err) == 0) {
        signal_all(peers, world, rank, SLOT_RS_DONE, seq);
        wait_all(flag_row(peers.p[rank], SLOT_RS_DONE), world, seq, err, timeout_ns);
      }
    }
  }
}

// out[i] = sum_p vals_p[i], i < n <= 64, summed in rank order on every rank.
__global__ void allreduce_f32_kernel(Ptrs peers, int world, int rank, const float* __restrict__ vals, int n,
                                     float* __restrict__ out, unsigned seq, int* err, uint64_t timeout_ns) {
  __shared__ int ok;
  const int half = seq & 1u;
  const int i = threadIdx.x;
  if (i == 0) ok = *reinterpret_cast<volatile int*>(err) == 0;
  __syncthreads();
  if (!ok) return;
  if (i < n) {
    const float v = vals[i];
    for (int p = 0; p < world; ++p) {
      float* x = reinterpret_cast<float*>(peers.p[p] + kXchgOff) + (half * kMaxWorld + rank) * kXchgN;
      x[i] = v;
    }
  }
  __syncthreads();
  if (i == 0) {
    signal_all(peers, world, rank, SLOT_AR, seq);
    ok = wait_all(flag_row(peers.p[rank], SLOT_AR), world, seq, err, timeout_ns);
  }
  __syncthreads();
  if (!ok) return;
  if (i < n) {
    float s = 0.f;
    const float* x = reinterpret_cast<const float*>(peers.p[rank] + kXchgOff) + half * kMaxWorld * kXchgN;
    for (int p = 0; p < world; ++p) s += __ldcg(x + p * kXchgN + i);
    out[i] = s;
  }
}

// ---------------------------------------------------------------------------------- host

static Ptrs to_ptrs(const std::vector<int64_t>& v) {
  TORCH_CHECK(!v.empty() && v.size() <= static_cast<size_t>(kMaxWorld), "peer: 1..16 ranks");
  Ptrs p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = v[i];
  return p;
}

static int grid_for(int64_t work, int threads, int cap) {
  int64_t g = (work + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(g, cap)));
}

int64_t alloc(int64_t bytes) {
  TORCH_CHECK(bytes > kHeaderBytes, "peer heap smaller than its header");
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, bytes));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  return reinterpret_cast<int64_t>(p);
}

at::Tensor handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  at::Tensor t = at::empty({static_cast<int64_t>(sizeof(h))}, at::TensorOptions().dtype(at::kByte));
  memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t open(const at::Tensor& h) {
  TORCH_CHECK(h.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)) && h.device().is_cpu(),
              "peer.open: a 64-byte CPU handle");
  cudaIpcMemHandle_t mh;
  memcpy(&mh, h.contiguous().data_ptr(), sizeof(mh));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, mh, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

void release(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

at::Tensor view(int64_t ptr, int64_t numel, const at::Tensor& like) {
  TORCH_CHECK(like.is_cuda(), "peer.view: `like` gives the device and dtype");
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {}, like.options());
}

void signal(const std::vector<int64_t>& peers, int64_t rank, int64_t slot, int64_t value) {
  const Ptrs P = to_ptrs(peers);
  signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(P, static_cast<int>(peers.size()),
                                                                  static_cast<int>(rank), static_cast<int>(slot),
                                                                  static_cast<unsigned>(value));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void all_gather(const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard_bytes, at::Tensor& out,
                int64_t epoch, int64_t max_blocks, double timeout_s) {
  const int world = static_cast<int>(peers.size());
  TORCH_CHECK(shard_bytes % 16 == 0 && src_off % 16 == 0, "all_gather: 16-byte shards");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.data_ptr() != nullptr &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "all_gather: aligned contiguous output");
  TORCH_CHECK(out.numel() * out.element_size() >= shard_bytes * world, "all_gather: output too small");
  const int64_t nvec = shard_bytes / 16;
  const int grid = grid_for(nvec * world, 512 * 4, static_cast<int>(max_blocks));
  all_gather_kernel<<<grid, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      to_ptrs(peers), world, static_cast<int>(rank), src_off, nvec, reinterpret_cast<uint4*>(out.data_ptr()),
      static_cast<unsigned>(epoch), error_word_ptr(), static_cast<uint64_t>(timeout_s * 1e9));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gather_range(const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard_bytes, at::Tensor& out,
                  int64_t lo, int64_t hi, int64_t epoch, double timeout_s) {
  lo = lo / 16 * 16;
  hi = (hi + 15) / 16 * 16;
  const int world = (int)peers.size();
  TORCH_CHECK(shard_bytes % 16 == 0 && src_off % 16 == 0 && hi <= shard_bytes * world && lo >= 0 && lo < hi,
              "gather_range: bounds");
  TORCH_CHECK(out.is_cuda() && out.numel() * out.element_size() >= hi &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "gather_range: output");
  const int grid = grid_for((hi - lo) / 16, 256, 64);
  gather_range_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      to_ptrs(peers), world, (int)rank, src_off, shard_bytes, lo, hi, reinterpret_cast<char*>(out.data_ptr()),
      (unsigned)epoch, error_word_ptr(), (uint64_t)(timeout_s * 1e9));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void reduce_scatter(const std::vector<int64_t>& peers, int64_t rank, int64_t src_off, int64_t shard, bool in_f32,
                    at::Tensor& out, double scale, const c10::optional<at::Tensor>& sq, int64_t seq,
                    int64_t max_blocks, double timeout_s, const std::vector<at::Tensor>& adam_state,
                    const std::vector<double>& adam_hp) {
  Adam A{};
  if (!adam_state.empty()) {  // {master, m, v, p} and {lr, b1, b2, eps, wd, bc1, bc2}
    TORCH_CHECK(adam_state.size() == 4 && adam_hp.size() == 7, "reduce_scatter: adam state/hyper-parameters");
    for (int i = 0; i < 3; ++i)
      TORCH_CHECK(adam_state[i].scalar_type() == at::kFloat && adam_state[i].numel() >= shard, "adam: fp32 shards");
    TORCH_CHECK(adam_state[3].scalar_type() == at::kBFloat16 && adam_state[3].numel() >= shard, "adam: bf16 shard");
    A.w = adam_state[0].data_ptr<float>();
    A.m = adam_state[1].data_ptr<float>();
    A.v = adam_state[2].data_ptr<float>();
    A.p = reinterpret_cast<__nv_bfloat16*>(adam_state[3].data_ptr());
    A.lr = (float)adam_hp[0], A.b1 = (float)adam_hp[1], A.b2 = (float)adam_hp[2], A.eps = (float)adam_hp[3];
    A.wd = (float)adam_hp[4], A.bc1 = (float)adam_hp[5], A.bc2 = (float)adam_hp[6];
  }
  const int world = static_cast<int>(peers.size());
  const int esz = in_f32 ? 4 : 2;
  TORCH_CHECK((shard * esz) % 16 == 0 && src_off % 16 == 0, "reduce_scatter: 16-byte shards");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() >= shard &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "reduce_scatter: fp32 aligned output of >= shard elements");
  float* sqp = nullptr;
  if (sq.has_value()) {
    TORCH_CHECK(sq->is_cuda() && sq->scalar_type() == at::kFloat, "reduce_scatter: fp32 sq accumulator");
    sqp = sq->data_ptr<float>();
  }
  const int64_t nvec = shard * esz / 16;
  const int grid = grid_for(nvec, 512, static_cast<int>(max_blocks));
  auto stream = at::cuda::getCurrentCUDAStream();
  const Ptrs P = to_ptrs(peers);
  const uint64_t tmo = static_cast<uint64_t>(timeout_s * 1e9);
  if (in_f32)
    reduce_scatter_kernel<float><<<grid, 512, 0, stream>>>(P, world, static_cast<int>(rank), src_off, shard,
                                                           out.data_ptr<float>(), static_cast<float>(scale), sqp,
                                                           static_cast<unsigned>(seq), error_word_ptr(), tmo, A);
  else
    reduce_scatter_kernel<__nv_bfloat16><<<grid, 512, 0, stream>>>(
        P, world, static_cast<int>(rank), src_off, shard, out.data_ptr<float>(), static_cast<float>(scale), sqp,
        static_cast<unsigned>(seq), error_word_ptr(), tmo, A);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void allreduce_f32(const std::vector<int64_t>& peers, int64_t rank, const at::Tensor& vals, at::Tensor& out,
                   int64_t seq, double timeout_s) {
  TORCH_CHECK(vals.is_cuda() && vals.scalar_type() == at::kFloat && vals.is_contiguous() && vals.numel() <= kXchgN,
              "allreduce_f32: <= 64 contiguous fp32 values");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.numel() >= vals.numel(), "allreduce_f32: out");
  allreduce_f32_kernel<<<1, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      to_ptrs(peers), static_cast<int>(peers.size()), static_cast<int>(rank), vals.data_ptr<float>(),
      static_cast<int>(vals.numel()), out.data_ptr<float>(), static_cast<unsigned>(seq), error_word_ptr(),
      static_cast<uint64_t>(timeout_s * 1e9));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace peer
}  // namespace bdllm
