// Block-diffusion decode kernels (the cached decoder's per-step device work).
//
//   conv_tail     causal depthwise conv (K = 4) + SiLU over one block per row, whose left context
//                 is the cached conv tail (the last K-1 pre-conv rows of the committed prefix);
//                 optionally writes the new tail (last K-1 rows of [tail || block]) in place
//   confidence    per logits row: softmax max probability and its argmax (first index on ties)
//                 in one pass (online max / sum of exponentials)
//   commit        the golden decoder's commit rule for every row of a batch, on the device:
//                 candidates = masked positions of the leftmost sub-block holding a mask;
//                 commit those with confidence >= threshold, else the single most confident;
//                 writes the picked ids, clears their mask bits, counts forwards and leftovers
// The rule is the reference's `decode.py:69-91`; all three replace host-side torch code.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {
namespace dec {

static inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

// ------------------------------------------------------------------------------- conv + tail
template <int K>
__global__ void conv_tail_kernel(const __nv_bfloat16* __restrict__ raw, int64_t ld, __nv_bfloat16* tail,
                                 const float* __restrict__ w, __nv_bfloat16* __restrict__ y, int T, int C,
                                 int update_tail) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= C) return;
  const int b = blockIdx.y;
  float wr[8][K];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float4 t = *reinterpret_cast<const float4*>(w + (c + e) * K);
    wr[e][0] = t.x, wr[e][1] = t.y, wr[e][2] = t.z, wr[e][3] = t.w;
  }
  const __nv_bfloat16* rb = raw + (int64_t)b * T * ld;
  __nv_bfloat16* tb = tail + (int64_t)b * (K - 1) * C;
  auto row = [&](int q) -> uint4 {  // pre-conv row q of [tail || block], q in [-(K-1), T)
    return q >= 0 ? *reinterpret_cast<const uint4*>(rb + (int64_t)q * ld + c)
                  : *reinterpret_cast<const uint4*>(tb + (int64_t)(K - 1 + q) * C + c);
  };
  for (int t = 0; t < T; ++t) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const uint4 p = row(t - (K - 1) + j);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p2[e]);
        acc[2 * e] += wr[2 * e][j] * f.x;
        acc[2 * e + 1] += wr[2 * e + 1][j] * f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) o2[e] = __floats2bfloat162_rn(silu_f(acc[2 * e]), silu_f(acc[2 * e + 1]));
    *reinterpret_cast<uint4*>(y + ((int64_t)b * T + t) * C + c) = o;
  }
  if (update_tail) {  // this thread owns these channels of the tail: read all, then write
    uint4 nt[K - 1];
#pragma unroll
    for (int r = 0; r < K - 1; ++r) nt[r] = row(T - (K - 1) + r);
#pragma unroll
    for (int r = 0; r < K - 1; ++r) *reinterpret_cast<uint4*>(tb + (int64_t)r * C + c) = nt[r];
  }
}

// ------------------------------------------------------------------------------- confidence
struct Best {
  float m;    // running max logit
  float s;    // sum exp(l - m)
  int idx;    // first index of the max
};

__device__ __forceinline__ Best merge(Best a, Best b) {
  if (b.m > a.m || (b.m == a.m && b.idx < a.idx && b.m != -INFINITY)) {
    const Best t = a;
    a = b;
    b = t;
  }
  // a holds the larger max (or equal max with the smaller index)
  const float s = a.s + (b.m == -INFINITY ? 0.f : b.s * __expf(b.m - a.m));
  return Best{a.m, s, a.idx};
}

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

// one 16-byte vector of 8 bf16 logits starting at index i0: a single rescale of the running sum
// per vector (at the vector's first maximum) instead of a dependent update per element
__device__ __forceinline__ void absorb8(Best& b, uint4 p, int i0) {
  const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
  float x[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(p2[e]);
    x[2 * e] = f.x, x[2 * e + 1] = f.y;
  }
  float mx = x[0];
  int am = 0;
#pragma unroll
  for (int e = 1; e < 8; ++e)
    if (x[e] > mx) mx = x[e], am = e;  // strict: the first index of the vector's max
  if (mx > b.m) {  // strict: an equal max keeps the thread's earlier index
    b.s = b.m == -INFINITY ? 0.f : b.s * __expf(b.m - mx);
    b.m = mx;
    b.idx = i0 + am;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) b.s += __expf(x[e] - b.m);
}

template <typename T>
__global__ void __launch_bounds__(512) confidence_kernel(const T* __restrict__ logits, int64_t ld, int V,
                                                         float* __restrict__ conf, int64_t* __restrict__ pick,
                                                         int vec) {
  const T* row = logits + (int64_t)blockIdx.x * ld;
  Best b{-INFINITY, 0.f, 0x7fffffff};
  if constexpr (sizeof(T) == 2) {
    if (vec) {  // bf16 rows of a multiple of 8 logits, 16-byte aligned
      const uint4* rv = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
      for (int j = threadIdx.x; j < V / 8; j += blockDim.x) absorb8(b, rv[j], j * 8);
      V = 0;  // nothing left for the element loop
    }
  }
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = to_f<T>(row[i]);
    if (x > b.m) {
      b.s = (b.m == -INFINITY ? 0.f : b.s * __expf(b.m - x)) + 1.f;
      b.m = x;
      b.idx = i;
    } else {
      b.s += __expf(x - b.m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best t{__shfl_xor_sync(0xffffffffu, b.m, o), __shfl_xor_sync(0xffffffffu, b.s, o),
           __shfl_xor_sync(0xffffffffu, b.idx, o)};
    b = merge(b, t);
  }
  __shared__ Best red[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = b;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    b = lane < nw ? red[lane] : Best{-INFINITY, 0.f, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best t{__shfl_xor_sync(0xffffffffu, b.m, o), __shfl_xor_sync(0xffffffffu, b.s, o),
             __shfl_xor_sync(0xffffffffu, b.idx, o)};
      b = merge(b, t);
    }
    if (lane == 0) {
      conf[blockIdx.x] = 1.f / b.s;  // exp(m - m) / sum exp(l - m)
      pick[blockIdx.x] = b.idx;
    }
  }
}

// ------------------------------------------------------------------------------- commit
// One warp per row; lane i = block position i (T <= 32).
__global__ void commit_kernel(const float* __restrict__ conf, const int64_t* __restrict__ pick,
                              uint8_t* __restrict__ masked, int64_t* __restrict__ ids, int T, float threshold,
                              int sub_block, int* __restrict__ forwards, int* __restrict__ remaining) {
  const int r = blockIdx.x, i = threadIdx.x;
  const bool valid = i < T;
  const int64_t o = (int64_t)r * T + i;
  const bool m = valid && masked[o] != 0;
  const unsigned mbits = __ballot_sync(0xffffffffu, m);
  if (mbits == 0u) {
    if (i == 0) remaining[r] = 0;
    return;
  }
  bool cand = m;
  if (sub_block > 0) {
    const int first = __ffs(mbits) - 1;
    const int s0 = (first / sub_block) * sub_block;
    cand = cand && i >= s0 && i < s0 + sub_block;
  }
  const float c = cand ? conf[o] : -1.f;
  bool commit = cand && c >= threshold;
  if (__ballot_sync(0xffffffffu, commit) == 0u) {  // none above threshold: the most confident one
    float best = c;
    int bi = i;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, d);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
      if (ob > best || (ob == best && oi < bi)) best = ob, bi = oi;
    }
    commit = (i == bi);
  }
  if (commit) {
    ids[o] = pick[o];
    masked[o] = 0;
  }
  const unsigned left = __ballot_sync(0xffffffffu, m && !commit);
  if (i == 0) {
    forwards[r] += 1;
    remaining[r] = __popc(left);
  }
}

}  // namespace dec

at::Tensor conv_tail(const at::Tensor& raw, at::Tensor& tail, const at::Tensor& w, bool update_tail) {
  TORCH_CHECK(raw.dim() == 3 && raw.stride(-1) == 1 && raw.scalar_type() == at::kBFloat16, "conv_tail: raw [B, T, C]");
  const int B = raw.size(0), T = raw.size(1), C = raw.size(2), K = w.size(1);
  TORCH_CHECK(K == 4 && C % 8 == 0 && raw.stride(1) % 8 == 0 && raw.stride(0) == (int64_t)T * raw.stride(1),
              "conv_tail: K = 4, C % 8 == 0, mergeable rows");
  TORCH_CHECK(tail.is_contiguous() && tail.scalar_type() == at::kBFloat16 && tail.size(0) == B &&
                  tail.size(1) == K - 1 && tail.size(2) == C,
              "conv_tail: tail [B, K-1, C] bf16 contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(raw.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(tail.data_ptr()) % 16 == 0,
              "conv_tail: raw and tail at 16-byte aligned bases (read in 16-byte vectors)");
  auto wf = w.reshape({C, K}).to(at::kFloat).contiguous();
  if (reinterpret_cast<uintptr_t>(wf.data_ptr()) % 16 != 0) wf = wf.clone();  // read as float4
  auto y = at::empty({B, T, C}, raw.options());
  c10::cuda::CUDAGuard g(raw.device());
  dec::conv_tail_kernel<4><<<dim3((C / 8 + 127) / 128, B), 128, 0, dec::stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(raw.data_ptr()), raw.stride(1),
      reinterpret_cast<__nv_bfloat16*>(tail.data_ptr()), wf.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), T, C, update_tail ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

void confidence(const at::Tensor& logits, at::Tensor& conf, at::Tensor& pick) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "confidence: logits [R, V] with unit inner stride");
  const int R = logits.size(0), V = logits.size(1);
  TORCH_CHECK(conf.is_contiguous() && conf.scalar_type() == at::kFloat && conf.numel() >= R, "confidence: conf fp32");
  TORCH_CHECK(pick.is_contiguous() && pick.scalar_type() == at::kLong && pick.numel() >= R, "confidence: pick int64");
  c10::cuda::CUDAGuard g(logits.device());
  if (logits.scalar_type() == at::kFloat)
    dec::confidence_kernel<float><<<R, 512, 0, dec::stream()>>>(logits.data_ptr<float>(), logits.stride(0), V,
                                                                 conf.data_ptr<float>(), pick.data_ptr<int64_t>(), 0);
  else {
    TORCH_CHECK(logits.scalar_type() == at::kBFloat16, "confidence: fp32 or bf16 logits");
    const int vec = V % 8 == 0 && logits.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0;
    dec::confidence_kernel<__nv_bfloat16><<<R, 512, 0, dec::stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V, conf.data_ptr<float>(),
        pick.data_ptr<int64_t>(), vec);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void commit(const at::Tensor& conf, const at::Tensor& pick, at::Tensor& masked, at::Tensor& ids, double threshold,
            int64_t sub_block, at::Tensor& forwards, at::Tensor& remaining) {
  TORCH_CHECK(ids.dim() == 2 && ids.is_contiguous() && ids.scalar_type() == at::kLong, "commit: ids [B, T] int64");
  const int B = ids.size(0), T = ids.size(1);
  TORCH_CHECK(T <= 32, "commit: block <= 32");
  TORCH_CHECK(masked.is_contiguous() && masked.numel() == (int64_t)B * T &&
                  (masked.scalar_type() == at::kBool || masked.scalar_type() == at::kByte),
              "commit: masked [B, T] bool");
  TORCH_CHECK(conf.numel() == (int64_t)B * T && pick.numel() == (int64_t)B * T, "commit: conf/pick [B, T]");
  TORCH_CHECK(forwards.scalar_type() == at::kInt && remaining.scalar_type() == at::kInt && forwards.numel() >= B &&
                  remaining.numel() >= B,
              "commit: int32 counters [B]");
  c10::cuda::CUDAGuard g(ids.device());
  dec::commit_kernel<<<B, 32, 0, dec::stream()>>>(conf.data_ptr<float>(), pick.data_ptr<int64_t>(),
                                                  reinterpret_cast<uint8_t*>(masked.data_ptr()), ids.data_ptr<int64_t>(),
                                                  T, (float)threshold, (int)sub_block, forwards.data_ptr<int>(),
                                                  remaining.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bdllm
