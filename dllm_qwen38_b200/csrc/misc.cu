// Memory-bound kernels of the training step:
//   dswiglu        dgate/dup from d(act) and the stored bf16 (gate | up)
//   conv_fwd/bwd   the state-fork short causal conv + SiLU over the [B, 2L, C] two-stream layout
//   ce_rows        per-row log-sum-exp over the vocabulary, loss, and dlogits written in place
//   adamw          fused clip-scale + AdamW on fp32 master weights, bf16 parameter write-back
//   group_sum      GQA: per-v-head gradients summed over each k-head's group, bf16 in and out
//   mask_sample    the complementary masks of a step and both noised views, one launch
// (Reference paths: mask sampling `src/dllm_qwen38/objective.py:26-57`, masked CE `objective.py:60-84`,
// AdamW `fsdp_train.py:779`, conv + SiLU `gdn.py:217-219`, gates `gdn.py:225-226`, embedding
// `blockdiff.py:140-141`.)
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <utility>

#include "common.cuh"

namespace bdllm {

static inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }
static inline const __nv_bfloat16* cbf(const at::Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr());
}
static inline __nv_bfloat16* bfp(at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
// the kernels below move bf16 / fp32 data in 16-byte vectors: base addresses must be 16-byte aligned
static inline bool al16(const at::Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; }
// a contiguous input whose base is 16-byte aligned: the tensor itself, or a copy when a view's
// offset breaks the alignment
static inline at::Tensor vec_input(const at::Tensor& t) {
  auto c = t.contiguous();
  return al16(c) ? c : c.clone();
}

// ------------------------------------------------------------------------------- dswiglu
// act = silu(g) * u; dg = dact * u * silu'(g), du = dact * silu(g). gu rows [g (F) | u (F)].
__global__ void dswiglu_kernel(const __nv_bfloat16* __restrict__ dact, const __nv_bfloat16* __restrict__ gu,
                               __nv_bfloat16* __restrict__ dgu, int64_t rows, int F) {
  const int64_t n = rows * (int64_t)(F / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (F / 8);
    const int c = (int)(i % (F / 8)) * 8;
    uint4 da = *reinterpret_cast<const uint4*>(dact + r * F + c);
    uint4 gg = *reinterpret_cast<const uint4*>(gu + r * 2 * F + c);
    uint4 uu = *reinterpret_cast<const uint4*>(gu + r * 2 * F + F + c);
    const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&da);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gg);
    const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uu);
    uint4 og, ou;
    __nv_bfloat162* og2 = reinterpret_cast<__nv_bfloat162*>(&og);
    __nv_bfloat162* ou2 = reinterpret_cast<__nv_bfloat162*>(&ou);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 d = __bfloat1622float2(d2[e]), g = __bfloat1622float2(g2[e]), u = __bfloat1622float2(u2[e]);
      float sx = sigmoid_f(g.x), sy = sigmoid_f(g.y);
      float dgx = d.x * u.x * sx * (1.f + g.x * (1.f - sx));
      float dgy = d.y * u.y * sy * (1.f + g.y * (1.f - sy));
      og2[e] = __floats2bfloat162_rn(dgx, dgy);
      ou2[e] = __floats2bfloat162_rn(d.x * g.x * sx, d.y * g.y * sy);
    }
    *reinterpret_cast<uint4*>(dgu + r * 2 * F + c) = og;
    *reinterpret_cast<uint4*>(dgu + r * 2 * F + F + c) = ou;
  }
}

at::Tensor dswiglu(const at::Tensor& dact, const at::Tensor& gu) {
  const int F = dact.size(-1);
  TORCH_CHECK(F % 8 == 0 && gu.size(-1) == 2 * F && gu.scalar_type() == at::kBFloat16, "dswiglu: shapes");
  auto d = vec_input(dact.to(at::kBFloat16));
  auto g = vec_input(gu);
  const int64_t rows = d.numel() / F;
  TORCH_CHECK(g.numel() == rows * 2 * F, "dswiglu: d(act) and (gate | up) rows differ");
  auto out = at::empty({rows, 2 * F}, gu.options());
  if (rows == 0) return out;
  c10::cuda::CUDAGuard guard(gu.device());
  const int64_t n = rows * (F / 8);
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  dswiglu_kernel<<<grid, 256, 0, stream()>>>(cbf(d), cbf(g), bfp(out), rows, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// act = silu(g) * u from the stored bf16 (gate | up), the value the SwiGLU GEMM epilogue wrote
// (same rounding: the epilogue applies silu to the bf16-rounded gate and up)
__global__ void swiglu_act_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ act,
                                  int64_t rows, int F) {
  const int64_t n = rows * (int64_t)(F / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (F / 8);
    const int c = (int)(i % (F / 8)) * 8;
    const uint4 gg = *reinterpret_cast<const uint4*>(gu + r * 2 * F + c);
    const uint4 uu = *reinterpret_cast<const uint4*>(gu + r * 2 * F + F + c);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gg);
    const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uu);
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 g = __bfloat1622float2(g2[e]), u = __bfloat1622float2(u2[e]);
      o2[e] = __floats2bfloat162_rn(silu_f(g.x) * u.x, silu_f(g.y) * u.y);
    }
    *reinterpret_cast<uint4*>(act + r * F + c) = o;
  }
}

at::Tensor swiglu_act(const at::Tensor& gu) {
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16 && gu.dim() >= 1 && gu.size(-1) % 16 == 0,
              "swiglu_act: bf16 [..., 2F], F % 8 == 0");
  const int F = gu.size(-1) / 2;
  auto gc = vec_input(gu);
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto out = at::empty(sizes, gu.options());
  const int64_t rows = gu.numel() / (2 * F);
  if (rows == 0) return out;
  c10::cuda::CUDAGuard g(gu.device());
  const int64_t n = rows * (F / 8);
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  swiglu_act_kernel<<<grid, 256, 0, stream()>>>(cbf(gc), bfp(out), rows, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Attention output gate: y = o * sigmoid(g) over rows of D (o and y contiguous, g with row stride
// ldg: the gate half of the q|gate projection read in place); backward do = dy s,
// dg = dy o s (1 - s), s recomputed. 8 elements per thread.
__global__ void out_gate_fwd_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ g,
                                    int64_t ldg, __nv_bfloat16* __restrict__ y, int64_t rows, int D) {
  const int64_t n = rows * (int64_t)(D / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (D / 8);
    const int c = (int)(i % (D / 8)) * 8;
    const uint4 ov = *reinterpret_cast<const uint4*>(o + r * D + c);
    const uint4 gv = *reinterpret_cast<const uint4*>(g + r * ldg + c);
    const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
    uint4 out;
    __nv_bfloat162* y2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 of = __bfloat1622float2(o2[e]), gf = __bfloat1622float2(g2[e]);
      y2[e] = __floats2bfloat162_rn(of.x * sigmoid_f(gf.x), of.y * sigmoid_f(gf.y));
    }
    *reinterpret_cast<uint4*>(y + r * D + c) = out;
  }
}

__global__ void out_gate_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ o,
                                    const __nv_bfloat16* __restrict__ g, int64_t ldg, __nv_bfloat16* __restrict__ dout,
                                    __nv_bfloat16* __restrict__ dg, int64_t rows, int D) {
  const int64_t n = rows * (int64_t)(D / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (D / 8);
    const int c = (int)(i % (D / 8)) * 8;
    const uint4 dv = *reinterpret_cast<const uint4*>(dy + r * D + c);
    const uint4 ov = *reinterpret_cast<const uint4*>(o + r * D + c);
    const uint4 gv = *reinterpret_cast<const uint4*>(g + r * ldg + c);
    const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dv);
    const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
    uint4 a, b;
    __nv_bfloat162* a2 = reinterpret_cast<__nv_bfloat162*>(&a);
    __nv_bfloat162* b2 = reinterpret_cast<__nv_bfloat162*>(&b);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 df = __bfloat1622float2(d2[e]), of = __bfloat1622float2(o2[e]), gf = __bfloat1622float2(g2[e]);
      const float sx = sigmoid_f(gf.x), sy = sigmoid_f(gf.y);
      a2[e] = __floats2bfloat162_rn(df.x * sx, df.y * sy);
      b2[e] = __floats2bfloat162_rn(df.x * of.x * sx * (1.f - sx), df.y * of.y * sy * (1.f - sy));
    }
    *reinterpret_cast<uint4*>(dout + r * D + c) = a;
    *reinterpret_cast<uint4*>(dg + r * D + c) = b;
  }
}

// the gate as rows of D at one row stride ld (row r at g + r * ld over the flattened leading dims,
// so every leading dim longer than 1 must step by ld times the rows inside it), read in place;
// otherwise a contiguous copy
static std::pair<at::Tensor, int64_t> gate_rows(const at::Tensor& g, int D) {
  if (g.dim() >= 2 && g.stride(-1) == 1 && al16(g)) {
    int64_t ld = -1, inner = 1;  // inner: rows spanned by the dims inside the current one
    bool ok = true;
    for (int d = g.dim() - 2; d >= 0 && ok; --d) {
      if (g.size(d) == 1) continue;
      if (ld < 0) ld = g.stride(d);
      else ok = g.stride(d) == ld * inner;
      inner *= g.size(d);
    }
    if (ld < 0) ld = D;  // a single row
    if (ok && ld >= D && ld % 8 == 0) return {g, ld};
  }
  return {vec_input(g), (int64_t)D};
}

at::Tensor out_gate_fwd(const at::Tensor& o, const at::Tensor& g) {
  const int D = o.size(-1);
  TORCH_CHECK(o.scalar_type() == at::kBFloat16 && g.scalar_type() == at::kBFloat16 && g.sizes() == o.sizes() &&
                  D % 8 == 0,
              "out_gate: bf16 o and gate of one shape, last dim % 8 == 0");
  auto oc = vec_input(o);
  auto [gr, ldg] = gate_rows(g, D);
  auto y = at::empty_like(oc);
  const int64_t rows = oc.numel() / D;
  if (rows == 0) return y;
  c10::cuda::CUDAGuard gd(o.device());
  const int64_t n = rows * (D / 8);
  out_gate_fwd_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, stream()>>>(
      cbf(oc), cbf(gr), ldg, bfp(y), rows, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

std::vector<at::Tensor> out_gate_bwd(const at::Tensor& dy, const at::Tensor& o, const at::Tensor& g) {
  const int D = o.size(-1);
  TORCH_CHECK(o.scalar_type() == at::kBFloat16 && g.scalar_type() == at::kBFloat16 && g.sizes() == o.sizes() &&
                  dy.numel() == o.numel() && D % 8 == 0,
              "out_gate: bf16 o and gate of one shape, dy of as many elements, last dim % 8 == 0");
  auto d = vec_input(dy.to(at::kBFloat16));
  auto oc = vec_input(o);
  auto [gr, ldg] = gate_rows(g, D);
  auto dout = at::empty_like(oc), dg = at::empty_like(oc);
  const int64_t rows = oc.numel() / D;
  if (rows == 0) return {dout, dg};
  c10::cuda::CUDAGuard gd(o.device());
  const int64_t n = rows * (D / 8);
  out_gate_bwd_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, stream()>>>(
      cbf(d), cbf(oc), cbf(gr), ldg, bfp(dout), bfp(dg), rows, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dout, dg};
}

// ------------------------------------------------------------------------------- conv
// raw [B, 2L, C] (row stride ld), w [C, K] fp32. Source position of tap j for output token t:
//   q = t - (K-1) + j in the stream's own coordinates; see source_of().
enum ConvMode : int { CONV_FORK = 0, CONV_NOPREFIX = 1, CONV_CONCAT = 2 };

// returns the [B, 2L] row index that tap q of output row t reads, or -1 for a zero
__device__ __forceinline__ int source_of(int t, int q_off, int L, int block, int mode) {
  if (mode == CONV_CONCAT) {
    int q = t + q_off;
    return q >= 0 ? q : -1;
  }
  if (t >= L) {  // clean stream: plain causal from a zero start
    int p = t - L + q_off;
    return p >= 0 ? L + p : -1;
  }
  int q = t + q_off;  // noised stream
  int s = (t / block) * block;
  if (q >= s) return q;
  if (mode == CONV_FORK && q >= 0) return L + q;  // the clean prefix before the block
  return -1;
}

// grid: x over 8-channel vectors, y over groups of CONV_ROWS rows (b * T2 + t). A thread keeps
// its 8 channels' taps (32 floats) in registers and walks its rows.
constexpr int CONV_ROWS = 16;

template <int K>
__device__ __forceinline__ void load_taps(const float* __restrict__ w, int c, float (&wr)[8][K]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float4 t = *reinterpret_cast<const float4*>(w + (c + e) * K);
    wr[e][0] = t.x, wr[e][1] = t.y, wr[e][2] = t.z, wr[e][3] = t.w;
  }
}

// the K source rows of output row t (same rule as source_of, one division per row)
template <int K>
__device__ __forceinline__ void sources_of(int t, int L, int block, int mode, int (&src)[K]) {
  if (mode == CONV_CONCAT || t >= L) {
    const int lo = (mode == CONV_CONCAT) ? 0 : L;  // first row of the stream
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int q = t + j - (K - 1);
      src[j] = q >= lo ? q : -1;
    }
    return;
  }
  const int s = (t / block) * block;  // noised stream: own block, then the clean prefix (fork)
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const int q = t + j - (K - 1);
    src[j] = q >= s ? q : ((mode == CONV_FORK && q >= 0) ? L + q : -1);
  }
}

template <int K>
__device__ __forceinline__ void conv_row(const __nv_bfloat16* __restrict__ raw, int64_t ld, const float (&wr)[8][K],
                                         int b, int t, int c, int T2, int L, int block, int mode, float (&acc)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  int src[K];
  sources_of<K>(t, L, block, mode, src);
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (src[j] < 0 || !BDLLM_IDX(src[j], T2)) continue;
    const uint4 p = *reinterpret_cast<const uint4*>(raw + ((int64_t)b * T2 + src[j]) * ld + c);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(p2[e]);
      acc[2 * e] += wr[2 * e][j] * f.x;
      acc[2 * e + 1] += wr[2 * e + 1][j] * f.y;
    }
  }
}

template <int K>
__global__ void conv_fwd_kernel(const __nv_bfloat16* __restrict__ raw, int64_t ld, const float* __restrict__ w,
                                __nv_bfloat16* __restrict__ y, int B, int T2, int C, int L, int block, int mode) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= C) return;
  float wr[8][K];
  load_taps<K>(w, c, wr);
  const int r1 = min(B * T2, (int)(blockIdx.y + 1) * CONV_ROWS);
  for (int row = blockIdx.y * CONV_ROWS; row < r1; ++row) {
    const int t = row % T2, b = row / T2;
    float acc[8];
    conv_row<K>(raw, ld, wr, b, t, c, T2, L, block, mode, acc);
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) o2[e] = __floats2bfloat162_rn(silu_f(acc[2 * e]), silu_f(acc[2 * e + 1]));
    *reinterpret_cast<uint4*>(y + (int64_t)row * C + c) = o;
  }
}

// dpre = dy * silu'(pre), pre recomputed; stored fp32 so the gather below accumulates without a
// second rounding.
template <int K>
__global__ void conv_dpre_kernel(const __nv_bfloat16* __restrict__ raw, int64_t ld, const float* __restrict__ w,
                                 const __nv_bfloat16* __restrict__ dy, float* __restrict__ dpre, int B, int T2,
                                 int C, int L, int block, int mode) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= C) return;
  float wr[8][K];
  load_taps<K>(w, c, wr);
  const int r1 = min(B * T2, (int)(blockIdx.y + 1) * CONV_ROWS);
  for (int row = blockIdx.y * CONV_ROWS; row < r1; ++row) {
    const int t = row % T2, b = row / T2;
    float acc[8];
    conv_row<K>(raw, ld, wr, b, t, c, T2, L, block, mode, acc);
    const uint4 g = *reinterpret_cast<const uint4*>(dy + (int64_t)row * C + c);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g);
    float4 o0, o1;
    float* op[2] = {&o0.x, &o1.x};
    (void)op;
    float out[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 gf = __bfloat1622float2(g2[e]);
      const float s0 = sigmoid_f(acc[2 * e]), s1 = sigmoid_f(acc[2 * e + 1]);
      out[2 * e] = gf.x * s0 * (1.f + acc[2 * e] * (1.f - s0));
      out[2 * e + 1] = gf.y * s1 * (1.f + acc[2 * e + 1] * (1.f - s1));
    }
    o0 = make_float4(out[0], out[1], out[2], out[3]);
    o1 = make_float4(out[4], out[5], out[6], out[7]);
    float* dst = dpre + (int64_t)row * C + c;
    *reinterpret_cast<float4*>(dst) = o0;
    *reinterpret_cast<float4*>(dst + 4) = o1;
  }
}

// draw[b, q, c] = sum over (t, j) with source_of(t, j-(K-1)) == q of dpre[b, t, c] * w[c, j].
// A source row r is read by the rows t = r + d (d < K, tap K-1-d) of its own stream -- within its
// block in the noised stream -- and, in fork mode, a clean row r = L + q also by the noised rows
// t = q + d of later blocks (it is their clean prefix). Grid and threads as in the forward: 8
// channels per thread, CONV_ROWS consecutive source rows per block row.
template <int K>
__device__ __forceinline__ void add_consumer(const float* __restrict__ dpre, int64_t row, int C, int c,
                                             const float (&wr)[8][K], int j, float (&acc)[8]) {
  const float4* p = reinterpret_cast<const float4*>(dpre + row * C + c);
  const float4 u = p[0], v = p[1];
  acc[0] += u.x * wr[0][j], acc[1] += u.y * wr[1][j], acc[2] += u.z * wr[2][j], acc[3] += u.w * wr[3][j];
  acc[4] += v.x * wr[4][j], acc[5] += v.y * wr[5][j], acc[6] += v.z * wr[6][j], acc[7] += v.w * wr[7][j];
}

template <int K>
__global__ void conv_dx_kernel(const float* __restrict__ dpre, const float* __restrict__ w,
                               __nv_bfloat16* __restrict__ draw, int64_t ldd, int B, int T2, int C, int L, int block,
                               int mode) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= C) return;
  float wr[8][K];
  load_taps<K>(w, c, wr);
  const int r1 = min(B * T2, (int)(blockIdx.y + 1) * CONV_ROWS);
  for (int row = blockIdx.y * CONV_ROWS; row < r1; ++row) {
    const int b = row / T2, r = row - b * T2;
    const int64_t base = (int64_t)b * T2;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int tend = (mode == CONV_CONCAT || r >= L) ? T2 : min(L, (r / block + 1) * block);
#pragma unroll
    for (int d = 0; d < K; ++d)
      if (r + d < tend && BDLLM_IDX(r + d, T2)) add_consumer<K>(dpre, base + r + d, C, c, wr, K - 1 - d, acc);
    if (mode == CONV_FORK && r >= L) {
      const int q = r - L, later = (q / block + 1) * block;  // noised rows of later blocks
#pragma unroll
      for (int d = 0; d < K; ++d) {
        const int t = q + d;
        if (t < L && t >= later && BDLLM_IDX(t, T2)) add_consumer<K>(dpre, base + t, C, c, wr, K - 1 - d, acc);
      }
    }
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) o2[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
    *reinterpret_cast<uint4*>(draw + (base + r) * ldd + c) = o;
  }
}

// dw partials: thread = 8 channels x K taps over `tokens_per_block` consecutive rows (grid.y);
// part[chunk, c, j] is summed over chunks afterwards.
template <int K>
__global__ void conv_dw_kernel(const __nv_bfloat16* __restrict__ raw, int64_t ld, const float* __restrict__ dpre,
                               float* __restrict__ part, int B, int T2, int C, int L, int block, int mode,
                               int tokens_per_block) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= C) return;
  float acc[8][K];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < K; ++j) acc[e][j] = 0.f;
  const int total = B * T2;
  const int r0 = blockIdx.y * tokens_per_block, r1 = min(total, r0 + tokens_per_block);
  for (int row = r0; row < r1; ++row) {
    const int b = row / T2, t = row - b * T2;
    const float4* pd = reinterpret_cast<const float4*>(dpre + (int64_t)row * C + c);
    const float4 u = pd[0], v = pd[1];
    const float dv[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
    int src[K];
    sources_of<K>(t, L, block, mode, src);
#pragma unroll
    for (int j = 0; j < K; ++j) {
      if (src[j] < 0 || !BDLLM_IDX(src[j], T2)) continue;
      const uint4 p = *reinterpret_cast<const uint4*>(raw + ((int64_t)b * T2 + src[j]) * ld + c);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p2[e]);
        acc[2 * e][j] += dv[2 * e] * f.x;
        acc[2 * e + 1][j] += dv[2 * e + 1] * f.y;
      }
    }
  }
  float* dst = part + ((int64_t)blockIdx.y * C + c) * K;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    *reinterpret_cast<float4*>(dst + e * K) = make_float4(acc[e][0], acc[e][1], acc[e][2], acc[e][3]);
}

__global__ void sum_parts_kernel(const float* __restrict__ part, int nparts, int64_t n, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < nparts; ++p) s += part[p * n + i];
    out[i] = s;
  }
}

static int grid_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 32)); }

// raw [B, 2L, C] read in place at token stride ld when its rows are 16-byte vectors and its batch
// and token dims merge, else a contiguous copy; w [C, 4] as an aligned fp32 copy
static std::pair<at::Tensor, int64_t> conv_raw(const at::Tensor& raw, const at::Tensor& w, int64_t L) {
  TORCH_CHECK(raw.dim() == 3 && raw.scalar_type() == at::kBFloat16, "conv: raw [B, 2L, C] bf16");
  TORCH_CHECK(raw.size(1) == 2 * L && raw.size(2) % 8 == 0, "conv: raw [B, 2L, C] with C % 8 == 0");
  TORCH_CHECK(w.dim() == 2 && w.size(0) == raw.size(2) && w.size(1) == 4, "conv: weight [C, 4] (kernel size 4)");
  if (raw.stride(-1) == 1 && raw.stride(1) % 8 == 0 && raw.stride(1) >= raw.size(2) &&
      (raw.size(0) == 1 || raw.stride(0) == raw.size(1) * raw.stride(1)) && al16(raw))
    return {raw, raw.stride(1)};
  return {vec_input(raw), raw.size(2)};
}

at::Tensor conv_fwd(const at::Tensor& raw_in, const at::Tensor& w, int64_t L, int64_t block, int64_t mode) {
  auto [raw, ld] = conv_raw(raw_in, w, L);
  const int B = raw.size(0), T2 = raw.size(1), C = raw.size(2);
  auto wf = vec_input(w.to(at::kFloat));
  auto y = at::empty({B, T2, C}, raw.options());
  c10::cuda::CUDAGuard g(raw.device());
  conv_fwd_kernel<4><<<dim3((C / 8 + 255) / 256, (B * T2 + CONV_ROWS - 1) / CONV_ROWS), 256, 0, stream()>>>(cbf(raw), ld, wf.data_ptr<float>(),
                                                                   bfp(y), B, T2, C, (int)L, (int)block, (int)mode);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

std::vector<at::Tensor> conv_bwd(const at::Tensor& dy, const at::Tensor& raw_in, const at::Tensor& w, int64_t L,
                                 int64_t block, int64_t mode) {
  auto [raw, ld] = conv_raw(raw_in, w, L);
  const int B = raw.size(0), T2 = raw.size(1), C = raw.size(2), K = 4;
  TORCH_CHECK(dy.numel() == raw.numel(), "conv: dy [B, 2L, C]");
  auto wf = vec_input(w.to(at::kFloat));
  auto d = vec_input(dy.to(at::kBFloat16));
  c10::cuda::CUDAGuard g(raw.device());
  auto dpre = at::empty({B, T2, C}, raw.options().dtype(at::kFloat));
  conv_dpre_kernel<4><<<dim3((C / 8 + 255) / 256, (B * T2 + CONV_ROWS - 1) / CONV_ROWS), 256, 0, stream()>>>(cbf(raw), ld, wf.data_ptr<float>(),
                                                                    cbf(d), dpre.data_ptr<float>(), B, T2, C, (int)L,
                                                                    (int)block, (int)mode);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  auto draw = at::empty({B, T2, C}, raw.options());
  conv_dx_kernel<4><<<dim3((C / 8 + 255) / 256, (B * T2 + CONV_ROWS - 1) / CONV_ROWS), 256, 0, stream()>>>(
      dpre.data_ptr<float>(), wf.data_ptr<float>(), bfp(draw), C, B, T2, C, (int)L, (int)block, (int)mode);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t total = (int64_t)B * T2;
  // enough (channel-group x token-chunk) threads to fill the GPU: chunks of >= 32 rows
  const int tpb = (int)std::max<int64_t>(32, (total + 255) / 256);
  const int nb = (int)((total + tpb - 1) / tpb);
  auto part = at::empty({nb, C, K}, raw.options().dtype(at::kFloat));
  dim3 grid((C / 8 + 127) / 128, nb);
  conv_dw_kernel<4><<<grid, 128, 0, stream()>>>(cbf(raw), ld, dpre.data_ptr<float>(), part.data_ptr<float>(),
                                                B, T2, C, (int)L, (int)block, (int)mode, tpb);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  auto dw = at::empty({C, K}, raw.options().dtype(at::kFloat));
  sum_parts_kernel<<<grid_for((int64_t)C * K), 256, 0, stream()>>>(part.data_ptr<float>(), nb, (int64_t)C * K,
                                                                    dw.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {draw, dw};
}

// ------------------------------------------------------------------------------- CE
// One CTA per row of `logits` [n, V] (bf16, row stride ld). Pass 1: online max / sum-exp in fp32.
// Pass 2 (row is L2-resident): dlogits = exp(x - lse) - onehot(target), written over the logits.
// loss[row] = lse - x[target].
__global__ void ce_rows_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, const int64_t* __restrict__ tgt,
                               float* __restrict__ loss, int V) {
  const int64_t row = blockIdx.x;
  __nv_bfloat16* x = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 p = *reinterpret_cast<const uint4*>(x + c);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
    float v[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(p2[e]);
      v[2 * e] = f.x, v[2 * e + 1] = f.y;
    }
    float mx = v[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) mx = fmaxf(mx, v[e]);
    float nm = fmaxf(m, mx);
    s *= __expf(m - nm);
#pragma unroll
    for (int e = 0; e < 8; ++e) s += __expf(v[e] - nm);
    m = nm;
  }
  // block reduction of (m, s)
  __shared__ float sm[32], ss[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  if (lane == 0) sm[warp] = m, ss[warp] = s;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
      float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (lane == 0) sm[0] = m + logf(s);
  }
  __syncthreads();
  const float lse = sm[0];
  const int64_t t = tgt[row];
  if (threadIdx.x == 0) {
    (void)BDLLM_CHECK(isfinite(lse), row, V);  // sentinel: a non-finite logit in the row
    loss[row] = BDLLM_IDX(t, V) ? lse - __bfloat162float(x[t]) : NAN;
  }
  __syncthreads();  // the target logit is read before pass 2 overwrites it
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 p = *reinterpret_cast<const uint4*>(x + c);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(p2[e]);
      float a = __expf(f.x - lse) - (c + 2 * e == t ? 1.f : 0.f);
      float b = __expf(f.y - lse) - (c + 2 * e + 1 == t ? 1.f : 0.f);
      o2[e] = __floats2bfloat162_rn(a, b);
    }
    *reinterpret_cast<uint4*>(x + c) = o;
  }
}

at::Tensor ce_rows_(at::Tensor& logits, const at::Tensor& tgt) {
  TORCH_CHECK(logits.dim() == 2 && logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1 &&
                  logits.size(1) % 8 == 0 && logits.stride(0) % 8 == 0 && al16(logits),
              "ce_rows: bf16 logits [n, V] in 16-byte aligned rows, V % 8 == 0");
  const int64_t n = logits.size(0);
  TORCH_CHECK(tgt.numel() == n, "ce_rows: one target per row");
  auto loss = at::empty({n}, logits.options().dtype(at::kFloat));
  if (n == 0) return loss;
  auto t = tgt.to(at::kLong).contiguous();
  c10::cuda::CUDAGuard g(logits.device());
  ce_rows_kernel<<<n, 512, 0, stream()>>>(bfp(logits), logits.stride(0), t.data_ptr<int64_t>(), loss.data_ptr<float>(),
                                          (int)logits.size(1));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return loss;
}

// ------------------------------------------------------------------------------- AdamW
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ void store_as(float* p, float x) { *p = x; }
__device__ __forceinline__ void store_as(__nv_bfloat16* p, float x) { *p = __float2bfloat16(x); }

// w (fp32 master, or the fp32 param itself), p (param storage, bf16 or fp32), g (grad, any of
// bf16/fp32), m, v fp32. coef = clip coefficient applied to g. bc1/bc2 = bias corrections.
template <typename TP, typename TG>
__global__ void adamw_kernel(float* __restrict__ w, TP* __restrict__ p, const TG* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v, int64_t n, float lr, float b1, float b2,
                             float eps, float wd, float coef, const float* __restrict__ coef_dev, float bc1,
                             float bc2) {
  if (coef_dev != nullptr) coef *= *coef_dev;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float gi = to_f(g[i]) * coef;
    (void)BDLLM_CHECK(isfinite(gi), i, n);  // sentinel: a non-finite gradient element
    float wi = w[i];
    if (wd != 0.f) wi *= 1.f - lr * wd;
    float mi = b1 * m[i] + (1.f - b1) * gi;
    float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    wi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    w[i] = wi;
    if (p != nullptr) store_as(p + i, wi);
  }
}

// The same update on 4 elements per thread and iteration (16-byte fp32 vectors, 8-byte bf16 gradient
// / parameter vectors); block 0 also takes the n % 4 tail element-wise.
__device__ __forceinline__ void ld4(const float* p, float (&f)[4]) {
  const float4 q = *reinterpret_cast<const float4*>(p);
  f[0] = q.x, f[1] = q.y, f[2] = q.z, f[3] = q.w;
}
__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
}
__device__ __forceinline__ void st4(float* p, const float (&f)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, const float (&f)[4]) {
  uint2 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
  h[0] = __floats2bfloat162_rn(f[0], f[1]);
  h[1] = __floats2bfloat162_rn(f[2], f[3]);
  *reinterpret_cast<uint2*>(p) = u;
}

template <typename TP, typename TG>
__global__ void __launch_bounds__(256) adamw4_kernel(float* __restrict__ w, TP* __restrict__ p,
                                                     const TG* __restrict__ g, float* __restrict__ m,
                                                     float* __restrict__ v, int64_t n, float lr, float b1, float b2,
                                                     float eps, float wd, float coef,
                                                     const float* __restrict__ coef_dev, float bc1, float bc2) {
  if (coef_dev != nullptr) coef *= *coef_dev;
  const float decay = 1.f - lr * wd;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float gi[4], wi[4], mi[4], vi[4];
    ld4(g + 4 * i, gi);
    ld4(w + 4 * i, wi);
    ld4(m + 4 * i, mi);
    ld4(v + 4 * i, vi);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float ge = gi[e] * coef;
      (void)BDLLM_CHECK(isfinite(ge), 4 * i + e, n);  // sentinel: a non-finite gradient element
      mi[e] = b1 * mi[e] + (1.f - b1) * ge;
      vi[e] = b2 * vi[e] + (1.f - b2) * ge * ge;
      wi[e] = wi[e] * decay - lr * (mi[e] / bc1) / (sqrtf(vi[e] / bc2) + eps);
    }
    st4(m + 4 * i, mi);
    st4(v + 4 * i, vi);
    st4(w + 4 * i, wi);
    if (p != nullptr) st4(p + 4 * i, wi);
  }
  if (blockIdx.x == 0) {
    for (int64_t i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) {
      const float ge = to_f(g[i]) * coef;
      const float mi = b1 * m[i] + (1.f - b1) * ge;
      const float vi = b2 * v[i] + (1.f - b2) * ge * ge;
      m[i] = mi;
      v[i] = vi;
      const float wi = w[i] * decay - lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
      w[i] = wi;
      if (p != nullptr) store_as(p + i, wi);
    }
  }
}

void adamw_step(at::Tensor& w, at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1,
                double b2, double eps, double wd, double coef, const c10::optional<at::Tensor>& coef_dev, double bc1,
                double bc2) {
  TORCH_CHECK(!coef_dev.has_value() || (coef_dev->scalar_type() == at::kFloat && coef_dev->numel() >= 1),
              "adamw: fp32 device clip coefficient");
  const float* cd = coef_dev.has_value() ? coef_dev->data_ptr<float>() : nullptr;
  TORCH_CHECK(w.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  TORCH_CHECK(w.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat,
              "adamw: fp32 master and moments");
  TORCH_CHECK(g.scalar_type() == at::kFloat || g.scalar_type() == at::kBFloat16, "adamw: fp32 or bf16 gradient");
  const int64_t n = w.numel();
  TORCH_CHECK(p.numel() == n && g.numel() == n && m.numel() == n && v.numel() == n,
              "adamw: master, parameter, gradient and moments of one length");
  if (n == 0) return;
  c10::cuda::CUDAGuard gd(w.device());
  const bool same = p.data_ptr() == w.data_ptr();
  auto a16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (!same && a16(w.data_ptr()) && a16(p.data_ptr()) && a16(g.data_ptr()) && a16(m.data_ptr()) &&
      a16(v.data_ptr())) {
    const int grid = grid_for((n + 3) / 4);
#define ADAMW4(TP, TG, PP, GP)                                                                                      \
  adamw4_kernel<TP, TG><<<grid, 256, 0, stream()>>>(w.data_ptr<float>(), PP, GP, m.data_ptr<float>(),              \
                                                    v.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2,      \
                                                    (float)eps, (float)wd, (float)coef, cd, (float)bc1, (float)bc2)
    const bool gbf4 = g.scalar_type() == at::kBFloat16;
    if (p.scalar_type() == at::kFloat) {
      if (gbf4) ADAMW4(float, __nv_bfloat16, p.data_ptr<float>(), cbf(g));
      else ADAMW4(float, float, p.data_ptr<float>(), g.data_ptr<float>());
    } else {
      TORCH_CHECK(p.scalar_type() == at::kBFloat16 && p.is_contiguous(), "adamw: bf16 param");
      if (gbf4) ADAMW4(__nv_bfloat16, __nv_bfloat16, bfp(p), cbf(g));
      else ADAMW4(__nv_bfloat16, float, bfp(p), g.data_ptr<float>());
    }
#undef ADAMW4
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const int grid = grid_for(n);
#define ADAMW(TP, TG, PP, GP)                                                                                        \
  adamw_kernel<TP, TG><<<grid, 256, 0, stream()>>>(w.data_ptr<float>(), PP, GP, m.data_ptr<float>(),                  \
                                                   v.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2,          \
                                                   (float)eps, (float)wd, (float)coef, cd, (float)bc1, (float)bc2)
  const bool gbf = g.scalar_type() == at::kBFloat16;
  if (same || p.scalar_type() == at::kFloat) {
    float* pp = same ? nullptr : p.data_ptr<float>();
    if (gbf) ADAMW(float, __nv_bfloat16, pp, cbf(g));
    else ADAMW(float, float, pp, g.data_ptr<float>());
  } else {
    TORCH_CHECK(p.scalar_type() == at::kBFloat16 && p.is_contiguous(), "adamw: bf16 param");
    if (gbf) ADAMW(__nv_bfloat16, __nv_bfloat16, bfp(p), cbf(g));
    else ADAMW(__nv_bfloat16, float, bfp(p), g.data_ptr<float>());
  }
#undef ADAMW
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------- grad norm
// sq += sum_i x_i^2 over an fp32 or bf16 vector (16-byte vectors, one fp32 atomic per block);
// with dst set, dst = x (converted to dst's type, fp32 or bf16) is written in the same pass.
__device__ __forceinline__ void put(float* d, int64_t i, float f) { d[i] = f; }
__device__ __forceinline__ void put(__nv_bfloat16* d, int64_t i, float f) { d[i] = __float2bfloat16(f); }

template <typename T, typename TD>
__global__ void sumsq_kernel(const T* __restrict__ x, int64_t n, TD* __restrict__ dst, float* __restrict__ sq) {
  constexpr int V = 16 / sizeof(T);
  float acc = 0.f;
  const int64_t nv = n / V;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 raw = reinterpret_cast<const uint4*>(x)[i];
    float f[V];
    if constexpr (sizeof(T) == 4) {
      const float4 q = *reinterpret_cast<const float4*>(&raw);
      f[0] = q.x, f[1] = q.y, f[2] = q.z, f[3] = q.w;
    } else {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 t = __bfloat1622float2(h[e]);
        f[2 * e] = t.x, f[2 * e + 1] = t.y;
      }
    }
#pragma unroll
    for (int e = 0; e < V; ++e) acc += f[e] * f[e];
    if (dst != nullptr) {
      if constexpr (sizeof(T) == sizeof(TD)) {  // same type: copy the 16 bytes
        reinterpret_cast<uint4*>(dst)[i] = raw;
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) put(dst, i * V + e, f[e]);
      }
    }
  }
  // tail (n not a multiple of the vector width)
  for (int64_t i = nv * V + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float f = to_f(x[i]);
    acc += f * f;
    if (dst != nullptr) put(dst, i, f);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(sq, t);
  }
}

// sq += ||x||^2 (x fp32 or bf16, contiguous); with dst (fp32 or bf16): dst = x as well
void sumsq_(const at::Tensor& x, at::Tensor& sq, const c10::optional<at::Tensor>& dst) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "sumsq: contiguous 16-byte aligned input");
  TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16, "sumsq: fp32 or bf16 input");
  TORCH_CHECK(sq.scalar_type() == at::kFloat && sq.numel() >= 1, "sumsq: fp32 accumulator");
  const bool has_dst = dst.has_value();
  if (has_dst)
    TORCH_CHECK((dst->scalar_type() == at::kFloat || dst->scalar_type() == at::kBFloat16) && dst->is_contiguous() &&
                    dst->numel() >= x.numel() && reinterpret_cast<uintptr_t>(dst->data_ptr()) % 16 == 0,
                "sumsq: fp32 or bf16 contiguous destination");
  const int64_t n = x.numel();
  if (n == 0) return;
  c10::cuda::CUDAGuard gd(x.device());
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n / 8 + 255) / 256, 148 * 8));
  float* sqp = sq.data_ptr<float>();
  const bool xf = x.scalar_type() == at::kFloat;
  const bool df = !has_dst || dst->scalar_type() == at::kFloat;
  if (xf && df)
    sumsq_kernel<float, float><<<grid, 256, 0, stream()>>>(x.data_ptr<float>(), n,
                                                           has_dst ? dst->data_ptr<float>() : nullptr, sqp);
  else if (xf)
    sumsq_kernel<float, __nv_bfloat16><<<grid, 256, 0, stream()>>>(
        x.data_ptr<float>(), n, reinterpret_cast<__nv_bfloat16*>(dst->data_ptr()), sqp);
  else if (df)
    sumsq_kernel<__nv_bfloat16, float><<<grid, 256, 0, stream()>>>(cbf(x), n, has_dst ? dst->data_ptr<float>() : nullptr,
                                                                   sqp);
  else
    sumsq_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, stream()>>>(
        cbf(x), n, reinterpret_cast<__nv_bfloat16*>(dst->data_ptr()), sqp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------- embedding
// out[i] = table[ids[i]] (bf16 rows, 16-byte vectors); one warp per row
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int D,
                                 int64_t V, __nv_bfloat16* __restrict__ out, int64_t N, int* err) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= N) return;
  const int64_t id = ids[row];
  if (id < 0 || id >= V) {  // out of range: record, write zeros (never read outside the table)
    if ((threadIdx.x & 31) == 0) record_error(err, ERR_BOUNDS);
    for (int c = (threadIdx.x & 31) * 8; c < D; c += 256)
      *reinterpret_cast<uint4*>(out + row * D + c) = make_uint4(0, 0, 0, 0);
    return;
  }
  for (int c = (threadIdx.x & 31) * 8; c < D; c += 256)
    *reinterpret_cast<uint4*>(out + row * D + c) = *reinterpret_cast<const uint4*>(table + id * D + c);
}

// grad[ids[i]] += dh[i] (fp32 accumulate); one warp per row
__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dh, int D,
                                 int64_t V, float* __restrict__ grad, int64_t N) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= N) return;
  const int64_t id = ids[row];
  if (id < 0 || id >= V) return;
  for (int c = (threadIdx.x & 31) * 8; c < D; c += 256) {
    const uint4 p = *reinterpret_cast<const uint4*>(dh + row * D + c);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(p2[e]);
      atomicAdd(grad + id * D + c + 2 * e, f.x);
      atomicAdd(grad + id * D + c + 2 * e + 1, f.y);
    }
  }
}

at::Tensor embed_fwd(const at::Tensor& ids, const at::Tensor& table) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "embed: int64 ids");
  TORCH_CHECK(table.dim() == 2 && table.is_contiguous() && table.scalar_type() == at::kBFloat16 &&
                  table.size(1) % 8 == 0 && al16(table),
              "embed: bf16 table [V, D] at a 16-byte aligned base, D % 8 == 0");
  const int64_t N = ids.numel(), V = table.size(0);
  const int D = table.size(1);
  auto sizes = ids.sizes().vec();
  sizes.push_back(D);
  auto out = at::empty(sizes, table.options());
  if (N == 0) return out;
  c10::cuda::CUDAGuard g(table.device());
  embed_fwd_kernel<<<(int)((N + 7) / 8), 256, 0, stream()>>>(ids.data_ptr<int64_t>(), cbf(table), D, V, bfp(out), N,
                                                             error_word_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void embed_bwd_(at::Tensor& grad, const at::Tensor& ids, const at::Tensor& dh) {
  TORCH_CHECK(grad.dim() == 2 && grad.is_contiguous() && grad.scalar_type() == at::kFloat, "embed_bwd: fp32 [V, D]");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "embed_bwd: int64 ids");
  const int64_t N = ids.numel(), V = grad.size(0);
  const int D = grad.size(1);
  auto d = vec_input(dh.to(at::kBFloat16));
  TORCH_CHECK(d.numel() == N * D && D % 8 == 0, "embed_bwd: dh [N, D]");
  if (N == 0) return;
  c10::cuda::CUDAGuard g(grad.device());
  embed_bwd_kernel<<<(int)((N + 7) / 8), 256, 0, stream()>>>(ids.data_ptr<int64_t>(), cbf(d), D, V,
                                                             grad.data_ptr<float>(), N);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Sorted variant straight into a bf16 gradient (no fp32 [V, D] table): sid = the ids sorted, perm
// their positions in dh. Grid (positions / 8, column chunks of 256): the warp at the first
// position of a run of equal ids finds the run's end by binary search and sums the run's dh rows
// for its 256 columns in fp32 (8 per lane, 8 rows in flight), then writes the bf16 row chunk.
// A long run (the mask token fills half the noised stream) is spread over the column chunks;
// rows of ids absent from the batch keep the zeros the caller wrote. Deterministic.
__global__ void embed_bwd_sorted_kernel(const int64_t* __restrict__ sid, const int64_t* __restrict__ perm,
                                        const __nv_bfloat16* __restrict__ dh, int D, int64_t V,
                                        __nv_bfloat16* __restrict__ grad, int64_t N) {
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int c = blockIdx.y * 256 + (threadIdx.x & 31) * 8;
  if (i >= N || c >= D) return;
  const int64_t id = sid[i];
  if ((i > 0 && sid[i - 1] == id) || id < 0 || id >= V) return;  // not the start of a run
  int64_t lo = i + 1, hi = N;  // first position past the run
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (sid[mid] == id) lo = mid + 1;
    else hi = mid;
  }
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
  for (int64_t j = i; j < lo; ++j) {
    const uint4 p = *reinterpret_cast<const uint4*>(dh + perm[j] * D + c);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(p2[e]);
      acc[2 * e] += f.x, acc[2 * e + 1] += f.y;
    }
  }
  uint4 o;
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int e = 0; e < 4; ++e) o2[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
  *reinterpret_cast<uint4*>(grad + id * D + c) = o;
}

void embed_bwd_sorted(at::Tensor& grad, const at::Tensor& sid, const at::Tensor& perm, const at::Tensor& dh) {
  TORCH_CHECK(grad.dim() == 2 && grad.is_contiguous() && grad.scalar_type() == at::kBFloat16 && al16(grad),
              "embed_bwd_sorted: bf16 [V, D] at a 16-byte aligned base");
  TORCH_CHECK(sid.scalar_type() == at::kLong && perm.scalar_type() == at::kLong && sid.is_contiguous() &&
                  perm.is_contiguous() && sid.numel() == perm.numel(),
              "embed_bwd_sorted: int64 sorted ids and positions");
  const int64_t N = sid.numel(), V = grad.size(0);
  const int D = grad.size(1);
  auto d = vec_input(dh.to(at::kBFloat16));
  TORCH_CHECK(d.numel() == N * D && D % 8 == 0, "embed_bwd_sorted: dh [N, D]");
  if (N == 0) return;
  c10::cuda::CUDAGuard g(grad.device());
  const dim3 grid((unsigned)((N + 7) / 8), (unsigned)((D + 255) / 256));
  embed_bwd_sorted_kernel<<<grid, 256, 0, stream()>>>(sid.data_ptr<int64_t>(), perm.data_ptr<int64_t>(), cbf(d), D, V,
                                                      bfp(grad), N);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------- GDN gates
// beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) (softplus linear above 20, as torch's)
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// a, b: [rows, H] views with row stride lda / ldb (bf16); g, beta: [rows, H] fp32
__global__ void gates_fwd_kernel(const __nv_bfloat16* __restrict__ a, int64_t lda, const __nv_bfloat16* __restrict__ b,
                                 int64_t ldb, const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                                 int H, int64_t rows, float* __restrict__ g, float* __restrict__ beta) {
  const int64_t n = rows * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H;
    const int h = (int)(i - r * H);
    const float x = __bfloat162float(a[r * lda + h]) + dt_bias[h];
    g[i] = -__expf(A_log[h]) * softplus_f(x);
    beta[i] = sigmoid_f(__bfloat162float(b[r * ldb + h]));
  }
}

// da = dg * (-exp(A_log)) * sigmoid(a + dt_bias); db = dbeta * beta (1 - beta);
// d dt_bias[h] = sum_r da; d A_log[h] = sum_r dg * g  (per-head sums: block partials + atomics)
__global__ void gates_bwd_kernel(const __nv_bfloat16* __restrict__ a, int64_t lda, const __nv_bfloat16* __restrict__ b,
                                 int64_t ldb, const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                                 const float* __restrict__ dg, const float* __restrict__ dbeta, int H, int64_t rows,
                                 __nv_bfloat16* __restrict__ da, __nv_bfloat16* __restrict__ db,
                                 float* __restrict__ dA_log, float* __restrict__ ddt) {
  extern __shared__ float red[];  // [2 * H]
  for (int i = threadIdx.x; i < 2 * H; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  const int64_t n = rows * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H;
    const int h = (int)(i - r * H);
    const float x = __bfloat162float(a[r * lda + h]) + dt_bias[h];
    const float ea = __expf(A_log[h]);
    const float gv = -ea * softplus_f(x);
    const float dav = dg[i] * (-ea) * sigmoid_f(x);
    const float be = sigmoid_f(__bfloat162float(b[r * ldb + h]));
    da[i] = __float2bfloat16(dav);
    db[i] = __float2bfloat16(dbeta[i] * be * (1.f - be));
    atomicAdd(&red[h], dav);
    atomicAdd(&red[H + h], dg[i] * gv);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    atomicAdd(&ddt[i], red[i]);
    atomicAdd(&dA_log[i], red[H + i]);
  }
}

static void check_gate_view(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.stride(-1) == 1, "gdn_gates: ", name, " bf16 with unit inner stride");
  TORCH_CHECK(t.dim() >= 2, "gdn_gates: ", name, " [..., H]");
  for (int d = 0; d < t.dim() - 2; ++d)
    TORCH_CHECK(t.stride(d) == t.size(d + 1) * t.stride(d + 1), "gdn_gates: ", name, " rows must merge");
}

std::vector<at::Tensor> gdn_gates_fwd(const at::Tensor& a, const at::Tensor& b, const at::Tensor& A_log,
                                      const at::Tensor& dt_bias) {
  check_gate_view(a, "a");
  check_gate_view(b, "b");
  const int H = a.size(-1);
  TORCH_CHECK(b.sizes() == a.sizes() && A_log.numel() == H && dt_bias.numel() == H,
              "gdn_gates: a and b of one shape, A_log and dt_bias [H]");
  const int64_t rows = a.numel() / H;
  auto Af = A_log.to(at::kFloat).contiguous(), df = dt_bias.to(at::kFloat).contiguous();
  auto g = at::empty(a.sizes(), a.options().dtype(at::kFloat));
  auto beta = at::empty(a.sizes(), a.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard gd(a.device());
  gates_fwd_kernel<<<grid_for(rows * H), 256, 0, stream()>>>(cbf(a), a.stride(-2), cbf(b), b.stride(-2),
                                                             Af.data_ptr<float>(), df.data_ptr<float>(), H, rows,
                                                             g.data_ptr<float>(), beta.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {g, beta};
}

std::vector<at::Tensor> gdn_gates_bwd(const at::Tensor& dg, const at::Tensor& dbeta, const at::Tensor& a,
                                      const at::Tensor& b, const at::Tensor& A_log, const at::Tensor& dt_bias) {
  check_gate_view(a, "a");
  check_gate_view(b, "b");
  const int H = a.size(-1);
  TORCH_CHECK(b.sizes() == a.sizes() && A_log.numel() == H && dt_bias.numel() == H && dg.numel() == a.numel() &&
                  dbeta.numel() == a.numel() && (int64_t)H * 2 * sizeof(float) <= 48 * 1024,
              "gdn_gates: a, b, dg and dbeta of one shape, A_log and dt_bias [H], H <= 6144");
  const int64_t rows = a.numel() / H;
  auto Af = A_log.to(at::kFloat).contiguous(), df = dt_bias.to(at::kFloat).contiguous();
  auto dgc = dg.to(at::kFloat).contiguous(), dbc = dbeta.to(at::kFloat).contiguous();
  auto da = at::empty(a.sizes(), a.options());
  auto db = at::empty(a.sizes(), a.options());
  auto dA = at::zeros({H}, a.options().dtype(at::kFloat));
  auto ddt = at::zeros({H}, a.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard gd(a.device());
  const int grid = std::min<int64_t>(grid_for(rows * H), 148 * 4);
  gates_bwd_kernel<<<grid, 256, 2 * H * sizeof(float), stream()>>>(
      cbf(a), a.stride(-2), cbf(b), b.stride(-2), Af.data_ptr<float>(), df.data_ptr<float>(), dgc.data_ptr<float>(),
      dbc.data_ptr<float>(), H, rows, bfp(da), bfp(db), dA.data_ptr<float>(), ddt.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {da, db, dA, ddt};
}

// ------------------------------------------------------------------------------- group_sum
// x [rows, G, R, D] bf16 -> out [rows, G, D] bf16, summed over R in fp32 (one pass, 16-byte vectors):
// the GDN kernels give dq / dk per v-head, and each k-head's gradient is the sum over its group.
__global__ void group_sum_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out, int64_t n8,
                                 int R, int D8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rg = i / D8;  // (row, group)
    const int c = (int)(i % D8);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < R; ++r) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + ((rg * R + r) * D8 + c) * 8);
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p[e]);
        acc[2 * e] += f.x, acc[2 * e + 1] += f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) po[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
    *reinterpret_cast<uint4*>(out + i * 8) = o;
  }
}

at::Tensor group_sum(const at::Tensor& x_in, int64_t groups) {
  TORCH_CHECK(x_in.scalar_type() == at::kBFloat16 && x_in.dim() >= 2, "group_sum: bf16 [..., H, D]");
  auto x = vec_input(x_in);
  const int64_t D = x.size(-1), H = x.size(-2);
  TORCH_CHECK(D % 8 == 0 && groups > 0 && H % groups == 0, "group_sum: D % 8 == 0 and H divisible by groups");
  const int R = (int)(H / groups);
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape[shape.size() - 2] = groups;
  auto out = at::empty(shape, x.options());
  const int64_t n8 = out.numel() / 8;
  if (n8 == 0) return out;
  c10::cuda::CUDAGuard gd(x.device());
  group_sum_kernel<<<grid_for(n8), 256, 0, stream()>>>(cbf(x), bfp(out), n8, R, (int)(D / 8));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// ------------------------------------------------------------------------------- mask_sample
// Counter-based uniforms: the SplitMix64 output function (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014) applied to a key made of (seed, row, position,
// stream), top 24 bits as a float in [0, 1). No state: any thread draws any element.
__device__ __forceinline__ float key_uniform(uint64_t seed, uint64_t a, uint64_t b) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (a * 0x100000001B3ull + b + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

// One thread per (row, position): t = U(row, block) (the block's mask ratio), u = U(row, position);
// m = u < t on scorable positions (prompt_len <= i < valid_len). Writes rows [0, B) of the outputs
// for view m and rows [B, 2B) for the complement: x0_2 = x0 twice, xt_2 = x0 with [MASK] where
// the view masks, m_2 the view's mask.
__global__ void mask_sample_kernel(const int64_t* __restrict__ x0, const int64_t* __restrict__ plen,
                                   const int64_t* __restrict__ vlen, int B, int L, int block, int64_t mask_id,
                                   uint64_t seed, int64_t* __restrict__ x0_2, int64_t* __restrict__ xt_2,
                                   bool* __restrict__ m_2) {
  const int64_t n = (int64_t)B * L;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(idx / L), i = (int)(idx % L);
    const float t = key_uniform(seed, (uint64_t)b, (uint64_t)(i / block) * 2 + 1);
    const float u = key_uniform(seed, (uint64_t)b + (1ull << 32), (uint64_t)i * 2);
    const bool scor = i >= plen[b] && (vlen == nullptr || i < vlen[b]);
    const bool m = scor && u < t, mc = scor && !m;
    const int64_t x = x0[idx], o = idx + n;
    x0_2[idx] = x, x0_2[o] = x;
    xt_2[idx] = m ? mask_id : x, xt_2[o] = mc ? mask_id : x;
    m_2[idx] = m, m_2[o] = mc;
  }
}

std::vector<at::Tensor> mask_sample(const at::Tensor& x0, const at::Tensor& prompt_len,
                                    const c10::optional<at::Tensor>& valid_len, int64_t block, int64_t mask_id,
                                    int64_t seed) {
  TORCH_CHECK(x0.is_cuda() && x0.dim() == 2 && x0.scalar_type() == at::kLong, "mask_sample: int64 [B, L] on CUDA");
  const int B = x0.size(0), L = x0.size(1);
  TORCH_CHECK(block > 0 && L % block == 0, "mask_sample: block must divide L");
  auto xc = x0.contiguous();
  auto pl = prompt_len.to(x0.device(), at::kLong).contiguous();
  at::Tensor vl;
  if (valid_len.has_value()) vl = valid_len->to(x0.device(), at::kLong).contiguous();
  TORCH_CHECK(pl.numel() == B && (!vl.defined() || vl.numel() == B), "mask_sample: one length per row");
  auto x0_2 = at::empty({2 * B, L}, x0.options());
  auto xt_2 = at::empty({2 * B, L}, x0.options());
  auto m_2 = at::empty({2 * B, L}, x0.options().dtype(at::kBool));
  c10::cuda::CUDAGuard gd(x0.device());
  mask_sample_kernel<<<grid_for((int64_t)B * L), 256, 0, stream()>>>(
      xc.data_ptr<int64_t>(), pl.data_ptr<int64_t>(), vl.defined() ? vl.data_ptr<int64_t>() : nullptr, B, L,
      (int)block, mask_id, (uint64_t)seed, x0_2.data_ptr<int64_t>(), xt_2.data_ptr<int64_t>(), m_2.data_ptr<bool>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {x0_2, xt_2, m_2};
}

}  // namespace bdllm
