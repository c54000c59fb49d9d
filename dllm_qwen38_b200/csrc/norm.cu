// Row-wise normalisation kernels (memory bound): one warp per row, fp32 math, bf16 I/O.
//
//   rmsnorm        y = x * rstd * (1 + w)                     (Qwen3.5 RMSNorm, HF:711-728)
//   gated_rmsnorm  y = bf16(w * bf16(x * rstd)) * silu(z)      (HF:175-190, per v-head row)
//   qk_norm_rope   per-head rmsnorm(1 + w) of q and k, then rotate_half RoPE on the first R dims
//
// Backward kernels recompute rstd from x (one extra read of x beats storing it for 2BL rows) and
// produce per-block partial weight gradients that a second tiny kernel reduces (deterministic).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace bdllm {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int NORM_ROWS_PER_BLOCK = 8;  // 8 warps per block, one row each
constexpr int MAX_D = 8192;

// --------------------------------------------------------------------------------- rmsnorm
// One warp per row, two passes over the row (the second pass re-reads from L1/L2): pass 1 the
// sum of squares, pass 2 the scaled output. D % 8 == 0 (16-byte vectors).
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const float* __restrict__ w1,
                                   __nv_bfloat16* __restrict__ y, int64_t ldy, int rows, int D, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row = blockIdx.x * NORM_ROWS_PER_BLOCK + warp;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (int64_t)row * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    uint4 p = *reinterpret_cast<const uint4*>(xr + c);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(p2[e]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) (void)BDLLM_CHECK(isfinite(ss), row, rows);  // sentinel: a non-finite input row
  const float r = rsqrtf(ss / D + eps);
  __nv_bfloat16* yr = y + (int64_t)row * ldy;
  for (int c = lane * 8; c < D; c += 256) {
    uint4 p = *reinterpret_cast<const uint4*>(xr + c);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
    float4 wa = *reinterpret_cast<const float4*>(w1 + c), wb = *reinterpret_cast<const float4*>(w1 + c + 4);
    const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(p2[e]);
      o2[e] = __floats2bfloat162_rn(f.x * r * wv[2 * e], f.y * r * wv[2 * e + 1]);
    }
    *reinterpret_cast<uint4*>(yr + c) = o;
  }
}

// dx = r * g - x * r^3 * mean(g * x), g = dy * (1 + w); the weight gradient sum_rows dy * x * r
// accumulates in shared memory (one float per column) and each block writes one partial row.
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const float* __restrict__ w1, __nv_bfloat16* __restrict__ dx,
                                   float* __restrict__ dw_part, int rows, int D, float eps, int rows_per_block) {
  extern __shared__ float wacc[];  // [D]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int c = threadIdx.x; c < D; c += blockDim.x) wacc[c] = 0.f;
  __syncthreads();
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += NORM_ROWS_PER_BLOCK) {
    const __nv_bfloat16* xr = x + (int64_t)row * D;
    const __nv_bfloat16* dyr = dy + (int64_t)row * D;
    float ss = 0.f, gx = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      uint4 p = *reinterpret_cast<const uint4*>(xr + c);
      uint4 q = *reinterpret_cast<const uint4*>(dyr + c);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 a = __bfloat1622float2(p2[e]), b = __bfloat1622float2(q2[e]);
        ss += a.x * a.x + a.y * a.y;
        gx += b.x * w1[c + 2 * e] * a.x + b.y * w1[c + 2 * e + 1] * a.y;
      }
    }
    ss = warp_sum(ss);
    gx = warp_sum(gx);
    const float r = rsqrtf(ss / D + eps);
    const float k = r * r * r * gx / D;
    __nv_bfloat16* dxr = dx + (int64_t)row * D;
    for (int c = lane * 8; c < D; c += 256) {
      uint4 p = *reinterpret_cast<const uint4*>(xr + c);
      uint4 q = *reinterpret_cast<const uint4*>(dyr + c);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&q);
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 a = __bfloat1622float2(p2[e]), b = __bfloat1622float2(q2[e]);
        atomicAdd(&wacc[c + 2 * e], b.x * a.x * r);
        atomicAdd(&wacc[c + 2 * e + 1], b.y * a.y * r);
        o2[e] = __floats2bfloat162_rn(r * b.x * w1[c + 2 * e] - a.x * k, r * b.y * w1[c + 2 * e + 1] - a.y * k);
      }
      *reinterpret_cast<uint4*>(dxr + c) = o;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) dw_part[(int64_t)blockIdx.x * D + c] = wacc[c];
}

__global__ void colsum_kernel(const float* __restrict__ part, int nparts, int D, float* __restrict__ out) {
  int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= D) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += part[(int64_t)p * D + c];
  out[c] = s;
}

// --------------------------------------------------------------------------------- gated
// rows of Dv (<= 256): x, z [rows, Dv] (z row stride ldz), w [Dv] (plain weight, not 1 + w)
__global__ void gated_rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ z,
                                         int64_t ldz, const float* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                         int rows, int D, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row = blockIdx.x * NORM_ROWS_PER_BLOCK + warp;
  if (row >= rows) return;
  const int per = D / 32;  // elements per lane (D % 32 == 0, D <= 256)
  float xv[8];
  float ss = 0.f;
  for (int e = 0; e < per; ++e) {
    xv[e] = __bfloat162float(x[(int64_t)row * D + lane * per + e]);
    ss += xv[e] * xv[e];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  for (int e = 0; e < per; ++e) {
    int c = lane * per + e;
    float n = __bfloat162float(__float2bfloat16(xv[e] * r));
    float a = __bfloat162float(__float2bfloat16(w[c] * n));
    float zz = __bfloat162float(z[(int64_t)row * ldz + c]);
    y[(int64_t)row * D + c] = __float2bfloat16(a * silu_f(zz));
  }
}

__global__ void gated_rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                         const __nv_bfloat16* __restrict__ z, int64_t ldz,
                                         const float* __restrict__ w, __nv_bfloat16* __restrict__ dx,
                                         __nv_bfloat16* __restrict__ dz, int64_t lddz, float* __restrict__ dw_part,
                                         int rows, int D, float eps, int rows_per_block) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int per = D / 32;
  float wacc[8];
  for (int e = 0; e < 8; ++e) wacc[e] = 0.f;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += NORM_ROWS_PER_BLOCK) {
    float xv[8], g[8];
    float ss = 0.f;
    for (int e = 0; e < per; ++e) {
      xv[e] = __bfloat162float(x[(int64_t)row * D + lane * per + e]);
      ss += xv[e] * xv[e];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
    float gx = 0.f;
    for (int e = 0; e < per; ++e) {
      int c = lane * per + e;
      float n = xv[e] * r;
      float zz = __bfloat162float(z[(int64_t)row * ldz + c]);
      float sg = sigmoid_f(zz);
      float s = zz * sg;
      float d = __bfloat162float(dy[(int64_t)row * D + c]);
      float a = w[c] * n;
      dz[(int64_t)row * lddz + c] = __float2bfloat16(d * a * sg * (1.f + zz * (1.f - sg)));
      float da = d * s;
      wacc[e] += da * n;
      g[e] = da * w[c];
      gx += g[e] * xv[e];
    }
    gx = warp_sum(gx);
    const float k = r * r * r * gx / D;
    for (int e = 0; e < per; ++e) dx[(int64_t)row * D + lane * per + e] = __float2bfloat16(r * g[e] - xv[e] * k);
  }
  __shared__ float red[NORM_ROWS_PER_BLOCK][256];
  for (int e = 0; e < per; ++e) red[warp][lane * per + e] = wacc[e];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s = 0.f;
    for (int wv = 0; wv < NORM_ROWS_PER_BLOCK; ++wv) s += red[wv][c];
    dw_part[(int64_t)blockIdx.x * D + c] = s;
  }
}

// --------------------------------------------------------------------------------- q/k norm + RoPE
// src rows: token t (0..T-1 over B*T2), head h; element (t, h, d) at src + t*ld_t + h*ld_h + d.
// out contiguous [T, H, Dh]. cos/sin [T2, R] indexed by (t % T2). One warp per (t, h); Dh <= 256.
__global__ void qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ src, int64_t ld_t, int64_t ld_h,
                                        const float* __restrict__ w1, const __nv_bfloat16* __restrict__ cs,
                                        const __nv_bfloat16* __restrict__ sn, __nv_bfloat16* __restrict__ out,
                                        int T, int H, int Dh, int T2, int R, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t idx = (int64_t)blockIdx.x * NORM_ROWS_PER_BLOCK + warp;
  if (idx >= (int64_t)T * H) return;
  const int t = idx / H, h = idx % H;
  const __nv_bfloat16* s = src + t * ld_t + h * ld_h;
  __shared__ float buf[NORM_ROWS_PER_BLOCK][256];
  float ss = 0.f;
  for (int d = lane; d < Dh; d += 32) {
    float v = __bfloat162float(s[d]);
    buf[warp][d] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / Dh + eps);
  __syncwarp();
  for (int d = lane; d < Dh; d += 32) buf[warp][d] = __bfloat162float(__float2bfloat16(buf[warp][d] * r * w1[d]));
  __syncwarp();
  const int pos = t % T2;
  const int half = R / 2;
  __nv_bfloat16* o = out + idx * Dh;
  for (int d = lane; d < Dh; d += 32) {
    float v = buf[warp][d];
    if (d < R) {
      float c = __bfloat162float(cs[pos * R + d]), sv = __bfloat162float(sn[pos * R + d]);
      float rot = d < half ? -buf[warp][d + half] : buf[warp][d - half];
      v = v * c + rot * sv;
    }
    o[d] = __float2bfloat16(v);
  }
}

// backward: dn = rope^T(dout) (rotation transposed), then rmsnorm backward; dw partial per block.
__global__ void qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ src,
                                        int64_t ld_t, int64_t ld_h, const float* __restrict__ w1,
                                        const __nv_bfloat16* __restrict__ cs, const __nv_bfloat16* __restrict__ sn,
                                        __nv_bfloat16* __restrict__ dsrc, int64_t dld_t, int64_t dld_h,
                                        float* __restrict__ dw_part, int T, int H, int Dh, int T2, int R, float eps,
                                        int items_per_block) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __shared__ float dbuf[NORM_ROWS_PER_BLOCK][256];
  __shared__ float wred[NORM_ROWS_PER_BLOCK][256];
  for (int d = lane; d < Dh; d += 32) wred[warp][d] = 0.f;
  const int64_t i0 = (int64_t)blockIdx.x * items_per_block;
  const int64_t i1 = min((int64_t)T * H, i0 + items_per_block);
  const int half = R / 2;
  for (int64_t idx = i0 + warp; idx < i1; idx += NORM_ROWS_PER_BLOCK) {
    const int t = idx / H, h = idx % H;
    const int pos = t % T2;
    const __nv_bfloat16* g = dout + idx * Dh;
    // dn[d] for d < R: y_d = n_d c_d + rot_d s_d, rot_d = -n_{d+half} (d<half) | n_{d-half}
    for (int d = lane; d < Dh; d += 32) {
      float v = __bfloat162float(g[d]);
      if (d < R) {
        float c = __bfloat162float(cs[pos * R + d]);
        int dp = d < half ? d + half : d - half;
        float gp = __bfloat162float(g[dp]);
        float sp = __bfloat162float(sn[pos * R + dp]);
        // n_d appears in y_d (coef c_d) and in y_dp (coef +s_dp if d < half else -s_dp)
        v = v * c + gp * sp * (d < half ? 1.f : -1.f);
      }
      dbuf[warp][d] = v;
    }
    const __nv_bfloat16* s = src + t * ld_t + h * ld_h;
    float ss = 0.f, gx = 0.f;
    for (int d = lane; d < Dh; d += 32) {
      float x = __bfloat162float(s[d]);
      ss += x * x;
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / Dh + eps);
    for (int d = lane; d < Dh; d += 32) {
      float x = __bfloat162float(s[d]);
      wred[warp][d] += dbuf[warp][d] * x * r;
      float gg = dbuf[warp][d] * w1[d];
      dbuf[warp][d] = gg;
      gx += gg * x;
    }
    gx = warp_sum(gx);
    const float k = r * r * r * gx / Dh;
    __nv_bfloat16* ds = dsrc + t * dld_t + h * dld_h;
    for (int d = lane; d < Dh; d += 32) {
      float x = __bfloat162float(s[d]);
      ds[d] = __float2bfloat16(r * dbuf[warp][d] - x * k);
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < Dh; d += blockDim.x) {
    float sacc = 0.f;
    for (int wv = 0; wv < NORM_ROWS_PER_BLOCK; ++wv) sacc += wred[wv][d];
    dw_part[(int64_t)blockIdx.x * Dh + d] = sacc;
  }
}

// ------------------------------------------------------------------------------------- host

static inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }
static inline const __nv_bfloat16* cbf(const at::Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr());
}
static inline __nv_bfloat16* bf(at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

static at::Tensor rows2d(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16, "norm: CUDA bf16 input expected");
  auto x2 = x.reshape({-1, x.size(-1)});
  if (x2.stride(-1) != 1 || x2.stride(0) % 8 || reinterpret_cast<uintptr_t>(x2.data_ptr()) % 16) x2 = x2.contiguous();
  return x2;
}

// y = x * rstd * w1 (w1 = 1 + w, fp32 [D])
at::Tensor rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w1, double eps) {
  const int D = x.size(-1);
  TORCH_CHECK(D % 8 == 0 && D <= MAX_D, "rmsnorm: D % 8 == 0 and D <= 8192");
  auto x2 = rows2d(x);
  const int rows = x2.size(0);
  auto y = at::empty({rows, D}, x.options());
  if (rows == 0) return y.view(x.sizes());
  c10::cuda::CUDAGuard g(x.device());
  auto w = w1.to(at::kFloat).contiguous();
  dim3 grid((rows + NORM_ROWS_PER_BLOCK - 1) / NORM_ROWS_PER_BLOCK), block(32 * NORM_ROWS_PER_BLOCK);
  rmsnorm_fwd_kernel<<<grid, block, 0, stream()>>>(cbf(x2), x2.stride(0), w.data_ptr<float>(), bf(y), D, rows, D,
                                                   (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y.view(x.sizes());
}

std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w1, double eps) {
  const int D = x.size(-1);
  auto x2 = x.reshape({-1, D}).contiguous();
  auto dy2 = dy.to(at::kBFloat16).reshape({-1, D}).contiguous();
  const int rows = x2.size(0);
  auto dx = at::empty_like(x2);
  c10::cuda::CUDAGuard g(x.device());
  auto w = w1.to(at::kFloat).contiguous();
  const int rows_per_block = std::max(64, (rows + 1023) / 1024);
  const int nblk = std::max(1, (rows + rows_per_block - 1) / rows_per_block);
  auto part = at::empty({nblk, D}, x.options().dtype(at::kFloat));
  auto dw = at::empty({D}, x.options().dtype(at::kFloat));
  if (rows > 0) {
    rmsnorm_bwd_kernel<<<nblk, 32 * NORM_ROWS_PER_BLOCK, D * sizeof(float), stream()>>>(
        cbf(dy2), cbf(x2), w.data_ptr<float>(), bf(dx), part.data_ptr<float>(), rows, D, (float)eps, rows_per_block);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    colsum_kernel<<<(D + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), nblk, D, dw.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    dw.zero_();
  }
  return {dx.view(x.sizes()), dw};
}

at::Tensor gated_rmsnorm_fwd(const at::Tensor& x, const at::Tensor& z, const at::Tensor& w, double eps) {
  const int D = x.size(-1);
  TORCH_CHECK(D % 32 == 0 && D <= 256, "gated_rmsnorm: D % 32 == 0 and D <= 256");
  auto x2 = x.reshape({-1, D}).contiguous();
  auto z2 = z.reshape({-1, D});
  if (z2.stride(-1) != 1) z2 = z2.contiguous();
  const int rows = x2.size(0);
  auto y = at::empty_like(x2);
  if (rows == 0) return y.view(x.sizes());
  c10::cuda::CUDAGuard g(x.device());
  auto wf = w.to(at::kFloat).contiguous();
  gated_rmsnorm_fwd_kernel<<<(rows + NORM_ROWS_PER_BLOCK - 1) / NORM_ROWS_PER_BLOCK, 32 * NORM_ROWS_PER_BLOCK, 0,
                             stream()>>>(cbf(x2), cbf(z2), z2.stride(0), wf.data_ptr<float>(), bf(y), rows, D,
                                         (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y.view(x.sizes());
}

std::vector<at::Tensor> gated_rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& z,
                                          const at::Tensor& w, double eps) {
  const int D = x.size(-1);
  auto x2 = x.reshape({-1, D}).contiguous();
  auto z2 = z.reshape({-1, D});
  if (z2.stride(-1) != 1) z2 = z2.contiguous();
  auto dy2 = dy.to(at::kBFloat16).reshape({-1, D}).contiguous();
  const int rows = x2.size(0);
  auto dx = at::empty_like(x2);
  auto dz = at::empty({rows, D}, x.options());
  const int rows_per_block = 128;
  const int nblk = std::max(1, (rows + rows_per_block - 1) / rows_per_block);
  auto part = at::empty({nblk, D}, x.options().dtype(at::kFloat));
  auto dw = at::zeros({D}, x.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard g(x.device());
  auto wf = w.to(at::kFloat).contiguous();
  if (rows > 0) {
    gated_rmsnorm_bwd_kernel<<<nblk, 32 * NORM_ROWS_PER_BLOCK, 0, stream()>>>(
        cbf(dy2), cbf(x2), cbf(z2), z2.stride(0), wf.data_ptr<float>(), bf(dx), bf(dz), D, part.data_ptr<float>(),
        rows, D, (float)eps, rows_per_block);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    colsum_kernel<<<(D + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), nblk, D, dw.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {dx.view(x.sizes()), dz.view(z.sizes()), dw};
}

// src: [..., T2, H, Dh]-shaped strided view (last dim contiguous); returns contiguous [N, H, Dh]
at::Tensor qk_norm_rope_fwd(const at::Tensor& src, const at::Tensor& w1, const at::Tensor& cs, const at::Tensor& sn,
                            double eps) {
  TORCH_CHECK(src.dim() == 4 && src.stride(-1) == 1, "qk_norm_rope: src [B, T2, H, Dh] with unit inner stride");
  const int B = src.size(0), T2 = src.size(1), H = src.size(2), Dh = src.size(3);
  TORCH_CHECK(Dh <= 256, "qk_norm_rope: Dh <= 256");
  TORCH_CHECK(src.stride(0) == (int64_t)T2 * src.stride(1), "qk_norm_rope: batch and token dims must merge");
  const int R = cs.size(-1);
  auto out = at::empty({B, T2, H, Dh}, src.options());
  const int T = B * T2;
  if (T == 0) return out;
  c10::cuda::CUDAGuard g(src.device());
  auto w = w1.to(at::kFloat).contiguous();
  auto c2 = cs.to(at::kBFloat16).contiguous(), s2 = sn.to(at::kBFloat16).contiguous();
  TORCH_CHECK(c2.size(0) == T2, "qk_norm_rope: cos/sin rows must equal T2");
  const int64_t items = (int64_t)T * H;
  qk_norm_rope_fwd_kernel<<<(items + NORM_ROWS_PER_BLOCK - 1) / NORM_ROWS_PER_BLOCK, 32 * NORM_ROWS_PER_BLOCK, 0,
                            stream()>>>(cbf(src), src.stride(1), src.stride(2), w.data_ptr<float>(), cbf(c2), cbf(s2),
                                        bf(out), T, H, Dh, T2, R, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> qk_norm_rope_bwd(const at::Tensor& dout, const at::Tensor& src, const at::Tensor& w1,
                                         const at::Tensor& cs, const at::Tensor& sn, double eps) {
  const int B = src.size(0), T2 = src.size(1), H = src.size(2), Dh = src.size(3);
  const int R = cs.size(-1);
  auto d = dout.to(at::kBFloat16).contiguous();
  auto dsrc = at::empty({B, T2, H, Dh}, src.options());
  const int T = B * T2;
  const int64_t items = (int64_t)T * H;
  // about four 8-warp blocks per SM whatever the head count (the k side has 6x fewer rows than q)
  const int per_block = (int)std::min<int64_t>(256, std::max<int64_t>(8, (items + 4 * 148 - 1) / (4 * 148)));
  const int nblk = std::max<int64_t>(1, (items + per_block - 1) / per_block);
  auto part = at::empty({nblk, Dh}, src.options().dtype(at::kFloat));
  auto dw = at::zeros({Dh}, src.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard g(src.device());
  auto w = w1.to(at::kFloat).contiguous();
  auto c2 = cs.to(at::kBFloat16).contiguous(), s2 = sn.to(at::kBFloat16).contiguous();
  if (items > 0) {
    qk_norm_rope_bwd_kernel<<<nblk, 32 * NORM_ROWS_PER_BLOCK, 0, stream()>>>(
        cbf(d), cbf(src), src.stride(1), src.stride(2), w.data_ptr<float>(), cbf(c2), cbf(s2), bf(dsrc),
        dsrc.stride(1), dsrc.stride(2), part.data_ptr<float>(), T, H, Dh, T2, R, (float)eps, per_block);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    colsum_kernel<<<(Dh + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), nblk, Dh, dw.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {dsrc, dw};
}

}  // namespace bdllm
