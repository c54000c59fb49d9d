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

#include <tuple>

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

// dx = r * g - x * r^3 * mean(g * x), g = dy * (1 + w); weight gradient sum_rows dy * x * r.
// A block takes RMS_BWD_ROWS rows. Phase 1: one warp per row computes r and mean(g * x) and writes
// dx; the rows' r go to shared memory. Phase 2: thread t sums dy * x * r over the block's rows for
// the 8-column groups t, t + 256, ... (16-byte loads of rows the block just read, mostly L2 hits)
// and writes one partial row; no atomics, so the result is deterministic.
constexpr int RMS_BWD_ROWS = 16;
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const float* __restrict__ w1, __nv_bfloat16* __restrict__ dx,
                                   float* __restrict__ dw_part, int rows, int D, float eps) {
  __shared__ float rr[RMS_BWD_ROWS];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int r0 = blockIdx.x * RMS_BWD_ROWS;
  const int r1 = min(rows, r0 + RMS_BWD_ROWS);
  for (int row = r0 + warp; row < r1; row += NORM_ROWS_PER_BLOCK) {
    const __nv_bfloat16* xr = x + (int64_t)row * D;
    const __nv_bfloat16* dyr = dy + (int64_t)row * D;
    float ss = 0.f, gx = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      uint4 p = *reinterpret_cast<const uint4*>(xr + c);
      uint4 q = *reinterpret_cast<const uint4*>(dyr + c);
      float4 wa = *reinterpret_cast<const float4*>(w1 + c), wb = *reinterpret_cast<const float4*>(w1 + c + 4);
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 a = __bfloat1622float2(p2[e]), b = __bfloat1622float2(q2[e]);
        ss += a.x * a.x + a.y * a.y;
        gx += b.x * wv[2 * e] * a.x + b.y * wv[2 * e + 1] * a.y;
      }
    }
    ss = warp_sum(ss);
    gx = warp_sum(gx);
    const float r = rsqrtf(ss / D + eps);
    const float k = r * r * r * gx / D;
    if (lane == 0) rr[row - r0] = r;
    __nv_bfloat16* dxr = dx + (int64_t)row * D;
    for (int c = lane * 8; c < D; c += 256) {
      uint4 p = *reinterpret_cast<const uint4*>(xr + c);
      uint4 q = *reinterpret_cast<const uint4*>(dyr + c);
      float4 wa = *reinterpret_cast<const float4*>(w1 + c), wb = *reinterpret_cast<const float4*>(w1 + c + 4);
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&q);
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 a = __bfloat1622float2(p2[e]), b = __bfloat1622float2(q2[e]);
        o2[e] = __floats2bfloat162_rn(r * b.x * wv[2 * e] - a.x * k, r * b.y * wv[2 * e + 1] - a.y * k);
      }
      *reinterpret_cast<uint4*>(dxr + c) = o;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int row = r0; row < r1; ++row) {
      uint4 p = *reinterpret_cast<const uint4*>(x + (int64_t)row * D + c);
      uint4 q = *reinterpret_cast<const uint4*>(dy + (int64_t)row * D + c);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&q);
      const float r = rr[row - r0];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 a = __bfloat1622float2(p2[e]), b = __bfloat1622float2(q2[e]);
        acc[2 * e] += b.x * a.x * r;
        acc[2 * e + 1] += b.y * a.y * r;
      }
    }
    float* out = dw_part + (int64_t)blockIdx.x * D + c;
    *reinterpret_cast<float4*>(out) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(out + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// out[c] = sum_p part[p][c]: a block of 32 x 8 threads per 32 columns; thread (tx, ty) sums the
// partial rows ty, ty + 8, ... of column tx (coalesced 128-byte row segments), then the 8 sums
// of a column are added in shared memory in a fixed order.
__global__ void colsum_kernel(const float* __restrict__ part, int nparts, int D, float* __restrict__ out) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.f;
  if (c < D)
    for (int p = ty; p < nparts; p += 8) s += part[(int64_t)p * D + c];
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < D) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][tx];
    out[c] = t;
  }
}

// --------------------------------------------------------------------------------- gated
// Rows of D = 32 * PER (<= 256) elements, one warp per row, lane l holding elements
// [PER l, PER l + PER) as one 2 / 4 / 8 / 16-byte vector (PER 1, 2, 4, 8; other PER element-wise).
// x, y, dy, dx, dz are [rows, D]; z is read in place from its projection: row = t * H + h lives at
// z + t * ldzt + h * D (the z slice of the fused input projection, no copy).
template <int PER>
__device__ __forceinline__ void ld_row(const __nv_bfloat16* p, float (&f)[PER], bool vec) {
  if constexpr (PER == 8) {
    if (vec) {
      uint4 u = *reinterpret_cast<const uint4*>(p);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 t = __bfloat1622float2(h[e]);
        f[2 * e] = t.x, f[2 * e + 1] = t.y;
      }
      return;
    }
  } else if constexpr (PER == 4) {
    if (vec) {
      uint2 u = *reinterpret_cast<const uint2*>(p);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float2 t = __bfloat1622float2(h[e]);
        f[2 * e] = t.x, f[2 * e + 1] = t.y;
      }
      return;
    }
  } else if constexpr (PER == 2) {
    if (vec) {
      float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
      f[0] = t.x, f[1] = t.y;
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < PER; ++e) f[e] = __bfloat162float(p[e]);
}
template <int PER>
__device__ __forceinline__ void st_row(__nv_bfloat16* p, const float (&f)[PER]) {
  if constexpr (PER == 8) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  } else if constexpr (PER == 4) {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 2; ++e) h[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
    *reinterpret_cast<uint2*>(p) = u;
  } else if constexpr (PER == 2) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(f[0], f[1]);
  } else {
#pragma unroll
    for (int e = 0; e < PER; ++e) p[e] = __float2bfloat16(f[e]);
  }
}

template <int PER>
__global__ void gated_rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ z,
                                         int64_t ldzt, int H, bool zvec, const float* __restrict__ w,
                                         __nv_bfloat16* __restrict__ y, int rows, float eps) {
  constexpr int D = 32 * PER;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row = blockIdx.x * NORM_ROWS_PER_BLOCK + warp;
  if (row >= rows) return;
  float xv[PER], zv[PER], o[PER];
  ld_row<PER>(x + (int64_t)row * D + lane * PER, xv, true);
  ld_row<PER>(z + (int64_t)(row / H) * ldzt + (int64_t)(row % H) * D + lane * PER, zv, zvec);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) ss += xv[e] * xv[e];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int c = lane * PER + e;
    const float n = __bfloat162float(__float2bfloat16(xv[e] * r));
    const float a = __bfloat162float(__float2bfloat16(w[c] * n));
    o[e] = a * silu_f(zv[e]);
  }
  st_row<PER>(y + (int64_t)row * D + lane * PER, o);
}

template <int PER>
__global__ void gated_rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                         const __nv_bfloat16* __restrict__ z, int64_t ldzt, int H, bool zvec,
                                         const float* __restrict__ w, __nv_bfloat16* __restrict__ dx,
                                         __nv_bfloat16* __restrict__ dz, float* __restrict__ dw_part, int rows,
                                         float eps, int rows_per_block) {
  constexpr int D = 32 * PER;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float wv[PER], wacc[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) wv[e] = w[lane * PER + e], wacc[e] = 0.f;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += NORM_ROWS_PER_BLOCK) {
    float xv[PER], zv[PER], dv[PER], g[PER], dzv[PER];
    ld_row<PER>(x + (int64_t)row * D + lane * PER, xv, true);
    ld_row<PER>(z + (int64_t)(row / H) * ldzt + (int64_t)(row % H) * D + lane * PER, zv, zvec);
    ld_row<PER>(dy + (int64_t)row * D + lane * PER, dv, true);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) ss += xv[e] * xv[e];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
    float gx = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const float n = xv[e] * r;
      const float zz = zv[e];
      const float sg = sigmoid_f(zz);
      const float a = wv[e] * n;
      dzv[e] = dv[e] * a * sg * (1.f + zz * (1.f - sg));
      const float da = dv[e] * zz * sg;
      wacc[e] += da * n;
      g[e] = da * wv[e];
      gx += g[e] * xv[e];
    }
    gx = warp_sum(gx);
    const float k = r * r * r * gx / D;
#pragma unroll
    for (int e = 0; e < PER; ++e) g[e] = r * g[e] - xv[e] * k;
    st_row<PER>(dz + (int64_t)row * D + lane * PER, dzv);
    st_row<PER>(dx + (int64_t)row * D + lane * PER, g);
  }
  __shared__ float red[NORM_ROWS_PER_BLOCK][D];
#pragma unroll
  for (int e = 0; e < PER; ++e) red[warp][lane * PER + e] = wacc[e];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s = 0.f;
    for (int wi = 0; wi < NORM_ROWS_PER_BLOCK; ++wi) s += red[wi][c];
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
static inline bool al16(const at::Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; }

// contiguous [rows, D] bf16 rows at a 16-byte aligned base (the kernels move rows in 16-byte
// vectors): the input itself, or a copy when its layout or a view's offset does not allow that
static at::Tensor vec_rows(const at::Tensor& x, int64_t D, const char* what) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, what, ": bf16 input expected");
  auto x2 = x.reshape({-1, D}).contiguous();
  return al16(x2) ? x2 : x2.clone();
}

// an fp32 weight of n elements at a 16-byte aligned base (read as float4)
static at::Tensor fvec(const at::Tensor& w, int64_t n, const char* what) {
  TORCH_CHECK(w.numel() == n, what, ": weight of ", n, " elements expected, got ", w.numel());
  auto f = w.to(at::kFloat).contiguous();
  return al16(f) ? f : f.clone();
}

static at::Tensor rows2d(const at::Tensor& x) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "norm: bf16 input expected");
  auto x2 = x.reshape({-1, x.size(-1)});
  if (x2.stride(-1) != 1 || x2.stride(0) % 8 || !al16(x2)) x2 = vec_rows(x2, x.size(-1), "norm");
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
  auto w = fvec(w1, D, "rmsnorm");
  dim3 grid((rows + NORM_ROWS_PER_BLOCK - 1) / NORM_ROWS_PER_BLOCK), block(32 * NORM_ROWS_PER_BLOCK);
  rmsnorm_fwd_kernel<<<grid, block, 0, stream()>>>(cbf(x2), x2.stride(0), w.data_ptr<float>(), bf(y), D, rows, D,
                                                   (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y.view(x.sizes());
}

std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w1, double eps) {
  const int D = x.size(-1);
  TORCH_CHECK(D % 8 == 0 && dy.numel() == x.numel(), "rmsnorm_bwd: D % 8 == 0, dy of x's size");
  auto x2 = vec_rows(x, D, "rmsnorm_bwd");
  auto dy2 = vec_rows(dy.to(at::kBFloat16), D, "rmsnorm_bwd");
  const int rows = x2.size(0);
  auto dx = at::empty_like(x2);
  c10::cuda::CUDAGuard g(x.device());
  auto w = fvec(w1, D, "rmsnorm_bwd");
  const int nblk = std::max(1, (rows + RMS_BWD_ROWS - 1) / RMS_BWD_ROWS);
  auto part = at::empty({nblk, D}, x.options().dtype(at::kFloat));
  auto dw = at::empty({D}, x.options().dtype(at::kFloat));
  if (rows > 0) {
    rmsnorm_bwd_kernel<<<nblk, 32 * NORM_ROWS_PER_BLOCK, 0, stream()>>>(
        cbf(dy2), cbf(x2), w.data_ptr<float>(), bf(dx), part.data_ptr<float>(), rows, D, (float)eps);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    colsum_kernel<<<(D + 31) / 32, 256, 0, stream()>>>(part.data_ptr<float>(), nblk, D, dw.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else {
    dw.zero_();
  }
  return {dx.view(x.sizes()), dw};
}

// z as [T, H, D] with unit inner stride and head stride D (any token stride): returns
// (base pointer, token stride, H, whether PER-element vector loads are aligned); other layouts
// are made contiguous first
static std::tuple<at::Tensor, int64_t, int> gated_z(const at::Tensor& z, int D, int rows) {
  at::Tensor zz = z;
  if (z.dim() >= 3 && z.stride(-1) == 1 && z.stride(-2) == D) {
    const int H = z.size(-2);
    // the leading dims must merge into one token index with a single stride
    int64_t ldt = z.dim() >= 3 ? z.stride(-3) : (int64_t)H * D;
    bool ok = true;
    for (int d = z.dim() - 4; d >= 0; --d)
      if (z.size(d) > 1 && z.stride(d) != z.stride(d + 1) * z.size(d + 1)) ok = false;
    if (ok && (int64_t)rows % H == 0) return {zz, ldt, H};
  }
  zz = z.reshape({-1, D}).contiguous();
  return {zz, (int64_t)D, 1};
}

#define BDLLM_GATED_PER(PER_, ...) \
  switch (per) {                   \
    case 1: { constexpr int PER_ = 1; __VA_ARGS__; break; } \
    case 2: { constexpr int PER_ = 2; __VA_ARGS__; break; } \
    case 3: { constexpr int PER_ = 3; __VA_ARGS__; break; } \
    case 4: { constexpr int PER_ = 4; __VA_ARGS__; break; } \
    case 5: { constexpr int PER_ = 5; __VA_ARGS__; break; } \
    case 6: { constexpr int PER_ = 6; __VA_ARGS__; break; } \
    case 7: { constexpr int PER_ = 7; __VA_ARGS__; break; } \
    default: { constexpr int PER_ = 8; __VA_ARGS__; break; } \
  }

at::Tensor gated_rmsnorm_fwd(const at::Tensor& x, const at::Tensor& z, const at::Tensor& w, double eps) {
  const int D = x.size(-1);
  TORCH_CHECK(D % 32 == 0 && D <= 256, "gated_rmsnorm: D % 32 == 0 and D <= 256");
  TORCH_CHECK(z.numel() == x.numel() && z.scalar_type() == at::kBFloat16, "gated_rmsnorm: bf16 z of x's size");
  auto x2 = vec_rows(x, D, "gated_rmsnorm");
  const int rows = x2.size(0);
  auto y = at::empty_like(x2);
  if (rows == 0) return y.view(x.sizes());
  c10::cuda::CUDAGuard g(x.device());
  auto [zz, ldzt, H] = gated_z(z, D, rows);
  const int per = D / 32;
  const bool zvec = ((reinterpret_cast<uintptr_t>(zz.data_ptr()) | (uintptr_t)(ldzt * 2)) % (per * 2)) == 0;
  auto wf = fvec(w, D, "gated_rmsnorm");
  const int nb = (rows + NORM_ROWS_PER_BLOCK - 1) / NORM_ROWS_PER_BLOCK;
  BDLLM_GATED_PER(P, gated_rmsnorm_fwd_kernel<P><<<nb, 32 * NORM_ROWS_PER_BLOCK, 0, stream()>>>(
                         cbf(x2), cbf(zz), ldzt, H, zvec, wf.data_ptr<float>(), bf(y), rows, (float)eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y.view(x.sizes());
}

std::vector<at::Tensor> gated_rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& z,
                                          const at::Tensor& w, double eps) {
  const int D = x.size(-1);
  TORCH_CHECK(D % 32 == 0 && D <= 256, "gated_rmsnorm: D % 32 == 0 and D <= 256");
  TORCH_CHECK(z.numel() == x.numel() && dy.numel() == x.numel() && z.scalar_type() == at::kBFloat16,
              "gated_rmsnorm: bf16 z and dy of x's size");
  auto x2 = vec_rows(x, D, "gated_rmsnorm_bwd");
  auto dy2 = vec_rows(dy.to(at::kBFloat16), D, "gated_rmsnorm_bwd");
  const int rows = x2.size(0);
  auto dx = at::empty_like(x2);
  auto dz = at::empty({rows, D}, x.options());
  const int rows_per_block = 128;
  const int nblk = std::max(1, (rows + rows_per_block - 1) / rows_per_block);
  auto part = at::empty({nblk, D}, x.options().dtype(at::kFloat));
  auto dw = at::zeros({D}, x.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard g(x.device());
  auto wf = fvec(w, D, "gated_rmsnorm_bwd");
  if (rows > 0) {
    auto [zz, ldzt, H] = gated_z(z, D, rows);
    const int per = D / 32;
    const bool zvec = ((reinterpret_cast<uintptr_t>(zz.data_ptr()) | (uintptr_t)(ldzt * 2)) % (per * 2)) == 0;
    BDLLM_GATED_PER(P, gated_rmsnorm_bwd_kernel<P><<<nblk, 32 * NORM_ROWS_PER_BLOCK, 0, stream()>>>(
                           cbf(dy2), cbf(x2), cbf(zz), ldzt, H, zvec, wf.data_ptr<float>(), bf(dx), bf(dz),
                           part.data_ptr<float>(), rows, (float)eps, rows_per_block));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    colsum_kernel<<<(D + 31) / 32, 256, 0, stream()>>>(part.data_ptr<float>(), nblk, D, dw.data_ptr<float>());
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
  TORCH_CHECK(cs.size(0) == T2 && cs.numel() == (int64_t)T2 * R && sn.numel() == cs.numel() && R % 2 == 0 && R <= Dh,
              "qk_norm_rope: cos / sin [T2, R], R even and <= Dh");
  auto out = at::empty({B, T2, H, Dh}, src.options());
  const int T = B * T2;
  if (T == 0) return out;
  c10::cuda::CUDAGuard g(src.device());
  auto w = fvec(w1, Dh, "qk_norm_rope");
  auto c2 = cs.to(at::kBFloat16).contiguous(), s2 = sn.to(at::kBFloat16).contiguous();
  const int64_t items = (int64_t)T * H;
  qk_norm_rope_fwd_kernel<<<(items + NORM_ROWS_PER_BLOCK - 1) / NORM_ROWS_PER_BLOCK, 32 * NORM_ROWS_PER_BLOCK, 0,
                            stream()>>>(cbf(src), src.stride(1), src.stride(2), w.data_ptr<float>(), cbf(c2), cbf(s2),
                                        bf(out), T, H, Dh, T2, R, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> qk_norm_rope_bwd(const at::Tensor& dout, const at::Tensor& src, const at::Tensor& w1,
                                         const at::Tensor& cs, const at::Tensor& sn, double eps) {
  TORCH_CHECK(src.dim() == 4 && src.stride(-1) == 1 && src.scalar_type() == at::kBFloat16,
              "qk_norm_rope: src [B, T2, H, Dh] bf16 with unit inner stride");
  const int B = src.size(0), T2 = src.size(1), H = src.size(2), Dh = src.size(3);
  TORCH_CHECK(Dh <= 256 && src.stride(0) == (int64_t)T2 * src.stride(1), "qk_norm_rope: Dh <= 256, batch and token dims merge");
  const int R = cs.size(-1);
  TORCH_CHECK(dout.numel() == (int64_t)B * T2 * H * Dh, "qk_norm_rope: dout of src's size");
  TORCH_CHECK(cs.size(0) == T2 && cs.numel() == (int64_t)T2 * R && sn.numel() == cs.numel() && R % 2 == 0 && R <= Dh,
              "qk_norm_rope: cos / sin [T2, R], R even and <= Dh");
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
  auto w = fvec(w1, Dh, "qk_norm_rope_bwd");
  auto c2 = cs.to(at::kBFloat16).contiguous(), s2 = sn.to(at::kBFloat16).contiguous();
  if (items > 0) {
    qk_norm_rope_bwd_kernel<<<nblk, 32 * NORM_ROWS_PER_BLOCK, 0, stream()>>>(
        cbf(d), cbf(src), src.stride(1), src.stride(2), w.data_ptr<float>(), cbf(c2), cbf(s2), bf(dsrc),
        dsrc.stride(1), dsrc.stride(2), part.data_ptr<float>(), T, H, Dh, T2, R, (float)eps, per_block);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    colsum_kernel<<<(Dh + 31) / 32, 256, 0, stream()>>>(part.data_ptr<float>(), nblk, Dh, dw.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {dsrc, dw};
}

}  // namespace bdllm
