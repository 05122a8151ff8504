// Task-batched LayerNorm with per-task affine parameters, fp32, and its first
// and second derivatives, for the full-MAML model (pre-LN encoder, one set of
// fast weights per task).
//
//   x [nt, R, D] rows, w, b [nt, D] (row stride ldw), eps inside the sqrt:
//   xhat = (x - mean) * rstd,  rstd = (var + eps)^-1/2,  y = xhat * w + b.
//
// With P(v) = v - mean(v) - xhat * mean(v * xhat) (symmetric in v; the
// Jacobian of xhat is rstd * P), the backward of y is
//   gx = rstd * P(gy * w),  gw = sum_rows gy * xhat,  gb = sum_rows gy,
// and the backward of that map, for cotangents (u, a, c) of (gx, gw, gb):
//   d gy = rstd * w * P(u) + a * xhat + c
//   d w  = sum_rows rstd * gy * P(u)
//   d x  = rstd * P(gy * a) - rstd^2 / D * (K * xhat + P(<u,xhat> g + <g,xhat> u)),
// with g = gy * w and K = <P(u), g> (per-row dot products over D).
//
// One warp per row (each lane keeps D/32 values in registers).  The sums over
// rows (gw, gb, d w) are formed per CTA of 16 rows of one task into a
// workspace and added up by a second, deterministic kernel.
#pragma once

#include "common.cuh"

namespace theria {
namespace ln {

constexpr int ROWS_PER_CTA = 16;  // 2 rows per warp: enough CTAs to hide the row latency
constexpr int WARPS = 8;

__device__ __forceinline__ float wsum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Row statistics: xhat in place of x, returns rstd.
template <int V>
__device__ __forceinline__ float normalize(float (&x)[V], int D, float eps) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
    if (lane + 32 * i < D) s += x[i];
  const float mean = wsum(s) / (float)D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    x[i] = lane + 32 * i < D ? x[i] - mean : 0.f;
    q = fmaf(x[i], x[i], q);
  }
  const float rstd = rsqrtf(wsum(q) / (float)D + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) x[i] *= rstd;
  return rstd;
}

// P(v) in place.
template <int V>
__device__ __forceinline__ void project(float (&v)[V], const float (&xh)[V], int D) {
  float s = 0.f, t = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    s += v[i];
    t = fmaf(v[i], xh[i], t);
  }
  const float mv = wsum(s) / (float)D, mt = wsum(t) / (float)D;
#pragma unroll
  for (int i = 0; i < V; ++i) v[i] = v[i] - mv - xh[i] * mt;
}

template <int V>
__device__ __forceinline__ void load_row(float (&r)[V], const float* p, int D) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < V; ++i) r[i] = (p && lane + 32 * i < D) ? p[lane + 32 * i] : 0.f;
}
template <int V>
__device__ __forceinline__ void store_row(float* p, const float (&r)[V], int D) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < V; ++i)
    if (lane + 32 * i < D) p[lane + 32 * i] = r[i];
}

// Grid (ceil(R / 16), nt); rows of one task per CTA.
template <int V>
__global__ void __launch_bounds__(WARPS * 32)
fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
           const float* __restrict__ b, int64_t ldw, float* __restrict__ y, int64_t R,
           int D, float eps) {
  const int warp = threadIdx.x >> 5;
  const int64_t t = blockIdx.y;
  float wr[V], br[V];
  load_row(wr, w + t * ldw, D);
  load_row(br, b + t * ldw, D);
  const int64_t r_end = R < (int64_t)(blockIdx.x + 1) * ROWS_PER_CTA
                            ? R : (int64_t)(blockIdx.x + 1) * ROWS_PER_CTA;
  for (int64_t r = (int64_t)blockIdx.x * ROWS_PER_CTA + warp; r < r_end; r += WARPS) {
    const int64_t off = (t * R + r) * D;
    float xr[V];
    load_row(xr, x + off, D);
    normalize(xr, D, eps);
#pragma unroll
    for (int i = 0; i < V; ++i) xr[i] = fmaf(xr[i], wr[i], br[i]);
    store_row(y + off, xr, D);
  }
}

// Per-CTA column sums of NS row-vectors into ws[t][cta][NS][D].
template <int V, int NS>
__device__ __forceinline__ void cta_colsum(float (&acc)[NS][V], float* smem, float* ws_cta, int D) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int i = 0; i < V; ++i) smem[(warp * NS + s) * (32 * V) + lane + 32 * i] = acc[s][i];
  __syncthreads();
  for (int e = threadIdx.x; e < NS * D; e += blockDim.x) {
    const int s = e / D, d = e - s * D;
    float v = 0.f;
#pragma unroll
    for (int wp = 0; wp < WARPS; ++wp) v += smem[(wp * NS + s) * (32 * V) + d];
    ws_cta[e] = v;
  }
}

template <int V>
__global__ void __launch_bounds__(WARPS * 32)
bwd_kernel(const float* __restrict__ x, const float* __restrict__ w, int64_t ldw,
           const float* __restrict__ gy, float* __restrict__ gx, float* __restrict__ ws,
           int64_t R, int D, float eps) {
  __shared__ float smem[WARPS * 2 * 32 * V];
  const int warp = threadIdx.x >> 5;
  const int64_t t = blockIdx.y;
  float wr[V];
  load_row(wr, w + t * ldw, D);
  float acc[2][V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[0][i] = acc[1][i] = 0.f;
  const int64_t r_end = R < (int64_t)(blockIdx.x + 1) * ROWS_PER_CTA
                            ? R : (int64_t)(blockIdx.x + 1) * ROWS_PER_CTA;
  for (int64_t r = (int64_t)blockIdx.x * ROWS_PER_CTA + warp; r < r_end; r += WARPS) {
    const int64_t off = (t * R + r) * D;
    float xh[V], g[V];
    load_row(xh, x + off, D);
    load_row(g, gy + off, D);
    const float rstd = normalize(xh, D, eps);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      acc[0][i] = fmaf(g[i], xh[i], acc[0][i]);  // gw
      acc[1][i] += g[i];                         // gb
      g[i] *= wr[i];
    }
    project(g, xh, D);
#pragma unroll
    for (int i = 0; i < V; ++i) g[i] *= rstd;
    store_row(gx + off, g, D);
  }
  cta_colsum<V, 2>(acc, smem, ws + ((int64_t)t * gridDim.x + blockIdx.x) * 2 * D, D);
}

template <int V>
__global__ void __launch_bounds__(WARPS * 32)
bwd2_kernel(const float* __restrict__ x, const float* __restrict__ w, int64_t ldw,
            const float* __restrict__ gy, const float* __restrict__ u,
            const float* __restrict__ a, int64_t lda, const float* __restrict__ c,
            int64_t ldc, float* __restrict__ dx, float* __restrict__ dgy, float* __restrict__ ws, int64_t R,
            int D, float eps) {
  __shared__ float smem[WARPS * 32 * V];
  const int warp = threadIdx.x >> 5;
  const int64_t t = blockIdx.y;
  float wr[V], ar[V], cr[V];
  load_row(wr, w + t * ldw, D);
  load_row(ar, a ? a + t * lda : nullptr, D);
  load_row(cr, c ? c + t * ldc : nullptr, D);
  float acc[1][V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[0][i] = 0.f;
  const float invD = 1.f / (float)D;
  const int64_t r_end = R < (int64_t)(blockIdx.x + 1) * ROWS_PER_CTA
                            ? R : (int64_t)(blockIdx.x + 1) * ROWS_PER_CTA;
  for (int64_t r = (int64_t)blockIdx.x * ROWS_PER_CTA + warp; r < r_end; r += WARPS) {
    const int64_t off = (t * R + r) * D;
    float xh[V], gyr[V], ur[V];
    load_row(xh, x + off, D);
    load_row(gyr, gy + off, D);
    load_row(ur, u ? u + off : nullptr, D);
    const float rstd = normalize(xh, D, eps);
    // <u, xhat>, <g, xhat> before u is projected
    float ux = 0.f, gxh = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      ux = fmaf(ur[i], xh[i], ux);
      gxh = fmaf(gyr[i] * wr[i], xh[i], gxh);
    }
    ux = wsum(ux);
    gxh = wsum(gxh);
    float v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = ux * gyr[i] * wr[i] + gxh * ur[i];
    project(v, xh, D);   // P(<u,xhat> g + <g,xhat> u)
    project(ur, xh, D);  // P(u)
    float k = 0.f;
    float o[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      k = fmaf(ur[i], gyr[i] * wr[i], k);
      o[i] = rstd * wr[i] * ur[i] + ar[i] * xh[i] + cr[i];  // d gy
      acc[0][i] = fmaf(rstd * gyr[i], ur[i], acc[0][i]);     // d w
    }
    k = wsum(k);
    store_row(dgy + off, o, D);
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = gyr[i] * ar[i];
    project(o, xh, D);  // P(gy * a)
    const float r2 = rstd * rstd * invD;
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = rstd * o[i] - r2 * (k * xh[i] + v[i]);
    store_row(dx + off, o, D);
  }
  cta_colsum<V, 1>(acc, smem, ws + ((int64_t)t * gridDim.x + blockIdx.x) * D, D);
}

// out[t][s][d] = sum_cta ws[t][cta][s][d]  (NS * D values per task); out rows
// for s = 0 .. NS-1 go to outs[s] (contiguous [nt][D]).  Grid (nt, NS*D/32):
// lanes over 32 of the NS*D columns, 32 warps over interleaved CTAs, the
// warps' partials added in a fixed order (deterministic).
constexpr int COLSUM_THREADS = 1024;
__global__ void __launch_bounds__(COLSUM_THREADS)
colsum_kernel(const float* __restrict__ ws, float* __restrict__ out0,
              float* __restrict__ out1, int n_cta, int NS, int D) {
  __shared__ float part[COLSUM_THREADS / 32][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x;
  const int W = NS * D, e = blockIdx.y * 32 + lane;
  float v = 0.f;
  if (e < W)
    for (int k = warp; k < n_cta; k += COLSUM_THREADS / 32) v += ws[((t * n_cta) + k) * W + e];
  part[warp][lane] = v;
  __syncthreads();
  if (warp == 0 && e < W) {
    float sum = 0.f;
#pragma unroll 8
    for (int w = 0; w < COLSUM_THREADS / 32; ++w) sum += part[w][lane];
    const int si = e / D, d = e - si * D;
    (si == 0 ? out0 : out1)[t * D + d] = sum;
  }
}

// Partial row sums for out[t][c] = sum_r x[t][r][c] (x [nt, R, C]
// contiguous; the bias gradient of the model's linears): grid (nt, C/32,
// ceil(R / ROWSUM_ROWS)), lanes over 32 columns, 8 warps over the CTA's rows,
// warps' partials added in a fixed order into ws[t][chunk][C]; colsum_kernel
// then adds the chunks (deterministic overall).
constexpr int ROWSUM_ROWS = 128;
__global__ void __launch_bounds__(WARPS * 32)
rowsum_partial_kernel(const float* __restrict__ x, float* __restrict__ ws, int64_t R, int C) {
  __shared__ float part[WARPS][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x;
  const int c = blockIdx.y * 32 + lane;
  const int64_t r0 = (int64_t)blockIdx.z * ROWSUM_ROWS;
  const int64_t r1 = R < r0 + ROWSUM_ROWS ? R : r0 + ROWSUM_ROWS;
  float v = 0.f;
  if (c < C) {
    const float* p = x + t * R * C + c;
#pragma unroll 4
    for (int64_t r = r0 + warp; r < r1; r += WARPS) v += p[r * C];
  }
  part[warp][lane] = v;
  __syncthreads();
  if (warp == 0 && c < C) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) sum += part[w][lane];
    ws[(t * gridDim.z + blockIdx.z) * C + c] = sum;
  }
}

// Second derivative of the exact (erf) GELU through its backward
// gx = gy * gelu'(x): for a cotangent u of gx,
//   d gy = u * gelu'(x),   d x = u * gy * gelu''(x),
// gelu'(x) = Phi(x) + x phi(x),  gelu''(x) = phi(x) (2 - x^2), with the
// standard normal cdf Phi and density phi.  Elementwise, grid-stride.
__global__ void gelu_bwd2_kernel(const float* __restrict__ x, const float* __restrict__ gy,
                                 const float* __restrict__ u, float* __restrict__ dx,
                                 float* __restrict__ dgy, int64_t n) {
  const float kInvSqrt2 = 0.70710678118654752f, kInvSqrt2Pi = 0.39894228040143268f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float xv = x[i], uv = u[i];
    const float pdf = kInvSqrt2Pi * expf(-0.5f * xv * xv);
    const float cdf = 0.5f * (1.f + erff(xv * kInvSqrt2));
    dgy[i] = uv * fmaf(xv, pdf, cdf);
    dx[i] = uv * gy[i] * pdf * (2.f - xv * xv);
  }
}

// out[t][e] = sum_c x[t][c][e] for x [nt, S, W] (the S partial products of a
// split reduction): one thread per output element, chunks added in order.
__global__ void chunk_sum_kernel(const float* __restrict__ x, float* __restrict__ out,
                                 int64_t nt, int S, int64_t W) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nt * W;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / W, e = i - t * W;
    const float* p = x + t * S * W + e;
    float v = 0.f;
    for (int c = 0; c < S; ++c) v += p[c * W];
    out[i] = v;
  }
}

// out[t][r][c] = x[t][r][c] + b[t][c] (+ res[t][r][c]) for x, res, out
// [nt, R, C] contiguous and b rows at stride ldb (0: one row for all tasks).
__global__ void add_bias_kernel(const float* __restrict__ x, const float* __restrict__ b,
                                int64_t ldb, const float* __restrict__ res,
                                float* __restrict__ out, int64_t nt, int64_t R, int64_t C) {
  const int64_t n = nt * R * C;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / (R * C), c = i % C;
    float v = x[i] + b[t * ldb + c];
    if (res) v += res[i];
    out[i] = v;
  }
}

}  // namespace ln
}  // namespace theria
