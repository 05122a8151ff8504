// CUDA-core (FFMA) SDPA kernels: forward, backward, frozen-stats JVP and
// HVP, all computed in fp32 from inputs of any supported element type.
//
// These carry the fp32 contract of the path (max relative error <= 1e-5
// against the reference's CPU fp32 math, which tensor-core TF32 cannot
// meet) and every shape the tensor-core kernels do not take (head dims
// other than 64/128, fp32 inputs).  Shapes on that path are small (the MAML
// classifier runs N=64, D=16) and latency-bound.
//
// Work split.  "Row" kernels give each warp one query row i and stream the
// keys through shared memory in tiles of 32 (lane l owns key j0+l of the
// tile); "column" kernels give each warp one key row j and stream queries
// the same way.  Row sums over keys are warp shuffles; the per-row
// accumulators over the head dim live in registers, lane l owning
// dims l, l+32, l+64, l+96.  No atomics: every output element has exactly
// one writer, so results are deterministic.
//
// Math (s = scale, P = softmax(sQK^T), LSE from the forward):
//   forward     O = P V, online softmax over key tiles
//   backward    z = rowsum(dO * O); dS = P (dO V^T - z)
//               dQ = s dS K (row), dK = s dS^T Q, dV = P^T dO (column)
//   JVP         Sdot = s (tQ K^T + Q tK^T); c = rowsum(P Sdot)
//               Odot = (P Sdot) V - c O + P tV
//   HVP of <O, W> along (tQ, tK, tV):
//               pass 1 (row): c, z = rowsum(W O), zdot = rowsum(W Odot), Odot
//               pass 2 (row): hQ = s (dSdot K + dS tK)
//               pass 3 (col): hK = s (dSdot^T Q + dS^T tQ), hV = Pdot^T W
//   with dS = P (W V^T - z), dSdot = Pdot (W V^T - z) + P (W tV^T - zdot),
//   Pdot = P (Sdot - c).
#pragma once

#include "common.cuh"

namespace theria {
namespace simt {

constexpr int KT = 32;     // keys (or queries) per shared-memory tile
constexpr int WARPS = 8;   // rows per CTA
constexpr int NC = 4;      // head-dim registers per lane (D <= 128)

// Cooperative load of rows [r0, r0+32) of a [rows, D] slice into a padded
// [32][D+1] fp32 tile; rows past `nrows` are zero.
template <typename T>
__device__ __forceinline__ void load_tile(float* dst, const T* __restrict__ src, int64_t r0,
                                          int64_t nrows, int D) {
  for (int e = threadIdx.x; e < KT * D; e += blockDim.x) {
    int r = e / D, d = e - r * D;
    int64_t gr = r0 + r;
    dst[r * (D + 1) + d] = gr < nrows ? to_f32<T>(src[gr * D + d]) : 0.f;
  }
}

// One warp loads a D-vector.
template <typename T>
__device__ __forceinline__ void load_vec(float* dst, const T* __restrict__ src, int D, int lane) {
  for (int d = lane; d < D; d += 32) dst[d] = to_f32<T>(src[d]);
}

__device__ __forceinline__ float dot_tile(const float* vec, const float* tile_row, int D) {
  float a = 0.f;
  for (int d = 0; d < D; ++d) a = fmaf(vec[d], tile_row[d], a);
  return a;
}

// acc[c] += sum_l coef(lane l) * tile[l][lane + 32c]
__device__ __forceinline__ void acc_tile(float (&acc)[NC], float coef, const float* tile, int D,
                                         int lane) {
#pragma unroll 4
  for (int l = 0; l < KT; ++l) {
    float w = __shfl_sync(0xffffffffu, coef, l);
    const float* row = tile + l * (D + 1);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      int d = lane + 32 * c;
      if (d < D) acc[c] = fmaf(w, row[d], acc[c]);
    }
  }
}

__device__ __forceinline__ float vec_dot_acc(const float (&acc)[NC], const float* vec, int D,
                                             int lane) {
  float a = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    int d = lane + 32 * c;
    if (d < D) a = fmaf(acc[c], vec[d], a);
  }
  return warp_sum(a);
}

template <typename OT>
__device__ __forceinline__ void store_acc(OT* dst, const float (&acc)[NC], float mul, int D,
                                          int lane) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    int d = lane + 32 * c;
    if (d < D) dst[d] = from_f32<OT>(acc[c] * mul);
  }
}

__device__ __forceinline__ void store_acc_any(void* dst, int64_t off, int dtype,
                                              const float (&acc)[NC], float mul, int D,
                                              int lane) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    int d = lane + 32 * c;
    if (d < D) store_any(dst, off + d, dtype, acc[c] * mul);
  }
}

// Last key a CTA of row kernels must visit (exclusive).
__device__ __forceinline__ int64_t row_kend(const Shape& s) {
  if (!s.causal) return s.M;
  int64_t last_row = (int64_t)blockIdx.x * WARPS + WARPS - 1;
  if (last_row > s.T - 1) last_row = s.T - 1;
  return last_row + 1 < s.M ? last_row + 1 : s.M;
}

// First query a CTA of column kernels must visit (tile aligned).
__device__ __forceinline__ int64_t col_qbegin(const Shape& s) {
  if (!s.causal) return 0;
  int64_t first_key = (int64_t)blockIdx.x * WARPS;
  return (first_key / KT) * KT;
}

// ---------------------------------------------------------------- forward
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
fwd_row_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               void* __restrict__ o, int o_dtype, float* __restrict__ lse, Shape s) {
  extern __shared__ float sm[];
  const int D = (int)s.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* Ks = sm;
  float* Vs = Ks + KT * (D + 1);
  float* qv = Vs + KT * (D + 1) + warp * D;
  const int64_t bh = blockIdx.y;
  const int64_t row = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = row < s.T;
  const T* kb = k + bh * s.M * D;
  const T* vb = v + bh * s.M * D;
  if (active) load_vec(qv, q + (bh * s.T + row) * D, D, lane);
  float m = -INFINITY, l = 0.f, acc[NC] = {0.f, 0.f, 0.f, 0.f};
  const int64_t kend = row_kend(s);
  for (int64_t j0 = 0; j0 < kend; j0 += KT) {
    __syncthreads();
    load_tile(Ks, kb, j0, s.M, D);
    load_tile(Vs, vb, j0, s.M, D);
    __syncthreads();
    if (!active) continue;
    int64_t j = j0 + lane;
    bool valid = j < s.M && (!s.causal || j <= row);
    float sc = valid ? s.scale * dot_tile(qv, Ks + lane * (D + 1), D) : -INFINITY;
    float mnew = fmaxf(m, warp_max(sc));
    if (mnew == -INFINITY) continue;
    float p = valid ? expf(sc - mnew) : 0.f;
    float corr = expf(m - mnew);
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[c] *= corr;
    acc_tile(acc, p, Vs, D, lane);
    m = mnew;
  }
  if (!active) return;
  float inv = l > 0.f ? 1.f / l : 0.f;
  store_acc_any(o, (bh * s.T + row) * D, o_dtype, acc, inv, D, lane);
  if (lse != nullptr && lane == 0) lse[bh * s.T + row] = l > 0.f ? m + logf(l) : -INFINITY;
}

// --------------------------------------------------- backward: z = rowsum(dO O)
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
delta_from_o_kernel(const void* __restrict__ o, int o_dtype, const T* __restrict__ dout,
                    float* __restrict__ z, int64_t rows, int D) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  float a = 0.f;
  for (int d = lane; d < D; d += 32)
    a = fmaf(to_f32<T>(dout[row * D + d]), load_any(o, row * D + d, o_dtype), a);
  a = warp_sum(a);
  if (lane == 0) z[row] = a;
}

// z = sum_j P_ij (dO_i . V_j), when the forward output is not at hand.
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
delta_from_stats_kernel(const T* __restrict__ q, const T* __restrict__ k,
                        const T* __restrict__ v, const T* __restrict__ dout,
                        const float* __restrict__ lse, float* __restrict__ z, Shape s) {
  extern __shared__ float sm[];
  const int D = (int)s.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* Ks = sm;
  float* Vs = Ks + KT * (D + 1);
  float* qv = Vs + KT * (D + 1) + warp * 2 * D;
  float* gv = qv + D;
  const int64_t bh = blockIdx.y;
  const int64_t row = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = row < s.T;
  if (active) {
    load_vec(qv, q + (bh * s.T + row) * D, D, lane);
    load_vec(gv, dout + (bh * s.T + row) * D, D, lane);
  }
  const float L = active ? lse[bh * s.T + row] : 0.f;
  float zacc = 0.f;
  const int64_t kend = row_kend(s);
  for (int64_t j0 = 0; j0 < kend; j0 += KT) {
    __syncthreads();
    load_tile(Ks, k + bh * s.M * D, j0, s.M, D);
    load_tile(Vs, v + bh * s.M * D, j0, s.M, D);
    __syncthreads();
    if (!active) continue;
    int64_t j = j0 + lane;
    bool valid = j < s.M && (!s.causal || j <= row);
    if (valid) {
      float p = expf(s.scale * dot_tile(qv, Ks + lane * (D + 1), D) - L);
      zacc = fmaf(p, dot_tile(gv, Vs + lane * (D + 1), D), zacc);
    }
  }
  zacc = warp_sum(zacc);
  if (active && lane == 0) z[bh * s.T + row] = zacc;
}

// ------------------------------------------------------- backward: dQ (row)
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
dq_row_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
              const T* __restrict__ dout, const float* __restrict__ lse,
              const float* __restrict__ z, T* __restrict__ dq, Shape s) {
  extern __shared__ float sm[];
  const int D = (int)s.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* Ks = sm;
  float* Vs = Ks + KT * (D + 1);
  float* qv = Vs + KT * (D + 1) + warp * 2 * D;
  float* gv = qv + D;
  const int64_t bh = blockIdx.y;
  const int64_t row = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = row < s.T;
  if (active) {
    load_vec(qv, q + (bh * s.T + row) * D, D, lane);
    load_vec(gv, dout + (bh * s.T + row) * D, D, lane);
  }
  const float L = active ? lse[bh * s.T + row] : 0.f;
  const float zi = active ? z[bh * s.T + row] : 0.f;
  float acc[NC] = {0.f, 0.f, 0.f, 0.f};
  const int64_t kend = row_kend(s);
  for (int64_t j0 = 0; j0 < kend; j0 += KT) {
    __syncthreads();
    load_tile(Ks, k + bh * s.M * D, j0, s.M, D);
    load_tile(Vs, v + bh * s.M * D, j0, s.M, D);
    __syncthreads();
    if (!active) continue;
    int64_t j = j0 + lane;
    bool valid = j < s.M && (!s.causal || j <= row);
    float ds = 0.f;
    if (valid) {
      float p = expf(s.scale * dot_tile(qv, Ks + lane * (D + 1), D) - L);
      ds = p * (dot_tile(gv, Vs + lane * (D + 1), D) - zi);
    }
    acc_tile(acc, ds, Ks, D, lane);
  }
  if (active) store_acc(dq + (bh * s.T + row) * D, acc, s.scale, D, lane);
}

// ---------------------------------------------- backward: dK, dV (column)
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
dkdv_col_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const T* __restrict__ dout, const float* __restrict__ lse,
                const float* __restrict__ z, T* __restrict__ dk, T* __restrict__ dv, Shape s) {
  extern __shared__ float sm[];
  const int D = (int)s.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* Qs = sm;
  float* Gs = Qs + KT * (D + 1);
  float* Ls = Gs + KT * (D + 1);
  float* Zs = Ls + KT;
  float* kv = Zs + KT + warp * 2 * D;
  float* vv = kv + D;
  const int64_t bh = blockIdx.y;
  const int64_t col = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = col < s.M;
  if (active) {
    load_vec(kv, k + (bh * s.M + col) * D, D, lane);
    load_vec(vv, v + (bh * s.M + col) * D, D, lane);
  }
  float ak[NC] = {0.f, 0.f, 0.f, 0.f}, av[NC] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t i0 = col_qbegin(s); i0 < s.T; i0 += KT) {
    __syncthreads();
    load_tile(Qs, q + bh * s.T * D, i0, s.T, D);
    load_tile(Gs, dout + bh * s.T * D, i0, s.T, D);
    if (threadIdx.x < KT) {
      int64_t i = i0 + threadIdx.x;
      Ls[threadIdx.x] = i < s.T ? lse[bh * s.T + i] : 0.f;
      Zs[threadIdx.x] = i < s.T ? z[bh * s.T + i] : 0.f;
    }
    __syncthreads();
    if (!active) continue;
    int64_t i = i0 + lane;
    bool valid = i < s.T && (!s.causal || col <= i);
    float p = 0.f, ds = 0.f;
    if (valid) {
      p = expf(s.scale * dot_tile(kv, Qs + lane * (D + 1), D) - Ls[lane]);
      ds = p * (dot_tile(vv, Gs + lane * (D + 1), D) - Zs[lane]);
    }
    acc_tile(ak, ds, Qs, D, lane);
    acc_tile(av, p, Gs, D, lane);
  }
  if (!active) return;
  if (dk) store_acc(dk + (bh * s.M + col) * D, ak, s.scale, D, lane);
  if (dv) store_acc(dv + (bh * s.M + col) * D, av, 1.f, D, lane);
}

// ------------------------------------------ JVP (and HVP pass 1), row
// Writes Odot (if o_tan); with w != nullptr also rows c, z, zdot into
// stats[0..3) (each [B*H*T]).
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
jvp_row_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const T* __restrict__ tq, const T* __restrict__ tk, const T* __restrict__ tv,
               const T* __restrict__ w, const float* __restrict__ lse,
               T* __restrict__ o_tan, float* __restrict__ stats, Shape s) {
  extern __shared__ float sm[];
  const int D = (int)s.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = KT * (D + 1);
  float* Ks = sm;
  float* Vs = Ks + tile;
  float* TKs = Vs + tile;
  float* TVs = TKs + tile;
  float* qv = TVs + tile + warp * 3 * D;
  float* tqv = qv + D;
  float* wv = tqv + D;
  const int64_t bh = blockIdx.y;
  const int64_t row = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = row < s.T;
  const int64_t roff = (bh * s.T + row) * D;
  if (active) {
    load_vec(qv, q + roff, D, lane);
    load_vec(tqv, tq + roff, D, lane);
    if (w) load_vec(wv, w + roff, D, lane);
  }
  const float L = active ? lse[bh * s.T + row] : 0.f;
  float aA[NC] = {0.f, 0.f, 0.f, 0.f}, aO[NC] = {0.f, 0.f, 0.f, 0.f},
        aB[NC] = {0.f, 0.f, 0.f, 0.f};
  float cacc = 0.f;
  const int64_t kend = row_kend(s);
  for (int64_t j0 = 0; j0 < kend; j0 += KT) {
    __syncthreads();
    load_tile(Ks, k + bh * s.M * D, j0, s.M, D);
    load_tile(Vs, v + bh * s.M * D, j0, s.M, D);
    load_tile(TKs, tk + bh * s.M * D, j0, s.M, D);
    load_tile(TVs, tv + bh * s.M * D, j0, s.M, D);
    __syncthreads();
    if (!active) continue;
    int64_t j = j0 + lane;
    bool valid = j < s.M && (!s.causal || j <= row);
    float p = 0.f, psd = 0.f;
    if (valid) {
      const float* kr = Ks + lane * (D + 1);
      p = expf(s.scale * dot_tile(qv, kr, D) - L);
      float sd = s.scale * (dot_tile(tqv, kr, D) + dot_tile(qv, TKs + lane * (D + 1), D));
      psd = p * sd;
    }
    cacc += psd;
    acc_tile(aA, psd, Vs, D, lane);
    acc_tile(aO, p, Vs, D, lane);
    acc_tile(aB, p, TVs, D, lane);
  }
  if (!active) return;
  const float c = warp_sum(cacc);
  float od[NC];
#pragma unroll
  for (int cc = 0; cc < NC; ++cc) od[cc] = aA[cc] - c * aO[cc] + aB[cc];
  if (o_tan) store_acc(o_tan + roff, od, 1.f, D, lane);
  if (w) {
    float zi = vec_dot_acc(aO, wv, D, lane);
    float zd = vec_dot_acc(od, wv, D, lane);
    if (lane == 0) {
      const int64_t n = s.B * s.H * s.T, r = bh * s.T + row;
      stats[r] = c;
      stats[n + r] = zi;
      stats[2 * n + r] = zd;
    }
  }
}

// Per-element HVP terms shared by the row and column kernels.
struct HvpTerms {
  float p, pd, ds, dsd;
};
__device__ __forceinline__ HvpTerms hvp_terms(float sc, float sd, float dp, float dpd, float L,
                                              float c, float zi, float zd) {
  HvpTerms t;
  t.p = expf(sc - L);
  t.pd = t.p * (sd - c);
  t.ds = t.p * (dp - zi);
  t.dsd = t.pd * (dp - zi) + t.p * (dpd - zd);
  return t;
}

// ------------------------------------------------------- HVP pass 2: hQ
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
hq_row_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
              const T* __restrict__ tq, const T* __restrict__ tk, const T* __restrict__ tv,
              const T* __restrict__ w, const float* __restrict__ lse,
              const float* __restrict__ stats, T* __restrict__ hq, Shape s) {
  extern __shared__ float sm[];
  const int D = (int)s.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = KT * (D + 1);
  float* Ks = sm;
  float* Vs = Ks + tile;
  float* TKs = Vs + tile;
  float* TVs = TKs + tile;
  float* qv = TVs + tile + warp * 3 * D;
  float* tqv = qv + D;
  float* wv = tqv + D;
  const int64_t bh = blockIdx.y;
  const int64_t row = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = row < s.T;
  const int64_t roff = (bh * s.T + row) * D;
  const int64_t n = s.B * s.H * s.T, r = bh * s.T + row;
  if (active) {
    load_vec(qv, q + roff, D, lane);
    load_vec(tqv, tq + roff, D, lane);
    load_vec(wv, w + roff, D, lane);
  }
  const float L = active ? lse[r] : 0.f;
  const float c = active ? stats[r] : 0.f;
  const float zi = active ? stats[n + r] : 0.f;
  const float zd = active ? stats[2 * n + r] : 0.f;
  float acc[NC] = {0.f, 0.f, 0.f, 0.f};
  const int64_t kend = row_kend(s);
  for (int64_t j0 = 0; j0 < kend; j0 += KT) {
    __syncthreads();
    load_tile(Ks, k + bh * s.M * D, j0, s.M, D);
    load_tile(Vs, v + bh * s.M * D, j0, s.M, D);
    load_tile(TKs, tk + bh * s.M * D, j0, s.M, D);
    load_tile(TVs, tv + bh * s.M * D, j0, s.M, D);
    __syncthreads();
    if (!active) continue;
    int64_t j = j0 + lane;
    bool valid = j < s.M && (!s.causal || j <= row);
    float ds = 0.f, dsd = 0.f;
    if (valid) {
      const float* kr = Ks + lane * (D + 1);
      const float* tkr = TKs + lane * (D + 1);
      float sc = s.scale * dot_tile(qv, kr, D);
      float sd = s.scale * (dot_tile(tqv, kr, D) + dot_tile(qv, tkr, D));
      float dp = dot_tile(wv, Vs + lane * (D + 1), D);
      float dpd = dot_tile(wv, TVs + lane * (D + 1), D);
      HvpTerms t = hvp_terms(sc, sd, dp, dpd, L, c, zi, zd);
      ds = t.ds;
      dsd = t.dsd;
    }
    acc_tile(acc, dsd, Ks, D, lane);
    acc_tile(acc, ds, TKs, D, lane);
  }
  if (active) store_acc(hq + roff, acc, s.scale, D, lane);
}

// ------------------------------------------------ HVP pass 3: hK, hV (column)
template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
hkhv_col_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const T* __restrict__ tq, const T* __restrict__ tk, const T* __restrict__ tv,
                const T* __restrict__ w, const float* __restrict__ lse,
                const float* __restrict__ stats, T* __restrict__ hk, T* __restrict__ hv,
                Shape s) {
  extern __shared__ float sm[];
  const int D = (int)s.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tile = KT * (D + 1);
  float* Qs = sm;
  float* TQs = Qs + tile;
  float* Ws = TQs + tile;
  float* Ls = Ws + tile;  // 4 x KT row scalars: lse, c, z, zdot
  float* kv = Ls + 4 * KT + warp * 4 * D;
  float* vv = kv + D;
  float* tkv = vv + D;
  float* tvv = tkv + D;
  const int64_t bh = blockIdx.y;
  const int64_t col = (int64_t)blockIdx.x * WARPS + warp;
  const bool active = col < s.M;
  const int64_t n = s.B * s.H * s.T;
  if (active) {
    const int64_t coff = (bh * s.M + col) * D;
    load_vec(kv, k + coff, D, lane);
    load_vec(vv, v + coff, D, lane);
    load_vec(tkv, tk + coff, D, lane);
    load_vec(tvv, tv + coff, D, lane);
  }
  float ak[NC] = {0.f, 0.f, 0.f, 0.f}, av[NC] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t i0 = col_qbegin(s); i0 < s.T; i0 += KT) {
    __syncthreads();
    load_tile(Qs, q + bh * s.T * D, i0, s.T, D);
    load_tile(TQs, tq + bh * s.T * D, i0, s.T, D);
    load_tile(Ws, w + bh * s.T * D, i0, s.T, D);
    if (threadIdx.x < KT) {
      int64_t i = i0 + threadIdx.x;
      bool ok = i < s.T;
      int64_t r = bh * s.T + i;
      Ls[threadIdx.x] = ok ? lse[r] : 0.f;
      Ls[KT + threadIdx.x] = ok ? stats[r] : 0.f;
      Ls[2 * KT + threadIdx.x] = ok ? stats[n + r] : 0.f;
      Ls[3 * KT + threadIdx.x] = ok ? stats[2 * n + r] : 0.f;
    }
    __syncthreads();
    if (!active) continue;
    int64_t i = i0 + lane;
    bool valid = i < s.T && (!s.causal || col <= i);
    float pd = 0.f, ds = 0.f, dsd = 0.f;
    if (valid) {
      const float* qr = Qs + lane * (D + 1);
      const float* wr = Ws + lane * (D + 1);
      float sc = s.scale * dot_tile(kv, qr, D);
      float sd = s.scale * (dot_tile(kv, TQs + lane * (D + 1), D) + dot_tile(tkv, qr, D));
      float dp = dot_tile(vv, wr, D);
      float dpd = dot_tile(tvv, wr, D);
      HvpTerms t = hvp_terms(sc, sd, dp, dpd, Ls[lane], Ls[KT + lane], Ls[2 * KT + lane],
                             Ls[3 * KT + lane]);
      pd = t.pd;
      ds = t.ds;
      dsd = t.dsd;
    }
    acc_tile(ak, dsd, Qs, D, lane);
    acc_tile(ak, ds, TQs, D, lane);
    acc_tile(av, pd, Ws, D, lane);
  }
  if (!active) return;
  const int64_t coff = (bh * s.M + col) * D;
  if (hk) store_acc(hk + coff, ak, s.scale, D, lane);
  if (hv) store_acc(hv + coff, av, 1.f, D, lane);
}

}  // namespace simt
}  // namespace theria
