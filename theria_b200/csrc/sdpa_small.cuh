// Whole-head SDPA kernels for short sequences (T, M <= 64, D <= 64), fp32
// compute from any input dtype.
//
// One CTA holds one (batch, head) entirely in shared memory -- its inputs
// and the T x M score-shaped matrices -- and runs a whole operator in one
// launch: forward, backward (dQ, dK, dV with z formed in place), JVP, or the
// full HVP (hQ, hK, hV and Odot).  This is the regime of the full-MAML
// classifier (N = 64, head dim 16, thousands of heads per call), where the
// tiled kernels would run one nearly empty tile per head.
//
// Every product is an element-parallel loop over the output (thread e
// computes elements e, e + blockDim, ...) with the reduction dimension read
// from padded shared rows (stride D+1 or M+1); row statistics are one
// thread per row.  Results are deterministic.
#pragma once

#include "common.cuh"

namespace theria {
namespace small {

constexpr int MAXN = 64;   // max T and M
constexpr int MAXD = 64;   // max head dim
constexpr int NTHREADS = 256;

// Arithmetic in the accumulator type A: float for fp32/fp16/bf16 inputs,
// double for fp64 inputs (the fp64 variant serves gradcheck-style checks).
__device__ __forceinline__ float fmaA(float a, float b, float c) { return fmaf(a, b, c); }
__device__ __forceinline__ double fmaA(double a, double b, double c) { return fma(a, b, c); }
__device__ __forceinline__ float expA(float x) { return expf(x); }
__device__ __forceinline__ double expA(double x) { return exp(x); }
__device__ __forceinline__ float logA(float x) { return logf(x); }
__device__ __forceinline__ double logA(double x) { return log(x); }
__device__ __forceinline__ float maxA(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double maxA(double a, double b) { return fmax(a, b); }
template <typename A, typename T>
__device__ __forceinline__ A load_as(T x) { return (A)to_f32<T>(x); }
template <>
__device__ __forceinline__ double load_as<double, double>(double x) { return x; }
template <typename OT, typename A>
__device__ __forceinline__ OT store_as(A x) { return from_f32<OT>((float)x); }
template <>
__device__ __forceinline__ double store_as<double, double>(double x) { return x; }

inline size_t smem_bytes(int T, int M, int D, int n_q_like, int n_k_like, int n_scores,
                         size_t elem = sizeof(float)) {
  return elem * ((size_t)n_q_like * T * (D + 1) + (size_t)n_k_like * M * (D + 1) +
                          (size_t)n_scores * T * (M + 1) + 4 * (size_t)T);
}

template <typename A, typename T>
__device__ __forceinline__ void load_mat(A* dst, const T* __restrict__ src, int rows, int D) {
  for (int e = threadIdx.x; e < rows * D; e += blockDim.x) {
    const int r = e / D, d = e - r * D;
    dst[r * (D + 1) + d] = load_as<A>(src[e]);
  }
}

// The products below give each thread 2 x 2 blocks of outputs, so every
// shared-memory value loaded feeds two FMAs (the single-output form was
// bound by shared-memory loads).  Odd extents are handled by clamping the
// second row/column to the first and not storing it.

// C[i][j] = alpha * (sum_d A1[i][d] B1[j][d] [+ A2[i][d] B2[j][d]])
template <bool TWO, typename A>
__device__ __forceinline__ void abt_impl(A* C, int ldc, const A* A1, const A* B1,
                                         const A* A2, const A* B2, int rA, int rB,
                                         int D, A alpha) {
  const int nbj = (rB + 1) >> 1, nb = ((rA + 1) >> 1) * nbj;
  for (int e = threadIdx.x; e < nb; e += blockDim.x) {
    const int i0 = 2 * (e / nbj), j0 = 2 * (e % nbj);
    const int i1 = min(i0 + 1, rA - 1), j1 = min(j0 + 1, rB - 1);
    A c00 = A(0), c01 = A(0), c10 = A(0), c11 = A(0);
    {
      const A *a0 = A1 + i0 * (D + 1), *a1 = A1 + i1 * (D + 1);
      const A *b0 = B1 + j0 * (D + 1), *b1 = B1 + j1 * (D + 1);
      for (int d = 0; d < D; ++d) {
        c00 = fmaA(a0[d], b0[d], c00);
        c01 = fmaA(a0[d], b1[d], c01);
        c10 = fmaA(a1[d], b0[d], c10);
        c11 = fmaA(a1[d], b1[d], c11);
      }
    }
    if (TWO) {
      const A *a0 = A2 + i0 * (D + 1), *a1 = A2 + i1 * (D + 1);
      const A *b0 = B2 + j0 * (D + 1), *b1 = B2 + j1 * (D + 1);
      for (int d = 0; d < D; ++d) {
        c00 = fmaA(a0[d], b0[d], c00);
        c01 = fmaA(a0[d], b1[d], c01);
        c10 = fmaA(a1[d], b0[d], c10);
        c11 = fmaA(a1[d], b1[d], c11);
      }
    }
    C[i0 * ldc + j0] = alpha * c00;
    if (j0 + 1 < rB) C[i0 * ldc + j0 + 1] = alpha * c01;
    if (i0 + 1 < rA) {
      C[(i0 + 1) * ldc + j0] = alpha * c10;
      if (j0 + 1 < rB) C[(i0 + 1) * ldc + j0 + 1] = alpha * c11;
    }
  }
}

template <typename A>
__device__ __forceinline__ void abt(A* C, int ldc, const A* X, const A* Y, int rA,
                                    int rB, int D, A alpha) {
  abt_impl<false, A>(C, ldc, X, Y, nullptr, nullptr, rA, rB, D, alpha);
}

// C = alpha * (A1 B1^T + A2 B2^T)
template <typename A>
__device__ __forceinline__ void abt2(A* C, int ldc, const A* A1, const A* B1,
                                     const A* A2, const A* B2, int rA, int rB, int D,
                                     A alpha) {
  abt_impl<true, A>(C, ldc, A1, B1, A2, B2, rA, rB, D, alpha);
}

template <typename OT, typename A>
__device__ __forceinline__ void store2x2(OT* out, int ldo, int i0, int d0, int nI, int nD,
                                         A alpha, A c00, A c01, A c10,
                                         A c11) {
  out[i0 * ldo + d0] = store_as<OT>(alpha * c00);
  if (d0 + 1 < nD) out[i0 * ldo + d0 + 1] = store_as<OT>(alpha * c01);
  if (i0 + 1 < nI) {
    out[(i0 + 1) * ldo + d0] = store_as<OT>(alpha * c10);
    if (d0 + 1 < nD) out[(i0 + 1) * ldo + d0 + 1] = store_as<OT>(alpha * c11);
  }
}

// out[i][d] = alpha * sum_j (S1[i][j] X1[j][d] [+ S2[i][j] X2[j][d]])
//   (S: [rS][cS] at stride lds; X: [cS][D]; out: [rS][D] dense)
template <bool TWO, typename OT, typename A>
__device__ __forceinline__ void sx_impl(OT* __restrict__ out, const A* S1, const A* X1,
                                        const A* S2, const A* X2, int lds, int rS,
                                        int cS, int D, A alpha) {
  const int nbd = (D + 1) >> 1, nb = ((rS + 1) >> 1) * nbd;
  for (int e = threadIdx.x; e < nb; e += blockDim.x) {
    const int i0 = 2 * (e / nbd), d0 = 2 * (e % nbd);
    const int i1 = min(i0 + 1, rS - 1), d1 = min(d0 + 1, D - 1);
    A c00 = A(0), c01 = A(0), c10 = A(0), c11 = A(0);
    for (int j = 0; j < cS; ++j) {
      const A s0 = S1[i0 * lds + j], s1 = S1[i1 * lds + j];
      const A x0 = X1[j * (D + 1) + d0], x1 = X1[j * (D + 1) + d1];
      c00 = fmaA(s0, x0, c00);
      c01 = fmaA(s0, x1, c01);
      c10 = fmaA(s1, x0, c10);
      c11 = fmaA(s1, x1, c11);
      if (TWO) {
        const A t0 = S2[i0 * lds + j], t1 = S2[i1 * lds + j];
        const A y0 = X2[j * (D + 1) + d0], y1 = X2[j * (D + 1) + d1];
        c00 = fmaA(t0, y0, c00);
        c01 = fmaA(t0, y1, c01);
        c10 = fmaA(t1, y0, c10);
        c11 = fmaA(t1, y1, c11);
      }
    }
    store2x2(out, D, i0, d0, rS, D, alpha, c00, c01, c10, c11);
  }
}

// out[j][d] = alpha * sum_i (S1[i][j] X1[i][d] [+ S2[i][j] X2[i][d]])  (S transposed)
template <bool TWO, typename OT, typename A>
__device__ __forceinline__ void stx_impl(OT* __restrict__ out, const A* S1, const A* X1,
                                         const A* S2, const A* X2, int lds, int rS,
                                         int cS, int D, A alpha) {
  const int nbd = (D + 1) >> 1, nb = ((cS + 1) >> 1) * nbd;
  for (int e = threadIdx.x; e < nb; e += blockDim.x) {
    const int j0 = 2 * (e / nbd), d0 = 2 * (e % nbd);
    const int j1 = min(j0 + 1, cS - 1), d1 = min(d0 + 1, D - 1);
    A c00 = A(0), c01 = A(0), c10 = A(0), c11 = A(0);
    for (int i = 0; i < rS; ++i) {
      const A s0 = S1[i * lds + j0], s1 = S1[i * lds + j1];
      const A x0 = X1[i * (D + 1) + d0], x1 = X1[i * (D + 1) + d1];
      c00 = fmaA(s0, x0, c00);
      c01 = fmaA(s0, x1, c01);
      c10 = fmaA(s1, x0, c10);
      c11 = fmaA(s1, x1, c11);
      if (TWO) {
        const A t0 = S2[i * lds + j0], t1 = S2[i * lds + j1];
        const A y0 = X2[i * (D + 1) + d0], y1 = X2[i * (D + 1) + d1];
        c00 = fmaA(t0, y0, c00);
        c01 = fmaA(t0, y1, c01);
        c10 = fmaA(t1, y0, c10);
        c11 = fmaA(t1, y1, c11);
      }
    }
    store2x2(out, D, j0, d0, cS, D, alpha, c00, c01, c10, c11);
  }
}

template <typename OT, typename A>
__device__ __forceinline__ void sx(OT* __restrict__ out, const A* S, int lds, const A* X,
                                   int rS, int cS, int D, A alpha) {
  sx_impl<false, OT, A>(out, S, X, nullptr, nullptr, lds, rS, cS, D, alpha);
}
template <typename OT, typename A>
__device__ __forceinline__ void sx2(OT* __restrict__ out, const A* S1, const A* X1,
                                    const A* S2, const A* X2, int lds, int rS, int cS,
                                    int D, A alpha) {
  sx_impl<true, OT, A>(out, S1, X1, S2, X2, lds, rS, cS, D, alpha);
}
template <typename OT, typename A>
__device__ __forceinline__ void stx(OT* __restrict__ out, const A* S, int lds,
                                    const A* X, int rS, int cS, int D, A alpha) {
  stx_impl<false, OT, A>(out, S, X, nullptr, nullptr, lds, rS, cS, D, alpha);
}
template <typename OT, typename A>
__device__ __forceinline__ void stx2(OT* __restrict__ out, const A* S1, const A* X1,
                                     const A* S2, const A* X2, int lds, int rS, int cS,
                                     int D, A alpha) {
  stx_impl<true, OT, A>(out, S1, X1, S2, X2, lds, rS, cS, D, alpha);
}

__device__ __forceinline__ bool masked(int i, int j, int causal) { return causal && j > i; }

// fp64 rebuilds the row logsumexp from the scores in double precision: the
// float32 lse the forward saved would make P (and so every derivative) a
// non-smooth function of the inputs at the 1e-7 level, which is what
// finite-difference checks in fp64 resolve.  Other types keep the saved lse.
template <typename A>
__device__ __forceinline__ void exact_lse(const A* S, int lds, A* lse_s, int T, int M,
                                          int causal) {
  if constexpr (sizeof(A) == sizeof(double)) {
    for (int i = threadIdx.x; i < T; i += blockDim.x) {
      A m = -INFINITY;
      for (int j = 0; j < M; ++j)
        if (!masked(i, j, causal)) m = maxA(m, S[i * lds + j]);
      A l = A(0);
      for (int j = 0; j < M; ++j)
        if (!masked(i, j, causal)) l += expA(S[i * lds + j] - m);
      lse_s[i] = m + logA(l);
    }
  }
}

// P[i][j] = exp(S[i][j] - lse_i) in place (0 where masked).
template <typename A>
__device__ __forceinline__ void probs_from_lse(A* S, int lds, const A* lse_s, int T,
                                               int M, int causal) {
  for (int e = threadIdx.x; e < T * M; e += blockDim.x) {
    const int i = e / M, j = e - i * M;
    S[i * lds + j] = masked(i, j, causal) ? A(0) : expA(S[i * lds + j] - lse_s[i]);
  }
}

// ---------------------------------------------------------------- forward
template <typename T, typename OT, typename A = float>
__global__ void __launch_bounds__(NTHREADS)
fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           OT* __restrict__ o, float* __restrict__ lse, Shape s) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  A* Q = sm;
  A* K = Q + Tq * (D + 1);
  A* V = K + M * (D + 1);
  A* S = V + M * (D + 1);
  load_mat(Q, q + bh * Tq * D, Tq, D);
  load_mat(K, k + bh * M * D, M, D);
  load_mat(V, v + bh * M * D, M, D);
  __syncthreads();
  abt(S, lm, Q, K, Tq, M, D, A(s.scale));
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    A m = -INFINITY;
    for (int j = 0; j < M; ++j)
      if (!masked(i, j, s.causal)) m = maxA(m, S[i * lm + j]);
    A l = A(0);
    for (int j = 0; j < M; ++j) {
      const A p = masked(i, j, s.causal) ? A(0) : expA(S[i * lm + j] - m);
      S[i * lm + j] = p;
      l += p;
    }
    const A inv = A(1) / l;
    for (int j = 0; j < M; ++j) S[i * lm + j] *= inv;
    if (lse) lse[bh * Tq + i] = m + logA(l);
  }
  __syncthreads();
  sx(o + bh * Tq * D, S, lm, V, Tq, M, D, A(1));
}

// ---------------------------------------------------------------- backward
template <typename T, typename A = float>
__global__ void __launch_bounds__(NTHREADS)
bwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ dout, const float* __restrict__ lse, T* __restrict__ dq,
           T* __restrict__ dk, T* __restrict__ dv, Shape s) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  A* Q = sm;
  A* G = Q + Tq * (D + 1);  // dO
  A* K = G + Tq * (D + 1);
  A* V = K + M * (D + 1);
  A* P = V + M * (D + 1);
  A* DS = P + Tq * lm;
  A* L = DS + Tq * lm;
  load_mat(Q, q + bh * Tq * D, Tq, D);
  load_mat(G, dout + bh * Tq * D, Tq, D);
  load_mat(K, k + bh * M * D, M, D);
  load_mat(V, v + bh * M * D, M, D);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  abt(P, lm, Q, K, Tq, M, D, A(s.scale));
  abt(DS, lm, G, V, Tq, M, D, A(1));  // dP
  __syncthreads();
  exact_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    A z = A(0);
    for (int j = 0; j < M; ++j) z = fmaA(P[i * lm + j], DS[i * lm + j], z);
    for (int j = 0; j < M; ++j) DS[i * lm + j] = P[i * lm + j] * (DS[i * lm + j] - z);
  }
  __syncthreads();
  if (dq) sx(dq + bh * Tq * D, DS, lm, K, Tq, M, D, A(s.scale));
  if (dk) stx(dk + bh * M * D, DS, lm, Q, Tq, M, D, A(s.scale));
  if (dv) stx(dv + bh * M * D, P, lm, G, Tq, M, D, A(1));
}

// ---------------------------------------------------------------- JVP
template <typename T, typename A = float>
__global__ void __launch_bounds__(NTHREADS)
jvp_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ tq, const T* __restrict__ tk, const T* __restrict__ tv,
           const float* __restrict__ lse, T* __restrict__ o_tan, Shape s) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  A* Q = sm;
  A* TQ = Q + Tq * (D + 1);
  A* K = TQ + Tq * (D + 1);
  A* TK = K + M * (D + 1);
  A* V = TK + M * (D + 1);
  A* TV = V + M * (D + 1);
  A* P = TV + M * (D + 1);
  A* SD = P + Tq * lm;
  A* L = SD + Tq * lm;
  load_mat(Q, q + bh * Tq * D, Tq, D);
  load_mat(TQ, tq + bh * Tq * D, Tq, D);
  load_mat(K, k + bh * M * D, M, D);
  load_mat(TK, tk + bh * M * D, M, D);
  load_mat(V, v + bh * M * D, M, D);
  load_mat(TV, tv + bh * M * D, M, D);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  abt(P, lm, Q, K, Tq, M, D, A(s.scale));
  abt2(SD, lm, TQ, K, Q, TK, Tq, M, D, A(s.scale));
  __syncthreads();
  exact_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    A c = A(0);
    for (int j = 0; j < M; ++j) c = fmaA(P[i * lm + j], SD[i * lm + j], c);
    for (int j = 0; j < M; ++j) SD[i * lm + j] = P[i * lm + j] * (SD[i * lm + j] - c);
  }
  __syncthreads();
  sx2(o_tan + bh * Tq * D, SD, V, P, TV, lm, Tq, M, D, A(1));
}

// ---------------------------------------------------------------- HVP
// Full HVP of L = <O, W> along (tQ, tK, tV): hQ, hK, hV and Odot.
template <typename T, typename A = float>
__global__ void __launch_bounds__(NTHREADS)
hvp_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ w, const float* __restrict__ lse, const T* __restrict__ tq,
           const T* __restrict__ tk, const T* __restrict__ tv, T* __restrict__ hq,
           T* __restrict__ hk, T* __restrict__ hv, T* __restrict__ o_tan, Shape s) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  const int qsz = Tq * (D + 1), ksz = M * (D + 1), ssz = Tq * lm;
  A* Q = sm;
  A* TQ = Q + qsz;
  A* W = TQ + qsz;
  A* K = W + qsz;
  A* TK = K + ksz;
  A* V = TK + ksz;
  A* TV = V + ksz;
  A* P = TV + ksz;
  A* PD = P + ssz;   // Sdot -> Pdot
  A* DS = PD + ssz;  // dP   -> dS
  A* DSD = DS + ssz; // dPd  -> dSd
  A* L = DSD + ssz;
  const int64_t qo = bh * Tq * D, ko = bh * M * D;
  load_mat(Q, q + qo, Tq, D);
  load_mat(TQ, tq + qo, Tq, D);
  load_mat(W, w + qo, Tq, D);
  load_mat(K, k + ko, M, D);
  load_mat(TK, tk + ko, M, D);
  load_mat(V, v + ko, M, D);
  load_mat(TV, tv + ko, M, D);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  abt(P, lm, Q, K, Tq, M, D, A(s.scale));
  abt2(PD, lm, TQ, K, Q, TK, Tq, M, D, A(s.scale));
  abt(DS, lm, W, V, Tq, M, D, A(1));
  abt(DSD, lm, W, TV, Tq, M, D, A(1));
  __syncthreads();
  exact_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    A* p = P + i * lm;
    A* pd = PD + i * lm;
    A* ds = DS + i * lm;
    A* dsd = DSD + i * lm;
    A c = A(0), z = A(0);
    for (int j = 0; j < M; ++j) {
      c = fmaA(p[j], pd[j], c);
      z = fmaA(p[j], ds[j], z);
    }
    A zd = A(0);
    for (int j = 0; j < M; ++j) {
      pd[j] = p[j] * (pd[j] - c);                 // Pdot
      zd = fmaA(pd[j], ds[j], fmaA(p[j], dsd[j], zd));  // rowsum(W Odot)
    }
    for (int j = 0; j < M; ++j) {
      const A g = ds[j] - z;
      dsd[j] = pd[j] * g + p[j] * (dsd[j] - zd);  // dSdot
      ds[j] = p[j] * g;                           // dS
    }
  }
  __syncthreads();
  if (hq) sx2(hq + qo, DSD, K, DS, TK, lm, Tq, M, D, A(s.scale));
  if (hk) stx2(hk + ko, DSD, Q, DS, TQ, lm, Tq, M, D, A(s.scale));
  if (hv) stx(hv + ko, PD, lm, W, Tq, M, D, A(1));
  if (o_tan) sx2(o_tan + qo, PD, V, P, TV, lm, Tq, M, D, A(1));
}

}  // namespace small
}  // namespace theria
