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

inline size_t smem_bytes(int T, int M, int D, int n_q_like, int n_k_like, int n_scores) {
  return sizeof(float) * ((size_t)n_q_like * T * (D + 1) + (size_t)n_k_like * M * (D + 1) +
                          (size_t)n_scores * T * (M + 1) + 4 * (size_t)T);
}

template <typename T>
__device__ __forceinline__ void load_mat(float* dst, const T* __restrict__ src, int rows, int D) {
  for (int e = threadIdx.x; e < rows * D; e += blockDim.x) {
    const int r = e / D, d = e - r * D;
    dst[r * (D + 1) + d] = to_f32<T>(src[e]);
  }
}

// C[i][j] = alpha * sum_d A[i][d] B[j][d]   (A: [rA][D], B: [rB][D])
__device__ __forceinline__ void abt(float* C, int ldc, const float* A, const float* B, int rA,
                                    int rB, int D, float alpha) {
  for (int e = threadIdx.x; e < rA * rB; e += blockDim.x) {
    const int i = e / rB, j = e - i * rB;
    const float* a = A + i * (D + 1);
    const float* b = B + j * (D + 1);
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(a[d], b[d], acc);
    C[i * ldc + j] = alpha * acc;
  }
}

// out[i][d] = alpha * sum_j S[i][j] X[j][d]       (S: [rS][cS] ld lds, X: [cS][D])
template <typename OT>
__device__ __forceinline__ void sx(OT* __restrict__ out, const float* S, int lds, const float* X,
                                   int rS, int cS, int D, float alpha) {
  for (int e = threadIdx.x; e < rS * D; e += blockDim.x) {
    const int i = e / D, d = e - i * D;
    float acc = 0.f;
    for (int j = 0; j < cS; ++j) acc = fmaf(S[i * lds + j], X[j * (D + 1) + d], acc);
    out[e] = from_f32<OT>(alpha * acc);
  }
}

// out[j][d] = alpha * sum_i S[i][j] X[i][d]       (transpose of S)
template <typename OT>
__device__ __forceinline__ void stx(OT* __restrict__ out, const float* S, int lds,
                                    const float* X, int rS, int cS, int D, float alpha) {
  for (int e = threadIdx.x; e < cS * D; e += blockDim.x) {
    const int j = e / D, d = e - j * D;
    float acc = 0.f;
    for (int i = 0; i < rS; ++i) acc = fmaf(S[i * lds + j], X[i * (D + 1) + d], acc);
    out[e] = from_f32<OT>(alpha * acc);
  }
}

// out[i][d] = alpha * sum_j (S1[i][j] X1[j][d] + S2[i][j] X2[j][d])
template <typename OT>
__device__ __forceinline__ void sx2(OT* __restrict__ out, const float* S1, const float* X1,
                                    const float* S2, const float* X2, int lds, int rS, int cS,
                                    int D, float alpha) {
  for (int e = threadIdx.x; e < rS * D; e += blockDim.x) {
    const int i = e / D, d = e - i * D;
    float acc = 0.f;
    for (int j = 0; j < cS; ++j) {
      acc = fmaf(S1[i * lds + j], X1[j * (D + 1) + d], acc);
      acc = fmaf(S2[i * lds + j], X2[j * (D + 1) + d], acc);
    }
    out[e] = from_f32<OT>(alpha * acc);
  }
}

// out[j][d] = alpha * sum_i (S1[i][j] X1[i][d] + S2[i][j] X2[i][d])
template <typename OT>
__device__ __forceinline__ void stx2(OT* __restrict__ out, const float* S1, const float* X1,
                                     const float* S2, const float* X2, int lds, int rS, int cS,
                                     int D, float alpha) {
  for (int e = threadIdx.x; e < cS * D; e += blockDim.x) {
    const int j = e / D, d = e - j * D;
    float acc = 0.f;
    for (int i = 0; i < rS; ++i) {
      acc = fmaf(S1[i * lds + j], X1[i * (D + 1) + d], acc);
      acc = fmaf(S2[i * lds + j], X2[i * (D + 1) + d], acc);
    }
    out[e] = from_f32<OT>(alpha * acc);
  }
}

__device__ __forceinline__ bool masked(int i, int j, int causal) { return causal && j > i; }

// C = alpha * (A1 B1^T + A2 B2^T)
__device__ __forceinline__ void abt2(float* C, int ldc, const float* A1, const float* B1,
                                     const float* A2, const float* B2, int rA, int rB, int D,
                                     float alpha) {
  for (int e = threadIdx.x; e < rA * rB; e += blockDim.x) {
    const int i = e / rB, j = e - i * rB;
    const float *a1 = A1 + i * (D + 1), *b1 = B1 + j * (D + 1);
    const float *a2 = A2 + i * (D + 1), *b2 = B2 + j * (D + 1);
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(a1[d], b1[d], fmaf(a2[d], b2[d], acc));
    C[i * ldc + j] = alpha * acc;
  }
}

// P[i][j] = exp(S[i][j] - lse_i) in place (0 where masked).
__device__ __forceinline__ void probs_from_lse(float* S, int lds, const float* lse_s, int T,
                                               int M, int causal) {
  for (int e = threadIdx.x; e < T * M; e += blockDim.x) {
    const int i = e / M, j = e - i * M;
    S[i * lds + j] = masked(i, j, causal) ? 0.f : expf(S[i * lds + j] - lse_s[i]);
  }
}

// ---------------------------------------------------------------- forward
template <typename T, typename OT>
__global__ void __launch_bounds__(NTHREADS)
fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           OT* __restrict__ o, float* __restrict__ lse, Shape s) {
  extern __shared__ float sm[];
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  float* Q = sm;
  float* K = Q + Tq * (D + 1);
  float* V = K + M * (D + 1);
  float* S = V + M * (D + 1);
  load_mat(Q, q + bh * Tq * D, Tq, D);
  load_mat(K, k + bh * M * D, M, D);
  load_mat(V, v + bh * M * D, M, D);
  __syncthreads();
  abt(S, lm, Q, K, Tq, M, D, s.scale);
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    float m = -INFINITY;
    for (int j = 0; j < M; ++j)
      if (!masked(i, j, s.causal)) m = fmaxf(m, S[i * lm + j]);
    float l = 0.f;
    for (int j = 0; j < M; ++j) {
      const float p = masked(i, j, s.causal) ? 0.f : expf(S[i * lm + j] - m);
      S[i * lm + j] = p;
      l += p;
    }
    const float inv = 1.f / l;
    for (int j = 0; j < M; ++j) S[i * lm + j] *= inv;
    if (lse) lse[bh * Tq + i] = m + logf(l);
  }
  __syncthreads();
  sx(o + bh * Tq * D, S, lm, V, Tq, M, D, 1.f);
}

// ---------------------------------------------------------------- backward
template <typename T>
__global__ void __launch_bounds__(NTHREADS)
bwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ dout, const float* __restrict__ lse, T* __restrict__ dq,
           T* __restrict__ dk, T* __restrict__ dv, Shape s) {
  extern __shared__ float sm[];
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  float* Q = sm;
  float* G = Q + Tq * (D + 1);  // dO
  float* K = G + Tq * (D + 1);
  float* V = K + M * (D + 1);
  float* P = V + M * (D + 1);
  float* DS = P + Tq * lm;
  float* L = DS + Tq * lm;
  load_mat(Q, q + bh * Tq * D, Tq, D);
  load_mat(G, dout + bh * Tq * D, Tq, D);
  load_mat(K, k + bh * M * D, M, D);
  load_mat(V, v + bh * M * D, M, D);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  abt(P, lm, Q, K, Tq, M, D, s.scale);
  abt(DS, lm, G, V, Tq, M, D, 1.f);  // dP
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    float z = 0.f;
    for (int j = 0; j < M; ++j) z = fmaf(P[i * lm + j], DS[i * lm + j], z);
    for (int j = 0; j < M; ++j) DS[i * lm + j] = P[i * lm + j] * (DS[i * lm + j] - z);
  }
  __syncthreads();
  if (dq) sx(dq + bh * Tq * D, DS, lm, K, Tq, M, D, s.scale);
  if (dk) stx(dk + bh * M * D, DS, lm, Q, Tq, M, D, s.scale);
  if (dv) stx(dv + bh * M * D, P, lm, G, Tq, M, D, 1.f);
}

// ---------------------------------------------------------------- JVP
template <typename T>
__global__ void __launch_bounds__(NTHREADS)
jvp_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ tq, const T* __restrict__ tk, const T* __restrict__ tv,
           const float* __restrict__ lse, T* __restrict__ o_tan, Shape s) {
  extern __shared__ float sm[];
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  float* Q = sm;
  float* TQ = Q + Tq * (D + 1);
  float* K = TQ + Tq * (D + 1);
  float* TK = K + M * (D + 1);
  float* V = TK + M * (D + 1);
  float* TV = V + M * (D + 1);
  float* P = TV + M * (D + 1);
  float* SD = P + Tq * lm;
  float* L = SD + Tq * lm;
  load_mat(Q, q + bh * Tq * D, Tq, D);
  load_mat(TQ, tq + bh * Tq * D, Tq, D);
  load_mat(K, k + bh * M * D, M, D);
  load_mat(TK, tk + bh * M * D, M, D);
  load_mat(V, v + bh * M * D, M, D);
  load_mat(TV, tv + bh * M * D, M, D);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  abt(P, lm, Q, K, Tq, M, D, s.scale);
  abt2(SD, lm, TQ, K, Q, TK, Tq, M, D, s.scale);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    float c = 0.f;
    for (int j = 0; j < M; ++j) c = fmaf(P[i * lm + j], SD[i * lm + j], c);
    for (int j = 0; j < M; ++j) SD[i * lm + j] = P[i * lm + j] * (SD[i * lm + j] - c);
  }
  __syncthreads();
  sx2(o_tan + bh * Tq * D, SD, V, P, TV, lm, Tq, M, D, 1.f);
}

// ---------------------------------------------------------------- HVP
// Full HVP of L = <O, W> along (tQ, tK, tV): hQ, hK, hV and Odot.
template <typename T>
__global__ void __launch_bounds__(NTHREADS)
hvp_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ w, const float* __restrict__ lse, const T* __restrict__ tq,
           const T* __restrict__ tk, const T* __restrict__ tv, T* __restrict__ hq,
           T* __restrict__ hk, T* __restrict__ hv, T* __restrict__ o_tan, Shape s) {
  extern __shared__ float sm[];
  const int Tq = (int)s.T, M = (int)s.M, D = (int)s.D, lm = M + 1;
  const int64_t bh = blockIdx.x;
  const int qsz = Tq * (D + 1), ksz = M * (D + 1), ssz = Tq * lm;
  float* Q = sm;
  float* TQ = Q + qsz;
  float* W = TQ + qsz;
  float* K = W + qsz;
  float* TK = K + ksz;
  float* V = TK + ksz;
  float* TV = V + ksz;
  float* P = TV + ksz;
  float* PD = P + ssz;   // Sdot -> Pdot
  float* DS = PD + ssz;  // dP   -> dS
  float* DSD = DS + ssz; // dPd  -> dSd
  float* L = DSD + ssz;
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
  abt(P, lm, Q, K, Tq, M, D, s.scale);
  abt2(PD, lm, TQ, K, Q, TK, Tq, M, D, s.scale);
  abt(DS, lm, W, V, Tq, M, D, 1.f);
  abt(DSD, lm, W, TV, Tq, M, D, 1.f);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) {
    float* p = P + i * lm;
    float* pd = PD + i * lm;
    float* ds = DS + i * lm;
    float* dsd = DSD + i * lm;
    float c = 0.f, z = 0.f;
    for (int j = 0; j < M; ++j) {
      c = fmaf(p[j], pd[j], c);
      z = fmaf(p[j], ds[j], z);
    }
    float zd = 0.f;
    for (int j = 0; j < M; ++j) {
      pd[j] = p[j] * (pd[j] - c);                 // Pdot
      zd = fmaf(pd[j], ds[j], fmaf(p[j], dsd[j], zd));  // rowsum(W Odot)
    }
    for (int j = 0; j < M; ++j) {
      const float g = ds[j] - z;
      dsd[j] = pd[j] * g + p[j] * (dsd[j] - zd);  // dSdot
      ds[j] = p[j] * g;                           // dS
    }
  }
  __syncthreads();
  if (hq) sx2(hq + qo, DSD, K, DS, TK, lm, Tq, M, D, s.scale);
  if (hk) stx2(hk + ko, DSD, Q, DS, TQ, lm, Tq, M, D, s.scale);
  if (hv) stx(hv + ko, PD, lm, W, Tq, M, D, 1.f);
  if (o_tan) sx2(o_tan + qo, PD, V, P, TV, lm, Tq, M, D, 1.f);
}

}  // namespace small
}  // namespace theria
