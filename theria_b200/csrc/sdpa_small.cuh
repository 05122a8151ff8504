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
// Every product is a register-blocked loop over the output (4 x 4 outputs
// per thread, reduction read from padded shared rows of stride D+1 or M+1);
// row statistics take one warp per row.  Results are deterministic.
#pragma once

#include "common.cuh"

namespace theria {
namespace small {

constexpr int MAXN = 64;   // max T and M
constexpr int MAXD = 64;   // max head dim
constexpr int NTHREADS = 256;

// Element strides (batch, head, row) of the three tensor families; the last
// dim is contiguous.  q-like: q, tq, dq, hq; k-like: k, v, tk, tv, dk, dv,
// hk, hv; o-like: o, dO / W, o_tan.  Contiguous [B, H, rows, D] tensors have
// (H*rows*D, rows*D, D); a packed self-attention projection [B, T, 3, H, D]
// has (3*H*D*T, D, 3*H*D) for q, k and v alike.
struct Layout {
  int64_t qb, qh, qt, kb, kh, kt, ob, oh, ot;
};

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
__device__ __forceinline__ void load_mat(A* dst, const T* __restrict__ src, int rows, int D,
                                         int64_t ld) {
  for (int e = threadIdx.x; e < rows * D; e += blockDim.x) {
    const int r = e / D, d = e - r * D;
    dst[r * (D + 1) + d] = load_as<A>(src[r * ld + d]);
  }
}

// Every product below is one generic block-wide kernel:
//   out(r, c) = alpha * sum_k [A1(r,k) B1(c,k) + A2(r,k) B2(c,k)]
// with A(r, k) = A[r*ar + k*ak] and B(c, k) = B[c*bc + k*bk] in shared memory.
// Each thread owns a 4 x 4 block of outputs, so every value it loads feeds
// four FMAs (shared-memory load bandwidth is the limit at these sizes), and
// when the output is too small to occupy the block the reduction over k is
// split over KS neighbouring lanes (k = ks, ks + KS, ...) and summed with
// shuffles.  The lane layout keeps the loads free of bank conflicts for the
// padded strides used here (D+1 for [rows][D], M+1 for score rows): the
// rows of the two row groups sharing a warp are 4 apart, and columns are
// blocked (c = 4 ct + n) when at most 8 column groups exist, interleaved
// (c = ct + CT n) otherwise.
constexpr int PB = 4;  // outputs per thread along rows and along columns

template <bool TWO, typename A, typename Store>
__device__ __forceinline__ void prod(int R, int C, int K, const A* A1, const A* B1,
                                     const A* A2, const A* B2, int ar, int ak, int bc,
                                     int bk, A alpha, Store store) {
  const int RT = (R + PB - 1) / PB, CT = (C + PB - 1) / PB;
  int KS = 1;
  while (KS < 8 && 2 * KS <= K && RT * CT * KS * 2 <= NTHREADS) KS *= 2;
  const int t = threadIdx.x;
  if (t >= RT * CT * KS) return;  // whole KS-lane groups drop out together
  const int ks = t & (KS - 1), u = t / KS;
  const int ct = u % CT;
  int rt = u / CT;
  if ((RT & 7) == 0) rt = (rt & ~7) | ((rt & 1) << 2) | ((rt >> 1) & 3);
  const bool blocked = CT <= 8;
  int ro[PB], co[PB];
  bool rv[PB], cv[PB];
#pragma unroll
  for (int m = 0; m < PB; ++m) {
    const int r = rt + RT * m;
    rv[m] = r < R;
    ro[m] = (rv[m] ? r : R - 1) * ar;
    const int c = blocked ? ct * PB + m : ct + CT * m;
    cv[m] = c < C;
    co[m] = (cv[m] ? c : C - 1) * bc;
  }
  A acc[PB][PB];
#pragma unroll
  for (int m = 0; m < PB; ++m)
#pragma unroll
    for (int n = 0; n < PB; ++n) acc[m][n] = A(0);
  // k = ks + KS * kk: with compile-time sizes (the specialised kernels) the
  // loop unrolls fully and every load is a base pointer plus an immediate.
  const int KQ = K / KS;
  auto step = [&](const A* x, const A* y) {
    A a[PB], b[PB];
#pragma unroll
    for (int m = 0; m < PB; ++m) a[m] = x[ro[m]];
#pragma unroll
    for (int n = 0; n < PB; ++n) b[n] = y[co[n]];
#pragma unroll
    for (int m = 0; m < PB; ++m)
#pragma unroll
      for (int n = 0; n < PB; ++n) acc[m][n] = fmaA(a[m], b[n], acc[m][n]);
  };
#pragma unroll
  for (int term = 0; term < (TWO ? 2 : 1); ++term) {
    const A* X = (term ? A2 : A1) + ks * ak;
    const A* Y = (term ? B2 : B1) + ks * bk;
#pragma unroll 4
    for (int kk = 0; kk < KQ; ++kk) step(X + kk * KS * ak, Y + kk * KS * bk);
    if (ks < K - KQ * KS) step(X + KQ * KS * ak, Y + KQ * KS * bk);
  }
  if (KS > 1) {
    const int lane = threadIdx.x & 31;
    const unsigned grp = (KS == 32 ? 0xffffffffu : ((1u << KS) - 1u) << (lane & ~(KS - 1)));
    for (int o = KS >> 1; o > 0; o >>= 1)
#pragma unroll
      for (int m = 0; m < PB; ++m)
#pragma unroll
        for (int n = 0; n < PB; ++n) acc[m][n] += __shfl_xor_sync(grp, acc[m][n], o);
  }
#pragma unroll
  for (int m = 0; m < PB; ++m)
#pragma unroll
    for (int n = 0; n < PB; ++n)
      if (((m * PB + n) & (KS - 1)) == ks && rv[m] && cv[n])
        store(rt + RT * m, blocked ? ct * PB + n : ct + CT * n, alpha * acc[m][n]);
}

// C[i][j] = alpha * (sum_d A1[i][d] B1[j][d] [+ A2[i][d] B2[j][d]])  (rows at stride D+1)
template <bool TWO, typename A>
__device__ __forceinline__ void abt_impl(A* C, int ldc, const A* A1, const A* B1,
                                         const A* A2, const A* B2, int rA, int rB,
                                         int D, A alpha) {
  prod<TWO, A>(rA, rB, D, A1, B1, A2, B2, D + 1, 1, D + 1, 1, alpha,
               [&](int i, int j, A x) { C[i * ldc + j] = x; });
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

// out[i][d] = alpha * sum_j (S1[i][j] X1[j][d] [+ S2[i][j] X2[j][d]])
//   (S: [rS][cS] at stride lds; X: [cS][D] at stride D+1; out: [rS][D] dense)
template <bool TWO, typename OT, typename A>
__device__ __forceinline__ void sx_impl(OT* __restrict__ out, int64_t ldo, const A* S1,
                                        const A* X1, const A* S2, const A* X2, int lds,
                                        int rS, int cS, int D, A alpha) {
  prod<TWO, A>(rS, D, cS, S1, X1, S2, X2, lds, 1, 1, D + 1, alpha,
               [&](int i, int d, A x) { out[i * ldo + d] = store_as<OT>(x); });
}

// out[j][d] = alpha * sum_i (S1[i][j] X1[i][d] [+ S2[i][j] X2[i][d]])  (S transposed)
template <bool TWO, typename OT, typename A>
__device__ __forceinline__ void stx_impl(OT* __restrict__ out, int64_t ldo, const A* S1,
                                         const A* X1, const A* S2, const A* X2, int lds,
                                         int rS, int cS, int D, A alpha) {
  prod<TWO, A>(cS, D, rS, S1, X1, S2, X2, 1, lds, 1, D + 1, alpha,
               [&](int j, int d, A x) { out[j * ldo + d] = store_as<OT>(x); });
}

template <typename OT, typename A>
__device__ __forceinline__ void sx(OT* __restrict__ out, int64_t ldo, const A* S, int lds,
                                   const A* X, int rS, int cS, int D, A alpha) {
  sx_impl<false, OT, A>(out, ldo, S, X, nullptr, nullptr, lds, rS, cS, D, alpha);
}
template <typename OT, typename A>
__device__ __forceinline__ void sx2(OT* __restrict__ out, int64_t ldo, const A* S1,
                                    const A* X1, const A* S2, const A* X2, int lds, int rS,
                                    int cS, int D, A alpha) {
  sx_impl<true, OT, A>(out, ldo, S1, X1, S2, X2, lds, rS, cS, D, alpha);
}
template <typename OT, typename A>
__device__ __forceinline__ void stx(OT* __restrict__ out, int64_t ldo, const A* S, int lds,
                                    const A* X, int rS, int cS, int D, A alpha) {
  stx_impl<false, OT, A>(out, ldo, S, X, nullptr, nullptr, lds, rS, cS, D, alpha);
}
template <typename OT, typename A>
__device__ __forceinline__ void stx2(OT* __restrict__ out, int64_t ldo, const A* S1,
                                     const A* X1, const A* S2, const A* X2, int lds, int rS,
                                     int cS, int D, A alpha) {
  stx_impl<true, OT, A>(out, ldo, S1, X1, S2, X2, lds, rS, cS, D, alpha);
}

__device__ __forceinline__ bool masked(int i, int j, int causal) { return causal && j > i; }

// Row passes run one warp per score row (lanes over the columns).
template <typename A>
__device__ __forceinline__ A warp_sum(A x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
template <typename A>
__device__ __forceinline__ A warp_max(A x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = maxA(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
#define THERIA_ROWS(i) \
  for (int i = threadIdx.x >> 5; i < Tq; i += blockDim.x >> 5)
#define THERIA_COLS(j) for (int j = threadIdx.x & 31; j < M; j += 32)

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
template <typename T, typename OT, typename A = float, int NC = 0, int DC = 0>
__global__ void __launch_bounds__(NTHREADS)
fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           OT* __restrict__ o, float* __restrict__ lse, Shape s, Layout ly) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  // NC, DC > 0: sequence lengths and head dim fixed at compile time
  const int Tq = NC ? NC : (int)s.T, M = NC ? NC : (int)s.M, D = DC ? DC : (int)s.D;
  const int lm = M + 1;
  const int64_t bh = blockIdx.x, hb = bh / s.H, hh = bh - hb * s.H;
  const int64_t qo = hb * ly.qb + hh * ly.qh, ko = hb * ly.kb + hh * ly.kh,
                oo = hb * ly.ob + hh * ly.oh;
  A* Q = sm;
  A* K = Q + Tq * (D + 1);
  A* V = K + M * (D + 1);
  A* S = V + M * (D + 1);
  load_mat(Q, q + qo, Tq, D, ly.qt);
  load_mat(K, k + ko, M, D, ly.kt);
  load_mat(V, v + ko, M, D, ly.kt);
  __syncthreads();
  abt(S, lm, Q, K, Tq, M, D, A(s.scale));
  __syncthreads();
  THERIA_ROWS(i) {
    A* row = S + i * lm;
    A m = -INFINITY;
    THERIA_COLS(j) if (!masked(i, j, s.causal)) m = maxA(m, row[j]);
    m = warp_max(m);
    A l = A(0);
    THERIA_COLS(j) {
      const A p = masked(i, j, s.causal) ? A(0) : expA(row[j] - m);
      row[j] = p;
      l += p;
    }
    l = warp_sum(l);
    const A inv = A(1) / l;
    THERIA_COLS(j) row[j] *= inv;
    if (lse && (threadIdx.x & 31) == 0) lse[bh * Tq + i] = m + logA(l);
  }
  __syncthreads();
  sx(o + oo, ly.ot, S, lm, V, Tq, M, D, A(1));
}

// ---------------------------------------------------------------- backward
template <typename T, typename A = float, int NC = 0, int DC = 0>
__global__ void __launch_bounds__(NTHREADS)
bwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ dout, const float* __restrict__ lse, T* __restrict__ dq,
           T* __restrict__ dk, T* __restrict__ dv, Shape s, Layout ly) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  // NC, DC > 0: sequence lengths and head dim fixed at compile time
  const int Tq = NC ? NC : (int)s.T, M = NC ? NC : (int)s.M, D = DC ? DC : (int)s.D;
  const int lm = M + 1;
  const int64_t bh = blockIdx.x, hb = bh / s.H, hh = bh - hb * s.H;
  const int64_t qo = hb * ly.qb + hh * ly.qh, ko = hb * ly.kb + hh * ly.kh,
                oo = hb * ly.ob + hh * ly.oh;
  A* Q = sm;
  A* G = Q + Tq * (D + 1);  // dO
  A* K = G + Tq * (D + 1);
  A* V = K + M * (D + 1);
  A* P = V + M * (D + 1);
  A* DS = P + Tq * lm;
  A* L = DS + Tq * lm;
  load_mat(Q, q + qo, Tq, D, ly.qt);
  load_mat(G, dout + oo, Tq, D, ly.ot);
  load_mat(K, k + ko, M, D, ly.kt);
  load_mat(V, v + ko, M, D, ly.kt);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  abt(P, lm, Q, K, Tq, M, D, A(s.scale));
  abt(DS, lm, G, V, Tq, M, D, A(1));  // dP
  __syncthreads();
  exact_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  THERIA_ROWS(i) {
    const A* p = P + i * lm;
    A* ds = DS + i * lm;
    A z = A(0);
    THERIA_COLS(j) z = fmaA(p[j], ds[j], z);
    z = warp_sum(z);
    THERIA_COLS(j) ds[j] = p[j] * (ds[j] - z);
  }
  __syncthreads();
  if (dq) sx(dq + qo, ly.qt, DS, lm, K, Tq, M, D, A(s.scale));
  if (dk) stx(dk + ko, ly.kt, DS, lm, Q, Tq, M, D, A(s.scale));
  if (dv) stx(dv + ko, ly.kt, P, lm, G, Tq, M, D, A(1));
}

// ---------------------------------------------------------------- JVP
template <typename T, typename A = float, int NC = 0, int DC = 0>
__global__ void __launch_bounds__(NTHREADS)
jvp_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ tq, const T* __restrict__ tk, const T* __restrict__ tv,
           const float* __restrict__ lse, T* __restrict__ o_tan, Shape s, Layout ly) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  // NC, DC > 0: sequence lengths and head dim fixed at compile time
  const int Tq = NC ? NC : (int)s.T, M = NC ? NC : (int)s.M, D = DC ? DC : (int)s.D;
  const int lm = M + 1;
  const int64_t bh = blockIdx.x, hb = bh / s.H, hh = bh - hb * s.H;
  const int64_t qo = hb * ly.qb + hh * ly.qh, ko = hb * ly.kb + hh * ly.kh,
                oo = hb * ly.ob + hh * ly.oh;
  A* Q = sm;
  A* TQ = Q + Tq * (D + 1);
  A* K = TQ + Tq * (D + 1);
  A* TK = K + M * (D + 1);
  A* V = TK + M * (D + 1);
  A* TV = V + M * (D + 1);
  A* P = TV + M * (D + 1);
  A* SD = P + Tq * lm;
  A* L = SD + Tq * lm;
  load_mat(Q, q + qo, Tq, D, ly.qt);
  load_mat(TQ, tq + qo, Tq, D, ly.qt);
  load_mat(K, k + ko, M, D, ly.kt);
  load_mat(TK, tk + ko, M, D, ly.kt);
  load_mat(V, v + ko, M, D, ly.kt);
  load_mat(TV, tv + ko, M, D, ly.kt);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  abt(P, lm, Q, K, Tq, M, D, A(s.scale));
  abt2(SD, lm, TQ, K, Q, TK, Tq, M, D, A(s.scale));
  __syncthreads();
  exact_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  THERIA_ROWS(i) {
    const A* p = P + i * lm;
    A* sd = SD + i * lm;
    A c = A(0);
    THERIA_COLS(j) c = fmaA(p[j], sd[j], c);
    c = warp_sum(c);
    THERIA_COLS(j) sd[j] = p[j] * (sd[j] - c);
  }
  __syncthreads();
  sx2(o_tan + oo, ly.ot, SD, V, P, TV, lm, Tq, M, D, A(1));
}

// ---------------------------------------------------------------- HVP
// Full HVP of L = <O, W> along (tQ, tK, tV): hQ, hK, hV and Odot.
//
// Shared memory is used in phases so that a MAML head (T = M = 64, D = 16,
// fp32) needs 74 KB and three CTAs fit per SM: never more than the four
// score-shaped matrices plus two operand matrices are resident.
//   R0 = [P | Pdot]          (first Q, tQ, K, tK are read from R1 instead)
//   R1 = [dP->dS | dPd->dSd] (holds Q, tQ, K, tK until S and Sdot exist)
//   OP0, OP1 = W and V, then W and tV, then V and tV
// and Q, tQ, K, tK are read again from global memory (L2) into R0 once P
// and Pdot are no longer needed.
inline size_t hvp_smem_bytes(int T, int M, int D, size_t elem) {
  const size_t ssz = (size_t)T * (M + 1), opq = (size_t)T * (D + 1), opk = (size_t)M * (D + 1);
  const size_t half = 2 * ssz > 2 * (opq + opk) ? 2 * ssz : 2 * (opq + opk);
  const size_t slot = opq > opk ? opq : opk;
  return elem * (2 * half + 2 * slot + (size_t)T);
}

template <typename T, typename A = float, int NC = 0, int DC = 0>
__global__ void __launch_bounds__(NTHREADS)
hvp_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
           const T* __restrict__ w, const float* __restrict__ lse, const T* __restrict__ tq,
           const T* __restrict__ tk, const T* __restrict__ tv, T* __restrict__ hq,
           T* __restrict__ hk, T* __restrict__ hv, T* __restrict__ o_tan, Shape s, Layout ly) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  A* sm = reinterpret_cast<A*>(sm_raw);
  // NC, DC > 0: sequence lengths and head dim fixed at compile time
  const int Tq = NC ? NC : (int)s.T, M = NC ? NC : (int)s.M, D = DC ? DC : (int)s.D;
  const int lm = M + 1;
  const int64_t bh = blockIdx.x, hb = bh / s.H, hh = bh - hb * s.H;
  const int64_t qo = hb * ly.qb + hh * ly.qh, ko = hb * ly.kb + hh * ly.kh,
                oo = hb * ly.ob + hh * ly.oh;
  const int ssz = Tq * lm, opq = Tq * (D + 1), opk = M * (D + 1);
  const int half = 2 * ssz > 2 * (opq + opk) ? 2 * ssz : 2 * (opq + opk);
  const int slot = opq > opk ? opq : opk;
  A* R0 = sm;
  A* R1 = R0 + half;
  A* OP0 = R1 + half;
  A* OP1 = OP0 + slot;
  A* L = OP1 + slot;
  A* P = R0;
  A* PD = R0 + ssz;   // Sdot -> Pdot
  A* DS = R1;         // dP   -> dS
  A* DSD = R1 + ssz;  // dPd  -> dSd
  auto load_qk = [&](A* base) {  // Q, tQ, K, tK packed at base
    load_mat(base, q + qo, Tq, D, ly.qt);
    load_mat(base + opq, tq + qo, Tq, D, ly.qt);
    load_mat(base + 2 * opq, k + ko, M, D, ly.kt);
    load_mat(base + 2 * opq + opk, tk + ko, M, D, ly.kt);
  };
  // S and Sdot from Q, tQ, K, tK held in R1
  load_qk(R1);
  load_mat(OP0, w + oo, Tq, D, ly.ot);
  load_mat(OP1, v + ko, M, D, ly.kt);
  for (int i = threadIdx.x; i < Tq; i += blockDim.x) L[i] = lse[bh * Tq + i];
  __syncthreads();
  {
    const A *Q = R1, *TQ = R1 + opq, *K = R1 + 2 * opq, *TK = K + opk;
    abt(P, lm, Q, K, Tq, M, D, A(s.scale));
    abt2(PD, lm, TQ, K, Q, TK, Tq, M, D, A(s.scale));
  }
  __syncthreads();
  // dP = W V^T over the dead Q/K copies, then dPd = W tV^T
  abt(DS, lm, OP0, OP1, Tq, M, D, A(1));
  __syncthreads();
  load_mat(OP1, tv + ko, M, D, ly.kt);
  __syncthreads();
  abt(DSD, lm, OP0, OP1, Tq, M, D, A(1));
  __syncthreads();
  exact_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  probs_from_lse(P, lm, L, Tq, M, s.causal);
  __syncthreads();
  THERIA_ROWS(i) {
    A* p = P + i * lm;
    A* pd = PD + i * lm;
    A* ds = DS + i * lm;
    A* dsd = DSD + i * lm;
    A c = A(0), z = A(0);
    THERIA_COLS(j) {
      c = fmaA(p[j], pd[j], c);
      z = fmaA(p[j], ds[j], z);
    }
    c = warp_sum(c);
    z = warp_sum(z);
    A zd = A(0);
    THERIA_COLS(j) {
      pd[j] = p[j] * (pd[j] - c);                 // Pdot
      zd = fmaA(pd[j], ds[j], fmaA(p[j], dsd[j], zd));  // rowsum(W Odot)
    }
    zd = warp_sum(zd);
    THERIA_COLS(j) {
      const A g = ds[j] - z;
      dsd[j] = pd[j] * g + p[j] * (dsd[j] - zd);  // dSdot
      ds[j] = p[j] * g;                           // dS
    }
  }
  __syncthreads();
  // hV = Pdot^T W (W still in OP0), then V into OP0 for Odot = Pdot V + P tV
  if (hv) stx(hv + ko, ly.kt, PD, lm, OP0, Tq, M, D, A(1));
  __syncthreads();
  load_mat(OP0, v + ko, M, D, ly.kt);
  __syncthreads();
  if (o_tan) sx2(o_tan + oo, ly.ot, PD, OP0, P, OP1, lm, Tq, M, D, A(1));
  __syncthreads();
  // P and Pdot are done: Q, tQ, K, tK again, into R0, for hQ and hK
  if (hq || hk) {
    load_qk(R0);
    __syncthreads();
    const A *Q = R0, *TQ = R0 + opq, *K = R0 + 2 * opq, *TK = K + opk;
    if (hq) sx2(hq + qo, ly.qt, DSD, K, DS, TK, lm, Tq, M, D, A(s.scale));
    if (hk) stx2(hk + ko, ly.kt, DSD, Q, DS, TQ, lm, Tq, M, D, A(s.scale));
  }
}

#undef THERIA_ROWS
#undef THERIA_COLS

}  // namespace small
}  // namespace theria
