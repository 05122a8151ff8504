// Attention scores and probabilities as dense [B, H, T, M] matrices.
//
// These serve the reference's partial kernels (QK^T with PyTorch softmax/PV,
// and fused QK^T + softmax with PyTorch PV).  Both are one tile pass:
//   scores  out = scale * Q K^T               (fp32 or the input dtype)
//   probs   out = exp(scale * Q K^T - LSE)    (fp32; zero above the causal
//                                             diagonal), LSE from the forward
// Two kernels: a tcgen05 tile kernel for 16-bit inputs with head dim 64/128
// (one 128x128 output tile per CTA, Q and K tiles by TMA, the product in
// TMEM, four warps writing one output row each), and a CUDA-core tiled kernel
// for every other case (fp32, other head dims, unaligned tensors).  The
// output write dominates (4 bytes per score), so both are memory-bound at
// large sizes.
#pragma once

#include "common.cuh"
#include "tc_common.cuh"

namespace theria {
namespace scores {

enum Mode { kScores = 0, kProbs = 1 };

// Store 32 consecutive values of one output row (columns m0 .. m0+31).
template <typename O>
__device__ __forceinline__ void store_row32(O* dst, const float (&v)[32], int valid, bool vec) {
  if (vec && valid >= 32) {
    if constexpr (sizeof(O) == 4) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float* e = v + 8 * i;
        d4[i] = make_uint4(tc::pack2<O>(e[0], e[1]), tc::pack2<O>(e[2], e[3]),
                           tc::pack2<O>(e[4], e[5]), tc::pack2<O>(e[6], e[7]));
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = from_f32<O>(v[i]);
  }
}

// ---------------------------------------------------------------- tcgen05
constexpr int TM = 128, TN = 128;

template <int HD>
struct TcSmem {
  static constexpr int kTile = TM * HD * 2;
  static constexpr int oQ = 0;
  static constexpr int oK = kTile;
  static constexpr int oBar = 2 * kTile;  // full, done
  static constexpr int oTmem = oBar + 16;
  static constexpr int oAbort = oTmem + 4;
  static constexpr int kAlloc = oAbort + 4 + 1024;
};

template <typename T, typename O, int HD>
__global__ void __launch_bounds__(128)
tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
          O* __restrict__ out, const float* __restrict__ lse, int Tq, int M, float scale,
          int mode, int causal, int vec) {
  using L = TcSmem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* done = full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::oAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * TM, m0 = blockIdx.y * TN, bh = blockIdx.z;

  if (threadIdx.x == 0) {
    tc::mbar_init(full, 1);
    tc::mbar_init(done, 1);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, 128);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Above the causal diagonal every probability is zero: skip the product.
  const bool skip = mode == kProbs && causal && m0 > t0 + TM - 1;
  if (threadIdx.x == 0 && !skip) {
    tc::mbar_expect_tx(full, 2 * L::kTile);
    for (int cb = 0; cb < HD / 64; ++cb) {
      tc::tma_load_3d(smem + L::oQ + cb * TM * 128, &tm_q, full, cb * 64, t0, bh);
      tc::tma_load_3d(smem + L::oK + cb * TN * 128, &tm_k, full, cb * 64, m0, bh);
    }
    if (tc::mbar_wait(full, 0, abort)) {
      tc::tc_fence_after();
      constexpr uint32_t id = tc::idesc_f16(TM, TN, tc::AbFmt<T>::v, 0, 0);
      const uint64_t dq = tc::sw128_desc(tc::smem_u32(smem + L::oQ), 16, 1024);
      const uint64_t dk = tc::sw128_desc(tc::smem_u32(smem + L::oK), 16, 1024);
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk)
        tc::mma_ss(tmem, tc::desc_at(dq, (kk / 4) * (TM * 128) + (kk % 4) * 32),
                   tc::desc_at(dk, (kk / 4) * (TN * 128) + (kk % 4) * 32), id, kk > 0 ? 1u : 0u);
      tc::mma_commit(done);
    } else {
      tc::mbar_wait_drain(full, 0);  // the copies land before the CTA may exit
      tc::mbar_arrive(done);          // release the epilogue warps (they see abort)
    }
  }
  const bool ok = skip || __all_sync(0xffffffffu, tc::mbar_wait(done, 0, abort));
  tc::tc_fence_after();
  const int r = warp * 32 + lane;
  const int t = t0 + r;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const float sl = scale * 1.4426950408889634f;
  const float row_l = (mode == kProbs && t < Tq) ? lse[(size_t)bh * Tq + t] * 1.4426950408889634f : 0.f;
  O* row = out + ((size_t)bh * Tq + (size_t)(t < Tq ? t : 0)) * M;
#pragma unroll 1
  for (int c = 0; c < TN / 32; ++c) {
    float v[32];
    if (ok && !skip) {
      tc::tmem_ld32(tmem + lane_off + c * 32, v);  // warp-collective
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    const int mc = m0 + c * 32;
    if (t >= Tq || mc >= M) continue;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (mode == kScores) {
        v[i] *= scale;
      } else {
        const bool masked = skip || (causal && mc + i > t);
        v[i] = masked ? 0.f : tc::ex2(fmaf(v[i], sl, -row_l));
      }
    }
    store_row32(row + mc, v, M - mc, vec != 0);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 128);
  }
}

// ---------------------------------------------------------------- CUDA cores
// 64 x 64 output tile per block of 16 x 16 threads (4 x 4 outputs each),
// head dim streamed through shared memory in chunks of 16.
constexpr int ST = 64, SK = 16;

template <typename T, typename O>
__global__ void __launch_bounds__(256)
simt_kernel(const T* __restrict__ q, const T* __restrict__ k, O* __restrict__ out,
            const float* __restrict__ lse, int Tq, int M, int D, float scale, int mode,
            int causal) {
  __shared__ float qs[ST][SK + 1], ks[ST][SK + 1];
  const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 16 + tx;
  const int t0 = blockIdx.y * ST, m0 = blockIdx.x * ST, bh = blockIdx.z;
  const T* qb = q + (size_t)bh * Tq * D;
  const T* kb = k + (size_t)bh * M * D;
  float acc[4][4] = {};
  for (int d0 = 0; d0 < D; d0 += SK) {
    for (int i = tid; i < ST * SK; i += 256) {
      const int rr = i / SK, dd = i % SK;
      qs[rr][dd] = (t0 + rr < Tq && d0 + dd < D) ? to_f32<T>(qb[(size_t)(t0 + rr) * D + d0 + dd]) : 0.f;
      ks[rr][dd] = (m0 + rr < M && d0 + dd < D) ? to_f32<T>(kb[(size_t)(m0 + rr) * D + d0 + dd]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int dd = 0; dd < SK; ++dd) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = qs[ty + 16 * i][dd];
        b[i] = ks[tx + 16 * i][dd];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty + 16 * i;
    if (t >= Tq) continue;
    const float l = mode == kProbs ? lse[(size_t)bh * Tq + t] : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + tx + 16 * j;
      if (m >= M) continue;
      float v = acc[i][j] * scale;
      if (mode == kProbs) v = (causal && m > t) ? 0.f : expf(v - l);
      out[((size_t)bh * Tq + t) * M + m] = from_f32<O>(v);
    }
  }
}

}  // namespace scores
}  // namespace theria
