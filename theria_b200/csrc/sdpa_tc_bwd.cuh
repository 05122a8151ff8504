// Tensor-core (tcgen05) SDPA backward for bf16/fp16, head dim 64 or 128.
//
// Three launches per call:
//   prep     z_i = rowsum(dO_i * O_i) and dQacc := 0        (memory bound)
//   main     one CTA per (128-key tile, batch*head), looping over 128-row
//            query tiles (key/value-stationary):
//              S^T  = K Q_i^T            (tcgen05, TMEM cols [0,128))
//              dP^T = V dO_i^T           (tcgen05, TMEM cols [128,256))
//              P^T  = exp(s S^T - LSE),  dS^T = P^T (dP^T - z)   (CUDA cores,
//                     one key row per thread, written as 16-bit SW128 tiles)
//              dV  += P^T dO_i           (TMEM cols [256, 256+D))
//              dK  += dS^T Q_i           (TMEM cols [256+D, 256+2D))
//              dQ_i = dS K               (TMEM cols [0, D), reusing S^T's)
//            dQ_i is added to the fp32 accumulator dQacc with vector
//            reductions (red.global.add.v4.f32); dK, dV are stored once.
//   finish   dQ = scale * dQacc in the input dtype
// Warp roles in main: warp 0 TMA, warp 1 MMA issuer + TMEM owner, warps
// 2..5 compute.  Operand majors: K, Q_i as K-major (S^T), V, dO_i likewise
// (dP^T); P^T / dS^T K-major with dO_i / Q_i MN-major (dV, dK); for dQ the
// stored dS^T is read as an MN-major A and K as an MN-major B.
#pragma once

#include "tc_common.cuh"

namespace theria {
namespace tcbwd {

constexpr int BK = 128;  // keys per CTA
constexpr int BQ = 128;  // query rows per iteration
constexpr int NTHREADS = 192;

template <int HD>
struct Smem {
  static constexpr int kTile = 128 * HD * 2;  // one 128-row operand tile
  static constexpr int kP = BK * BQ * 2;
  static constexpr int oK = 0;
  static constexpr int oV = oK + kTile;
  static constexpr int oQ = oV + kTile;
  static constexpr int oDO = oQ + kTile;
  static constexpr int oP = oDO + kTile;     // P^T  [key][q]
  static constexpr int oDS = oP + kP;        // dS^T [key][q]
  static constexpr int oBar = oDS + kP;
  // kv_full, qdo_full, qdo_empty, s_full, p_full, mma2_done, s_free, drain
  static constexpr int nBar = 8;
  static constexpr int oTmem = oBar + nBar * 8;
  static constexpr int oAbort = oTmem + 4;
  static constexpr int kBytes = oAbort + 4;
  static constexpr int kAlloc = kBytes + 1024;
};

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// z = rowsum(dO * O) (O in o_dtype) and zero the fp32 dQ accumulator; one
// warp per row.
template <typename T>
__global__ void __launch_bounds__(256)
prep_kernel(const void* __restrict__ o, int o_f32, const T* __restrict__ dout,
            float* __restrict__ z, float* __restrict__ dq_acc, int64_t rows, int D) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float a = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float ov = o_f32 ? static_cast<const float*>(o)[row * D + d]
                           : to_f32<T>(static_cast<const T*>(o)[row * D + d]);
    a = fmaf(to_f32<T>(dout[row * D + d]), ov, a);
    dq_acc[row * D + d] = 0.f;
  }
  a = warp_sum(a);
  if (lane == 0) z[row] = a;
}

// dQacc (already scaled) -> dQ in the input dtype.
template <typename T>
__global__ void __launch_bounds__(256)
finish_kernel(const float* __restrict__ dq_acc, T* __restrict__ dq, int64_t n) {
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n;
       i += (int64_t)gridDim.x * blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(dq_acc + i);
    uint2 p = make_uint2(tc::pack2<T>(v.x, v.y), tc::pack2<T>(v.z, v.w));
    *reinterpret_cast<uint2*>(dq + i) = p;
  }
}

template <typename T, int HD, bool CAUSAL>
__global__ void __launch_bounds__(NTHREADS, 1)
bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
           const float* __restrict__ lse, const float* __restrict__ z,
           float* __restrict__ dq_acc, T* __restrict__ dk, T* __restrict__ dv, int Tq, int M,
           float scale, float scale_log2) {
  using L = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* p_full = bars + 4;
  uint64_t* mma2_done = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* drain = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::oAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int k0 = blockIdx.x * BK;
  const int n_qt = (Tq + BQ - 1) / BQ;
  const int i_begin = CAUSAL ? k0 / BQ : 0;  // first query tile that sees these keys
  const int n_iter = n_qt > i_begin ? n_qt - i_begin : 0;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 8; ++b) tc::mbar_init(bars + b, (b == 4 || b == 6) ? 128 : 1);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 256 + HD;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_iter > 0) {
      tc::prefetch_tmap(&tm_q);
      tc::prefetch_tmap(&tm_do);
      tc::mbar_expect_tx(kv_full, 2 * L::kTile);
      for (int cb = 0; cb < HD / 64; ++cb) {
        tc::tma_load_3d(smem + L::oK + cb * BK * 128, &tm_k, kv_full, cb * 64, k0, bh);
        tc::tma_load_3d(smem + L::oV + cb * BK * 128, &tm_v, kv_full, cb * 64, k0, bh);
      }
      int issued = 0;
      for (int t = 0; t < n_iter; ++t) {
        if (t > 0 && !tc::mbar_wait(qdo_empty, (t - 1) & 1, abort)) break;
        const int q0 = (i_begin + t) * BQ;
        tc::mbar_expect_tx(qdo_full, 2 * L::kTile);
        for (int cb = 0; cb < HD / 64; ++cb) {
          tc::tma_load_3d(smem + L::oQ + cb * BQ * 128, &tm_q, qdo_full, cb * 64, q0, bh);
          tc::tma_load_3d(smem + L::oDO + cb * BQ * 128, &tm_do, qdo_full, cb * 64, q0, bh);
        }
        issued = t + 1;
      }
      tc::mbar_wait_drain(kv_full, 0);
      if (issued > 0) tc::mbar_wait_drain(qdo_full, (issued - 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_iter > 0) {
      constexpr int ab = tc::AbFmt<T>::v;
      constexpr uint32_t id_s = tc::idesc_f16(BK, BQ, ab, 0, 0);    // S^T, dP^T
      constexpr uint32_t id_kv = tc::idesc_f16(BK, HD, ab, 0, 1);   // dV, dK
      constexpr uint32_t id_q = tc::idesc_f16(BQ, HD, ab, 1, 1);    // dQ
      const uint32_t a_k = tc::smem_u32(smem + L::oK), a_v = tc::smem_u32(smem + L::oV);
      const uint32_t a_q = tc::smem_u32(smem + L::oQ), a_do = tc::smem_u32(smem + L::oDO);
      const uint32_t a_p = tc::smem_u32(smem + L::oP), a_ds = tc::smem_u32(smem + L::oDS);
      bool ok = tc::mbar_wait(kv_full, 0, abort);
      for (int t = 0; ok && t < n_iter; ++t) {
        if (!tc::mbar_wait(qdo_full, t & 1, abort)) break;
        if (t > 0 && !tc::mbar_wait(s_free, (t - 1) & 1, abort)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk / 4) * (128 * 128) + (kk % 4) * 32;
          tc::mma_ss(t_s, tc::sw128_desc(a_k + off, 16, 1024), tc::sw128_desc(a_q + off, 16, 1024),
                     id_s, kk > 0 ? 1u : 0u);
          tc::mma_ss(t_dp, tc::sw128_desc(a_v + off, 16, 1024),
                     tc::sw128_desc(a_do + off, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(s_full);
        if (!tc::mbar_wait(p_full, t & 1, abort)) break;
        tc::tc_fence_after();
        const uint32_t acc = t > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          // contraction over queries: P^T / dS^T K-major, dO / Q MN-major
          const uint32_t off_a = (kk / 4) * (BK * 128) + (kk % 4) * 32;
          const uint32_t off_b = kk * 16 * 128;
          tc::mma_ss(t_dv, tc::sw128_desc(a_p + off_a, 16, 1024),
                     tc::sw128_desc(a_do + off_b, BQ * 128, 1024), id_kv, (acc | kk) ? 1u : 0u);
          tc::mma_ss(t_dk, tc::sw128_desc(a_ds + off_a, 16, 1024),
                     tc::sw128_desc(a_q + off_b, BQ * 128, 1024), id_kv, (acc | kk) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // contraction over keys: dS^T read as MN-major A, K as MN-major B
          const uint32_t off = kk * 16 * 128;
          tc::mma_ss(t_s, tc::sw128_desc(a_ds + off, BK * 128, 1024),
                     tc::sw128_desc(a_k + off, BK * 128, 1024), id_q, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(mma2_done);
        tc::mma_commit(qdo_empty);
      }
      tc::mma_commit(drain);
      tc::mbar_wait_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ compute
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane: key row (S^T, dV, dK) or query row (dQ)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int key = k0 + r;
    bool ok = true;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, abort));
    };
    const uint32_t a_p = tc::smem_u32(smem + L::oP), a_ds = tc::smem_u32(smem + L::oDS);
    for (int t = 0; t < n_iter; ++t) {
      const int q0 = (i_begin + t) * BQ;
      if (!wait(s_full, t & 1)) { ok = false; break; }
      tc::tc_fence_after();
      const bool diag = CAUSAL && (q0 < k0 + BK);
#pragma unroll 1
      for (int c = 0; c < BQ / 32; ++c) {
        float s[32], dp[32];
        tc::tmem_ld32(t_s + lane_off + c * 32, s);
        tc::tmem_ld32(t_dp + lane_off + c * 32, dp);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int qi = c * 32 + e;
          // Row statistics straight from global memory: every lane reads
          // the same address, so each is one broadcast load through L1.
          const int q = q0 + qi;
          const bool in = q < Tq;
          const float lq = in ? __ldg(lse + (size_t)bh * Tq + q) * 1.4426950408889634f : 0.f;
          const float zq = in ? __ldg(z + (size_t)bh * Tq + q) : 0.f;
          float p = tc::ex2(s[e] * scale_log2 - lq);
          if (!in || key >= M || (diag && q < key)) p = 0.f;
          s[e] = p;                   // P^T
          dp[e] = p * (dp[e] - zq);   // dS^T
        }
        // 32 query columns = 4 chunks of 8 in column block c/2
        const uint32_t blk = (uint32_t)(c >> 1) * (BK * 128);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint32_t ch = (uint32_t)((c & 1) * 4 + h);
          const float* pe = s + h * 8;
          const float* de = dp + h * 8;
          tc::st_shared_v4(a_p + blk + tc::sw128_off(r, ch), tc::pack2<T>(pe[0], pe[1]),
                           tc::pack2<T>(pe[2], pe[3]), tc::pack2<T>(pe[4], pe[5]),
                           tc::pack2<T>(pe[6], pe[7]));
          tc::st_shared_v4(a_ds + blk + tc::sw128_off(r, ch), tc::pack2<T>(de[0], de[1]),
                           tc::pack2<T>(de[2], de[3]), tc::pack2<T>(de[4], de[5]),
                           tc::pack2<T>(de[6], de[7]));
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full);
      // dQ_i partial of this key tile -> fp32 accumulator
      if (!wait(mma2_done, t & 1)) { ok = false; break; }
      tc::tc_fence_after();
      const int qrow = q0 + r;
      float* dst = dq_acc + ((size_t)bh * Tq + (size_t)(qrow < Tq ? qrow : 0)) * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        float v[32];
        tc::tmem_ld32(t_s + lane_off + c * 32, v);
        if (qrow < Tq) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            red_add_v4(dst + c * 32 + 4 * i, v[4 * i] * scale, v[4 * i + 1] * scale,
                       v[4 * i + 2] * scale, v[4 * i + 3] * scale);
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(s_free);
    }
    // ------------------------------------------------------------ dK, dV
    if (ok) {
      const bool store = key < M;
      const size_t base = ((size_t)bh * M + (store ? key : 0)) * HD;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        T* out = which == 0 ? dv : dk;
        const float mul = which == 0 ? 1.f : scale;
        const uint32_t col = which == 0 ? t_dv : t_dk;
        if (out == nullptr) continue;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          float v[32];
          if (n_iter > 0) {
            tc::tmem_ld32(col + lane_off + c * 32, v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;  // keys no query attends to
          }
          if (!store) continue;
          uint4* d4 = reinterpret_cast<uint4*>(out + base + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float* e = v + 8 * i;
            d4[i] = make_uint4(tc::pack2<T>(e[0] * mul, e[1] * mul),
                               tc::pack2<T>(e[2] * mul, e[3] * mul),
                               tc::pack2<T>(e[4] * mul, e[5] * mul),
                               tc::pack2<T>(e[6] * mul, e[7] * mul));
          }
        }
      }
    }
  }
  // ------------------------------------------------------------ teardown
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace tcbwd
}  // namespace theria
