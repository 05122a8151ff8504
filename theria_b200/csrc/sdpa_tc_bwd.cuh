// Tensor-core (tcgen05) SDPA backward for bf16/fp16, head dim 64 or 128.
//
// Three launches per call:
//   prep     z_i = rowsum(dO_i * O_i) and dQacc := 0        (memory bound)
//   main     one CTA per (128-key tile, batch*head), looping over 64-row
//            query tiles t (key/value-stationary), pipelined so the tensor
//            core works on tile t+1 while CUDA cores finish tile t:
//              S^T  = K Q_t^T,  dP^T = V dO_t^T      (tcgen05 -> TMEM)
//              P^T  = exp(s S^T - LSE),  dS^T = P^T (dP^T - z)   (CUDA cores,
//                     one key row per thread, 16-bit SW128 tiles in smem)
//              dV  += P^T dO_t,  dK += dS^T Q_t       (TMEM accumulators)
//              dQ   = dS K, staged in shared memory and added to the fp32
//                     accumulator dQacc by TMA bulk reductions; dK, dV are
//                     stored once at the end.
//   finish   dQ = dQacc in the input dtype (dQacc is pre-scaled)
// TMEM (512 columns): S^T [0,64) and dP^T [64,128), released as soon as the
// CUDA cores have loaded them; dV [128, 128+D); dK [128+D, 128+2D).
// dQ: for D = 128 as dQ^T = K^T dS^T (M = D = 128 lanes, 64 columns) into a
// double buffer [384 + 64b, 448 + 64b); for D = 64 as dQ = dS K for a PAIR of
// query tiles at once (M = 128 query rows, the two adjacent dS^T buffers read
// as one MN-major operand) into [256, 320).
// Warp roles: warp 0 TMA (for D = 64 non-causal also each tile's row terms
// LSE and z, staged in shared memory for broadcast loads); warp 1
// issues S^T/dP^T and owns TMEM; warp 2 issues dV/dK/dQ; warps 3..10 two
// groups of four (one per TMEM lane quarter) splitting the columns; warps
// 11..14 flush dQ.  Two issuing threads: one
// thread issues a tcgen05.mma only every ~60 cycles, slower than the tensor
// core runs the N = 64 products, and each barrier wait between groups stalls
// its issue stream; with the two groups on separate threads each hides the
// other's waits.  The groups touch disjoint TMEM columns, and every
// cross-group dependency already passes through the compute warps' barriers.
#pragma once

#include "tc_common.cuh"

namespace theria {
namespace tcbwd {

constexpr int BK = 128;        // keys per CTA (M of S^T, dP^T, dV, dK)
constexpr int BQ = 64;         // query rows per iteration (N of S^T, dP^T)
constexpr int NCOMPUTE = 256;  // 8 compute warps: 2 groups x 4 TMEM lane quarters
constexpr int NDQ = 128;       // 4 warps that flush dQ (one per TMEM lane quarter)
constexpr int NTHREADS = 96 + NCOMPUTE + NDQ;
constexpr int kFirstCompute = 3;  // warps 0..2: TMA, S/dP issuer, dV/dK/dQ issuer

template <int HD>
struct Smem {
  static constexpr int kKV = BK * HD * 2;   // K or V tile
  static constexpr int kQ = BQ * HD * 2;    // one Q or dO tile
  // Q/dO ring depth: a stage is released only when the tile's last MMAs
  // complete, so the ring must cover that latency plus the TMA refill.
  static constexpr int QST = HD == 128 ? 3 : 4;
  static constexpr int kP = BK * BQ * 2;    // one dS^T buffer [key][q]
  // fp32 dQ staged for the bulk reduction: 64 query rows of dQ^T as rows
  // [q][d] (D = 128), or a pair's 128 query rows of dQ as two 128-byte-swizzled
  // halves [q][32 d] (D = 64); 32 KB either way
  static constexpr int kStage = 32768;
  static constexpr int oK = 0;
  static constexpr int oV = oK + kKV;
  static constexpr int oQ = oV + kKV;       // QST stages
  static constexpr int oDO = oQ + QST * kQ; // QST stages
  static constexpr int oDS = oDO + QST * kQ;  // 2 buffers (adjacent: a pair is one M=128 operand)
  static constexpr int oStage = oDS + 2 * kP;
  // per Q/dO stage: the row terms {-LSE*log2(e), -z} of the tile's 64 queries
  static constexpr int kRow = BQ * 8;
  static constexpr int oRow = oStage + kStage;
  static constexpr int oBar = oRow + QST * kRow;
  // kv_full, q_full[4], q_empty[4], s_full, s_read, p_full[2], mma2_done[2],
  // dq_free[2], drain[2], stage_free, stage_full, kv_tmem
  static constexpr int nBar = 1 + 8 + 2 + 6 + 2 + 2 + 1;
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

// z = rowsum(dO * O) (O in o_dtype) and zero the fp32 dQ accumulator.
// D / 8 threads per row (D in {64, 128}), each on 8 consecutive elements with
// 16-byte loads and stores; the row sum is finished by shuffles among them.
template <typename T>
__global__ void __launch_bounds__(256)
prep_kernel(const void* __restrict__ o, int o_f32, const T* __restrict__ dout,
            float* __restrict__ z, float* __restrict__ dq_acc, int64_t rows, int D) {
  const int tpr = D / 8;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = gid / tpr;
  const int part = (int)(gid % tpr);
  float a = 0.f;
  if (row < rows) {
    const int64_t base = row * D + part * 8;
    const uint4 dr = *reinterpret_cast<const uint4*>(dout + base);
    const T* dv = reinterpret_cast<const T*>(&dr);
    float ov[8];
    if (o_f32) {
      const float4 x = *reinterpret_cast<const float4*>(static_cast<const float*>(o) + base);
      const float4 y = *reinterpret_cast<const float4*>(static_cast<const float*>(o) + base + 4);
      ov[0] = x.x; ov[1] = x.y; ov[2] = x.z; ov[3] = x.w;
      ov[4] = y.x; ov[5] = y.y; ov[6] = y.z; ov[7] = y.w;
    } else {
      const uint4 orr = *reinterpret_cast<const uint4*>(static_cast<const T*>(o) + base);
      const T* op = reinterpret_cast<const T*>(&orr);
#pragma unroll
      for (int i = 0; i < 8; ++i) ov[i] = to_f32<T>(op[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) a = fmaf(to_f32<T>(dv[i]), ov[i], a);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(dq_acc + base) = zero;
    *reinterpret_cast<float4*>(dq_acc + base + 4) = zero;
  }
  for (int off = tpr / 2; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
  if (row < rows && part == 0) z[row] = a;
}

// dQacc (already scaled) -> dQ in the input dtype; 8 elements per thread
// and step (two 16-byte loads, one 16-byte store; n is a multiple of 8).
template <typename T>
__global__ void __launch_bounds__(256)
finish_kernel(const float* __restrict__ dq_acc, T* __restrict__ dq, int64_t n) {
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < n;
       i += (int64_t)gridDim.x * blockDim.x * 8) {
    const float4 a = *reinterpret_cast<const float4*>(dq_acc + i);
    const float4 b = *reinterpret_cast<const float4*>(dq_acc + i + 4);
    *reinterpret_cast<uint4*>(dq + i) = make_uint4(tc::pack2<T>(a.x, a.y), tc::pack2<T>(a.z, a.w),
                                                   tc::pack2<T>(b.x, b.y), tc::pack2<T>(b.z, b.w));
  }
}


template <typename T, int HD, bool CAUSAL>
__global__ void __launch_bounds__(NTHREADS, 1)
bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
           const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse,
           const float* __restrict__ z,
           float* __restrict__ dq_acc, T* __restrict__ dk, T* __restrict__ dv, int Tq, int M,
           float scale, float scale_log2) {
  using L = Smem<HD>;
  constexpr bool kPairDq = (HD == 64);  // dQ per pair of query tiles (see header)
  // The compute warps take each query's row terms (LSE, z) from a copy the
  // producer warp stages in shared memory (broadcast loads) for D = 64
  // non-causal, where they were issue-bound on the per-query shuffles
  // (+9 %); elsewhere from shuffles of one load per lane, which keep the
  // shared-memory pipe (the D = 128 limit) free and measured faster.
  constexpr bool kRowStage = (HD == 64) && !CAUSAL;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* kv_full = bars;
  constexpr int QST = L::QST;
  uint64_t* q_full = bars + 1;      // [QST] Q_t, dO_t and the tile's row terms landed
  uint64_t* q_empty = bars + 5;     // [QST] stage free (MMAs reading it done)
  uint64_t* s_full = bars + 9;      // S^T, dP^T of the current tile computed
  uint64_t* s_read = bars + 10;     // ... and loaded by the compute warps (256 arrivals)
  uint64_t* p_full = bars + 11;     // [2] P^T (TMEM), dS^T (smem) of buffer b written (256 arrivals)
  uint64_t* mma2_done = bars + 13;  // [2] dV, dK (and dQ) MMAs of the tile done
  uint64_t* dq_free = bars + 15;    // dQ read out of TMEM (128 arrivals); [1] unused
  uint64_t* drain = bars + 17;      // [2] each issuer's last MMAs done
  uint64_t* stage_free = bars + 19; // dQ staging buffer read by the previous reduction
  uint64_t* stage_full = bars + 20; // dQ staging buffer written (128 arrivals)
  uint64_t* kv_tmem = bars + 21;    // D = 64: K and V copied into TMEM (256 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::oAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Causal grids put the head index in x so the heaviest tiles of every head
  // are dispatched first (longest-first over the whole grid).
  const int bh = CAUSAL ? blockIdx.x : blockIdx.y;
  const int k0 = (CAUSAL ? blockIdx.y : blockIdx.x) * BK;
  const int n_qt = (Tq + BQ - 1) / BQ;
  const int i_begin = CAUSAL ? k0 / BQ : 0;  // first query tile that sees these keys
  const int n_iter = n_qt > i_begin ? n_qt - i_begin : 0;
  auto tile_of = [&](int t) { return i_begin + t; };

  if (threadIdx.x == 0) {
    tc::mbar_init(kv_full, 1);
    for (int b = 0; b < QST; ++b) {
      tc::mbar_init(q_full + b, kRowStage ? 2 : 1);  // TMA bytes (+ the row-term stores)
      tc::mbar_init(q_empty + b, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(p_full + b, NCOMPUTE);
      tc::mbar_init(mma2_done + b, 1);
      tc::mbar_init(dq_free + b, NDQ);
    }
    tc::mbar_init(s_full, 1);
    tc::mbar_init(s_read, NCOMPUTE);
    tc::mbar_init(drain, 1);
    tc::mbar_init(drain + 1, 1);
    tc::mbar_init(stage_free, 1);
    tc::mbar_init(stage_full, NDQ);
    tc::mbar_init(kv_tmem, NCOMPUTE);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: S^T [0,64), dP^T [64,128), dV [128,128+D), dK [128+D,128+2D),
  // dQ^T [384,448) (D=128) or the pair dQ [256,320) (D=64), and the packed
  // 16-bit P^T buffers [448+32b, 480+32b).
  const uint32_t t_dv = tmem + 128, t_dk = tmem + 128 + HD, t_dqp = tmem + 256;
  const uint32_t t_dqt = tmem + 384, t_pt = tmem + 448;
  // D = 64: K and V as TMEM A operands of S^T and dP^T (packed 16-bit pairs,
  // lane = key, 32 columns each): they are read by every tile's products,
  // and from TMEM they no longer take shared-memory bandwidth.
  const uint32_t t_kt = tmem + 320, t_vt = tmem + 352;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Lane 0 issues the TMA copies; the whole warp stages each tile's row
    // terms in shared memory, where the compute warps read them as
    // broadcast vector loads (instead of one shuffle per query and term).
    if (n_iter > 0) {
      if (lane == 0) {
        tc::prefetch_tmap(&tm_q);
        tc::prefetch_tmap(&tm_do);
        tc::mbar_expect_tx(kv_full, 2 * L::kKV);
        for (int cb = 0; cb < HD / 64; ++cb) {
          tc::tma_load_3d(smem + L::oK + cb * BK * 128, &tm_k, kv_full, cb * 64, k0, bh);
          tc::tma_load_3d(smem + L::oV + cb * BK * 128, &tm_v, kv_full, cb * 64, k0, bh);
        }
      }
      const size_t row_base = (size_t)bh * Tq;
      // row terms of tile t, loaded one tile ahead so their latency never
      // delays a TMA issue; negated, so they enter paired adds / fmas
      // directly (rows past the end: P = exp2(-inf) = 0)
      float2 rv[2];
      auto load_rows = [&](int t) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int q = tile_of(t) * BQ + h * 32 + lane;
          rv[h] = q < Tq ? make_float2(-__ldg(lse + row_base + q) * 1.4426950408889634f,
                                       -__ldg(z + row_base + q))
                         : make_float2(-INFINITY, 0.f);
        }
      };
      if (kRowStage) load_rows(0);
      int issued = 0;
      for (int t = 0; t < n_iter; ++t) {
        // without staged row terms only lane 0 runs this loop
        if (!kRowStage && lane != 0) break;
        const int st = t % QST;
        bool ok = true;
        if (lane == 0 && t >= QST) ok = tc::mbar_wait(q_empty + st, ((t / QST) - 1) & 1, abort);
        if (kRowStage) ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        const int q0 = tile_of(t) * BQ;
        if (lane == 0) {
          tc::mbar_expect_tx(q_full + st, 2 * L::kQ);
          for (int cb = 0; cb < HD / 64; ++cb) {
            tc::tma_load_3d(smem + L::oQ + st * L::kQ + cb * BQ * 128, &tm_q, q_full + st,
                            cb * 64, q0, bh);
            tc::tma_load_3d(smem + L::oDO + st * L::kQ + cb * BQ * 128, &tm_do, q_full + st,
                            cb * 64, q0, bh);
          }
        }
        if (kRowStage) {
          float2* rt = reinterpret_cast<float2*>(smem + L::oRow + st * L::kRow);
          rt[lane] = rv[0];
          rt[32 + lane] = rv[1];
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(q_full + st);
          if (t + 1 < n_iter) load_rows(t + 1);
        }
        issued = t + 1;
      }
      if (lane == 0) {
        tc::mbar_wait_drain(kv_full, 0);
        for (int t = issued > QST ? issued - QST : 0; t < issued; ++t)
          tc::mbar_wait_drain(q_full + t % QST, (t / QST) & 1);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0 && n_iter > 0) {
      constexpr int ab = tc::AbFmt<T>::v;
      constexpr uint32_t id_s = tc::idesc_f16(BK, BQ, ab, 0, 0);    // S^T, dP^T
      constexpr uint32_t id_kv = tc::idesc_f16(BK, HD, ab, 0, 1);   // dV, dK
      constexpr uint32_t id_dqt = tc::idesc_f16(HD, BQ, ab, 1, 1);  // dQ^T (HD == 128)
      constexpr uint32_t id_dqp = tc::idesc_f16(2 * BQ, HD, ab, 1, 1);  // pair dQ (HD == 64)
      const uint32_t a_k = tc::smem_u32(smem + L::oK), a_v = tc::smem_u32(smem + L::oV);
      const uint32_t a_q = tc::smem_u32(smem + L::oQ), a_do = tc::smem_u32(smem + L::oDO);
      const uint32_t a_ds = tc::smem_u32(smem + L::oDS);
      bool ok = tc::mbar_wait(kv_full, 0, abort);
      if (warp == 1) {
        // S^T = K Q_t^T and dP^T = V dO_t^T into the single S/dP buffer,
        // which is free once the compute warps loaded the previous tile.
        const uint64_t kK = tc::sw128_desc(a_k, 16, 1024), kV = tc::sw128_desc(a_v, 16, 1024);
        const uint64_t kQ = tc::sw128_desc(a_q, 16, 1024), kDO = tc::sw128_desc(a_do, 16, 1024);
        if (kPairDq) ok = ok && tc::mbar_wait(kv_tmem, 0, abort);
        for (int t = 0; ok && t < n_iter; ++t) {
          const int st = t % QST;
          if (!tc::mbar_wait(q_full + st, (t / QST) & 1, abort)) break;
          if (t >= 1 && !tc::mbar_wait(s_read, (t - 1) & 1, abort)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off_a = (kk / 4) * (BK * 128) + (kk % 4) * 32;
            const uint32_t off_b = st * L::kQ + (kk / 4) * (BQ * 128) + (kk % 4) * 32;
            if constexpr (kPairDq) {
              tc::mma_ts(tmem + 64, t_vt + kk * 8, tc::desc_at(kDO, off_b), id_s,
                         kk > 0 ? 1u : 0u);
              tc::mma_ts(tmem, t_kt + kk * 8, tc::desc_at(kQ, off_b), id_s, kk > 0 ? 1u : 0u);
            } else {
              tc::mma_ss(tmem + 64, tc::desc_at(kV, off_a), tc::desc_at(kDO, off_b), id_s,
                         kk > 0 ? 1u : 0u);
              tc::mma_ss(tmem, tc::desc_at(kK, off_a), tc::desc_at(kQ, off_b), id_s,
                         kk > 0 ? 1u : 0u);
            }
          }
          tc::mma_commit(s_full);
        }
        tc::mma_commit(drain);
        tc::mbar_wait_drain(drain, 0);
      } else {
        // dV += P^T dO_t, dK += dS^T Q_t, then dQ; releases the Q/dO stage.
        const uint64_t kDS = tc::sw128_desc(a_ds, 16, 1024);
        const uint64_t mQ = tc::sw128_desc(a_q, BQ * 128, 1024);
        const uint64_t mDO = tc::sw128_desc(a_do, BQ * 128, 1024);
        const uint64_t mK = tc::sw128_desc(a_k, BK * 128, 1024);
        const uint64_t mDS = tc::sw128_desc(a_ds, BK * 128, 1024);
        const uint64_t mDSpair = tc::sw128_desc(a_ds, L::kP, 1024);
        for (int t = 0; ok && t < n_iter; ++t) {
          const int b = t & 1;
          // D = 64: the pair-dQ buffer wait comes first.  It is normally
          // satisfied, but any wait costs this (MMA-issuing) thread a few
          // hundred cycles, better spent while the compute warps still produce
          // P^T / dS^T.  (For D = 128 the previous dQ^T flush can still be
          // running here, and waiting for it would hold back dV/dK.)
          if (kPairDq && ((t & 1) || t == n_iter - 1) && (t >> 1) > 0 &&
              !tc::mbar_wait(dq_free, ((t >> 1) - 1) & 1, abort))
            break;
          if (!tc::mbar_wait(p_full + b, (t >> 1) & 1, abort)) break;
          tc::tc_fence_after();
          const uint32_t pbo = b * L::kP;  // this tile's dS^T buffer offset
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {
            // contraction over the tile's queries: P^T from TMEM (8 packed
            // columns per 16 queries), dS^T K-major in smem, dO / Q MN-major
            const uint32_t off_b = (t % QST) * L::kQ + kk * 16 * 128;
            const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
            tc::mma_ts(t_dv, t_pt + b * 32 + kk * 8, tc::desc_at(mDO, off_b), id_kv, acc);
            tc::mma_ss(t_dk, tc::desc_at(kDS, pbo + kk * 32), tc::desc_at(mQ, off_b), id_kv,
                       acc);
          }
          if constexpr (!kPairDq) {
            // dQ^T = K^T dS^T over the keys, once the previous dQ^T was read
            if (t >= 1 && !tc::mbar_wait(dq_free, (t - 1) & 1, abort)) break;
            tc::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              tc::mma_ss(t_dqt, tc::desc_at(mK, kk * 2048),
                         tc::desc_at(mDS, pbo + kk * 2048), id_dqt, kk > 0 ? 1u : 0u);
          } else if ((t & 1) || t == n_iter - 1) {
            // dQ for the pair (2p, 2p+1): both dS^T buffers as one M = 128 operand
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              tc::mma_ss(t_dqp, tc::desc_at(mDSpair, kk * 2048), tc::desc_at(mK, kk * 2048),
                         id_dqp, kk > 0 ? 1u : 0u);
          }
          tc::mma_commit(mma2_done + b);
          // S^T/dP^T of tile t also read this stage; they completed before
          // the compute warps could publish p_full for tile t.
          tc::mma_commit(q_empty + t % QST);
        }
        tc::mma_commit(drain + 1);
        tc::mbar_wait_drain(drain + 1, 0);
      }
    }
  } else if (warp < kFirstCompute + NCOMPUTE / 32) {
    // ------------------------------------------------------------ compute
    // Warps 3..10: P^T and dS^T, then dK / dV at the end.  Group `grp`
    // handles query columns [32 grp, 32 grp + 32) of each tile.
    const int grp = (warp - kFirstCompute) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane = key row
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int key = k0 + r;
    bool ok = true;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, abort));
    };
    const uint32_t a_ds = tc::smem_u32(smem + L::oDS);
    const size_t row_base = (size_t)bh * Tq;
    if (kPairDq && n_iter > 0) {
      // copy this thread's key row of K (group 0) or V (group 1) into TMEM:
      // the 128-byte SW128 row is 32 packed pairs, one per column
      ok = wait(kv_full, 0);
      if (ok) {
        const uint32_t row = tc::smem_u32(smem + (grp == 0 ? L::oK : L::oV)) + (uint32_t)r * 128;
        uint32_t w[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 x = tc::ld_shared_f4(row + (uint32_t)((c ^ (r & 7)) << 4));
          w[4 * c] = __float_as_uint(x.x);
          w[4 * c + 1] = __float_as_uint(x.y);
          w[4 * c + 2] = __float_as_uint(x.z);
          w[4 * c + 3] = __float_as_uint(x.w);
        }
        tc::tmem_st32u((grp == 0 ? t_kt : t_vt) + lane_off, w);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        tc::mbar_arrive(kv_tmem);
      }
    }
    for (int t = 0; ok && t < n_iter; ++t) {
      const int b = t & 1;
      const int q0 = tile_of(t) * BQ;
      // Row terms of this group's 32 queries: staged by the producer warp,
      // or one load per lane broadcast by shuffles below.
      const uint32_t rows_at = tc::smem_u32(smem + L::oRow + (t % QST) * L::kRow) + grp * 32 * 8;
      float my_l = 0.f, my_z = 0.f;
      if (kRowStage) {
        if (!wait(q_full + t % QST, (t / QST) & 1)) { ok = false; break; }
      } else {
        const int ql = q0 + grp * 32 + lane;
        // negated, so the row terms enter paired adds / fmas directly
        my_l = ql < Tq ? -__ldg(lse + row_base + ql) * 1.4426950408889634f : -INFINITY;
        my_z = ql < Tq ? -__ldg(z + row_base + ql) : 0.f;
      }
      if (!wait(s_full, t & 1)) { ok = false; break; }
      tc::tc_fence_after();
      float s[32], dp[32];
      tc::tmem_ld32(tmem + lane_off + grp * 32, s);
      tc::tmem_ld32(tmem + 64 + lane_off + grp * 32, dp);
      tc::tc_fence_before();
      tc::mbar_arrive(s_read);  // the tensor core may start on the next tile
      // P^T / dS^T buffers b are free once the MMAs that read them are done:
      // tile t-2's dV/dK (and dQ); with paired dQ, an even tile's buffer is
      // also read by the pair MMA issued with tile t-1.
      if (t >= 2) {
        const int tw = (kPairDq && !(t & 1)) ? t - 1 : t - 2;
        if (!wait(mma2_done + (tw & 1), (tw >> 1) & 1)) { ok = false; break; }
      }
      // Masking is needed only on the causal diagonal and for a ragged last
      // key tile; the test is uniform per tile, so other tiles skip it.
      const bool diag = CAUSAL && (q0 < k0 + BK);
      const bool edge = diag || (k0 + BK > M);
      // valid columns e satisfy e >= e_min (causal: query >= key); none if key >= M
      const int e_min = key >= M ? 32 : (diag ? key - (q0 + grp * 32) : 0);
      // two columns at a time on paired fp32 instructions
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float nl0, nl1, nz0, nz1;
        if (kRowStage) {
          // {-l, -z} of queries e and e+1: one broadcast 16-byte load
          const float4 rr = tc::ld_shared_f4(rows_at + e * 8);
          nl0 = rr.x; nz0 = rr.y; nl1 = rr.z; nz1 = rr.w;
        } else {
          nl0 = __shfl_sync(0xffffffffu, my_l, e);
          nl1 = __shfl_sync(0xffffffffu, my_l, e + 1);
          nz0 = __shfl_sync(0xffffffffu, my_z, e);
          nz1 = __shfl_sync(0xffffffffu, my_z, e + 1);
        }
        float x0, x1, g0, g1;
        tc::fma2(x0, x1, s[e], s[e + 1], scale_log2, scale_log2, nl0, nl1);
        float p0 = tc::ex2(x0), p1 = tc::ex2(x1);  // rows past the end: -inf -> 0
        if (edge && e < e_min) p0 = 0.f;
        if (edge && e + 1 < e_min) p1 = 0.f;
        s[e] = p0;  // P^T
        s[e + 1] = p1;
        tc::add2(g0, g1, dp[e], dp[e + 1], nz0, nz1);
        tc::mul2(dp[e], dp[e + 1], p0, p1, g0, g1);  // dS^T = P^T (dP^T - z)
      }
      // P^T stays in TMEM as packed 16-bit pairs (A operand of dV += P^T dO);
      // dS^T goes to shared memory (operand of dK and dQ).
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = tc::pack2<T>(s[2 * i], s[2 * i + 1]);
      tc::tmem_st16(t_pt + b * 32 + grp * 16 + lane_off, pk);
      const uint32_t db = a_ds + b * L::kP;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t off = tc::sw128_off(r, grp * 4 + h);
        const float* de = dp + h * 8;
        tc::st_shared_v4(db + off, tc::pack2<T>(de[0], de[1]), tc::pack2<T>(de[2], de[3]),
                         tc::pack2<T>(de[4], de[5]), tc::pack2<T>(de[6], de[7]));
      }
      tc::tmem_wait_st();
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full + b);
    }
    // ------------------------------------------------------------ dK, dV
    if (ok && n_iter > 0) {
      const int tl = n_iter - 1;
      ok = wait(mma2_done + (tl & 1), (tl >> 1) & 1);
      if (ok) tc::tc_fence_after();
    }
    if (ok) {
      const bool store = key < M;
      const size_t base = ((size_t)bh * M + (store ? key : 0)) * HD;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        T* out = which == 0 ? dv : dk;
        if (out == nullptr) continue;
        const float mul = which == 0 ? 1.f : scale;
        const uint32_t col = which == 0 ? t_dv : t_dk;
#pragma unroll 1
        for (int c = grp * (HD / 64); c < (grp + 1) * (HD / 64); ++c) {
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
  } else {
    // ------------------------------------------------------------ dQ flush
    // Warps 11..14: read each finished dQ out of TMEM and add it (scaled)
    // into the fp32 accumulator, concurrently with the next tile's compute.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const size_t row_base = (size_t)bh * Tq;
    const bool bulk_issuer = warp == kFirstCompute + NCOMPUTE / 32 && lane == 0;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, abort));
    };
    for (int t = 0; t < n_iter; ++t) {
      if (kPairDq && !(t & 1) && t != n_iter - 1) continue;  // pairs finish on odd tiles
      if (!wait(mma2_done + (t & 1), (t >> 1) & 1)) break;
      tc::tc_fence_after();
      if constexpr (!kPairDq) {
        // dQ^T of tile t (lane = head-dim index r, 64 query columns): read
        // it out of TMEM, release the buffer, stage it scaled as fp32 rows
        // [q][d] and add the tile to dQacc with one bulk reduction.  The
        // staging buffer is reused once the previous reduction has read it.
        const int qb = tile_of(t) * BQ;
        float v0[32], v1[32];
        tc::tmem_ld32(t_dqt + lane_off, v0);
        tc::tmem_ld32(t_dqt + lane_off + 32, v1);
        tc::tc_fence_before();
        tc::mbar_arrive(dq_free);
        if (bulk_issuer) {
          tc::bulk_wait_read_all();
          tc::mbar_arrive(stage_free);
        }
        if (!wait(stage_free, t & 1)) break;
        float* stage = reinterpret_cast<float*>(smem + L::oStage);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          stage[e * HD + r] = v0[e] * scale;
          stage[(32 + e) * HD + r] = v1[e] * scale;
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(stage_full);
        bool staged = true;
        if (bulk_issuer) {
          staged = tc::mbar_wait(stage_full, t & 1, abort);
          const int rows = Tq - qb < BQ ? Tq - qb : BQ;
          if (staged)
            tc::bulk_reduce_add_f32(dq_acc + (row_base + qb) * HD, smem + L::oStage,
                                    (uint32_t)(rows * HD * 4));
        }
        if (!__shfl_sync(0xffffffffu, staged, 0)) break;
      } else {
        // dQ of the pair ending at tile t (lane = query row, 64 head dims):
        // read out of TMEM, release the buffer, stage it scaled in two
        // 128-byte-swizzled halves [q][32 d] (the swizzle spreads a warp's
        // 16-byte stores over all banks) and add the pair's rows to dQacc with
        // two bulk tensor reductions (rows past the end are clipped).
        const int qb = tile_of(t & ~1) * BQ;
        float v0[32], v1[32];
        tc::tmem_ld32(t_dqp + lane_off, v0);
        tc::tmem_ld32(t_dqp + lane_off + 32, v1);
        tc::tc_fence_before();
        tc::mbar_arrive(dq_free);
        const int pi = t >> 1;  // pair index: phase of the staging barriers
        if (bulk_issuer) {
          tc::bulk_wait_read_all();
          tc::mbar_arrive(stage_free);
        }
        if (!wait(stage_free, pi & 1)) break;
        const uint32_t srow = tc::smem_u32(smem + L::oStage) + (uint32_t)r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t off = (uint32_t)((c ^ (r & 7)) << 4);
          tc::st_shared_v4(srow + off, __float_as_uint(v0[4 * c] * scale),
                           __float_as_uint(v0[4 * c + 1] * scale),
                           __float_as_uint(v0[4 * c + 2] * scale),
                           __float_as_uint(v0[4 * c + 3] * scale));
          tc::st_shared_v4(srow + 16384 + off, __float_as_uint(v1[4 * c] * scale),
                           __float_as_uint(v1[4 * c + 1] * scale),
                           __float_as_uint(v1[4 * c + 2] * scale),
                           __float_as_uint(v1[4 * c + 3] * scale));
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(stage_full);
        bool staged = true;
        if (bulk_issuer) {
          staged = tc::mbar_wait(stage_full, pi & 1, abort);
          if (staged) {
            tc::bulk_tensor_reduce_add_3d(&tm_dq, smem + L::oStage, 0, qb, bh);
            tc::bulk_tensor_reduce_add_3d(&tm_dq, smem + L::oStage + 16384, 32, qb, bh);
          }
        }
        if (!__shfl_sync(0xffffffffu, staged, 0)) break;
      }
    }
    // the last reductions must finish before the CTA (and its staging
    // buffer) goes away
    if (bulk_issuer) tc::bulk_wait_all();
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
