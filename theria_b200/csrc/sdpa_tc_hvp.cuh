// Tensor-core (tcgen05) HVP backward pass for bf16/fp16, head dim 64 or 128.
//
// Hessian-vector product of L = <O, W> along u = (tQ, tK, tV), given the
// forward LSE and the row terms of pass 1 (c = rowsum(P Sdot),
// z = rowsum(W O), zdot = rowsum(W Odot); see sdpa_tc_jvp.cuh).
// One CTA per (128-key tile, batch*head), looping over 64-row query tiles:
//   S^T  = K Q^T,   Sd'^T = K tQ^T + tK Q^T,   dP^T = V W^T,   dPd^T = tV W^T
//   P = exp(s S - LSE), Pd = P (s Sd' - c), dS = P (dP - z),
//   dSd = Pd (dP - z) + P (dPd - zdot)                     (CUDA cores)
//   hK += dSd^T Q + dS^T tQ,   hV += Pd^T W                 (TMEM accumulators)
//   hQ  = dSd K + dS tK   -> fp32 accumulator via global reductions
// hQ is formed like dQ in the backward: for D = 128 as hQ^T (M = D lanes)
// over the S^T columns once read, for D = 64 per pair of query tiles
// (M = 128 query rows) in its own columns.
// TMEM: S^T [0,64), Sd^T [64,128), dP^T [128,192), dPd^T [192,256),
// hV [256, 256+D), hK [256+D, 256+2D), pair hQ [384, 448) for D = 64.
// Warp roles: 0 TMA, 1 issues the S-group products (and owns TMEM), 2
// issues hK, hV and hQ, 3 stages the row terms, 4..11 compute, 12..15 hQ
// flush.  With the two groups on separate threads the next tile's S-group
// (D = 64) runs on the tensor core while the CUDA cores still work on the
// current tile; for D = 128 the S-group waits for hQ^T to leave the S^T
// columns.
#pragma once

#include "sdpa_tc_bwd.cuh"

namespace theria {
namespace tchvp {

constexpr int BK = 128, BQ = 64;
constexpr int NCOMPUTE = 256, NDQ = 128;
// Four warpgroups: control (TMA, two MMA issuers, one idle warp), two of
// compute, one of hQ flush.  Registers are moved from the control and flush
// groups to the compute groups (setmaxnreg), whose threads hold four
// 32-column rows of scores at once.
constexpr int NTHREADS = 128 + NCOMPUTE + NDQ;
constexpr int kFirstCompute = 4;
// Per head dim (control, compute, flush), registers per thread; measured
// at configs[2] and B1 H32 N4096: D = 64 gains 1-3 % from a leaner control
// and flush group, D = 128 (whose control and flush code needs the room)
// does not.
#ifndef THERIA_HVP64_RC
#define THERIA_HVP64_RC 96
#define THERIA_HVP64_RM 160
#define THERIA_HVP64_RF 96
#endif
#ifndef THERIA_HVP128_RC
#define THERIA_HVP128_RC 112
#define THERIA_HVP128_RM 144
#define THERIA_HVP128_RF 112
#endif
template <int HD>
struct RegSplit {
  static constexpr int ctl = HD == 64 ? THERIA_HVP64_RC : THERIA_HVP128_RC;
  static constexpr int compute = HD == 64 ? THERIA_HVP64_RM : THERIA_HVP128_RM;
  static constexpr int flush = HD == 64 ? THERIA_HVP64_RF : THERIA_HVP128_RF;
  static constexpr int total = ctl + 2 * compute + flush;
  // a warp's launch allocation is the largest multiple of 8 registers that
  // fits NTHREADS threads in 64K; a split above it would wait forever
  static_assert(total * 128 <= (65536 / NTHREADS) / 8 * 8 * NTHREADS,
                "register split exceeds the launch allocation");
};

template <int HD>
struct Cfg {
  static constexpr int ST = HD == 64 ? 2 : 1;  // Q/tQ/W ring depth (what smem allows)
  static constexpr int kKV = BK * HD * 2;
  static constexpr int kQ = BQ * HD * 2;
  static constexpr int kP = BK * BQ * 2;
  static constexpr int oK = 0, oV = kKV, oTK = 2 * kKV, oTV = 3 * kKV;
  static constexpr int oQ = 4 * kKV;             // stage s: Q, tQ, W at oQ + s*3*kQ
  static constexpr int oPd = oQ + ST * 3 * kQ;   // Pd^T [key][q]
  static constexpr int NB = HD == 64 ? 2 : 1;   // dS/dSd buffers (2: pair operand)
  static constexpr int oDS = oPd + kP;           // dS^T  x NB (adjacent)
  static constexpr int oDSd = oDS + NB * kP;     // dSd^T x NB (adjacent)
  // fp32 hQ of a pair of query tiles, staged as two 128-byte-swizzled halves
  // [128 q][32 d] for the bulk tensor reduction (D = 64 only)
  static constexpr int oStage = oDSd + NB * kP;
  static constexpr int kStage = HD == 64 ? 32768 : 0;
  // per Q/tQ/W stage, row terms of the tile's 64 queries staged by warp 3:
  // {-LSE*log2(e), -z} (D = 64; c and zdot stay on shuffles: the shared
  // memory has room for no more) or {-LSE*log2(e), -c, -z, -zdot} (D = 128)
  static constexpr int NTERM = HD == 64 ? 2 : 4;
  static constexpr int kRow = BQ * NTERM * 4;
  static constexpr int oRow = oStage + kStage;
  static constexpr int oBar = oRow + ST * kRow;
  // kv_full, q_full[3], q_empty[3], s_full, s_read, p_full, mma2_done[2],
  // hq_free, drain[2], stage_free, stage_full
  static constexpr int nBar = 17;
  static constexpr int oTmem = oBar + nBar * 8;
  static constexpr int oAbort = oTmem + 4;
  static constexpr int kAlloc = oAbort + 4 + 1024;
};

template <typename T, int HD, bool CAUSAL>
__global__ void __launch_bounds__(NTHREADS, 1)
hvp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_tq,
           const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_k,
           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_tk,
           const __grid_constant__ CUtensorMap tm_tv, const __grid_constant__ CUtensorMap tm_hq,
           const float* __restrict__ lse,
           const float* __restrict__ stats, int64_t n_rows_total, float* __restrict__ hq_acc,
           T* __restrict__ hk, T* __restrict__ hv, int Tq, int M, float scale,
           float scale_log2, float* __restrict__ hkv_acc, int n_split) {
  using C = Cfg<HD>;
  constexpr bool kPair = (HD == 64);
  // Row terms staged in shared memory by warp 3 (see there): measured
  // +4-7 % non-causal; causal grids (many short CTAs) measured 0-5 % slower
  // with it, so they keep the shuffles.
  constexpr bool kRowStage = !CAUSAL;
  constexpr int ST = C::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::oBar);
  uint64_t *kv_full = bars, *q_full = bars + 1, *q_empty = bars + 4, *s_full = bars + 7,
           *s_read = bars + 8, *p_full = bars + 9, *mma2_done = bars + 10, *hq_free = bars + 12,
           *drain = bars + 13, *stage_free = bars + 15, *stage_full = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + C::oAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Causal grids put the head index in x so the heaviest tiles of every head
  // are dispatched first (longest-first over the whole grid).
  const int bh = CAUSAL ? blockIdx.x : blockIdx.y;
  const int k0 = (CAUSAL ? blockIdx.y : blockIdx.x) * BK;
  const int n_qt = (Tq + BQ - 1) / BQ;
  // With n_split > 1 the query tiles that see this key tile are divided into
  // n_split chunks (gridDim.z), each an even number of tiles so that dQ-style
  // pairs never straddle two CTAs; hK and hV are then partial sums, added in
  // fp32 into hkv_acc [2][B*H][M][D] (hV, then hK already scaled).
  const int i_first = CAUSAL ? k0 / BQ : 0;
  const int n_all = n_qt > i_first ? n_qt - i_first : 0;
  const int chunk = n_split > 1 ? (((n_all + n_split - 1) / n_split + 1) & ~1) : n_all;
  const int i_begin = i_first + (int)blockIdx.z * chunk;
  const int n_iter = n_qt - i_begin < chunk ? (n_qt > i_begin ? n_qt - i_begin : 0) : chunk;

  if (threadIdx.x == 0) {
    tc::mbar_init(kv_full, 1);
    for (int b = 0; b < 3; ++b) {
      tc::mbar_init(q_full + b, kRowStage ? 2 : 1);  // TMA bytes (+ warp 3's row terms)
      tc::mbar_init(q_empty + b, 1);
    }
    for (int b = 0; b < 2; ++b) tc::mbar_init(mma2_done + b, 1);
    tc::mbar_init(s_full, 1);
    tc::mbar_init(s_read, NCOMPUTE);
    tc::mbar_init(p_full, NCOMPUTE);
    tc::mbar_init(hq_free, NDQ);
    tc::mbar_init(drain, 1);
    tc::mbar_init(drain + 1, 1);
    tc::mbar_init(stage_free, 1);
    tc::mbar_init(stage_full, NDQ);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_hv = tmem + 256, t_hk = tmem + 256 + HD, t_hqp = tmem + 384;

  if (warp < kFirstCompute)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RegSplit<HD>::ctl));
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_iter > 0) {
      tc::mbar_expect_tx(kv_full, 4 * C::kKV);
      for (int cb = 0; cb < HD / 64; ++cb) {
        const int o = cb * BK * 128;
        tc::tma_load_3d(smem + C::oK + o, &tm_k, kv_full, cb * 64, k0, bh);
        tc::tma_load_3d(smem + C::oV + o, &tm_v, kv_full, cb * 64, k0, bh);
        tc::tma_load_3d(smem + C::oTK + o, &tm_tk, kv_full, cb * 64, k0, bh);
        tc::tma_load_3d(smem + C::oTV + o, &tm_tv, kv_full, cb * 64, k0, bh);
      }
      int issued = 0;
      for (int t = 0; t < n_iter; ++t) {
        const int st = t % ST;
        if (t >= ST && !tc::mbar_wait(q_empty + st, ((t / ST) - 1) & 1, abort)) break;
        const int q0 = (i_begin + t) * BQ;
        uint8_t* base = smem + C::oQ + st * 3 * C::kQ;
        tc::mbar_expect_tx(q_full + st, 3 * C::kQ);
        for (int cb = 0; cb < HD / 64; ++cb) {
          const int o = cb * BQ * 128;
          tc::tma_load_3d(base + o, &tm_q, q_full + st, cb * 64, q0, bh);
          tc::tma_load_3d(base + C::kQ + o, &tm_tq, q_full + st, cb * 64, q0, bh);
          tc::tma_load_3d(base + 2 * C::kQ + o, &tm_w, q_full + st, cb * 64, q0, bh);
        }
        issued = t + 1;
      }
      tc::mbar_wait_drain(kv_full, 0);
      for (int t = issued > ST ? issued - ST : 0; t < issued; ++t)
        tc::mbar_wait_drain(q_full + t % ST, (t / ST) & 1);
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0 && n_iter > 0) {
      constexpr int ab = tc::AbFmt<T>::v;
      constexpr uint32_t id_s = tc::idesc_f16(BK, BQ, ab, 0, 0);
      constexpr uint32_t id_kv = tc::idesc_f16(BK, HD, ab, 0, 1);
      constexpr uint32_t id_hqt = tc::idesc_f16(HD, BQ, ab, 1, 1);      // HD == 128
      constexpr uint32_t id_hqp = tc::idesc_f16(2 * BQ, HD, ab, 1, 1);  // HD == 64
      const uint32_t a_k = tc::smem_u32(smem + C::oK), a_v = tc::smem_u32(smem + C::oV);
      const uint32_t a_tk = tc::smem_u32(smem + C::oTK), a_tv = tc::smem_u32(smem + C::oTV);
      const uint32_t a_q0 = tc::smem_u32(smem + C::oQ);
      // base descriptors (K-major "k", MN-major "m"), advanced by constant adds
      const uint64_t kK = tc::sw128_desc(a_k, 16, 1024), kV = tc::sw128_desc(a_v, 16, 1024);
      const uint64_t kTK = tc::sw128_desc(a_tk, 16, 1024), kTV = tc::sw128_desc(a_tv, 16, 1024);
      const uint64_t kQ0 = tc::sw128_desc(a_q0, 16, 1024);              // + stage, Q/tQ/W
      const uint64_t mQ0 = tc::sw128_desc(a_q0, BQ * 128, 1024);
      const uint64_t kPd = tc::sw128_desc(tc::smem_u32(smem + C::oPd), 16, 1024);
      const uint64_t kDS = tc::sw128_desc(tc::smem_u32(smem + C::oDS), 16, 1024);
      const uint64_t kDSd = tc::sw128_desc(tc::smem_u32(smem + C::oDSd), 16, 1024);
      const uint64_t mK = tc::sw128_desc(a_k, BK * 128, 1024);
      const uint64_t mTK = tc::sw128_desc(a_tk, BK * 128, 1024);
      const uint64_t mDS = tc::sw128_desc(tc::smem_u32(smem + C::oDS), BK * 128, 1024);
      const uint64_t mDSd = tc::sw128_desc(tc::smem_u32(smem + C::oDSd), BK * 128, 1024);
      const uint64_t mDSp = tc::sw128_desc(tc::smem_u32(smem + C::oDS), C::kP, 1024);
      const uint64_t mDSdp = tc::sw128_desc(tc::smem_u32(smem + C::oDSd), C::kP, 1024);
      bool ok = tc::mbar_wait(kv_full, 0, abort);
      if (warp == 1) {
        for (int t = 0; ok && t < n_iter; ++t) {
          const int st = t % ST;
          const uint32_t qo = st * 3 * C::kQ, to = qo + C::kQ, wo = qo + 2 * C::kQ;
          if (!tc::mbar_wait(q_full + st, (t / ST) & 1, abort)) break;
          if (t >= 1 && !tc::mbar_wait(s_read, (t - 1) & 1, abort)) break;
          // D = 128: hQ^T(t-1) sits in the S^T columns until it is flushed
          if (!kPair && t >= 1 && !tc::mbar_wait(hq_free, (t - 1) & 1, abort)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t oa = (kk / 4) * (BK * 128) + (kk % 4) * 32;
            const uint32_t ob = (kk / 4) * (BQ * 128) + (kk % 4) * 32;
            const uint32_t acc = kk > 0 ? 1u : 0u;
            tc::mma_ss(tmem + 0, tc::desc_at(kK, oa), tc::desc_at(kQ0, qo + ob), id_s, acc);
            tc::mma_ss(tmem + 64, tc::desc_at(kK, oa), tc::desc_at(kQ0, to + ob), id_s, acc);
            tc::mma_ss(tmem + 64, tc::desc_at(kTK, oa), tc::desc_at(kQ0, qo + ob), id_s, 1u);
            tc::mma_ss(tmem + 128, tc::desc_at(kV, oa), tc::desc_at(kQ0, wo + ob), id_s, acc);
            tc::mma_ss(tmem + 192, tc::desc_at(kTV, oa), tc::desc_at(kQ0, wo + ob), id_s, acc);
          }
          tc::mma_commit(s_full);
        }
        tc::mma_commit(drain);
        tc::mbar_wait_drain(drain, 0);
      } else {
        for (int t = 0; ok && t < n_iter; ++t) {
          const int st = t % ST;
          const uint32_t bo = (kPair ? (t & 1) : 0) * C::kP;  // dS/dSd buffer offset
          const uint32_t qo = st * 3 * C::kQ, to = qo + C::kQ, wo = qo + 2 * C::kQ;
          // D = 64: the pair-hQ buffer wait comes before the P wait (a wait
          // costs this MMA-issuing thread a few hundred cycles even when
          // satisfied; here it overlaps the compute warps' work)
          if (kPair && ((t & 1) || t == n_iter - 1) && (t >> 1) > 0 &&
              !tc::mbar_wait(hq_free, ((t >> 1) - 1) & 1, abort))
            break;
          if (!tc::mbar_wait(p_full, t & 1, abort)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {
            const uint32_t ob = kk * 16 * 128;
            const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
            tc::mma_ss(t_hk, tc::desc_at(kDSd, bo + kk * 32), tc::desc_at(mQ0, qo + ob), id_kv,
                       acc);                                                       // dSd^T Q
            tc::mma_ss(t_hk, tc::desc_at(kDS, bo + kk * 32), tc::desc_at(mQ0, to + ob), id_kv,
                       1u);                                                        // dS^T tQ
            tc::mma_ss(t_hv, tc::desc_at(kPd, kk * 32), tc::desc_at(mQ0, wo + ob), id_kv,
                       acc);                                                       // Pd^T W
          }
          if constexpr (!kPair) {
            // hQ^T = K^T dSd^T + tK^T dS^T, into the S^T columns (the compute
            // warps loaded S^T(t) before publishing p_full)
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint32_t o = kk * 2048;
              tc::mma_ss(tmem, tc::desc_at(mK, o), tc::desc_at(mDSd, bo + o), id_hqt,
                         kk > 0 ? 1u : 0u);
              tc::mma_ss(tmem, tc::desc_at(mTK, o), tc::desc_at(mDS, bo + o), id_hqt, 1u);
            }
          } else if ((t & 1) || t == n_iter - 1) {
            // hQ = dSd K + dS tK for the pair (2p, 2p+1) (buffer free: above)
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint32_t o = kk * 2048;
              tc::mma_ss(t_hqp, tc::desc_at(mDSdp, o), tc::desc_at(mK, o), id_hqp,
                         kk > 0 ? 1u : 0u);
              tc::mma_ss(t_hqp, tc::desc_at(mDSp, o), tc::desc_at(mTK, o), id_hqp, 1u);
            }
          }
          tc::mma_commit(mma2_done + (t & 1));
          // the S-group products of tile t also read this stage; they were
          // complete before the compute warps could publish p_full(t)
          tc::mma_commit(q_empty + st);
        }
        tc::mma_commit(drain + 1);
        tc::mbar_wait_drain(drain + 1, 0);
      }
    }
  } else if (warp < kFirstCompute) {
    // ------------------------------------------------------------ row terms
    // Warp 3 stages each tile's per-query row terms in shared memory (one
    // tile ahead of their use), where the compute warps read them as
    // broadcast vector loads instead of one shuffle per query and term.
    if (kRowStage && n_iter > 0) {
      const size_t row_base = (size_t)bh * Tq;
      float rv[2][C::NTERM];
      auto load_rows = [&](int t) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int q = (i_begin + t) * BQ + h * 32 + lane;
          const bool in = q < Tq;
          // negated, so they enter paired adds / fmas directly
          rv[h][0] = in ? -__ldg(lse + row_base + q) * 1.4426950408889634f : -INFINITY;
          if constexpr (C::NTERM == 2) {
            rv[h][1] = in ? -__ldg(stats + n_rows_total + row_base + q) : 0.f;
          } else {
            rv[h][1] = in ? -__ldg(stats + row_base + q) : 0.f;
            rv[h][2] = in ? -__ldg(stats + n_rows_total + row_base + q) : 0.f;
            rv[h][3] = in ? -__ldg(stats + 2 * n_rows_total + row_base + q) : 0.f;
          }
        }
      };
      load_rows(0);
      for (int t = 0; t < n_iter; ++t) {
        const int st = t % ST;
        bool ok = true;
        if (lane == 0 && t >= ST) ok = tc::mbar_wait(q_empty + st, ((t / ST) - 1) & 1, abort);
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        float* rt = reinterpret_cast<float*>(smem + C::oRow + st * C::kRow);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < C::NTERM; ++i) rt[(h * 32 + lane) * C::NTERM + i] = rv[h][i];
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(q_full + st);
        if (t + 1 < n_iter) load_rows(t + 1);
      }
    }
  } else if (warp < kFirstCompute + NCOMPUTE / 32) {
    // ------------------------------------------------------------ compute
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(RegSplit<HD>::compute));
    const int grp = (warp - kFirstCompute) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane = key row
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int key = k0 + r;
    bool ok = true;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, abort));
    };
    const uint32_t a_pd = tc::smem_u32(smem + C::oPd);
    const uint32_t a_ds = tc::smem_u32(smem + C::oDS), a_dsd = tc::smem_u32(smem + C::oDSd);
    const size_t row_base = (size_t)bh * Tq;
    for (int t = 0; t < n_iter; ++t) {
      const int b = kPair ? (t & 1) : 0;
      const int q0 = (i_begin + t) * BQ;
      const int ql = q0 + grp * 32 + lane;
      const bool qin = ql < Tq;
      // Row terms of this group's 32 queries: staged in shared memory by
      // warp 3 (all four for D = 128; LSE and z for D = 64), the others one
      // load per lane broadcast by shuffles.  Negated, so they enter paired
      // adds / fmas directly.
      const uint32_t rows_at =
          tc::smem_u32(smem + C::oRow + (t % ST) * C::kRow) + grp * 32 * C::NTERM * 4;
      float my_l = 0.f, my_c = 0.f, my_z = 0.f, my_zd = 0.f;
      if (kRowStage) {
        if (!wait(q_full + t % ST, (t / ST) & 1)) { ok = false; break; }
      } else {
        my_l = qin ? -__ldg(lse + row_base + ql) * 1.4426950408889634f : -INFINITY;
        my_z = qin ? -__ldg(stats + n_rows_total + row_base + ql) : 0.f;
      }
      if (!kRowStage || C::NTERM == 2) {
        my_c = qin ? -__ldg(stats + row_base + ql) : 0.f;
        my_zd = qin ? -__ldg(stats + 2 * n_rows_total + row_base + ql) : 0.f;
      }
      if (!wait(s_full, t & 1)) { ok = false; break; }
      tc::tc_fence_after();
      float sv[32], sd[32], dp[32], dpd[32];
      const uint32_t c0 = tmem + lane_off + grp * 32;
      tc::tmem_ld32(c0, sv);
      tc::tmem_ld32(c0 + 64, sd);
      tc::tmem_ld32(c0 + 128, dp);
      tc::tmem_ld32(c0 + 192, dpd);
      tc::tc_fence_before();
      tc::mbar_arrive(s_read);
      const bool diag = CAUSAL && (q0 < k0 + BK);
      const bool edge = diag || (k0 + BK > M);  // uniform per tile
      const int e_min = key >= M ? 32 : (diag ? key - (q0 + grp * 32) : 0);
      // two columns at a time on paired fp32 instructions
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float nl[2], nc[2], nz[2], nzd[2];
        if (kRowStage && C::NTERM == 4) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float4 rr = tc::ld_shared_f4(rows_at + (e + i) * 16);
            nl[i] = rr.x; nc[i] = rr.y; nz[i] = rr.z; nzd[i] = rr.w;
          }
        } else {
          if (kRowStage) {
            const float4 rr = tc::ld_shared_f4(rows_at + e * 8);  // {l, z} of e, e+1
            nl[0] = rr.x; nz[0] = rr.y; nl[1] = rr.z; nz[1] = rr.w;
          }
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (!kRowStage) {
              nl[i] = __shfl_sync(0xffffffffu, my_l, e + i);
              nz[i] = __shfl_sync(0xffffffffu, my_z, e + i);
            }
            nc[i] = __shfl_sync(0xffffffffu, my_c, e + i);
            nzd[i] = __shfl_sync(0xffffffffu, my_zd, e + i);
          }
        }
        float x0, x1, pd0, pd1, g0, g1, h0, h1;
        tc::fma2(x0, x1, sv[e], sv[e + 1], scale_log2, scale_log2, nl[0], nl[1]);
        float p0 = tc::ex2(x0), p1 = tc::ex2(x1);
        if (edge && e < e_min) p0 = 0.f;
        if (edge && e + 1 < e_min) p1 = 0.f;
        tc::fma2(pd0, pd1, sd[e], sd[e + 1], scale, scale, nc[0], nc[1]);
        tc::mul2(pd0, pd1, p0, p1, pd0, pd1);                       // Pd^T
        tc::add2(g0, g1, dp[e], dp[e + 1], nz[0], nz[1]);           // dP - z
        tc::add2(h0, h1, dpd[e], dpd[e + 1], nzd[0], nzd[1]);       // dPd - zdot
        tc::mul2(sd[e], sd[e + 1], p0, p1, g0, g1);                 // dS^T
        tc::mul2(h0, h1, p0, p1, h0, h1);
        tc::fma2(dp[e], dp[e + 1], pd0, pd1, g0, g1, h0, h1);       // dSd^T
        sv[e] = pd0;
        sv[e + 1] = pd1;
      }
      // every tile written below was last read by tile t-1's MMAs
      if (t >= 1 && !wait(mma2_done + ((t - 1) & 1), ((t - 1) >> 1) & 1)) { ok = false; break; }
      const uint32_t bpd = a_pd, bds = a_ds + b * C::kP, bdsd = a_dsd + b * C::kP;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t off = tc::sw128_off(r, grp * 4 + h);
        const float* x = sv + h * 8;
        const float* y = sd + h * 8;
        const float* zz = dp + h * 8;
        tc::st_shared_v4(bpd + off, tc::pack2<T>(x[0], x[1]), tc::pack2<T>(x[2], x[3]),
                         tc::pack2<T>(x[4], x[5]), tc::pack2<T>(x[6], x[7]));
        tc::st_shared_v4(bds + off, tc::pack2<T>(y[0], y[1]), tc::pack2<T>(y[2], y[3]),
                         tc::pack2<T>(y[4], y[5]), tc::pack2<T>(y[6], y[7]));
        tc::st_shared_v4(bdsd + off, tc::pack2<T>(zz[0], zz[1]), tc::pack2<T>(zz[2], zz[3]),
                         tc::pack2<T>(zz[4], zz[5]), tc::pack2<T>(zz[6], zz[7]));
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full);
    }
    // ------------------------------------------------------------ hK, hV
    if (ok && n_iter > 0) {
      const int tl = n_iter - 1;
      ok = wait(mma2_done + (tl & 1), (tl >> 1) & 1);
      if (ok) tc::tc_fence_after();
    }
    if (ok && n_split > 1) {
      // partial sums of this chunk of queries, added in fp32 (the TMEM loads
      // are warp-collective: every lane loads, lanes past M skip the add)
      if (n_iter > 0) {
        const bool store = key < M;
        const size_t base = ((size_t)bh * M + (store ? key : 0)) * HD;
        const size_t plane = (size_t)(CAUSAL ? gridDim.x : gridDim.y) * M * HD;  // B*H*M*D
#pragma unroll 1
        for (int which = 0; which < 2; ++which) {
          if ((which == 0 ? (void*)hv : (void*)hk) == nullptr) continue;
          const float mul = which == 0 ? 1.f : scale;
          const uint32_t col = which == 0 ? t_hv : t_hk;
          float* acc = hkv_acc + which * plane + base;
#pragma unroll 1
          for (int c = grp * (HD / 64); c < (grp + 1) * (HD / 64); ++c) {
            float v[32];
            tc::tmem_ld32(col + lane_off + c * 32, v);
            if (!store) continue;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              tcbwd::red_add_v4(acc + c * 32 + 4 * i, v[4 * i] * mul, v[4 * i + 1] * mul,
                                v[4 * i + 2] * mul, v[4 * i + 3] * mul);
          }
        }
      }
    } else if (ok) {
      const bool store = key < M;
      const size_t base = ((size_t)bh * M + (store ? key : 0)) * HD;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        T* out = which == 0 ? hv : hk;
        if (out == nullptr) continue;
        const float mul = which == 0 ? 1.f : scale;
        const uint32_t col = which == 0 ? t_hv : t_hk;
#pragma unroll 1
        for (int c = grp * (HD / 64); c < (grp + 1) * (HD / 64); ++c) {
          float v[32];
          if (n_iter > 0) {
            tc::tmem_ld32(col + lane_off + c * 32, v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
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
    // ------------------------------------------------------------ hQ flush
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RegSplit<HD>::flush));
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const size_t row_base = (size_t)bh * Tq;
    const bool bulk_issuer = warp == kFirstCompute + NCOMPUTE / 32 && lane == 0;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, abort));
    };
    for (int t = 0; t < n_iter; ++t) {
      if (kPair && !(t & 1) && t != n_iter - 1) continue;
      if (!wait(mma2_done + (t & 1), (t >> 1) & 1)) break;
      tc::tc_fence_after();
      if constexpr (!kPair) {
        // hQ^T of tile t sits in the S^T columns, which the next tile's
        // S-group waits for: read it out, release the columns, then add it.
        const int qb = (i_begin + t) * BQ;
        float v0[32], v1[32];
        tc::tmem_ld32(tmem + lane_off, v0);
        tc::tmem_ld32(tmem + lane_off + 32, v1);
        tc::tc_fence_before();
        tc::mbar_arrive(hq_free);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int q = qb + e;
          if (q < Tq) atomicAdd(hq_acc + (row_base + q) * HD + r, v0[e] * scale);
          if (q + 32 < Tq) atomicAdd(hq_acc + (row_base + q + 32) * HD + r, v1[e] * scale);
        }
        continue;
      } else {
        // hQ of the pair ending at tile t (lane = query row, 64 head dims):
        // read out of TMEM, release the buffer, stage it scaled in two
        // 128-byte-swizzled halves and add the pair's rows to hQacc with two
        // bulk tensor reductions (rows past the end are clipped).
        const int qb = (i_begin + (t & ~1)) * BQ;
        float v0[32], v1[32];
        tc::tmem_ld32(t_hqp + lane_off, v0);
        tc::tmem_ld32(t_hqp + lane_off + 32, v1);
        tc::tc_fence_before();
        tc::mbar_arrive(hq_free);
        const int pi = t >> 1;  // pair index: phase of the staging barriers
        if (bulk_issuer) {
          tc::bulk_wait_read_all();
          tc::mbar_arrive(stage_free);
        }
        if (!wait(stage_free, pi & 1)) break;
        const uint32_t srow = tc::smem_u32(smem + C::oStage) + (uint32_t)r * 128;
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
            tc::bulk_tensor_reduce_add_3d(&tm_hq, smem + C::oStage, 0, qb, bh);
            tc::bulk_tensor_reduce_add_3d(&tm_hq, smem + C::oStage + 16384, 32, qb, bh);
          }
        }
        if (!__shfl_sync(0xffffffffu, staged, 0)) break;
        continue;
      }
      tc::tc_fence_before();
      tc::mbar_arrive(hq_free);
    }
    // the last reductions must finish before the CTA (and its stage) goes away
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

}  // namespace tchvp
}  // namespace theria
