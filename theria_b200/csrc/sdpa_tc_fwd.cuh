// Tensor-core (tcgen05) SDPA forward for bf16/fp16 with head dim 64 or 128.
//
// One CTA owns TWO 128-row query tiles of one (batch, head) and streams the
// keys in tiles of 128 through a 2-stage K/V ring.  Warp roles:
//   warp 0       TMA producer: both Q tiles once, then K and V tiles
//   warp 1       MMA issuer (one thread) and TMEM owner
//   warps 4..7   softmax + epilogue of query tile 0 (one row per thread)
//   warps 8..11  softmax + epilogue of query tile 1
// TMEM (512 columns): S_t at [128t, 128t+128) and O_t at [256 + t*D, ...);
// for D = 64 also P_t at [384 + 64t, 448 + 64t) (see below).
// The tensor core alternates between the tiles (S_0, S_1, PV_0, PV_1, ...)
// so that one tile's softmax runs while the other tile's MMAs do.
// Softmax reads a thread's whole row of S with one TMEM load (128 registers),
// takes the row max and the exponentials from registers, and writes P as
// packed 16-bit pairs over the
// first 64 columns of its own S; the PV MMA then takes P straight from TMEM
// as its A operand (no shared-memory round trip).  In-order completion of
// one thread's tcgen05 operations makes this safe: S_t(j+1) is issued after
// PV_t(j), and the softmax waits for S_t(j+1) before touching S_t again,
// which also guarantees PV_t(j) has finished with P and with O_t.
// D = 64 (O_t is 64 columns, so TMEM has room): P_t has columns of its own,
// warp 1 issues S_t(j+1) as soon as the softmax warps have loaded S_t(j)
// and warp 2 issues the PV products; the softmax waits for PV_t(j) only
// before it overwrites P_t (or rescales O_t), so the tile's softmax steps
// follow each other without the PV and S products in between.
// Softmax runs in the log2 domain with a lazily updated row maximum (O and
// l rescaled only when the maximum grows by more than 8).  The epilogue
// writes O (input dtype or fp32) and LSE = ln(2) * (m + log2 l).
#pragma once

#include "tc_common.cuh"

namespace theria {
namespace tcfwd {

constexpr int BM = 128;      // rows per query tile
constexpr int NQT = 2;       // query tiles per CTA
constexpr int BN = 128;      // keys per tile
constexpr int STAGES = 2;    // K/V ring depth
// Warps per CTA.  D = 128: 2 control warps (TMA, MMA) and 16 softmax warps,
// two per TMEM lane quarter and query tile, each on one 64-column half of
// the S rows; at 5 warps per SM sub-partition that leaves 96 registers per
// thread, so a half reads its S columns from TMEM twice (once for the row
// maximum, once in 32-column chunks for the exponentials).  D = 64: 3
// control warps (TMA, S issuer, PV issuer) and 8 softmax warps, one per row,
// holding the whole row in registers (168 per thread).
template <int HD>
struct Cfg {
  static constexpr int kHalves = HD == 64 ? 1 : 2;
  static constexpr int kCtl = HD == 64 ? 3 : 2;
  static constexpr int kThreads = 32 * (kCtl + 8 * kHalves);
};
constexpr float kRescaleThreshold = 8.f;  // log2 units

template <int HD>
struct Smem {
  static constexpr int kQ = BM * HD * 2;  // one query tile
  static constexpr int kKV = BN * HD * 2;
  static constexpr int oQ = 0;
  static constexpr int oK = oQ + NQT * kQ;
  static constexpr int oV = oK + STAGES * kKV;
  static constexpr int oRed = oV + STAGES * kKV;  // softmax row-term exchange, 4 KB
  static constexpr int oBar = oRed + 2 * 2 * 2 * BM * 4;
  // q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[2],
  // p_full[2], o_done[2], drain, (D = 64) s_read[2], pv_done[2], drain2
  static constexpr int nBar = 1 + 4 * STAGES + 6 + 1 + 5;
  static constexpr int oTmem = oBar + nBar * 8;
  static constexpr int oAbort = oTmem + 4;
  static constexpr int kBytes = oAbort + 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024
};

template <typename T, int HD, bool CAUSAL>
__global__ void __launch_bounds__(Cfg<HD>::kThreads, 1)
fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
           const __grid_constant__ CUtensorMap tm_v, void* __restrict__ out, int out_f32,
           float* __restrict__ lse, int Tq, int M, float scale_log2) {
  using L = Smem<HD>;
  // D = 64: O_t takes 64 TMEM columns, so P_t gets columns of its own
  // instead of overwriting S_t.  S_t(j+1) is then issued as soon as the
  // softmax warps have loaded S_t(j), and runs while they form P_t(j): the
  // softmax of a tile no longer waits for PV_t(j) and S_t(j+1) in between.
  // S products and PV products come from two issuing threads (warps 1, 2).
  constexpr bool kSepP = (HD == 64);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  // K and V stages are released separately: K_j once both S_t(j) are done
  // (a step before V_j, which PV_t(j) reads), so the next K load starts early.
  uint64_t* k_empty = v_full + STAGES;
  uint64_t* v_empty = k_empty + STAGES;
  uint64_t* s_full = v_empty + STAGES;  // [2] per query tile
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* o_done = p_full + 2;         // [2]
  uint64_t* drain = o_done + 2;
  uint64_t* s_read = drain + 1;   // [2] D = 64: S_t loaded by the softmax warps (one per warp)
  uint64_t* pv_done = s_read + 2; // [2] D = 64: PV_t(j) complete (P_t and O_t free)
  uint64_t* drain2 = pv_done + 2;  // D = 64: the PV issuer's last MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::oAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Causal grids put the head index in x so the heaviest tiles of every head
  // are dispatched first (longest-first over the whole grid).
  const int bh = CAUSAL ? blockIdx.x : blockIdx.y;
  const int cta = CAUSAL ? (gridDim.y - 1 - blockIdx.y) : blockIdx.x;
  const int q0 = cta * (NQT * BM);
  int n_tiles = (M + BN - 1) / BN;
  if (CAUSAL) n_tiles = min(n_tiles, (q0 + NQT * BM - 1) / BN + 1);
  // Key tiles query tile t needs: causal, the first tile stops one key
  // tile before the second (that tile would be masked out entirely).
  auto tiles_of = [&](int t) {
    return CAUSAL ? min(n_tiles, (q0 + t * BM + BM - 1) / BN + 1) : n_tiles;
  };

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(k_full + s, 1);
      tc::mbar_init(v_full + s, 1);
      tc::mbar_init(k_empty + s, 1);
      tc::mbar_init(v_empty + s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      tc::mbar_init(s_full + t, 1);
      tc::mbar_init(p_full + t, 128 * Cfg<HD>::kHalves);
      tc::mbar_init(o_done + t, 1);
    }
    tc::mbar_init(drain, 1);
    for (int t = 0; t < 2; ++t) {
      tc::mbar_init(s_read + t, 4 * Cfg<HD>::kHalves);
      tc::mbar_init(pv_done + t, 1);
    }
    tc::mbar_init(drain2, 1);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tc::prefetch_tmap(&tm_q);
      tc::prefetch_tmap(&tm_k);
      tc::prefetch_tmap(&tm_v);
      int issued = 0;
      tc::mbar_expect_tx(q_full, NQT * L::kQ);
      for (int t = 0; t < NQT; ++t)
        for (int cb = 0; cb < HD / 64; ++cb)
          tc::tma_load_3d(smem + L::oQ + t * L::kQ + cb * BM * 128, &tm_q, q_full, cb * 64,
                          q0 + t * BM, bh);
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES && !tc::mbar_wait(k_empty + st, ((j / STAGES) - 1) & 1, abort)) break;
        tc::mbar_expect_tx(k_full + st, L::kKV);
        for (int cb = 0; cb < HD / 64; ++cb)
          tc::tma_load_3d(smem + L::oK + st * L::kKV + cb * BN * 128, &tm_k, k_full + st,
                          cb * 64, j * BN, bh);
        if (j >= STAGES && !tc::mbar_wait(v_empty + st, ((j / STAGES) - 1) & 1, abort)) {
          issued = j;  // K_j was issued; the drain below waits for it separately
          tc::mbar_wait_drain(k_full + st, (j / STAGES) & 1);
          break;
        }
        tc::mbar_expect_tx(v_full + st, L::kKV);
        for (int cb = 0; cb < HD / 64; ++cb)
          tc::tma_load_3d(smem + L::oV + st * L::kKV + cb * BN * 128, &tm_v, v_full + st,
                          cb * 64, j * BN, bh);
        issued = j + 1;
      }
      // Every copy issued into this CTA's shared memory lands before it may
      // exit (bounded; returns at once on the normal path).
      tc::mbar_wait_drain(q_full, 0);
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j) {
        tc::mbar_wait_drain(k_full + j % STAGES, (j / STAGES) & 1);
        tc::mbar_wait_drain(v_full + j % STAGES, (j / STAGES) & 1);
      }
    }
  } else if (kSepP && (warp == 1 || warp == 2)) {
    // ------------------------------------------------------------ MMA issuers (D = 64)
    // Warp 1 issues S_t(j) = Q_t K_j^T once the softmax warps have loaded
    // S_t(j-1); warp 2 issues O_t += P_t(j) V_j from P_t's own columns.
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_f16(BM, BN, tc::AbFmt<T>::v, 0, 0);
      constexpr uint32_t id_pv = tc::idesc_f16(BM, HD, tc::AbFmt<T>::v, 0, 1);
      if (warp == 1) {
        const uint64_t dq0 = tc::sw128_desc(tc::smem_u32(smem + L::oQ), 16, 1024);
        const uint64_t dk0 = tc::sw128_desc(tc::smem_u32(smem + L::oK), 16, 1024);
        bool ok = tc::mbar_wait(q_full, 0, abort);
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int st = j % STAGES;
          if (!tc::mbar_wait(k_full + st, (j / STAGES) & 1, abort)) break;
          const uint64_t dk = tc::desc_at(dk0, st * L::kKV);
          for (int t = 0; t < NQT; ++t) {
            if (j >= tiles_of(t)) continue;
            if (j >= 1 && !tc::mbar_wait(s_read + t, (j - 1) & 1, abort)) { ok = false; break; }
            tc::tc_fence_after();
            const uint64_t dq = tc::desc_at(dq0, t * L::kQ);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
              tc::mma_ss(tmem + t * 128, tc::desc_at(dq, kk * 32), tc::desc_at(dk, kk * 32),
                         id_s, kk > 0 ? 1u : 0u);
            tc::mma_commit(s_full + t);
          }
          if (!ok) break;
          tc::mma_commit(k_empty + st);
        }
        tc::mma_commit(drain);
        tc::mbar_wait_drain(drain, 0);
      } else {
        const uint64_t dv0 = tc::sw128_desc(tc::smem_u32(smem + L::oV), BN * 128, 1024);
        bool ok = true;
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int st = j % STAGES;
          if (!tc::mbar_wait(v_full + st, (j / STAGES) & 1, abort)) break;
          const uint64_t dv = tc::desc_at(dv0, st * L::kKV);
          for (int t = 0; t < NQT; ++t) {
            const int nt = tiles_of(t);
            if (j >= nt) continue;
            if (!tc::mbar_wait(p_full + t, j & 1, abort)) { ok = false; break; }
            tc::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              tc::mma_ts(tmem + 256 + t * HD, tmem + 384 + t * 64 + kk * 8,
                         tc::desc_at(dv, kk * 2048), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
            tc::mma_commit(pv_done + t);
            if (j + 1 == nt) tc::mma_commit(o_done + t);
          }
          if (!ok) break;
          tc::mma_commit(v_empty + st);
        }
        tc::mma_commit(drain2);
        tc::mbar_wait_drain(drain2, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_f16(BM, BN, tc::AbFmt<T>::v, 0, 0);
      constexpr uint32_t id_pv = tc::idesc_f16(BM, HD, tc::AbFmt<T>::v, 0, 1);
      // base descriptors, advanced per instruction by constant adds
      const uint64_t dq0 = tc::sw128_desc(tc::smem_u32(smem + L::oQ), 16, 1024);
      const uint64_t dk0 = tc::sw128_desc(tc::smem_u32(smem + L::oK), 16, 1024);
      const uint64_t dv0 = tc::sw128_desc(tc::smem_u32(smem + L::oV), BN * 128, 1024);
      // S_t(j) = Q_t K_j^T into TMEM columns [128t, 128t+128)
      auto issue_s = [&](int t, int j) {
        const uint64_t dq = tc::desc_at(dq0, t * L::kQ);
        const uint64_t dk = tc::desc_at(dk0, (j % STAGES) * L::kKV);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          tc::mma_ss(tmem + t * 128, tc::desc_at(dq, (kk / 4) * (BM * 128) + (kk % 4) * 32),
                     tc::desc_at(dk, (kk / 4) * (BN * 128) + (kk % 4) * 32), id_s,
                     kk > 0 ? 1u : 0u);
        tc::mma_commit(s_full + t);
        if (t == NQT - 1) tc::mma_commit(k_empty + j % STAGES);
      };
      bool ok = tc::mbar_wait(q_full, 0, abort) && tc::mbar_wait(k_full, 0, abort);
      if (ok) {
        tc::tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j % STAGES;
        const bool more = j + 1 < n_tiles;
        const uint64_t dv = tc::desc_at(dv0, st * L::kKV);
        // The operand waits of this step come first: they are normally long
        // satisfied, but each wait still costs the issuing thread a few
        // hundred cycles, which must not sit between a softmax publishing
        // P and the MMAs that consume it.
        if (!tc::mbar_wait(v_full + st, (j / STAGES) & 1, abort)) break;
        if (more && !tc::mbar_wait(k_full + (j + 1) % STAGES, ((j + 1) / STAGES) & 1, abort))
          break;
        for (int t = 0; t < NQT; ++t) {
          const int nt = tiles_of(t);
          if (j < nt) {
            if (!tc::mbar_wait(p_full + t, j & 1, abort)) { ok = false; break; }
            tc::tc_fence_after();
            // O_t += P_t V_j, P_t read from TMEM (packed pairs, 8 columns per
            // 16 keys; keys 64.. start at the second half's S columns)
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              tc::mma_ts(tmem + 256 + t * HD, tmem + t * 128 + (kk / 4) * 64 + (kk % 4) * 8,
                         tc::desc_at(dv, kk * 2048), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
            if (j + 1 == nt) tc::mma_commit(o_done + t);
          }
          if (t == NQT - 1) tc::mma_commit(v_empty + st);
          if (j + 1 < nt) issue_s(t, j + 1);
        }
      }
      // Every MMA issued above completes before TMEM is freed.
      tc::mma_commit(drain);
      tc::mbar_wait_drain(drain, 0);
    }
  } else if (warp >= Cfg<HD>::kCtl) {
    // ------------------------------------------------------------ softmax
    // kHalves warps per TMEM lane quarter and query tile; with two, half h
    // takes key columns [64h, 64h + 64) of every S tile and the halves
    // combine their row maxima (and at the end their row sums) through
    // shared memory under a named barrier of the two warps.
    constexpr int kHalves = Cfg<HD>::kHalves;
    constexpr int CW = BN / kHalves;      // S columns per warp
    const int idx = warp - Cfg<HD>::kCtl;
    const int t = idx / (4 * kHalves);    // query tile of this warp
    const int h = kHalves == 2 ? (idx >> 2) & 1 : 0;  // column half
    const int quarter = warp & 3;         // TMEM lanes this warp may access
    const int r = quarter * 32 + lane;    // row within the tile
    const int row = q0 + t * BM + r;
    const uint32_t bar_id = 1 + t * 4 + quarter;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t t_s = tmem + t * 128 + h * CW + lane_off;
    constexpr int HO = HD / kHalves;      // O columns this warp rescales and stores
    const uint32_t t_o = tmem + 256 + t * HD + h * HO + lane_off;
    // P_t (packed 16-bit pairs): D = 64 in its own columns [384 + 64t, +64);
    // D = 128 over the first 32 of the half's own S columns, [128t + 64h, +32),
    // which the half has read by then.
    const uint32_t t_p = (kSepP ? tmem + 384 + t * 64 : tmem + t * 128 + h * 64) + lane_off;
    float* red = reinterpret_cast<float*>(smem + L::oRed);  // [2 parity][2 t][2 h][128]
    auto red_at = [&](int par, int hh) { return red + ((par * 2 + t) * 2 + hh) * BM + r; };
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // Waits are warp-uniform: the TMEM accesses that follow are warp-collective.
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, abort));
    };
    const int nt = tiles_of(t);
    for (int j = 0; j < nt; ++j) {
      if (!wait(s_full + t, j & 1)) { ok = false; break; }
      tc::tc_fence_after();
      const int col0 = j * BN + h * CW;
      // Tiles that need masking (the causal diagonal, the ragged last key
      // tile) take a separate, slower path; the test is uniform per warp.
      const bool edge = (col0 + CW > M) || (CAUSAL && col0 + CW - 1 > q0 + t * BM);
      const int lim = CAUSAL ? min(M, row + 1) - col0 : M - col0;  // valid columns < lim
      // The maximum uses 8 independent partial maxima so the reduction is
      // not one long dependent chain.
      float v[CW];
      if constexpr (CW == 128) tc::tmem_ld128(t_s, v);
      else tc::tmem_ld64(t_s, v);  // for the row maximum only
      if constexpr (kSepP) {
        // S_t is in registers: the next S_t may be written
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(s_read + t);
      }
      float mp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mp[i] = -INFINITY;
      if (!edge) {
#pragma unroll
        for (int i = 0; i < CW; i += 2) mp[(i >> 1) & 7] = tc::max3(mp[(i >> 1) & 7], v[i], v[i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < CW; ++i) mp[i & 7] = fmaxf(mp[i & 7], i < lim ? v[i] : -INFINITY);
      }
      float mt = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                       fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      if constexpr (kHalves == 2) {
        *red_at(j & 1, h) = mt;
        tc::named_bar(bar_id, 64);
        mt = fmaxf(mt, *red_at(j & 1, h ^ 1));
      }
      mt *= scale_log2;
      const float m_new = fmaxf(m, mt);
      float m_use = m;
      bool rescale = false;
      if (m == -INFINITY) {
        m_use = m_new;
      } else if (m_new - m > kRescaleThreshold) {
        m_use = m_new;
        rescale = true;
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // O_t holds PV_t(0..j-1), all complete: D = 128, S_t(j) was issued
        // after them; D = 64, the wait below.
        if (kSepP && j >= 1) {
          if (!wait(pv_done + t, (j - 1) & 1)) { ok = false; break; }
          tc::tc_fence_after();
        }
        const float alpha = rescale ? tc::ex2(m - m_use) : 1.f;
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < HO / 32; ++c) {
          float o[32];
          tc::tmem_ld32(t_o + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tc::tmem_st32(t_o + c * 32, o);
        }
      }
      m = m_use;
      const float m_sub = (m_use == -INFINITY) ? 0.f : m_use;
      float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // partial row sums
      if constexpr (kHalves == 1) {
        // P = exp2(s - m) from the registers: exponentials, row sums and
        // 16-bit packing in one pass (each pair of S values dies as it is
        // packed), then one wide TMEM store once PV_t(j-1) has read P_t
        uint32_t pk[CW / 2];
        if (!edge) {
#pragma unroll
          for (int i = 0; i < CW; i += 2) {
            float x0, x1;
            tc::fma2(x0, x1, v[i], v[i + 1], scale_log2, scale_log2, -m_sub, -m_sub);
            x0 = tc::ex2(x0);
            x1 = tc::ex2(x1);
            const int k = 2 * ((i >> 1) & 3);  // four chains of paired partial sums
            tc::add2(rs[k], rs[k + 1], rs[k], rs[k + 1], x0, x1);
            pk[i / 2] = tc::pack2<T>(x0, x1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < CW; i += 2) {
            const float x0 = i < lim ? tc::ex2(fmaf(v[i], scale_log2, -m_sub)) : 0.f;
            const float x1 = i + 1 < lim ? tc::ex2(fmaf(v[i + 1], scale_log2, -m_sub)) : 0.f;
            const int k = 2 * ((i >> 1) & 3);
            tc::add2(rs[k], rs[k + 1], rs[k], rs[k + 1], x0, x1);
            pk[i / 2] = tc::pack2<T>(x0, x1);
          }
        }
        if (kSepP && j >= 1) {
          if (!wait(pv_done + t, (j - 1) & 1)) { ok = false; break; }
          tc::tc_fence_after();
        }
        tc::tmem_st64u(t_p, pk);
      } else {
        // P = exp2(s - m): S re-read from TMEM in two 32-column chunks;
        // exponentials, row sums and 16-bit packing in one pass per chunk
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float x[32];
          tc::tmem_ld32(t_s + c * 32, x);
          uint32_t pk[16];
          if (!edge) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float x0, x1;
              tc::fma2(x0, x1, x[i], x[i + 1], scale_log2, scale_log2, -m_sub, -m_sub);
              x0 = tc::ex2(x0);
              x1 = tc::ex2(x1);
              const int k = 2 * ((i >> 1) & 3);
              tc::add2(rs[k], rs[k + 1], rs[k], rs[k + 1], x0, x1);
              pk[i / 2] = tc::pack2<T>(x0, x1);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const int cc = c * 32 + i;
              const float x0 = cc < lim ? tc::ex2(fmaf(x[i], scale_log2, -m_sub)) : 0.f;
              const float x1 = cc + 1 < lim ? tc::ex2(fmaf(x[i + 1], scale_log2, -m_sub)) : 0.f;
              const int k = 2 * ((i >> 1) & 3);
              tc::add2(rs[k], rs[k + 1], rs[k], rs[k + 1], x0, x1);
              pk[i / 2] = tc::pack2<T>(x0, x1);
            }
          }
          // packed P of these 32 keys: 16 columns over S columns this half
          // has already read
          tc::tmem_st16(t_p + c * 16, pk);
        }
      }
      l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full + t);
    }
    // ------------------------------------------------------------ epilogue
    if constexpr (kHalves == 2) {
      // Both halves reach this barrier once (same trip count; a timed-out
      // wait makes every later wait of the CTA give up, so both leave the
      // loop), and combine their row sums here.
      *red_at(nt & 1, h) = l;
      tc::named_bar(bar_id, 64);
      l += *red_at(nt & 1, h ^ 1);
    }
    if (ok && wait(o_done + t, 0)) {
      tc::tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool store = row < Tq;
      const size_t base = ((size_t)bh * Tq + (size_t)(store ? row : 0)) * HD + h * HO;
#pragma unroll
      for (int c = 0; c < HO / 32; ++c) {
        float v[32];
        tc::tmem_ld32(t_o + c * 32, v);  // warp-collective: before any branch
        if (!store) continue;
        if (out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + base + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv,
                                 v[4 * i + 3] * inv);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(out) + base + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float* e = v + 8 * i;
            dst[i] = make_uint4(tc::pack2<T>(e[0] * inv, e[1] * inv),
                                tc::pack2<T>(e[2] * inv, e[3] * inv),
                                tc::pack2<T>(e[4] * inv, e[5] * inv),
                                tc::pack2<T>(e[6] * inv, e[7] * inv));
          }
        }
      }
      if (store && h == 0 && lse != nullptr)
        lse[(size_t)bh * Tq + row] =
            l > 0.f ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
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

}  // namespace tcfwd
}  // namespace theria
