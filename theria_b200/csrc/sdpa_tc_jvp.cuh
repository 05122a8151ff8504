// Tensor-core (tcgen05) frozen-stats JVP for bf16/fp16, head dim 64 or 128,
// and the first pass of the HVP (same kernel with W).
//
// One CTA owns 128 query rows of one (batch, head); P is rebuilt exactly
// from the forward's LSE, so there is no online rescaling.  Per key tile j:
//   S   = Q K^T                       (tcgen05 -> TMEM)
//   Sd' = tQ K^T + Q tK^T             (tcgen05 -> TMEM, one accumulator)
//   P   = exp(s S - LSE),  U = P * (s Sd')         (CUDA cores, 16-bit tiles)
//   OA += U V,   [OP | OT] += P [V | tV]           (tcgen05; V and tV sit
//                                                   side by side in smem, so
//                                                   one N = 2D MMA covers both)
//   c  += rowsum(U)
// and at the end Odot = OA - c OP + OT.  With W (HVP pass 1) the kernel also
// stores the row terms c, z = rowsum(W OP), zdot = rowsum(W Odot).
// Key tile BN = 128 for D = 64 and 64 for D = 128, so that
// TMEM = S (BN) + Sd (BN) + OA (D) + [OP|OT] (2D) fits in 512 columns.
// Warp roles: 0 TMA for Q/tQ and the K/tK ring (2 stages), 1 issues the S
// and Sd' products and owns TMEM, 2 issues the PV products, 3 TMA for V/tV,
// 4..11 compute (two groups splitting each tile's key columns, four TMEM
// lane quarters each).  With S and PV on separate issuing threads, S(j+1)
// runs on the tensor core while the CUDA cores still work on tile j.
#pragma once

#include "tc_common.cuh"

namespace theria {
namespace tcjvp {

constexpr int BM = 128;
constexpr int NCOMPUTE = 256;
constexpr int NTHREADS = 128 + NCOMPUTE;
constexpr int kFirstCompute = 4;
constexpr int KST = 2;  // K/tK ring depth

template <int HD>
struct Cfg {
  static constexpr int BN = HD == 128 ? 64 : 128;
  static constexpr int kQ = BM * HD * 2;
  static constexpr int kKV = BN * HD * 2;
  static constexpr int kP = BM * BN * 2;
  static constexpr int oQ = 0;
  static constexpr int oTQ = oQ + kQ;
  static constexpr int oK = oTQ + kQ;         // stage s: K at oK + 2s*kKV, tK after it
  static constexpr int oTK = oK + kKV;
  static constexpr int oV = oK + KST * 2 * kKV;
  static constexpr int oTV = oV + kKV;  // directly after V: [V | tV] is one B operand
  static constexpr int oP = oTV + kKV;
  static constexpr int oU = oP + kP;
  static constexpr int oStat = oU + kP;  // 3 x 128 floats: c, z, zdot partial sums
  static constexpr int oBar = oStat + 3 * BM * 4;
  // q_full, kt_full, kt_empty, vt_full, vt_empty, s_full, s_free, p_full,
  // pv_done, c_ready, w_ready, drain, kt_full[1], kt_empty[1], drain[1]
  static constexpr int nBar = 15;
  static constexpr int oTmem = oBar + nBar * 8;
  static constexpr int oAbort = oTmem + 4;
  static constexpr int kAlloc = oAbort + 4 + 1024;
  // TMEM columns
  static constexpr int tS = 0, tSd = BN, tOA = 2 * BN, tOP = 2 * BN + HD, tOT = 2 * BN + 2 * HD;
};

template <typename T, int HD, bool CAUSAL, bool WITH_W>
__global__ void __launch_bounds__(NTHREADS, 1)
jvp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_tq,
           const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_tk,
           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_tv,
           const float* __restrict__ lse, const T* __restrict__ w, T* __restrict__ o_tan,
           float* __restrict__ stats, int64_t n_rows_total, int Tq, int M, float scale,
           float scale_log2) {
  using C = Cfg<HD>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::oBar);
  uint64_t *q_full = bars, *kt_full = bars + 1, *kt_empty = bars + 2, *vt_full = bars + 3,
           *vt_empty = bars + 4, *s_full = bars + 5, *s_free = bars + 6, *p_full = bars + 7,
           *pv_done = bars + 8, *c_ready = bars + 9, *w_ready = bars + 10, *drain = bars + 11;
  // second K/tK stage and the second issuer's drain
  auto kt_full_s = [&](int st) { return st == 0 ? kt_full : bars + 12; };
  auto kt_empty_s = [&](int st) { return st == 0 ? kt_empty : bars + 13; };
  uint64_t* drain_b = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::oTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + C::oAbort);
  float* stat_s = reinterpret_cast<float*>(smem + C::oStat);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Causal grids put the head index in x so the heaviest tiles of every head
  // are dispatched first (longest-first over the whole grid).
  const int bh = CAUSAL ? blockIdx.x : blockIdx.y;
  const int qt = CAUSAL ? (gridDim.y - 1 - blockIdx.y) : blockIdx.x;
  const int q0 = qt * BM;
  int n_tiles = (M + BN - 1) / BN;
  if (CAUSAL) n_tiles = min(n_tiles, (q0 + BM - 1) / BN + 1);

  if (threadIdx.x == 0) {
    for (int b = 0; b < C::nBar; ++b) {
      const bool many = (bars + b == s_free) || (bars + b == p_full) || (bars + b == c_ready) ||
                        (bars + b == w_ready);
      tc::mbar_init(bars + b, many ? NCOMPUTE : 1);
    }
    *abort = 0;
    tc::fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 3 * BM; i += blockDim.x) stat_s[i] = 0.f;
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer: Q/tQ, K/tK
    if (lane == 0) {
      tc::mbar_expect_tx(q_full, 2 * C::kQ);
      for (int cb = 0; cb < HD / 64; ++cb) {
        tc::tma_load_3d(smem + C::oQ + cb * BM * 128, &tm_q, q_full, cb * 64, q0, bh);
        tc::tma_load_3d(smem + C::oTQ + cb * BM * 128, &tm_tq, q_full, cb * 64, q0, bh);
      }
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % KST;
        if (j >= KST && !tc::mbar_wait(kt_empty_s(st), ((j / KST) - 1) & 1, abort)) break;
        uint8_t* base = smem + C::oK + st * 2 * C::kKV;
        tc::mbar_expect_tx(kt_full_s(st), 2 * C::kKV);
        for (int cb = 0; cb < HD / 64; ++cb) {
          tc::tma_load_3d(base + cb * BN * 128, &tm_k, kt_full_s(st), cb * 64, j * BN, bh);
          tc::tma_load_3d(base + C::kKV + cb * BN * 128, &tm_tk, kt_full_s(st), cb * 64, j * BN,
                          bh);
        }
        issued = j + 1;
      }
      tc::mbar_wait_drain(q_full, 0);
      for (int j = issued > KST ? issued - KST : 0; j < issued; ++j)
        tc::mbar_wait_drain(kt_full_s(j % KST), (j / KST) & 1);
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ producer: V/tV
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        if (j >= 1 && !tc::mbar_wait(vt_empty, (j - 1) & 1, abort)) break;
        tc::mbar_expect_tx(vt_full, 2 * C::kKV);
        for (int cb = 0; cb < HD / 64; ++cb) {
          tc::tma_load_3d(smem + C::oV + cb * BN * 128, &tm_v, vt_full, cb * 64, j * BN, bh);
          tc::tma_load_3d(smem + C::oTV + cb * BN * 128, &tm_tv, vt_full, cb * 64, j * BN, bh);
        }
        issued = j + 1;
      }
      if (issued > 0) tc::mbar_wait_drain(vt_full, (issued - 1) & 1);
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      constexpr int ab = tc::AbFmt<T>::v;
      constexpr uint32_t id_s = tc::idesc_f16(BM, BN, ab, 0, 0);
      constexpr uint32_t id_a = tc::idesc_f16(BM, HD, ab, 0, 1);
      constexpr uint32_t id_pt = tc::idesc_f16(BM, 2 * HD, ab, 0, 1);
      const uint32_t a_q = tc::smem_u32(smem + C::oQ), a_tq = tc::smem_u32(smem + C::oTQ);
      const uint32_t a_k = tc::smem_u32(smem + C::oK), a_tk = tc::smem_u32(smem + C::oTK);
      const uint32_t a_v = tc::smem_u32(smem + C::oV);
      const uint32_t a_p = tc::smem_u32(smem + C::oP), a_u = tc::smem_u32(smem + C::oU);
      // base descriptors, advanced by constant adds
      const uint64_t kQ = tc::sw128_desc(a_q, 16, 1024), kTQ = tc::sw128_desc(a_tq, 16, 1024);
      const uint64_t kK = tc::sw128_desc(a_k, 16, 1024), kTK = tc::sw128_desc(a_tk, 16, 1024);
      const uint64_t kP = tc::sw128_desc(a_p, 16, 1024), kU = tc::sw128_desc(a_u, 16, 1024);
      const uint64_t mV = tc::sw128_desc(a_v, BN * 128, 1024);
      bool ok = tc::mbar_wait(q_full, 0, abort);
      if (warp == 1) {
        // S = Q K^T and Sd' = tQ K^T + Q tK^T into the single S/Sd buffer,
        // free once the compute warps loaded the previous tile's.
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int st = j % KST;
          if (!tc::mbar_wait(kt_full_s(st), (j / KST) & 1, abort)) break;
          if (j >= 1 && !tc::mbar_wait(s_free, (j - 1) & 1, abort)) break;
          tc::tc_fence_after();
          const uint32_t so = st * 2 * C::kKV;  // K/tK stage offset
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t oq = (kk / 4) * (BM * 128) + (kk % 4) * 32;
            const uint32_t ok_ = so + (kk / 4) * (BN * 128) + (kk % 4) * 32;
            const uint32_t acc = kk > 0 ? 1u : 0u;
            tc::mma_ss(tmem + C::tS, tc::desc_at(kQ, oq), tc::desc_at(kK, ok_), id_s, acc);
            tc::mma_ss(tmem + C::tSd, tc::desc_at(kTQ, oq), tc::desc_at(kK, ok_), id_s, acc);
            tc::mma_ss(tmem + C::tSd, tc::desc_at(kQ, oq), tc::desc_at(kTK, ok_), id_s, 1u);
          }
          tc::mma_commit(s_full);
          tc::mma_commit(kt_empty_s(st));
        }
        tc::mma_commit(drain);
        tc::mbar_wait_drain(drain, 0);
      } else {
        // OA += U V and [OP | OT] += P [V | tV] (one N = 2D product)
        for (int j = 0; ok && j < n_tiles; ++j) {
          if (!tc::mbar_wait(vt_full, j & 1, abort)) break;  // operands before P
          if (!tc::mbar_wait(p_full, j & 1, abort)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint32_t oa = (kk / 4) * (BM * 128) + (kk % 4) * 32;
            const uint32_t ob = kk * 16 * 128;
            const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
            tc::mma_ss(tmem + C::tOA, tc::desc_at(kU, oa), tc::desc_at(mV, ob), id_a, acc);
            tc::mma_ss(tmem + C::tOP, tc::desc_at(kP, oa), tc::desc_at(mV, ob), id_pt, acc);
          }
          tc::mma_commit(pv_done);
          tc::mma_commit(vt_empty);
        }
        tc::mma_commit(drain_b);
        tc::mbar_wait_drain(drain_b, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ compute
    constexpr int HALF = BN / 2;  // key columns per group
    const int grp = (warp - kFirstCompute) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane = query row in tile
    const int row = q0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const bool row_ok = row < Tq;
    const float lse2 = row_ok ? lse[(size_t)bh * Tq + row] * 1.4426950408889634f : INFINITY;
    bool ok = true;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity, abort));
    };
    const uint32_t a_p = tc::smem_u32(smem + C::oP), a_u = tc::smem_u32(smem + C::oU);
    float c_pair[2] = {0.f, 0.f};
    for (int j = 0; j < n_tiles; ++j) {
      if (!wait(s_full, j & 1)) { ok = false; break; }
      tc::tc_fence_after();
      float sv[HALF], sd[HALF];
#pragma unroll
      for (int c = 0; c < HALF / 32; ++c) {
        float a[32], b[32];
        tc::tmem_ld32(tmem + C::tS + lane_off + grp * HALF + c * 32, a);
        tc::tmem_ld32(tmem + C::tSd + lane_off + grp * HALF + c * 32, b);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          sv[c * 32 + e] = a[e];
          sd[c * 32 + e] = b[e];
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(s_free);  // S / Sd columns may be overwritten by tile j+1
      const int col0 = j * BN + grp * HALF;
      // masking only where a tile crosses the causal diagonal or the last key
      const bool edge = (col0 + HALF > M) || (CAUSAL && col0 + HALF - 1 > q0);
      const int lim = (CAUSAL ? min(M, row + 1) : M) - col0;  // valid: e < lim
      // two columns at a time on paired fp32 instructions
#pragma unroll
      for (int e = 0; e < HALF; e += 2) {
        float x0, x1, a0, a1, u0, u1;
        tc::fma2(x0, x1, sv[e], sv[e + 1], scale_log2, scale_log2, -lse2, -lse2);
        float p0 = tc::ex2(x0), p1 = tc::ex2(x1);
        if (edge && e >= lim) p0 = 0.f;
        if (edge && e + 1 >= lim) p1 = 0.f;
        tc::mul2(a0, a1, sd[e], sd[e + 1], scale, scale);
        tc::mul2(a0, a1, p0, p1, a0, a1);
        // c is summed from U as rounded for the MMA, so that OA - c OP
        // cancels consistently (a row with one key gives Odot = tV exactly).
        tc::unpack2<T>(tc::pack2<T>(a0, a1), u0, u1);
        tc::add2(c_pair[0], c_pair[1], c_pair[0], c_pair[1], u0, u1);
        sv[e] = p0;
        sv[e + 1] = p1;
        sd[e] = u0;
        sd[e + 1] = u1;
      }
      // P / U tiles were read by tile j-1's MMAs.
      if (j >= 1 && !wait(pv_done, (j - 1) & 1)) { ok = false; break; }
#pragma unroll
      for (int h = 0; h < HALF / 8; ++h) {
        const int colt = grp * HALF + h * 8;  // column within the tile
        const uint32_t off = (uint32_t)(colt / 64) * (BM * 128) + tc::sw128_off(r, (colt % 64) / 8);
        const float* pe = sv + h * 8;
        const float* ue = sd + h * 8;
        tc::st_shared_v4(a_p + off, tc::pack2<T>(pe[0], pe[1]), tc::pack2<T>(pe[2], pe[3]),
                         tc::pack2<T>(pe[4], pe[5]), tc::pack2<T>(pe[6], pe[7]));
        tc::st_shared_v4(a_u + off, tc::pack2<T>(ue[0], ue[1]), tc::pack2<T>(ue[2], ue[3]),
                         tc::pack2<T>(ue[4], ue[5]), tc::pack2<T>(ue[6], ue[7]));
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full);
    }
    // ------------------------------------------------------------ epilogue
    // c = rowsum(P Sd) over both groups' columns.
    atomicAdd(stat_s + r, c_pair[0] + c_pair[1]);
    tc::mbar_arrive(c_ready);
    if (ok) ok = wait(c_ready, 0);
    if (ok) ok = wait(pv_done, (n_tiles - 1) & 1);
    if (ok) {
      tc::tc_fence_after();
      const float c = stat_s[r];
      const size_t base = ((size_t)bh * Tq + (size_t)(row_ok ? row : 0)) * HD;
      float zp = 0.f, zdp = 0.f;
#pragma unroll 1
      for (int cc = grp * (HD / 64); cc < (grp + 1) * (HD / 64); ++cc) {
        float oa[32], op[32], ot[32];
        tc::tmem_ld32(tmem + C::tOA + lane_off + cc * 32, oa);
        tc::tmem_ld32(tmem + C::tOP + lane_off + cc * 32, op);
        tc::tmem_ld32(tmem + C::tOT + lane_off + cc * 32, ot);
#pragma unroll
        for (int e = 0; e < 32; ++e) oa[e] = oa[e] - c * op[e] + ot[e];  // Odot
        if (!row_ok) continue;
        if (WITH_W) {
          const uint4* w4 = reinterpret_cast<const uint4*>(w + base + cc * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 pk = w4[i];
            const uint32_t wv[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const T* two = reinterpret_cast<const T*>(&wv[h]);
              const float w0 = to_f32<T>(two[0]), w1 = to_f32<T>(two[1]);
              const int e = i * 8 + h * 2;
              zp += w0 * op[e] + w1 * op[e + 1];
              zdp += w0 * oa[e] + w1 * oa[e + 1];
            }
          }
        }
        if (o_tan != nullptr) {
          uint4* d4 = reinterpret_cast<uint4*>(o_tan + base + cc * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float* e = oa + 8 * i;
            d4[i] = make_uint4(tc::pack2<T>(e[0], e[1]), tc::pack2<T>(e[2], e[3]),
                               tc::pack2<T>(e[4], e[5]), tc::pack2<T>(e[6], e[7]));
          }
        }
      }
      if (WITH_W) {
        atomicAdd(stat_s + BM + r, zp);
        atomicAdd(stat_s + 2 * BM + r, zdp);
        tc::mbar_arrive(w_ready);
        if (wait(w_ready, 0) && grp == 0 && row_ok) {
          const int64_t gr = (int64_t)bh * Tq + row;
          stats[gr] = c;
          stats[n_rows_total + gr] = stat_s[BM + r];
          stats[2 * n_rows_total + gr] = stat_s[2 * BM + r];
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

}  // namespace tcjvp
}  // namespace theria
