// libtheria_sm100.so: the C ABI declared in include/theria_sdpa.h.
//
// The whole library is one translation unit (no relocatable device code):
// this file includes the kernel headers and implements argument checking,
// workspace carving and kernel selection for each entry point.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <type_traits>
#include <initializer_list>
#include <mutex>

#include "common.cuh"
#include "sdpa_scores.cuh"
#include "sdpa_simt.cuh"
#include "sdpa_small.cuh"
#include "maml_ln.cuh"
#include "../../include/theria_ln.h"
#include "sdpa_tc_bwd.cuh"
#include "sdpa_tc_fwd.cuh"
#include "sdpa_tc_jvp.cuh"
#include "sdpa_tc_hvp.cuh"
#include "tc_host.cuh"

namespace theria {
namespace {

constexpr int64_t kAlign = 256;

int64_t align_up(int64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

bool valid_dtype(int dt) {
  return dt == THERIA_F32 || dt == THERIA_F16 || dt == THERIA_BF16 || dt == THERIA_F64;
}

// Shared argument checks; returns THERIA_OK or an error status.
int check_shape(int64_t B, int64_t H, int64_t T, int64_t M, int64_t D, int dtype) {
  if (B < 0 || H < 0 || T < 0 || M < 0 || D <= 0) return THERIA_ERR_INVALID_ARG;
  if (!valid_dtype(dtype)) return THERIA_ERR_INVALID_ARG;
  if (D > THERIA_MAX_HEAD_DIM) return THERIA_ERR_UNSUPPORTED;
  if (B * H > 65535) return THERIA_ERR_UNSUPPORTED;  // grid.y carries batch*head
  if (M == 0 && T > 0) return THERIA_ERR_INVALID_ARG; // softmax over no keys
  return THERIA_OK;
}

bool empty_problem(int64_t B, int64_t H, int64_t T) { return B == 0 || H == 0 || T == 0; }

template <typename K>
void set_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

size_t tile_floats(int64_t D) { return (size_t)simt::KT * (D + 1); }

dim3 row_grid(const Shape& s) {
  return dim3((unsigned)((s.T + simt::WARPS - 1) / simt::WARPS), (unsigned)(s.B * s.H));
}
dim3 col_grid(const Shape& s) {
  return dim3((unsigned)((s.M + simt::WARPS - 1) / simt::WARPS), (unsigned)(s.B * s.H));
}

// ------------------------------------------------------------- SIMT launches
template <typename T>
int simt_fwd(const void* q, const void* k, const void* v, void* o, int o_dtype, float* lse,
             const Shape& s, cudaStream_t st) {
  size_t sm = (2 * tile_floats(s.D) + simt::WARPS * s.D) * sizeof(float);
  auto kern = simt::fwd_row_kernel<T>;
  set_smem(kern, sm);
  kern<<<row_grid(s), simt::WARPS * 32, sm, st>>>((const T*)q, (const T*)k, (const T*)v, o,
                                                  o_dtype, lse, s);
  return launch_status();
}

template <typename T>
int simt_bwd(const void* q, const void* k, const void* v, const void* o, int o_dtype,
             const void* dout, const float* lse, void* dq, void* dk, void* dv, float* z,
             const Shape& s, cudaStream_t st) {
  const int64_t rows = s.B * s.H * s.T;
  if (o != nullptr) {
    simt::delta_from_o_kernel<T><<<(unsigned)((rows + simt::WARPS - 1) / simt::WARPS),
                                   simt::WARPS * 32, 0, st>>>(o, o_dtype, (const T*)dout, z,
                                                              rows, (int)s.D);
  } else {
    size_t sm = (2 * tile_floats(s.D) + simt::WARPS * 2 * s.D) * sizeof(float);
    auto kern = simt::delta_from_stats_kernel<T>;
    set_smem(kern, sm);
    kern<<<row_grid(s), simt::WARPS * 32, sm, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                    (const T*)dout, lse, z, s);
  }
  if (int e = launch_status()) return e;
  if (dq != nullptr) {
    size_t sm = (2 * tile_floats(s.D) + simt::WARPS * 2 * s.D) * sizeof(float);
    auto kern = simt::dq_row_kernel<T>;
    set_smem(kern, sm);
    kern<<<row_grid(s), simt::WARPS * 32, sm, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                    (const T*)dout, lse, z, (T*)dq, s);
    if (int e = launch_status()) return e;
  }
  if (dk != nullptr || dv != nullptr) {
    size_t sm = (2 * tile_floats(s.D) + 2 * simt::KT + simt::WARPS * 2 * s.D) * sizeof(float);
    auto kern = simt::dkdv_col_kernel<T>;
    set_smem(kern, sm);
    kern<<<col_grid(s), simt::WARPS * 32, sm, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                    (const T*)dout, lse, z, (T*)dk, (T*)dv, s);
    if (int e = launch_status()) return e;
  }
  return THERIA_OK;
}

template <typename T>
int simt_jvp(const void* q, const void* k, const void* v, const void* tq, const void* tk,
             const void* tv, const void* w, const float* lse, void* o_tan, float* stats,
             const Shape& s, cudaStream_t st) {
  size_t sm = (4 * tile_floats(s.D) + simt::WARPS * 3 * s.D) * sizeof(float);
  auto kern = simt::jvp_row_kernel<T>;
  set_smem(kern, sm);
  kern<<<row_grid(s), simt::WARPS * 32, sm, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)tq, (const T*)tk, (const T*)tv,
      (const T*)w, lse, (T*)o_tan, stats, s);
  return launch_status();
}

template <typename T>
int tc_jvp(const void* q, const void* k, const void* v, const void* tq, const void* tk,
           const void* tv, const void* w, const float* lse, void* o_tan, float* stats,
           const Shape& s, int dtype, cudaStream_t st);
bool use_tc(int dtype, const Shape& s, std::initializer_list<const void*> ptrs);

template <typename T> constexpr int dtype_of() {
  return std::is_same<T, float>::value ? THERIA_F32
         : std::is_same<T, __half>::value ? THERIA_F16 : THERIA_BF16;
}

template <typename T>
int simt_hvp(const void* q, const void* k, const void* v, const void* w, const float* lse,
             const void* tq, const void* tk, const void* tv, void* hq, void* hk, void* hv,
             void* o_tan, float* stats, const Shape& s, cudaStream_t st) {
  int e1 = -1;
  if constexpr (!std::is_same<T, float>::value) {
    if (use_tc(dtype_of<T>(), s, {q, k, v, tq, tk, tv, w, o_tan}))
      e1 = tc_jvp<T>(q, k, v, tq, tk, tv, w, lse, o_tan, stats, s, dtype_of<T>(), st);
  }
  if (e1 > 0) return e1;
  if (e1 < 0)
    if (int e = simt_jvp<T>(q, k, v, tq, tk, tv, w, lse, o_tan, stats, s, st)) return e;
  if (hq != nullptr) {
    size_t sm = (4 * tile_floats(s.D) + simt::WARPS * 3 * s.D) * sizeof(float);
    auto kern = simt::hq_row_kernel<T>;
    set_smem(kern, sm);
    kern<<<row_grid(s), simt::WARPS * 32, sm, st>>>(
        (const T*)q, (const T*)k, (const T*)v, (const T*)tq, (const T*)tk, (const T*)tv,
        (const T*)w, lse, stats, (T*)hq, s);
    if (int e = launch_status()) return e;
  }
  if (hk != nullptr || hv != nullptr) {
    size_t sm = (3 * tile_floats(s.D) + 4 * simt::KT + simt::WARPS * 4 * s.D) * sizeof(float);
    auto kern = simt::hkhv_col_kernel<T>;
    set_smem(kern, sm);
    kern<<<col_grid(s), simt::WARPS * 32, sm, st>>>(
        (const T*)q, (const T*)k, (const T*)v, (const T*)tq, (const T*)tk, (const T*)tv,
        (const T*)w, lse, stats, (T*)hk, (T*)hv, s);
    if (int e = launch_status()) return e;
  }
  return THERIA_OK;
}

// ------------------------------------------------------ whole-head launches
bool small_eligible(const Shape& s) {
  return s.T <= small::MAXN && s.M <= small::MAXN && s.D <= small::MAXD && s.B * s.H < (1ll << 31);
}

// fp64 runs only in the whole-head kernels, in double precision throughout,
// and only where the head (inputs and score-shaped matrices, as doubles)
// fits in one CTA's shared memory.
constexpr size_t kMaxSmem = 227 * 1024;
bool f64_fits(const Shape& s, int n_q, int n_k, int n_s) {
  return small_eligible(s) &&
         small::smem_bytes((int)s.T, (int)s.M, (int)s.D, n_q, n_k, n_s, sizeof(double)) <= kMaxSmem;
}
bool f64_fits_hvp(const Shape& s) {
  return small_eligible(s) &&
         small::hvp_smem_bytes((int)s.T, (int)s.M, (int)s.D, sizeof(double)) <= kMaxSmem;
}

// The full-MAML head shape (T = M = 64, head dim 16, fp32) runs kernels
// specialised at compile time; every other shape the generic ones.
template <typename T, typename A>
bool small_spec(const Shape& s) {
  return std::is_same<T, float>::value && std::is_same<A, float>::value && s.T == 64 &&
         s.M == 64 && s.D == 16;
}

// Strides of contiguous [B, H, rows, D] tensors.
small::Layout contiguous_layout(const Shape& s) {
  const int64_t q = s.T * s.D, k = s.M * s.D;
  return small::Layout{s.H * q, q, s.D, s.H * k, k, s.D, s.H * q, q, s.D};
}
// Packed self-attention: q, k, v (and their gradients) at offsets 0, H*D,
// 2*H*D of [B, T, 3, H, D]; O-shaped tensors [B, T, H, D].
small::Layout packed_layout(const Shape& s) {
  const int64_t hd = s.H * s.D;
  return small::Layout{3 * hd * s.T, s.D, 3 * hd, 3 * hd * s.T, s.D, 3 * hd,
                       hd * s.T, s.D, hd};
}

template <typename K>
void small_setup(K kern, size_t bytes) {
  if (bytes > 48 * 1024)
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <typename T, typename A = float>
int small_fwd(const void* q, const void* k, const void* v, void* o, int o_dtype, float* lse,
              const Shape& s, cudaStream_t st, const small::Layout* lyp = nullptr) {
  const small::Layout ly = lyp ? *lyp : contiguous_layout(s);
  const size_t sm = small::smem_bytes((int)s.T, (int)s.M, (int)s.D, 1, 2, 1, sizeof(A));
  const unsigned grid = (unsigned)(s.B * s.H);
  if (o_dtype == THERIA_F32) {
    auto kern = small::fwd_kernel<T, float, A>;
    if constexpr (std::is_same<T, float>::value && std::is_same<A, float>::value)
      if (small_spec<T, A>(s)) kern = small::fwd_kernel<T, float, A, 64, 16>;
    small_setup(kern, sm);
    kern<<<grid, small::NTHREADS, sm, st>>>((const T*)q, (const T*)k, (const T*)v, (float*)o,
                                            lse, s, ly);
  } else {
    auto kern = small::fwd_kernel<T, T, A>;
    if constexpr (std::is_same<T, float>::value && std::is_same<A, float>::value)
      if (small_spec<T, A>(s)) kern = small::fwd_kernel<T, T, A, 64, 16>;
    small_setup(kern, sm);
    kern<<<grid, small::NTHREADS, sm, st>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, lse,
                                            s, ly);
  }
  return launch_status();
}

template <typename T, typename A = float>
int small_bwd(const void* q, const void* k, const void* v, const void* dout, const float* lse,
              void* dq, void* dk, void* dv, const Shape& s, cudaStream_t st,
              const small::Layout* lyp = nullptr) {
  const small::Layout ly = lyp ? *lyp : contiguous_layout(s);
  const size_t sm = small::smem_bytes((int)s.T, (int)s.M, (int)s.D, 2, 2, 2, sizeof(A));
  auto kern = small::bwd_kernel<T, A>;
  if constexpr (std::is_same<T, float>::value && std::is_same<A, float>::value)
    if (small_spec<T, A>(s)) kern = small::bwd_kernel<T, A, 64, 16>;
  small_setup(kern, sm);
  kern<<<(unsigned)(s.B * s.H), small::NTHREADS, sm, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)dout, lse, (T*)dq, (T*)dk, (T*)dv, s,
      ly);
  return launch_status();
}

template <typename T, typename A = float>
int small_jvp(const void* q, const void* k, const void* v, const void* tq, const void* tk,
              const void* tv, const float* lse, void* o_tan, const Shape& s, cudaStream_t st,
              const small::Layout* lyp = nullptr) {
  const small::Layout ly = lyp ? *lyp : contiguous_layout(s);
  const size_t sm = small::smem_bytes((int)s.T, (int)s.M, (int)s.D, 2, 4, 2, sizeof(A));
  auto kern = small::jvp_kernel<T, A>;
  if constexpr (std::is_same<T, float>::value && std::is_same<A, float>::value)
    if (small_spec<T, A>(s)) kern = small::jvp_kernel<T, A, 64, 16>;
  small_setup(kern, sm);
  kern<<<(unsigned)(s.B * s.H), small::NTHREADS, sm, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)tq, (const T*)tk, (const T*)tv, lse,
      (T*)o_tan, s, ly);
  return launch_status();
}

template <typename T, typename A = float>
int small_hvp(const void* q, const void* k, const void* v, const void* w, const float* lse,
              const void* tq, const void* tk, const void* tv, void* hq, void* hk, void* hv,
              void* o_tan, const Shape& s, cudaStream_t st, const small::Layout* lyp = nullptr) {
  const small::Layout ly = lyp ? *lyp : contiguous_layout(s);
  const size_t sm = small::hvp_smem_bytes((int)s.T, (int)s.M, (int)s.D, sizeof(A));
  auto kern = small::hvp_kernel<T, A>;
  if constexpr (std::is_same<T, float>::value && std::is_same<A, float>::value)
    if (small_spec<T, A>(s)) kern = small::hvp_kernel<T, A, 64, 16>;
  small_setup(kern, sm);
  kern<<<(unsigned)(s.B * s.H), small::NTHREADS, sm, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)w, lse, (const T*)tq, (const T*)tk,
      (const T*)tv, (T*)hq, (T*)hk, (T*)hv, (T*)o_tan, s, ly);
  return launch_status();
}

// Kernels that move registers between warpgroups (setmaxnreg) need the
// launch allocation their split assumes, or the raising warps would wait
// forever; checked once per kernel before its first launch.
template <typename K>
bool regs_cover_split(K kern, int nthreads, int split_sum_per_128) {
  cudaFuncAttributes a{};
  if (cudaFuncGetAttributes(&a, kern) != cudaSuccess) return false;
  return (int64_t)a.numRegs * nthreads >= (int64_t)split_sum_per_128 * 128;
}

// ------------------------------------------------------ tensor-core launches
template <typename T, int HD, bool CAUSAL>
int tc_fwd_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, void* o,
                  int out_f32, float* lse, const Shape& s, cudaStream_t st) {
  auto kern = tcfwd::fwd_kernel<T, HD, CAUSAL>;
  constexpr int smem = tcfwd::Smem<HD>::kAlloc;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((unsigned)((s.T + tcfwd::NQT * tcfwd::BM - 1) / (tcfwd::NQT * tcfwd::BM)),
            (unsigned)(s.B * s.H));
  if (CAUSAL) grid = dim3(grid.y, grid.x);  // head index in x: longest tiles first
  kern<<<grid, tcfwd::Cfg<HD>::kThreads, smem, st>>>(mq, mk, mv, o, out_f32, lse, (int)s.T, (int)s.M,
                                            s.scale * 1.4426950408889634f);
  return launch_status();
}

// Returns -1 when no TMA descriptor can describe the tensors (the caller
// then runs the SIMT kernel), else a THERIA_* status.
template <typename T>
int tc_fwd(const void* q, const void* k, const void* v, void* o, int o_dtype, float* lse,
           const Shape& s, int dtype, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  const int64_t bh = s.B * s.H;
  if (!tc::make_map_3d(&mq, q, dtype, bh, s.T, s.D, tcfwd::BM) ||
      !tc::make_map_3d(&mk, k, dtype, bh, s.M, s.D, tcfwd::BN) ||
      !tc::make_map_3d(&mv, v, dtype, bh, s.M, s.D, tcfwd::BN))
    return -1;
  const int f32 = o_dtype == THERIA_F32;
  if (s.D == 64)
    return s.causal ? tc_fwd_launch<T, 64, true>(mq, mk, mv, o, f32, lse, s, st)
                    : tc_fwd_launch<T, 64, false>(mq, mk, mv, o, f32, lse, s, st);
  return s.causal ? tc_fwd_launch<T, 128, true>(mq, mk, mv, o, f32, lse, s, st)
                  : tc_fwd_launch<T, 128, false>(mq, mk, mv, o, f32, lse, s, st);
}

int64_t simt_bwd_ws(const Shape& s) { return align_up(s.B * s.H * s.T * 4); }
int64_t tc_bwd_ws(const Shape& s) {
  return align_up(s.B * s.H * s.T * 4) + align_up(s.B * s.H * s.T * s.D * 4);
}

template <typename T, int HD, bool CAUSAL>
int tc_bwd_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                  const CUtensorMap& mdo, const CUtensorMap& mdq, const float* lse,
                  const float* z, float* dq_acc, void* dk, void* dv, const Shape& s,
                  cudaStream_t st) {
  auto kern = tcbwd::bwd_kernel<T, HD, CAUSAL>;
  constexpr int smem = tcbwd::Smem<HD>::kAlloc;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((unsigned)((s.M + tcbwd::BK - 1) / tcbwd::BK), (unsigned)(s.B * s.H));
  if (CAUSAL) grid = dim3(grid.y, grid.x);  // head index in x: longest tiles first
  kern<<<grid, tcbwd::NTHREADS, smem, st>>>(mq, mk, mv, mdo, mdq, lse, z, dq_acc, (T*)dk, (T*)dv,
                                            (int)s.T, (int)s.M, s.scale,
                                            s.scale * 1.4426950408889634f);
  return launch_status();
}

// Tensor-core backward; -1 when no TMA descriptor fits (caller falls back).
template <typename T>
int tc_bwd(const void* q, const void* k, const void* v, const void* o, int o_dtype,
           const void* dout, const float* lse, void* dq, void* dk, void* dv, void* ws,
           const Shape& s, int dtype, cudaStream_t st) {
  CUtensorMap mq, mk, mv, mdo;
  const int64_t bh = s.B * s.H;
  if (!tc::make_map_3d(&mq, q, dtype, bh, s.T, s.D, tcbwd::BQ) ||
      !tc::make_map_3d(&mk, k, dtype, bh, s.M, s.D, tcbwd::BK) ||
      !tc::make_map_3d(&mv, v, dtype, bh, s.M, s.D, tcbwd::BK) ||
      !tc::make_map_3d(&mdo, dout, dtype, bh, s.T, s.D, tcbwd::BQ))
    return -1;
  float* z = (float*)ws;
  float* dq_acc = (float*)((char*)ws + align_up(bh * s.T * 4));
  const int64_t rows = bh * s.T;
  // D = 64 adds its dQ tiles through a swizzled fp32 map of the accumulator
  CUtensorMap mdq;
  std::memset(&mdq, 0, sizeof(mdq));
  if (s.D == 64 && !tc::make_map_3d_f32(&mdq, dq_acc, bh, s.T, s.D, 2 * tcbwd::BQ)) return -1;
  if (o != nullptr) {
    tcbwd::prep_kernel<T><<<(unsigned)((rows * (s.D / 8) + 255) / 256), 256, 0, st>>>(
        o, o_dtype == THERIA_F32, (const T*)dout, z, dq_acc, rows, (int)s.D);
    if (int e = launch_status()) return e;
  } else {
    size_t sm = (2 * tile_floats(s.D) + simt::WARPS * 2 * s.D) * sizeof(float);
    auto kern = simt::delta_from_stats_kernel<T>;
    set_smem(kern, sm);
    kern<<<row_grid(s), simt::WARPS * 32, sm, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                    (const T*)dout, lse, z, s);
    if (int e = launch_status()) return e;
    if (cudaMemsetAsync(dq_acc, 0, rows * s.D * 4, st) != cudaSuccess) return THERIA_ERR_LAUNCH;
  }
  int e;
  if (s.D == 64)
    e = s.causal ? tc_bwd_launch<T, 64, true>(mq, mk, mv, mdo, mdq, lse, z, dq_acc, dk, dv, s, st)
                 : tc_bwd_launch<T, 64, false>(mq, mk, mv, mdo, mdq, lse, z, dq_acc, dk, dv, s, st);
  else
    e = s.causal ? tc_bwd_launch<T, 128, true>(mq, mk, mv, mdo, mdq, lse, z, dq_acc, dk, dv, s, st)
                 : tc_bwd_launch<T, 128, false>(mq, mk, mv, mdo, mdq, lse, z, dq_acc, dk, dv, s, st);
  if (e) return e;
  if (dq != nullptr) {
    const int64_t n = rows * s.D;
    const unsigned blocks = (unsigned)std::min<int64_t>((n / 8 + 255) / 256, 148 * 16);
    tcbwd::finish_kernel<T><<<blocks, 256, 0, st>>>(dq_acc, (T*)dq, n);
    return launch_status();
  }
  return THERIA_OK;
}

template <typename T, int HD, bool CAUSAL, bool W>
int tc_jvp_launch(const CUtensorMap* m, const float* lse, const void* w, void* o_tan,
                  float* stats, const Shape& s, cudaStream_t st) {
  using C = tcjvp::Cfg<HD>;
  auto kern = tcjvp::jvp_kernel<T, HD, CAUSAL, W>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
  dim3 grid((unsigned)((s.T + tcjvp::BM - 1) / tcjvp::BM), (unsigned)(s.B * s.H));
  if (CAUSAL) grid = dim3(grid.y, grid.x);  // head index in x: longest tiles first
  kern<<<grid, tcjvp::NTHREADS, C::kAlloc, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], lse,
                                                 (const T*)w, (T*)o_tan, stats,
                                                 s.B * s.H * s.T, (int)s.T, (int)s.M, s.scale,
                                                 s.scale * 1.4426950408889634f);
  return launch_status();
}

// Tensor-core JVP (w == nullptr) or HVP pass 1 (row terms into `stats`);
// -1 when no TMA descriptor fits.
template <typename T>
int tc_jvp(const void* q, const void* k, const void* v, const void* tq, const void* tk,
           const void* tv, const void* w, const float* lse, void* o_tan, float* stats,
           const Shape& s, int dtype, cudaStream_t st) {
  CUtensorMap m[6];
  const int64_t bh = s.B * s.H;
  const uint32_t bn = s.D == 128 ? tcjvp::Cfg<128>::BN : tcjvp::Cfg<64>::BN;
  const void* src[6] = {q, tq, k, tk, v, tv};
  for (int i = 0; i < 6; ++i)
    if (!tc::make_map_3d(&m[i], src[i], dtype, bh, i < 2 ? s.T : s.M, s.D,
                         i < 2 ? (uint32_t)tcjvp::BM : bn))
      return -1;
  const bool hw = w != nullptr;
#define THERIA_JVP(HD, C, W) tc_jvp_launch<T, HD, C, W>(m, lse, w, o_tan, stats, s, st)
  if (s.D == 64) {
    if (s.causal) return hw ? THERIA_JVP(64, true, true) : THERIA_JVP(64, true, false);
    return hw ? THERIA_JVP(64, false, true) : THERIA_JVP(64, false, false);
  }
  if (s.causal) return hw ? THERIA_JVP(128, true, true) : THERIA_JVP(128, true, false);
  return hw ? THERIA_JVP(128, false, true) : THERIA_JVP(128, false, false);
#undef THERIA_JVP
}

int64_t simt_hvp_ws(const Shape& s) { return align_up(3 * s.B * s.H * s.T * 4); }
// Query-chunk count of the HVP's second pass: the (key tile, b*h) units are
// few against the SMs at small B*H (configs[2]: 256 CTAs = 1.7 waves on 148
// SMs), so the queries of each key tile may be split over up to 4 CTAs
// whose hK/hV partial sums are added in fp32; chosen for the fullest last
// wave, preferring fewer chunks unless that wave fills >= 5 % better.  Each
// chunk keeps at least 16 query tiles: with 8 (configs[2] in 4 chunks) the
// per-CTA start-up cost outweighed the fuller wave (505 -> 447 TFLOP/s).
int hvp_split(const Shape& s, int sms) {
  const int64_t units = s.B * s.H * ((s.M + tchvp::BK - 1) / tchvp::BK);
  const int64_t n_qt = (s.T + tchvp::BQ - 1) / tchvp::BQ;
  if (s.causal || units >= 8 * (int64_t)sms) return 1;
  int best = 1;
  double best_eff = 0.0;
  for (int k = 1; k <= 4; ++k) {
    if (k > 1 && n_qt / k < 16) break;
    const int64_t ctas = units * k;
    const double eff = (double)ctas / (double)(((ctas + sms - 1) / sms) * sms);
    if (eff > best_eff + 0.05) {
      best = k;
      best_eff = eff;
    }
  }
  return best;
}

int64_t tc_hvp_ws(const Shape& s, int split) {
  return align_up(3 * s.B * s.H * s.T * 4) + align_up(s.B * s.H * s.T * s.D * 4) +
         (split > 1 ? align_up(2 * s.B * s.H * s.M * s.D * 4) : 0);
}
int64_t tc_hvp_ws(const Shape& s) { return tc_hvp_ws(s, hvp_split(s, 148)); }

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

template <typename T, int HD, bool CAUSAL>
int tc_hvp_launch(const CUtensorMap* m, const float* lse, const float* stats, float* hq_acc,
                  void* hk, void* hv, float* hkv_acc, int split, const Shape& s,
                  cudaStream_t st) {
  using C = tchvp::Cfg<HD>;
  auto kern = tchvp::hvp_kernel<T, HD, CAUSAL>;
  static const bool regs_ok = regs_cover_split(
      kern, tchvp::NTHREADS, tchvp::RegSplit<HD>::total);
  if (!regs_ok) return THERIA_ERR_LAUNCH;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
  dim3 grid((unsigned)((s.M + tchvp::BK - 1) / tchvp::BK), (unsigned)(s.B * s.H), split);
  if (CAUSAL) grid = dim3(grid.y, grid.x, split);  // head index in x: longest tiles first
  kern<<<grid, tchvp::NTHREADS, C::kAlloc, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7],
                                                 lse,
                                                 stats, s.B * s.H * s.T, hq_acc, (T*)hk,
                                                 (T*)hv, (int)s.T, (int)s.M, s.scale,
                                                 s.scale * 1.4426950408889634f, hkv_acc, split);
  return launch_status();
}

// Tensor-core HVP: pass 1 (JVP kernel with W) then the fused hQ/hK/hV pass;
// -1 when no TMA descriptor fits.
template <typename T>
int tc_hvp(const void* q, const void* k, const void* v, const void* w, const float* lse,
           const void* tq, const void* tk, const void* tv, void* hq, void* hk, void* hv,
           void* o_tan, void* ws, int64_t ws_bytes, const Shape& s, int dtype,
           cudaStream_t st) {
  CUtensorMap m[8];
  const int64_t bh = s.B * s.H;
  const void* src[7] = {q, tq, w, k, v, tk, tv};
  for (int i = 0; i < 7; ++i)
    if (!tc::make_map_3d(&m[i], src[i], dtype, bh, i < 3 ? s.T : s.M, s.D,
                         i < 3 ? (uint32_t)tchvp::BQ : (uint32_t)tchvp::BK))
      return -1;
  float* stats = (float*)ws;
  float* hq_acc = (float*)((char*)ws + align_up(3 * bh * s.T * 4));
  // D = 64 adds its hQ tiles through a swizzled fp32 map of the accumulator
  std::memset(&m[7], 0, sizeof(m[7]));
  if (s.D == 64 && !tc::make_map_3d_f32(&m[7], hq_acc, bh, s.T, s.D, 2 * tchvp::BQ)) return -1;
  // query chunks of the second pass, when the workspace has room for the
  // fp32 hK/hV partial sums
  int split = hvp_split(s, sm_count());
  if (split > 1 && ws_bytes < tc_hvp_ws(s, split)) split = 1;
  float* hkv_acc = split > 1 ? (float*)((char*)hq_acc + align_up(bh * s.T * s.D * 4)) : nullptr;
  const int64_t nkv = bh * s.M * s.D;
  int e = tc_jvp<T>(q, k, v, tq, tk, tv, w, lse, o_tan, stats, s, dtype, st);
  if (e != 0) return e;
  const int64_t n = bh * s.T * s.D;
  if (cudaMemsetAsync(hq_acc, 0, n * 4, st) != cudaSuccess) return THERIA_ERR_LAUNCH;
  if (split > 1 && cudaMemsetAsync(hkv_acc, 0, 2 * nkv * 4, st) != cudaSuccess)
    return THERIA_ERR_LAUNCH;
#define THERIA_HVP2(HD, C) \
  tc_hvp_launch<T, HD, C>(m, lse, stats, hq_acc, hk, hv, hkv_acc, split, s, st)
  if (s.D == 64)
    e = s.causal ? THERIA_HVP2(64, true) : THERIA_HVP2(64, false);
  else
    e = s.causal ? THERIA_HVP2(128, true) : THERIA_HVP2(128, false);
#undef THERIA_HVP2
  if (e) return e;
  if (split > 1) {
    const unsigned blocks = (unsigned)std::min<int64_t>((nkv / 8 + 255) / 256, 148 * 16);
    if (hv != nullptr) {
      tcbwd::finish_kernel<T><<<blocks, 256, 0, st>>>(hkv_acc, (T*)hv, nkv);
      if (int e2 = launch_status()) return e2;
    }
    if (hk != nullptr) {
      tcbwd::finish_kernel<T><<<blocks, 256, 0, st>>>(hkv_acc + nkv, (T*)hk, nkv);
      if (int e2 = launch_status()) return e2;
    }
  }
  if (hq != nullptr) {
    const unsigned blocks = (unsigned)std::min<int64_t>((n / 8 + 255) / 256, 148 * 16);
    tcbwd::finish_kernel<T><<<blocks, 256, 0, st>>>(hq_acc, (T*)hq, n);
    return launch_status();
  }
  return THERIA_OK;
}

bool use_tc(int dtype, const Shape& s, std::initializer_list<const void*> ptrs) {
  if (!tc::tc_eligible(dtype, s.T, s.M, s.D, s.B * s.H)) return false;
  for (const void* p : ptrs)
    if (p != nullptr && !tc::aligned16(p)) return false;
  return true;
}

// Dense scores / probabilities (sdpa_scores.cuh).  Output element type O is
// float, or T itself for 16-bit scores.
template <typename T, typename O>
int scores_launch(const void* q, const void* k, void* out, const float* lse, const Shape& s,
                  int dtype, int mode, cudaStream_t st) {
  const int vec = tc::aligned16(out) && (s.M * (int64_t)sizeof(O)) % 16 == 0;
  if constexpr (!std::is_same<T, float>::value) {
    if (use_tc(dtype, s, {q, k})) {
      CUtensorMap mq, mk;
      const int64_t bh = s.B * s.H;
      if (tc::make_map_3d(&mq, q, dtype, bh, s.T, s.D, scores::TM) &&
          tc::make_map_3d(&mk, k, dtype, bh, s.M, s.D, scores::TN)) {
        dim3 grid((unsigned)((s.T + scores::TM - 1) / scores::TM),
                  (unsigned)((s.M + scores::TN - 1) / scores::TN), (unsigned)bh);
        if (s.D == 64) {
          auto kern = scores::tc_kernel<T, O, 64>;
          constexpr int smem = scores::TcSmem<64>::kAlloc;
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
          kern<<<grid, 128, smem, st>>>(mq, mk, (O*)out, lse, (int)s.T, (int)s.M, s.scale, mode,
                                        s.causal, vec);
        } else {
          auto kern = scores::tc_kernel<T, O, 128>;
          constexpr int smem = scores::TcSmem<128>::kAlloc;
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
          kern<<<grid, 128, smem, st>>>(mq, mk, (O*)out, lse, (int)s.T, (int)s.M, s.scale, mode,
                                        s.causal, vec);
        }
        return launch_status();
      }
    }
  }
  dim3 grid((unsigned)((s.M + scores::ST - 1) / scores::ST),
            (unsigned)((s.T + scores::ST - 1) / scores::ST), (unsigned)(s.B * s.H));
  if (grid.y > 65535) return THERIA_ERR_UNSUPPORTED;
  scores::simt_kernel<T, O><<<grid, dim3(16, 16), 0, st>>>(
      (const T*)q, (const T*)k, (O*)out, lse, (int)s.T, (int)s.M, (int)s.D, s.scale, mode,
      s.causal);
  return launch_status();
}

template <typename T>
int scores_dispatch(const void* q, const void* k, void* out, int out_dtype, const float* lse,
                    const Shape& s, int dtype, int mode, cudaStream_t st) {
  if (out_dtype == THERIA_F32) return scores_launch<T, float>(q, k, out, lse, s, dtype, mode, st);
  return scores_launch<T, T>(q, k, out, lse, s, dtype, mode, st);
}

#define THERIA_DISPATCH(dtype, FN, ...)                          \
  ((dtype) == THERIA_F32   ? FN<float>(__VA_ARGS__)              \
   : (dtype) == THERIA_F16 ? FN<__half>(__VA_ARGS__)             \
                           : FN<__nv_bfloat16>(__VA_ARGS__))

}  // namespace
}  // namespace theria

using namespace theria;

extern "C" {

const char* theria_status_string(int status) {
  switch (status) {
    case THERIA_OK: return "ok";
    case THERIA_ERR_INVALID_ARG: return "invalid argument";
    case THERIA_ERR_UNSUPPORTED: return "unsupported shape (head_dim <= 128, batch*heads <= 65535)";
    case THERIA_ERR_LAUNCH: return "CUDA kernel launch failed";
    case THERIA_ERR_WORKSPACE: return "workspace missing or too small";
    case THERIA_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case THERIA_ERR_SCRATCH_LIMIT:
      return "problem too large for the fixed scratch of theria_sdpa_bwd_noalloc "
             "(B*H*T*4 bytes must fit in THERIA_NOALLOC_SCRATCH_BYTES); use theria_sdpa_bwd";
    default: return "unknown status";
  }
}

const char* theria_version(void) { return "theria-sm100 0.1.0"; }

int64_t theria_launch_count(void) { return (int64_t)launch_counter().load(); }

int theria_sdpa_fwd(const void* q, const void* k, const void* v, void* o, int o_dtype,
                    float* lse, int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                    int dtype, float scale, int causal, void* stream) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return e;
  if (o_dtype != THERIA_F32 && o_dtype != dtype) return THERIA_ERR_INVALID_ARG;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!q || !k || !v || !o) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, M, D, scale, causal ? 1 : 0};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == THERIA_F64)
    return f64_fits(s, 1, 2, 1) ? small_fwd<double, double>(q, k, v, o, o_dtype, lse, s, st)
                                : THERIA_ERR_UNSUPPORTED;
  if (small_eligible(s)) return THERIA_DISPATCH(dtype, small_fwd, q, k, v, o, o_dtype, lse, s, st);
  if (use_tc(dtype, s, {q, k, v, o})) {
    int e = dtype == THERIA_BF16 ? tc_fwd<__nv_bfloat16>(q, k, v, o, o_dtype, lse, s, dtype, st)
                                 : tc_fwd<__half>(q, k, v, o, o_dtype, lse, s, dtype, st);
    if (e >= 0) return e;
  }
  return THERIA_DISPATCH(dtype, simt_fwd, q, k, v, o, o_dtype, lse, s, st);
}

int theria_sdpa_scores(const void* q, const void* k, void* out, int out_dtype, int64_t B,
                       int64_t H, int64_t T, int64_t M, int64_t D, int dtype, float scale,
                       void* stream) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return e;
  if (out_dtype != THERIA_F32 && out_dtype != dtype) return THERIA_ERR_INVALID_ARG;
  if (dtype == THERIA_F64) return THERIA_ERR_UNSUPPORTED;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!q || !k || !out) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, M, D, scale, 0};
  return THERIA_DISPATCH(dtype, scores_dispatch, q, k, out, out_dtype, nullptr, s, dtype,
                         scores::kScores, (cudaStream_t)stream);
}

int theria_sdpa_probs(const void* q, const void* k, const float* lse, float* out, int64_t B,
                      int64_t H, int64_t T, int64_t M, int64_t D, int dtype, float scale,
                      int causal, void* stream) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return e;
  if (dtype == THERIA_F64) return THERIA_ERR_UNSUPPORTED;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!q || !k || !lse || !out) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, M, D, scale, causal ? 1 : 0};
  return THERIA_DISPATCH(dtype, scores_dispatch, q, k, out, THERIA_F32, lse, s, dtype,
                         scores::kProbs, (cudaStream_t)stream);
}

int64_t theria_sdpa_bwd_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t M,
                                        int64_t D) {
  Shape s{B, H, T, M, D, 1.f, 0};
  // Enough for the tensor-core path (row terms + fp32 dQ accumulator) where
  // the head dim allows it; the CUDA-core path needs only the row terms.
  return (D == 64 || D == 128) ? tc_bwd_ws(s) : simt_bwd_ws(s);
}

int64_t theria_sdpa_hvp_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t M,
                                        int64_t D) {
  Shape s{B, H, T, M, D, 1.f, 0};
  // Row terms (c, z, zdot), plus the fp32 hQ accumulator of the tensor-core
  // path where the head dim allows it.
  return (D == 64 || D == 128) ? tc_hvp_ws(s) : simt_hvp_ws(s);
}

int theria_sdpa_bwd(const void* q, const void* k, const void* v, const void* o, int o_dtype,
                    const void* dout, const float* lse, void* dq, void* dk, void* dv,
                    void* workspace, int64_t workspace_bytes, int64_t B, int64_t H, int64_t T,
                    int64_t M, int64_t D, int dtype, float scale, int causal, void* stream) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return e;
  if (o != nullptr && !valid_dtype(o_dtype)) return THERIA_ERR_INVALID_ARG;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!q || !k || !v || !dout || !lse) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, M, D, scale, causal ? 1 : 0};
  if (!workspace || workspace_bytes < simt_bwd_ws(s)) return THERIA_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == THERIA_F64)
    return f64_fits(s, 2, 2, 2) ? small_bwd<double, double>(q, k, v, dout, lse, dq, dk, dv, s, st)
                                : THERIA_ERR_UNSUPPORTED;
  if (small_eligible(s))
    return THERIA_DISPATCH(dtype, small_bwd, q, k, v, dout, lse, dq, dk, dv, s, st);
  // The tensor-core path needs the larger workspace; a caller that passes
  // only the minimum (row terms) gets the CUDA-core kernels.
  if (workspace_bytes >= tc_bwd_ws(s) && use_tc(dtype, s, {q, k, v, o, dout, dq, dk, dv})) {
    int e = dtype == THERIA_BF16
                ? tc_bwd<__nv_bfloat16>(q, k, v, o, o_dtype, dout, lse, dq, dk, dv, workspace, s,
                                        dtype, st)
                : tc_bwd<__half>(q, k, v, o, o_dtype, dout, lse, dq, dk, dv, workspace, s, dtype,
                                 st);
    if (e >= 0) return e;
  }
  return THERIA_DISPATCH(dtype, simt_bwd, q, k, v, o, o_dtype, dout, lse, dq, dk, dv,
                         (float*)workspace, s, st);
}

int theria_sdpa_jvp(const void* q, const void* k, const void* v, const void* tq,
                    const void* tk, const void* tv, const float* lse, void* o_tan, int64_t B,
                    int64_t H, int64_t T, int64_t M, int64_t D, int dtype, float scale,
                    int causal, void* stream) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return e;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!q || !k || !v || !tq || !tk || !tv || !lse || !o_tan) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, M, D, scale, causal ? 1 : 0};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == THERIA_F64)
    return f64_fits(s, 2, 4, 2)
               ? small_jvp<double, double>(q, k, v, tq, tk, tv, lse, o_tan, s, st)
               : THERIA_ERR_UNSUPPORTED;
  if (small_eligible(s))
    return THERIA_DISPATCH(dtype, small_jvp, q, k, v, tq, tk, tv, lse, o_tan, s, st);
  if (use_tc(dtype, s, {q, k, v, tq, tk, tv, o_tan})) {
    int e = dtype == THERIA_BF16
                ? tc_jvp<__nv_bfloat16>(q, k, v, tq, tk, tv, nullptr, lse, o_tan, nullptr, s,
                                        dtype, st)
                : tc_jvp<__half>(q, k, v, tq, tk, tv, nullptr, lse, o_tan, nullptr, s, dtype, st);
    if (e >= 0) return e;
  }
  return THERIA_DISPATCH(dtype, simt_jvp, q, k, v, tq, tk, tv, nullptr, lse, o_tan, nullptr, s,
                         st);
}

int theria_sdpa_hvp(const void* q, const void* k, const void* v, const void* w,
                    const float* lse, const void* tq, const void* tk, const void* tv, void* hq,
                    void* hk, void* hv, void* o_tan, void* workspace, int64_t workspace_bytes,
                    int64_t B, int64_t H, int64_t T, int64_t M, int64_t D, int dtype,
                    float scale, int causal, void* stream) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return e;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!q || !k || !v || !w || !lse || !tq || !tk || !tv) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, M, D, scale, causal ? 1 : 0};
  if (!workspace || workspace_bytes < simt_hvp_ws(s)) return THERIA_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == THERIA_F64)
    return f64_fits_hvp(s) ? small_hvp<double, double>(q, k, v, w, lse, tq, tk, tv, hq, hk,
                                                            hv, o_tan, s, st)
                                : THERIA_ERR_UNSUPPORTED;
  if (small_eligible(s))
    return THERIA_DISPATCH(dtype, small_hvp, q, k, v, w, lse, tq, tk, tv, hq, hk, hv, o_tan, s,
                           st);
  if (workspace_bytes >= tc_hvp_ws(s, 1) &&
      use_tc(dtype, s, {q, k, v, w, tq, tk, tv, hq, hk, hv, o_tan})) {
    int e = dtype == THERIA_BF16
                ? tc_hvp<__nv_bfloat16>(q, k, v, w, lse, tq, tk, tv, hq, hk, hv, o_tan,
                                        workspace, workspace_bytes, s, dtype, st)
                : tc_hvp<__half>(q, k, v, w, lse, tq, tk, tv, hq, hk, hv, o_tan, workspace,
                                 workspace_bytes, s, dtype, st);
    if (e >= 0) return e;
  }
  return THERIA_DISPATCH(dtype, simt_hvp, q, k, v, w, lse, tq, tk, tv, hq, hk, hv, o_tan,
                         (float*)workspace, s, st);
}

}  // extern "C"

namespace theria {
namespace {
// Diagnostic of the bounded-wait machinery every tensor-core kernel uses:
// warp 0 waits on an mbarrier phase that nothing completes, with a poll
// limit of `max_polls`, and must give up (setting the abort flag and the
// device error word); warp 1 waits on the same phase with the kernels'
// normal limit and must unwind when it sees the abort flag.  out[0] = 1 if
// warp 0 gave up, out[1] = 1 if warp 1 unwound.  The barrier's phase is
// then completed by an arrival so the CTA exits with nothing pending.
__global__ void __launch_bounds__(64) diag_bounded_wait_kernel(uint32_t max_polls, int* out) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    const bool ok = warp == 0 ? tc::mbar_wait(&bar, 0, &abort_flag, max_polls)
                              : tc::mbar_wait(&bar, 0, &abort_flag);
    out[warp] = ok ? 0 : 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) tc::mbar_arrive(&bar);
}
}  // namespace
}  // namespace theria

extern "C" {

int theria_diag_bounded_wait(int max_polls, int* out, void* stream) {
  if (max_polls < 1 || max_polls > (1 << 20) || out == nullptr) return THERIA_ERR_INVALID_ARG;
  theria::diag_bounded_wait_kernel<<<1, 64, 0, (cudaStream_t)stream>>>((uint32_t)max_polls, out);
  return theria::launch_status();
}

int theria_get_device_error(int* out_flag, void* stream) {
  if (!out_flag) return THERIA_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemcpyFromSymbolAsync(out_flag, g_device_error, sizeof(int), 0,
                                cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return THERIA_ERR_LAUNCH;
  return cudaStreamSynchronize(st) == cudaSuccess ? THERIA_OK : THERIA_ERR_LAUNCH;
}

int theria_clear_device_error(void* stream) {
  static const int zero = 0;
  return cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                 (cudaStream_t)stream) == cudaSuccess
             ? THERIA_OK
             : THERIA_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// Allocation-free backward.  Its scratch is this file-scope device array, one
// copy per GPU that loads the library.  On the host, `g_noalloc_scratch` only
// names the symbol: its device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and cached.
static __device__ __align__(256) unsigned char g_noalloc_scratch[THERIA_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, or nullptr.
void* noalloc_scratch_ptr() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    g_noalloc_ptr[dev] = p;
  }
  return g_noalloc_ptr[dev];
}
}  // namespace

int theria_sdpa_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                            int o_dtype, const void* dout, const float* lse, void* dq,
                            void* dk, void* dv, int64_t B, int64_t H, int64_t T, int64_t M,
                            int64_t D, int dtype, float scale, int causal, void* stream) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return e;
  if (B * H * T * 4 > (int64_t)THERIA_NOALLOC_SCRATCH_BYTES) return THERIA_ERR_SCRATCH_LIMIT;
  if (empty_problem(B, H, T)) return THERIA_OK;
  void* scratch = noalloc_scratch_ptr();
  if (scratch == nullptr) return THERIA_ERR_LAUNCH;
  return theria_sdpa_bwd(q, k, v, o, o_dtype, dout, lse, dq, dk, dv, scratch,
                         (int64_t)THERIA_NOALLOC_SCRATCH_BYTES, B, H, T, M, D, dtype, scale,
                         causal, stream);
}

int theria_sdpa_bwd_noalloc_uses_tc(int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                                    int dtype) {
  if (int e = check_shape(B, H, T, M, D, dtype)) return -e;
  if (B * H * T * 4 > (int64_t)THERIA_NOALLOC_SCRATCH_BYTES) return -THERIA_ERR_SCRATCH_LIMIT;
  Shape s{B, H, T, M, D, 1.f, 0};
  if (dtype == THERIA_F64 || small_eligible(s)) return 0;
  return tc::tc_shape_ok(dtype, T, M, D, B * H) &&
         tc_bwd_ws(s) <= (int64_t)THERIA_NOALLOC_SCRATCH_BYTES;
}

}  // extern "C"

// ------------------------------------------------------ packed self-attention
namespace {
int qkv_check(int64_t B, int64_t H, int64_t T, int64_t D, int dtype) {
  if (int e = check_shape(B, H, T, T, D, dtype)) return e;
  Shape s{B, H, T, T, D, 1.f, 0};
  if (!small_eligible(s)) return THERIA_ERR_UNSUPPORTED;
  return THERIA_OK;
}
template <typename T>
const T* part(const void* qkv, int which, int64_t H, int64_t D) {
  return (const T*)qkv + which * H * D;
}
template <typename T>
T* part(void* qkv, int which, int64_t H, int64_t D) {
  return (T*)qkv + which * H * D;
}
template <typename T, typename A = float>
int qkv_fwd(const void* qkv, void* o, float* lse, const Shape& s, cudaStream_t st) {
  const small::Layout ly = packed_layout(s);
  const int od = std::is_same<T, float>::value ? THERIA_F32
                 : std::is_same<T, double>::value ? THERIA_F64 : -1;
  return small_fwd<T, A>(part<T>(qkv, 0, s.H, s.D), part<T>(qkv, 1, s.H, s.D),
                         part<T>(qkv, 2, s.H, s.D), o, od, lse, s, st, &ly);
}
template <typename T, typename A = float>
int qkv_bwd(const void* qkv, const void* dout, const float* lse, void* dqkv, const Shape& s,
            cudaStream_t st) {
  const small::Layout ly = packed_layout(s);
  return small_bwd<T, A>(part<T>(qkv, 0, s.H, s.D), part<T>(qkv, 1, s.H, s.D),
                         part<T>(qkv, 2, s.H, s.D), dout, lse, part<T>(dqkv, 0, s.H, s.D),
                         part<T>(dqkv, 1, s.H, s.D), part<T>(dqkv, 2, s.H, s.D), s, st, &ly);
}
template <typename T, typename A = float>
int qkv_hvp(const void* qkv, const void* w, const float* lse, const void* tqkv, void* hqkv,
            void* o_tan, const Shape& s, cudaStream_t st) {
  const small::Layout ly = packed_layout(s);
  T* h[3] = {nullptr, nullptr, nullptr};
  if (hqkv)
    for (int i = 0; i < 3; ++i) h[i] = part<T>(hqkv, i, s.H, s.D);
  return small_hvp<T, A>(part<T>(qkv, 0, s.H, s.D), part<T>(qkv, 1, s.H, s.D),
                         part<T>(qkv, 2, s.H, s.D), w, lse, part<T>(tqkv, 0, s.H, s.D),
                         part<T>(tqkv, 1, s.H, s.D), part<T>(tqkv, 2, s.H, s.D), h[0], h[1],
                         h[2], o_tan, s, st, &ly);
}
}  // namespace

extern "C" {

int theria_sdpa_qkv_fwd(const void* qkv, void* o, float* lse, int64_t B, int64_t H, int64_t T,
                        int64_t D, int dtype, float scale, int causal, void* stream) {
  if (int e = qkv_check(B, H, T, D, dtype)) return e;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!qkv || !o || !lse) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, T, D, scale, causal ? 1 : 0};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == THERIA_F64)
    return f64_fits(s, 1, 2, 1) ? qkv_fwd<double, double>(qkv, o, lse, s, st)
                                : THERIA_ERR_UNSUPPORTED;
  return THERIA_DISPATCH(dtype, qkv_fwd, qkv, o, lse, s, st);
}

int theria_sdpa_qkv_bwd(const void* qkv, const void* dout, const float* lse, void* dqkv,
                        int64_t B, int64_t H, int64_t T, int64_t D, int dtype, float scale,
                        int causal, void* stream) {
  if (int e = qkv_check(B, H, T, D, dtype)) return e;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!qkv || !dout || !lse || !dqkv) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, T, D, scale, causal ? 1 : 0};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == THERIA_F64)
    return f64_fits(s, 2, 2, 2) ? qkv_bwd<double, double>(qkv, dout, lse, dqkv, s, st)
                                : THERIA_ERR_UNSUPPORTED;
  return THERIA_DISPATCH(dtype, qkv_bwd, qkv, dout, lse, dqkv, s, st);
}

int theria_sdpa_qkv_hvp(const void* qkv, const void* w, const float* lse, const void* tqkv,
                        void* hqkv, void* o_tan, int64_t B, int64_t H, int64_t T, int64_t D,
                        int dtype, float scale, int causal, void* stream) {
  if (int e = qkv_check(B, H, T, D, dtype)) return e;
  if (empty_problem(B, H, T)) return THERIA_OK;
  if (!qkv || !w || !lse || !tqkv || (!hqkv && !o_tan)) return THERIA_ERR_INVALID_ARG;
  Shape s{B, H, T, T, D, scale, causal ? 1 : 0};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == THERIA_F64)
    return f64_fits_hvp(s)
               ? qkv_hvp<double, double>(qkv, w, lse, tqkv, hqkv, o_tan, s, st)
               : THERIA_ERR_UNSUPPORTED;
  return THERIA_DISPATCH(dtype, qkv_hvp, qkv, w, lse, tqkv, hqkv, o_tan, s, st);
}

}  // extern "C"

// ------------------------------------------------------ MAML LayerNorm
namespace {
int ln_check(int64_t nt, int64_t R, int64_t D, int64_t ldw) {
  // ldw == 0: every task reads the same affine row (a broadcast view)
  if (nt < 0 || R < 0 || D <= 0 || (ldw < D && ldw != 0)) return THERIA_ERR_INVALID_ARG;
  if (D > THERIA_LN_MAX_D || nt > 65535) return THERIA_ERR_UNSUPPORTED;
  return THERIA_OK;
}
int64_t ln_ctas(int64_t R) { return (R + ln::ROWS_PER_CTA - 1) / ln::ROWS_PER_CTA; }

// V = values per lane: D <= 32 V.
template <template <int> class F, typename... Args>
int ln_dispatch(int64_t D, Args... args) {
  if (D <= 32) return F<1>::run(args...);
  if (D <= 64) return F<2>::run(args...);
  if (D <= 128) return F<4>::run(args...);
  return F<8>::run(args...);
}

template <int V>
struct LnFwd {
  static int run(const float* x, const float* w, const float* b, int64_t ldw, float* y,
                 int64_t nt, int64_t R, int D, float eps, cudaStream_t st) {
    dim3 grid((unsigned)ln_ctas(R), (unsigned)nt);
    ln::fwd_kernel<V><<<grid, ln::WARPS * 32, 0, st>>>(x, w, b, ldw, y, R, D, eps);
    return launch_status();
  }
};
template <int V>
struct LnBwd {
  static int run(const float* x, const float* w, int64_t ldw, const float* gy, float* gx,
                 float* gw, float* gb, float* ws, int64_t nt, int64_t R, int D, float eps,
                 cudaStream_t st) {
    dim3 grid((unsigned)ln_ctas(R), (unsigned)nt);
    ln::bwd_kernel<V><<<grid, ln::WARPS * 32, 0, st>>>(x, w, ldw, gy, gx, ws, R, D, eps);
    if (int e = launch_status()) return e;
    ln::colsum_kernel<<<dim3((unsigned)nt, (unsigned)((2 * D + 31) / 32)), ln::COLSUM_THREADS, 0, st>>>(
        ws, gw, gb, (int)grid.x, 2, D);
    return launch_status();
  }
};
template <int V>
struct LnBwd2 {
  static int run(const float* x, const float* w, int64_t ldw, const float* gy, const float* u,
                 const float* a, int64_t lda, const float* c, int64_t ldc, float* dx, float* dw,
                 float* dgy, float* ws, int64_t nt, int64_t R, int D, float eps,
                 cudaStream_t st) {
    dim3 grid((unsigned)ln_ctas(R), (unsigned)nt);
    ln::bwd2_kernel<V><<<grid, ln::WARPS * 32, 0, st>>>(x, w, ldw, gy, u, a, lda, c, ldc, dx,
                                                       dgy, ws, R, D, eps);
    if (int e = launch_status()) return e;
    ln::colsum_kernel<<<dim3((unsigned)nt, (unsigned)((D + 31) / 32)), ln::COLSUM_THREADS, 0, st>>>(
        ws, dw, dw, (int)grid.x, 1, D);
    return launch_status();
  }
};
}  // namespace

extern "C" {

int64_t theria_ln_workspace_bytes(int64_t nt, int64_t R, int64_t D) {
  return nt * ln_ctas(R) * 2 * D * (int64_t)sizeof(float);
}

int theria_ln_fwd(const float* x, const float* w, const float* b, int64_t ldw, float* y,
                  int64_t nt, int64_t R, int64_t D, float eps, void* stream) {
  if (int e = ln_check(nt, R, D, ldw)) return e;
  if (nt == 0 || R == 0) return THERIA_OK;
  if (!x || !w || !b || !y) return THERIA_ERR_INVALID_ARG;
  return ln_dispatch<LnFwd>(D, x, w, b, ldw, y, nt, R, (int)D, eps, (cudaStream_t)stream);
}

int theria_ln_bwd(const float* x, const float* w, int64_t ldw, const float* gy, float* gx,
                  float* gw, float* gb, void* workspace, int64_t workspace_bytes,
                  int64_t nt, int64_t R, int64_t D, float eps, void* stream) {
  if (int e = ln_check(nt, R, D, ldw)) return e;
  if (nt == 0) return THERIA_OK;
  if (!x || !w || !gy || !gx || !gw || !gb) return THERIA_ERR_INVALID_ARG;
  if (R == 0) {
    cudaMemsetAsync(gw, 0, nt * D * sizeof(float), (cudaStream_t)stream);
    cudaMemsetAsync(gb, 0, nt * D * sizeof(float), (cudaStream_t)stream);
    return THERIA_OK;
  }
  if (!workspace || workspace_bytes < theria_ln_workspace_bytes(nt, R, D))
    return THERIA_ERR_WORKSPACE;
  return ln_dispatch<LnBwd>(D, x, w, ldw, gy, gx, gw, gb, (float*)workspace, nt, R, (int)D,
                            eps, (cudaStream_t)stream);
}

int theria_add_bias(const float* x, const float* b, int64_t ldb, const float* res, float* out,
                    int64_t nt, int64_t R, int64_t C, void* stream) {
  if (nt < 0 || R < 0 || C <= 0 || (ldb < C && ldb != 0)) return THERIA_ERR_INVALID_ARG;
  if (nt == 0 || R == 0) return THERIA_OK;
  if (!x || !b || !out) return THERIA_ERR_INVALID_ARG;
  const int64_t blocks = std::min<int64_t>((nt * R * C + 255) / 256, 148 * 16);
  ln::add_bias_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, b, ldb, res, out, nt,
                                                                           R, C);
  return launch_status();
}

int theria_chunk_sum(const float* x, float* out, int64_t nt, int64_t S, int64_t W,
                     void* stream) {
  if (nt < 0 || S < 0 || W < 0 || S > 65535) return THERIA_ERR_INVALID_ARG;
  if (nt == 0 || W == 0) return THERIA_OK;
  if (!x || !out) return THERIA_ERR_INVALID_ARG;
  if (S == 0) {
    cudaMemsetAsync(out, 0, nt * W * sizeof(float), (cudaStream_t)stream);
    return THERIA_OK;
  }
  const int64_t blocks = std::min<int64_t>((nt * W + 255) / 256, 148 * 16);
  ln::chunk_sum_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, out, nt, (int)S, W);
  return launch_status();
}

int theria_gelu_bwd2(const float* x, const float* gy, const float* u, float* dx, float* dgy,
                     int64_t n, void* stream) {
  if (n < 0) return THERIA_ERR_INVALID_ARG;
  if (n == 0) return THERIA_OK;
  if (!x || !gy || !u || !dx || !dgy) return THERIA_ERR_INVALID_ARG;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  ln::gelu_bwd2_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, gy, u, dx, dgy, n);
  return launch_status();
}

int64_t theria_rowsum_workspace_bytes(int64_t nt, int64_t R, int64_t C) {
  return nt * ((R + ln::ROWSUM_ROWS - 1) / ln::ROWSUM_ROWS) * C * (int64_t)sizeof(float);
}

int theria_rowsum(const float* x, float* out, void* workspace, int64_t workspace_bytes,
                  int64_t nt, int64_t R, int64_t C, void* stream) {
  if (nt < 0 || R < 0 || C <= 0) return THERIA_ERR_INVALID_ARG;
  const int64_t chunks = (R + ln::ROWSUM_ROWS - 1) / ln::ROWSUM_ROWS;
  if (nt > 2147483647ll || (C + 31) / 32 > 65535 || chunks > 65535 || C > 1024)
    return THERIA_ERR_UNSUPPORTED;
  if (nt == 0) return THERIA_OK;
  if (!x || !out) return THERIA_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (R == 0) {
    cudaMemsetAsync(out, 0, nt * C * sizeof(float), st);
    return THERIA_OK;
  }
  if (!workspace || workspace_bytes < theria_rowsum_workspace_bytes(nt, R, C))
    return THERIA_ERR_WORKSPACE;
  float* ws = (float*)workspace;
  dim3 grid((unsigned)nt, (unsigned)((C + 31) / 32), (unsigned)chunks);
  ln::rowsum_partial_kernel<<<grid, ln::WARPS * 32, 0, st>>>(x, ws, R, (int)C);
  if (int e = launch_status()) return e;
  ln::colsum_kernel<<<dim3((unsigned)nt, (unsigned)((C + 31) / 32)), ln::COLSUM_THREADS, 0, st>>>(
      ws, out, out, (int)chunks, 1, (int)C);
  return launch_status();
}

int theria_ln_bwd2(const float* x, const float* w, int64_t ldw, const float* gy,
                   const float* u, const float* a, int64_t lda, const float* c, int64_t ldc,
                   float* dx, float* dw, float* dgy, void* workspace, int64_t workspace_bytes,
                   int64_t nt, int64_t R, int64_t D, float eps, void* stream) {
  if (int e = ln_check(nt, R, D, ldw)) return e;
  if ((a && lda < D && lda != 0) || (c && ldc < D && ldc != 0)) return THERIA_ERR_INVALID_ARG;
  if (nt == 0) return THERIA_OK;
  if (!x || !w || !gy || !dx || !dw || !dgy) return THERIA_ERR_INVALID_ARG;
  if (R == 0) {
    cudaMemsetAsync(dw, 0, nt * D * sizeof(float), (cudaStream_t)stream);
    return THERIA_OK;
  }
  if (!workspace || workspace_bytes < theria_ln_workspace_bytes(nt, R, D))
    return THERIA_ERR_WORKSPACE;
  return ln_dispatch<LnBwd2>(D, x, w, ldw, gy, u, a, lda, c, ldc, dx, dw, dgy,
                             (float*)workspace, nt, R, (int)D, eps, (cudaStream_t)stream);
}

}  // extern "C"
