// Host side of the tensor-core kernels: TMA descriptor encoding and the
// shape rules that pick them.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace theria {
namespace tc {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).  Resolved once per process; thread-safe.
inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// TMA map of a contiguous [bh, rows, hd] 16-bit tensor, box {64, box_rows, 1},
// 128-byte swizzle, zero fill out of bounds (per (batch, head) slice, so a
// ragged last tile never reads the next head's rows).
inline bool make_map_3d(CUtensorMap* map, const void* base, int dtype, int64_t bh,
                        int64_t rows, int64_t hd, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  CUtensorMapDataType t =
      dtype == THERIA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)rows, (cuuint64_t)bh};
  cuuint64_t strides[2] = {(cuuint64_t)(hd * 2), (cuuint64_t)(rows * hd * 2)};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, t, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D fp32 map over [B*H, rows, hd] with box {32 floats (128 B), box_rows, 1}
// and 128-byte swizzle: the destination of bulk tensor reductions from a
// swizzled shared-memory stage.
inline bool make_map_3d_f32(CUtensorMap* map, void* base, int64_t bh, int64_t rows, int64_t hd,
                            uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)rows, (cuuint64_t)bh};
  cuuint64_t strides[2] = {(cuuint64_t)(hd * 4), (cuuint64_t)(rows * hd * 4)};
  cuuint32_t box[3] = {32, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The tensor-core kernels take 16-bit inputs with head dim 64 or 128 and
// sizes that fit TMA's 32-bit coordinates.
// Dtype and size conditions of the tensor-core kernels alone.
inline bool tc_shape_ok(int dtype, int64_t T, int64_t M, int64_t D, int64_t BH) {
  if (dtype != THERIA_BF16 && dtype != THERIA_F16) return false;
  if (D != 64 && D != 128) return false;
  return T < (1ll << 31) && M < (1ll << 31) && BH < 65536;
}

inline bool tc_eligible(int dtype, int64_t T, int64_t M, int64_t D, int64_t BH) {
  return tc_shape_ok(dtype, T, M, D, BH) && encode_fn() != nullptr;
}

}  // namespace tc
}  // namespace theria
