// qrb200 -- host-side TMA tensor-map encoding for the batched (b, n, n) float32 buffers.
// The driver entry point is fetched through the runtime (no libcuda link dependency).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

namespace qrb {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Map over `batch` row-major n x n float32 matrices at `base`, box {32 columns, box_rows rows},
// 128-byte swizzle, zero fill out of range.  Requires n % 4 == 0 and a 16-byte aligned base.
inline bool encode_batched(CUtensorMap* map, const void* base, int n, int64_t batch,
                           int box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (n & 3) || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)n, (cuuint64_t)n, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)n * 4, (cuuint64_t)n * n * 4};
  const cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Map over `batch` row-major n x n float32 matrices read as k-major operand tiles: box
// {128 columns, 32 rows}, no swizzle (512-byte rows in shared memory), zero fill out of range.
inline bool encode_batched_wide(CUtensorMap* map, const void* base, int n, int64_t batch) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (n & 3) || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)n, (cuuint64_t)n, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)n * 4, (cuuint64_t)n * n * 4};
  const cuuint32_t box[3] = {128, 32, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// General 3-D float32 map: dims {d0 (contiguous), d1, d2}, byte strides s1 (between d1 rows)
// and s2 (between d2 planes), box {b0, b1, 1}; 128-byte swizzle when b0 * 4 == 128, none
// otherwise; zero fill out of range.  Requires a 16-byte aligned base and 16-byte strides.
inline bool encode_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (s1 & 15) || (s2 & 15)) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {b0, b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            b0 * 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace qrb
