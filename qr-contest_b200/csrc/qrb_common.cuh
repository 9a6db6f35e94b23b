// qrb200 -- shared device helpers for the batched square QR kernels (sm_100a).
//
// Conventions used by every kernel in this library:
//   * one matrix = n x n, row-major, contiguous; a batch is b such matrices back to back
//     (matrix stride n*n elements).  Working buffers are float32 with the same layout.
//   * grid.z (or grid.x for one-CTA-per-matrix kernels) indexes the matrix in the batch.
//   * per-matrix status words (int32) collect INFO_* bits; no kernel traps or asserts.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace qrb {

#ifdef QRB_PANEL_TIMERS
// phase-timer slots of the test kit's profiling build (off in the library)
__device__ long long g_panel_timers[8];
#endif

enum Dtype : int { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

// Per-matrix status bits written into info[b] (0 = clean).
enum InfoBits : int {
  INFO_NONFINITE_INPUT = 1,   // a NaN/Inf reached a pivot (LU stage)
  INFO_CHOL1_NOT_PD = 2,      // first CholeskyQR pass: Gram pivot <= 0 after jitter
  INFO_CHOL2_NOT_PD = 4,      // second pass
  INFO_LU_ZERO_PIVOT = 8,     // an exactly singular column (informational, like getrf info>0)
  INFO_DEVICE_TIMEOUT = 16,   // a bounded in-kernel wait gave up (never expected)
  INFO_BOUNDS = 32,           // bounds-check build: a pivot-map row index was out of range
};

// Row indices read from the LU's pivot maps (srcmap, orig, the panels' position maps) are the
// only data-dependent indices of the pipeline.  The bounds-check build (-DQRB_BOUNDS_CHECK,
// libqrb200_checked.so) tests each against its range; an index outside it raises INFO_BOUNDS
// in the matrix's info word and is replaced by `lo`, so the access stays inside the buffer and
// nothing traps.  In the regular build this is the identity.
__device__ __forceinline__ int checked_row(int r, int lo, int hi, int* info) {
#ifdef QRB_BOUNDS_CHECK
  if (r < lo || r >= hi) {
    if (info) atomicOr(info, INFO_BOUNDS);
    return lo;
  }
#endif
  return r;
}

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ int64_t mat_off(int64_t b, int n) { return b * (int64_t)n * n; }

}  // namespace qrb
