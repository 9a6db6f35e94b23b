// qrb200 -- row-block triangular solve X = M R^{-1} (R upper, non-unit).
//
// Replaces solve_triangular(R, M, upper=True, left=False) of reflection_no_reflectors.py:77.
// Each row of X depends only on the same row of M, so one CTA owns BMR full rows: they are
// loaded once into shared memory, solved column panel by column panel (GEMM against the
// already-solved columns, then a warp-per-row substitution with the 32x32 diagonal block),
// and written once.  HBM traffic is one read of M and one write of X; R is re-read from L2.
#pragma once
#include "qrb_common.cuh"

namespace qrb {

__host__ __device__ inline size_t trsm_smem_bytes(int bmr, int n) {
  return (size_t)bmr * (n + 1) * sizeof(float) + 32 * 33 * sizeof(float);
}

template <int BMR>
__global__ void __launch_bounds__(256) trsm_rows_kernel(const float* __restrict__ Mg,
                                                        const float* __restrict__ Rg,
                                                        float* __restrict__ Xg, int n) {
  extern __shared__ __align__(16) float sm[];
  const int ldx = n + 1;
  float* Xs = sm;                           // [BMR][n+1]
  float* Rs = sm + (size_t)BMR * ldx;       // [32][33]
  const int64_t b = blockIdx.y;
  const int r0 = blockIdx.x * BMR;
  const int rows = min(BMR, n - r0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* M = Mg + mat_off(b, n);
  const float* R = Rg + mat_off(b, n);
  float* X = Xg + mat_off(b, n);

  for (int idx = tid; idx < rows * n; idx += 256) {
    const int r = idx / n, c = idx - r * n;
    Xs[r * ldx + c] = M[(int64_t)(r0 + r) * n + c];
  }
  __syncthreads();

  constexpr int RPT = BMR / 8;  // rows per thread in the GEMM part (8 row groups of 32 lanes)
  for (int c0 = 0; c0 < n; c0 += 32) {
    const int cw = min(32, n - c0);
    // ---- X[:, c0:c0+cw] -= X[:, 0:c0] * R[0:c0, c0:c0+cw] ----
    float acc[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) acc[i] = 0.f;
    for (int kb = 0; kb < c0; kb += 32) {
      for (int idx = tid; idx < 32 * 32; idx += 256) {
        const int kk = idx >> 5, cc = idx & 31;
        Rs[kk * 33 + cc] = (cc < cw) ? R[(int64_t)(kb + kk) * n + c0 + cc] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int r = warp + 8 * i;
        if (r < rows) {
          const float* xr = Xs + r * ldx + kb;
          float t = acc[i];
#pragma unroll 8
          for (int kk = 0; kk < 32; ++kk) t = fmaf(xr[kk], Rs[kk * 33 + lane], t);
          acc[i] = t;
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = warp + 8 * i;
      if (r < rows && lane < cw) Xs[r * ldx + c0 + lane] -= acc[i];
    }
    // ---- diagonal block ----
    for (int idx = tid; idx < 32 * 32; idx += 256) {
      const int kk = idx >> 5, cc = idx & 31;
      Rs[kk * 33 + cc] = (kk < cw && cc < cw) ? R[(int64_t)(c0 + kk) * n + c0 + cc] : 0.f;
    }
    __syncthreads();
    for (int r = warp; r < rows; r += 8) {
      float v = (lane < cw) ? Xs[r * ldx + c0 + lane] : 0.f;
      for (int c = 0; c < cw; ++c) {
        float xc = 0.f;
        if (lane == c) { v = v / Rs[c * 33 + c]; }
        xc = __shfl_sync(0xffffffffu, v, c);
        if (lane > c) v = fmaf(-xc, Rs[c * 33 + lane], v);
      }
      if (lane < cw) Xs[r * ldx + c0 + lane] = v;
    }
    __syncthreads();
  }

  for (int idx = tid; idx < rows * n; idx += 256) {
    const int r = idx / n, c = idx - r * n;
    X[(int64_t)(r0 + r) * n + c] = Xs[r * ldx + c];
  }
}

}  // namespace qrb
