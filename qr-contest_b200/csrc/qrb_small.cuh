// qrb200 -- fused small-n QR: the whole pipeline for one matrix in one CTA's shared memory.
//
// For small n every stage of reflection_no_reflectors.py runs in a single kernel launch, one
// CTA per matrix, with three padded n x (n+1) float32 arrays in shared memory and no global
// workspace: the input is loaded once with 128-bit loads, H and tau are written once.
//   M : LU work array (getrf, :66), later the closure's copy of A (:186)
//   X : P*L (rows in original order), then Q1, then the frame Q (CholeskyQR2, :68-81)
//   G : Gram / Cholesky factor of each pass (:73-76), then the chart's working copy (:86-176)
// Work is mapped warp-per-row with lanes across columns (no index division, conflict-free
// shared-memory rows); the triangular solves X <- X R^{-1} need no block barrier at all
// (rows are independent; x_k is broadcast within the warp by a shuffle).  Unblocked forms of
// the same eliminations as the large-n path: the LU scales by the reciprocal pivot (getrf),
// the Cholesky is potf2's right-looking form, the chart divides by 1 + |d| (:158).
#pragma once
#include "qrb_common.cuh"
#include "qrb_panel.cuh"  // QRB_PT phase timers (test kit build)
#include <limits.h>

namespace qrb {

template <int NMAX, int NT>
__host__ __device__ inline size_t small_smem_bytes() {
  return (3 * (size_t)NMAX * (NMAX + 1) + 4 * NMAX + (NT / 32) * NMAX + 64) * sizeof(float);
}

template <int NMAX, int NT, typename T>
__global__ void __launch_bounds__(NT) small_qr_kernel(const T* __restrict__ Ag, T* __restrict__ Hg,
                                                      T* __restrict__ taug, int* __restrict__ info,
                                                      int n, T* __restrict__ Qg = nullptr,
                                                      int nmu = 0) {
  constexpr int LD = NMAX + 1;
  constexpr int NW = NT / 32;
  constexpr int CPL = (NMAX + 31) / 32;  // columns per lane
  extern __shared__ __align__(16) float sm[];
  float* M = sm;
  float* X = M + NMAX * LD;
  float* G = X + NMAX * LD;
  float* colk = G + NMAX * LD;        // [NMAX]
  float* sgn = colk + NMAX;            // [NMAX]
  float* rdg = sgn + NMAX;             // [NMAX] 1 / R[k][k] of the current pass
  int* perm = reinterpret_cast<int*>(rdg + NMAX);    // [NMAX]
  float* tpart = reinterpret_cast<float*>(perm + NMAX);  // [NW][NMAX] chart tau partials
  __shared__ int s_flags;
  __shared__ float s_f;

  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const T* A = Ag + mat_off(b, n);
  if (tid == 0) s_flags = 0;

  auto load_A = [&](float* dst) {
    const int nn = n * n;
    if (sizeof(T) == 4 && (nn & 3) == 0 && ((reinterpret_cast<uintptr_t>(A) & 15) == 0)) {
      const float4* A4 = reinterpret_cast<const float4*>(A);
      for (int q = tid; q < (nn >> 2); q += NT) {
        const float4 v = __ldg(A4 + q);
        const int e = q << 2;
        const float t[4] = {v.x, v.y, v.z, v.w};
        int r = e / n, c = e - r * n;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          dst[r * LD + c] = t[u];
          if (++c == n) { c = 0; ++r; }
        }
      }
    } else {
      for (int r = warp; r < n; r += NW)
        for (int c = lane; c < n; c += 32) dst[r * LD + c] = to_f32(A[(int64_t)r * n + c]);
    }
  };

  QRB_PT(0);
  load_A(M);
  for (int i = tid; i < n; i += NT) perm[i] = i;
  __syncthreads();

  // ---- I-a: LU with partial pivoting (getrf order, rows swapped in shared memory) ----
  for (int k = 0; k < n; ++k) {
    // every warp finds the pivot itself (first maximal |a| at or below the diagonal)
    float bv = -1.f;
    int bi = INT_MAX;
    bool bad = false;
    for (int r = k + lane; r < n; r += 32) {
      const float x = M[r * LD + k];
      bad |= !isfinite(x);
      const float v = fabsf(x);
      if (v > bv) { bv = v; bi = r; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int p = (bi == INT_MAX) ? k : bi;
    const bool anybad = __any_sync(0xffffffffu, bad);  // every lane votes
    if (tid == 0 && anybad) s_flags |= INFO_NONFINITE_INPUT;
    if (p != k) {
      __syncthreads();  // every warp has read column k before the swap
      if (warp == 0) {
        for (int c = lane; c < n; c += 32) {
          const float t = M[k * LD + c];
          M[k * LD + c] = M[p * LD + c];
          M[p * LD + c] = t;
        }
        if (lane == 0) { const int t = perm[k]; perm[k] = perm[p]; perm[p] = t; }
      }
      __syncthreads();
    }
    const float pv = M[k * LD + k];
    const float inv = (pv != 0.f) ? 1.f / pv : 1.f;
    if (pv == 0.f && tid == 0) s_flags |= INFO_LU_ZERO_PIVOT;
    // rows r, r + NW, r + 2NW, r + 3NW per warp iteration: independent loads overlap
    for (int r = k + 1 + warp; r < n; r += 4 * NW) {
      float l[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int rr = r + u * NW;
        l[u] = (rr < n) ? M[rr * LD + k] * inv : 0.f;  // read by every lane before lane 0 stores
      }
      for (int c = k + 1 + lane; c < n; c += 32) {
        const float pk = M[k * LD + c];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int rr = r + u * NW;
          if (rr < n) M[rr * LD + c] = fmaf(-l[u], pk, M[rr * LD + c]);
        }
      }
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (r + u * NW < n) M[(r + u * NW) * LD + k] = l[u];
      }
    }
    __syncthreads();
  }
  // P*L in original row order: X[perm[j]][c] = L[j][c]
  for (int j = warp; j < n; j += NW) {
    float* dst = X + perm[j] * LD;
    for (int c = lane; c < n; c += 32) dst[c] = (c < j) ? M[j * LD + c] : (c == j ? 1.f : 0.f);
  }
  __syncthreads();

  QRB_PT(1);
  // ---- I-b..d: two CholeskyQR passes, X <- X R^{-1} in place ----
  for (int pass = 0; pass < 2; ++pass) {
    // G = X^T X, lower triangle: warp per output row a, lanes over columns c <= a
    for (int a = warp; a < n; a += NW) {
      float acc[CPL];
#pragma unroll
      for (int q = 0; q < CPL; ++q) acc[q] = 0.f;
      for (int r = 0; r < n; ++r) {
        const float xa = X[r * LD + a];
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = lane + 32 * q;
          if (c <= a) acc[q] = fmaf(xa, X[r * LD + c], acc[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = lane + 32 * q;
        if (c <= a) G[a * LD + c] = acc[q];
      }
    }
    __syncthreads();
    if (pass == 0) QRB_PT(2);
    if (warp == 0) {  // mu = 1e-7 mean(diag G)  (:74)
      float acc = 0.f;
      const int nm = nmu > 0 ? nmu : n;  // the rectangular entry point's padding is left out
      for (int i = lane; i < nm; i += 32) acc += G[i * LD + i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (lane == 0) s_f = 1e-7f * (acc / (float)nm);
    }
    __syncthreads();
    // Cholesky (potf2, right-looking on the lower triangle): column k of G becomes R[k][k..]
    for (int k = 0; k < n; ++k) {
      float d = G[k * LD + k] + s_f;
      if (!(d > 0.f)) {
        if (tid == 0) s_flags |= (pass == 0 ? INFO_CHOL1_NOT_PD : INFO_CHOL2_NOT_PD);
        d = 1.f;
      }
      const float r = sqrtf(d), rinv = 1.f / r;
      for (int i = k + 1 + tid; i < n; i += NT) colk[i] = G[i * LD + k] * rinv;
      __syncthreads();
      if (tid == 0) rdg[k] = rinv;
      for (int i = k + 1 + warp; i < n; i += 4 * NW) {
        float li[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) li[u] = (i + u * NW < n) ? colk[i + u * NW] : 0.f;
        const int ilast = min(n - 1, i + 3 * NW);
        for (int j = k + 1 + lane; j <= ilast; j += 32) {
          const float cj = colk[j];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int ii = i + u * NW;
            if (ii < n && j <= ii) G[ii * LD + j] = fmaf(-li[u], cj, G[ii * LD + j]);
          }
        }
        if (lane == 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (i + u * NW < n) G[(i + u * NW) * LD + k] = li[u];
        }
      }
      __syncthreads();
    }
    if (pass == 0) QRB_PT(3);
    // X <- X R^{-1} with R[k][c] = G[c][k] (c > k), 1/R[k][k] = rdg[k]: every warp owns
    // whole rows (two at a time, interleaved); x_k is broadcast by one shuffle per step,
    // with branch-free selects so the serial chain stays short; no block barrier
    for (int r0 = warp * 2; r0 < n; r0 += 2 * NW) {
      const int r1 = r0 + 1;
      float x0[CPL], x1[CPL];
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = lane + 32 * q;
        x0[q] = (c < n) ? X[r0 * LD + c] : 0.f;
        x1[q] = (c < n && r1 < n) ? X[r1 * LD + c] : 0.f;
      }
      for (int k = 0; k < n; ++k) {
        const int qk = k >> 5, lk = k & 31;
        float s0 = x0[0], s1 = x1[0];
#pragma unroll
        for (int q = 1; q < CPL; ++q) {
          s0 = (q == qk) ? x0[q] : s0;
          s1 = (q == qk) ? x1[q] : s1;
        }
        const float ri = rdg[k];
        const float xk0 = __shfl_sync(0xffffffffu, s0, lk) * ri;
        const float xk1 = __shfl_sync(0xffffffffu, s1, lk) * ri;
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c = lane + 32 * q;
          const float rkc = (c > k && c < n) ? G[c * LD + k] : 0.f;
          x0[q] = (c == k) ? xk0 : fmaf(-xk0, rkc, x0[q]);
          x1[q] = (c == k) ? xk1 : fmaf(-xk1, rkc, x1[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = lane + 32 * q;
        if (c < n) {
          X[r0 * LD + c] = x0[q];
          if (r1 < n) X[r1 * LD + c] = x1[q];
        }
      }
    }
    __syncthreads();
    if (pass == 0) QRB_PT(4);
  }

  // ---- III: chart on a copy of Q (in G) ----
  for (int r = warp; r < n; r += NW)
    for (int c = lane; c < n; c += 32) G[r * LD + c] = X[r * LD + c];
  for (int i = tid; i < NW * NMAX; i += NT) tpart[i] = 0.f;
  __syncthreads();
  for (int k = 0; k < n; ++k) {
    const float dk = G[k * LD + k];
    const float pp = 1.f - dk, pm = 1.f + dk;
    const float sk = (fabsf(pp) >= fabsf(pm)) ? 1.f : -1.f;
    const float piv = (sk > 0.f) ? pp : pm;
    if (tid == 0) sgn[k] = sk;
    float part = 0.f;
    for (int r = k + 1 + warp; r < n; r += 4 * NW) {
      float y[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int rr = r + u * NW;
        y[u] = (rr < n) ? (-sk * G[rr * LD + k]) / piv : 0.f;  // Y[rr][k] (:158)
        part = fmaf(y[u], y[u], part);
      }
      for (int c = k + 1 + lane; c < n; c += 32) {
        const float gk = G[k * LD + c];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int rr = r + u * NW;
          if (rr < n) G[rr * LD + c] = fmaf(-y[u], gk, G[rr * LD + c]);
        }
      }
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (r + u * NW < n) G[(r + u * NW) * LD + k] = y[u];
      }
    }
    if (lane == 0) tpart[warp * NMAX + k] = part;
    __syncthreads();
  }

  QRB_PT(5);
  // ---- II: closure H_ij = s_i (Q^T A)_ij (j >= i), Y below the diagonal; tau ----
  load_A(M);
  __syncthreads();
  T* H = Hg + mat_off(b, n);
  for (int i = warp; i < n; i += NW) {
    float acc[CPL];
#pragma unroll
    for (int q = 0; q < CPL; ++q) acc[q] = 0.f;
    for (int r = 0; r < n; ++r) {
      const float qi = X[r * LD + i];
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = lane + 32 * q;
        if (c >= i && c < n) acc[q] = fmaf(qi, M[r * LD + c], acc[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = lane + 32 * q;
      if (c < n) H[(int64_t)i * n + c] = from_f32<T>(c >= i ? sgn[i] * acc[q] : G[i * LD + c]);
    }
  }
  for (int k = tid; k < n; k += NT) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) acc += tpart[w * NMAX + k];
    taug[b * n + k] = from_f32<T>(2.f / (acc + 1.f));
  }
  if (Qg) {  // explicit Q = householder_product(H, tau) = frame * diag(s)
    T* Q = Qg + mat_off(b, n);
    for (int r = warp; r < n; r += NW)
      for (int c = lane; c < n; c += 32) Q[(int64_t)r * n + c] = from_f32<T>(X[r * LD + c] * sgn[c]);
  }
  QRB_PT(6);
  __syncthreads();
  if (tid == 0) info[b] = s_flags;
}

}  // namespace qrb
