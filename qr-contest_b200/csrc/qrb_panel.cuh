// qrb200 -- panel elimination kernel (one CTA per matrix, panel resident in shared memory).
//
// One kernel template serves the three eliminations of the pipeline
// (reflection_no_reflectors.py):
//   PM_PIVOT : partial-pivot LU of A (torch.linalg.lu, :66).  Pivot = first row holding the
//              maximum |a| of the live column (getrf / i?amax semantics).  Rows never move in
//              HBM: the trailing block is kept "compact" (live rows at [k0,n) in current order)
//              and the unit-lower factor is written in ORIGINAL row order, i.e. the kernel
//              emits P*L directly -- the frame Q = P*Q_L (:81) then needs no permutation.
//   PM_CHOL  : unpivoted LU of the jittered Gram G + mu*I (:74-76) = L_G D L_G^T, emitting
//              the upper Cholesky rows R = D^{1/2} L_G^T (upper triangle of the R buffer),
//              the pivots D, L21 D^{1/2} (Cholesky trailing update), and what the L_G^{-1}
//              update needs (L11^{-1}, W = L21 L11^{-1}, the panel rows of L_G^{-1}); L_G^{-1}
//              itself accumulates in the strict lower triangle of the R buffer, so that
//              R^{-1} = L_G^{-T} D^{-1/2} is available without a triangular solve.  Only the
//              lower triangle of G is read (the diagonal block is mirrored in shared memory).
//   PM_CHART : the chart (:144-162): sign rule s_k = +1 iff |1-d| >= |1+d|, pivot 1 + |d|,
//              multipliers Y[i,k] = -s_k M[i,k] / piv, written straight into H's strict
//              lower triangle; tau_k = 2 / (1 + sum_{i>k} Y[i,k]^2) (:192).
// For PM_PIVOT and PM_CHART the kernel also emits W = L21 * L11^{-1} so that the trailing
// update is the single rank-w product  C22' = C22 - W * C12  (C12 = the panel rows' raw
// trailing columns), which equals the reference's "forward the panel rows, then
// M22 -= L21 U12" (:165-174) up to reassociation.
#pragma once
#include "qrb_common.cuh"
#include <float.h>
#include <limits.h>

// Phase timers for the test kit's profiling build only (off in the library).
#ifdef QRB_PANEL_TIMERS
#define QRB_PT(i)                                                         \
  do {                                                                    \
    __syncthreads();                                                      \
    if (threadIdx.x == 0 && blockIdx.x == 0) g_panel_timers[i] = clock64(); \
  } while (0)
#else
#define QRB_PT(i) do { } while (0)
#endif

namespace qrb {

enum PanelMode : int { PM_PIVOT = 0, PM_CHOL = 1, PM_CHART = 2 };

struct PanelArgs {
  int n, k0, w, ldw;
  const void* src;   // current trailing buffer: rows/cols [k0, n) valid (input dtype at k0 == 0)
  int* orig;         // PIVOT: [b][n] original row id of each current row
  int* srcmap;       // PIVOT: [b][n] out: new row -> old absolute row in src
  float* W;          // [b][n][ldw] out, rows [k0+w, n): W; CHOL also rows [k0, k0+w): L11^{-1}
  float* L;          // PIVOT: [b][n][n] out, P*L (original row order)
  float* R;          // CHOL: [b][n][n] out, upper rows [k0, k0+w) of R; strict lower rows
                     //       [k0, k0+w) of L_G^{-1} (columns < row), read back for k0 > 0
  float* D;          // CHOL: [b][n] out, pivots d_k (G = L_G D L_G^T)
  float* Wc;         // CHOL: [b][n][ldw] out, rows [k0+w, n): L21 D^{1/2}
  float* Bp;         // CHOL: [b][ldw][n] out, rows of L_G^{-1} [k0, k0+w) before the panel
                     //       (columns < k0+w, identity block included)
  int bp_ready;      // CHOL: Bp's columns < k0 were already written by the previous update
  float* mu;         // CHOL: [b] jitter, computed when k0 == 0
  int nmu;           // CHOL: diagonal entries in the jitter's mean (0 = n; the rectangular
                     //       entry point's zero-padded columns are left out of it)
  void* H;           // CHART: [b][n][n] out (output dtype), strict lower part
  void* tau;         // CHART: [b][n] out (output dtype)
  float* s;          // CHART: [b][n] out, signs
  int* info;         // [b]
  int info_bit;      // CHOL: bit to raise on a non-positive pivot
};

// Shared-memory bytes the panel kernel needs for an m-row, w-column panel.
__host__ __device__ inline size_t panel_smem_bytes(int m, int w) {
  return (size_t)m * (w + 1) * sizeof(float) + 3 * (size_t)m * sizeof(int) +
         (size_t)(w + 16) * sizeof(float) + 16 * sizeof(int);
}

template <int MODE, typename TIn, typename TOut>
__global__ void __launch_bounds__(256) panel_kernel(PanelArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int n = a.n, k0 = a.k0, w = a.w, m = n - k0, ldp = w + 1;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  float* P = sm;                                     // [m][ldp]
  int* lid = reinterpret_cast<int*>(P + (size_t)m * ldp);  // local row permutation
  int* oid = lid + m;                                // original ids (old order)
  int* nid = oid + m;                                // original ids (new order)
  float* dpiv = reinterpret_cast<float*>(nid + m);   // [w] pivots (CHOL) / signs (CHART)
  float* red_v = dpiv + w;                           // [8]
  float* red_x = red_v + 8;                          // [8]
  int* red_i = reinterpret_cast<int*>(red_x + 8);    // [8]
  int* s_pivrow = red_i + 8;
  __shared__ int s_flags;
  __shared__ float s_mu;

  const TIn* src = reinterpret_cast<const TIn*>(a.src) + mat_off(b, n);
  if (tid == 0) s_flags = 0;

  QRB_PT(0);
  // ---- jitter (CHOL): mu = 1e-7 * mean(diag G)  (reflection_no_reflectors.py:74) ----
  if (MODE == PM_CHOL) {
    if (k0 == 0) {
      float acc = 0.f;
      for (int i = tid; i < (a.nmu > 0 ? a.nmu : n); i += 256) acc += to_f32(src[(int64_t)i * n + i]);
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (lane == 0) red_x[warp] = acc;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < 8; ++i) t += red_x[i];
        s_mu = 1e-7f * (t / (float)(a.nmu > 0 ? a.nmu : n));
        a.mu[b] = s_mu;
      }
    } else if (tid == 0) {
      s_mu = a.mu[b];
    }
  }

  // ---- load the panel: rows [k0, n), columns [k0, k0 + w) ----
  for (int idx = tid; idx < m * w; idx += 256) {
    const int r = idx / w, c = idx - r * w;
    P[r * ldp + c] = to_f32(src[(int64_t)(k0 + r) * n + k0 + c]);
  }
  for (int r = tid; r < m; r += 256) lid[r] = r;
  __syncthreads();
  if (MODE == PM_CHOL) {
    // lower triangle only: mirror the diagonal block, add the jitter on the diagonal
    for (int idx = tid; idx < w * w; idx += 256) {
      const int r = idx / w, c = idx - r * w;
      if (r < c) P[r * ldp + c] = P[c * ldp + r];
    }
    __syncthreads();
    if (tid < w) P[tid * ldp + tid] += s_mu;
    __syncthreads();
  }

  QRB_PT(1);
  // ---- column-by-column elimination inside the panel ----
  for (int c = 0; c < w; ++c) {
    if (MODE == PM_PIVOT) {
      float bv = -1.f;
      int bi = INT_MAX;
      bool bad = false;
      for (int r = c + tid; r < m; r += 256) {
        const float x = P[r * ldp + c];
        const float v = fabsf(x);
        bad |= !isfinite(x);
        if (v > bv) { bv = v; bi = r; }
      }
      if (bad) atomicOr(&s_flags, INFO_NONFINITE_INPUT);
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, bv, o);
        const int oi = __shfl_down_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
      __syncthreads();
      if (tid == 0) {
        float v = red_v[0];
        int i0 = red_i[0];
        for (int q = 1; q < 8; ++q)
          if (red_v[q] > v || (red_v[q] == v && red_i[q] < i0)) { v = red_v[q]; i0 = red_i[q]; }
        *s_pivrow = (i0 == INT_MAX) ? c : i0;
      }
      __syncthreads();
      const int p = *s_pivrow;
      if (p != c) {
        for (int j = tid; j < w; j += 256) {
          const float t = P[c * ldp + j];
          P[c * ldp + j] = P[p * ldp + j];
          P[p * ldp + j] = t;
        }
        if (tid == 0) { const int t = lid[c]; lid[c] = lid[p]; lid[p] = t; }
      }
      __syncthreads();
    }

    const float pv = P[c * ldp + c];
    float scale = 1.f, piv = pv, sgn = 1.f;
    if (MODE == PM_PIVOT) {
      // getrf scales the column by the reciprocal pivot; an all-zero column is left as is
      scale = (pv != 0.f) ? 1.f / pv : 1.f;
      if (pv == 0.f && tid == 0) atomicOr(&s_flags, INFO_LU_ZERO_PIVOT);
    } else if (MODE == PM_CHOL) {
      if (!(pv > 0.f)) {
        if (tid == 0) atomicOr(&s_flags, a.info_bit);
        piv = 1.f;  // keep the arithmetic finite; the host reports the failure
      }
      if (tid == 0) dpiv[c] = piv;
    } else {  // PM_CHART
      const float pp = 1.f - pv, pm = 1.f + pv;
      sgn = (fabsf(pp) >= fabsf(pm)) ? 1.f : -1.f;
      piv = (sgn > 0.f) ? pp : pm;
      if (tid == 0) dpiv[c] = sgn;
    }

    for (int r = c + 1 + tid; r < m; r += 256) {
      float* row = P + r * ldp;
      float l;
      if (MODE == PM_PIVOT) l = row[c] * scale;
      else if (MODE == PM_CHOL) l = row[c] / piv;
      else l = (-sgn * row[c]) / piv;
      row[c] = l;
      const float* prow = P + c * ldp;
      for (int j = c + 1; j < w; ++j) row[j] = fmaf(-l, prow[j], row[j]);
    }
    __syncthreads();
  }

  int* info = a.info + b;

  QRB_PT(2);
  // ---- outputs ----
  if (MODE == PM_PIVOT) {
    int* orig = a.orig + b * n;
    for (int r = tid; r < m; r += 256) oid[r] = (k0 == 0) ? r : checked_row(orig[k0 + r], 0, n, info);
    __syncthreads();
    for (int r = tid; r < m; r += 256) {
      const int o = oid[checked_row(lid[r], 0, m, info)];
      nid[r] = o;
      orig[k0 + r] = o;
      a.srcmap[b * n + k0 + r] = k0 + lid[r];
    }
    __syncthreads();
    // P*L in original row order: row nid[p] gets columns [k0, k0+w) of L
    float* L = a.L + mat_off(b, n);
    for (int p = warp; p < m; p += 8) {
      float* Lrow = L + (int64_t)nid[p] * n;
      for (int c = lane; c < w; c += 32)
        Lrow[k0 + c] = (p > c) ? P[p * ldp + c] : (p == c ? 1.f : 0.f);
      if (p < w)  // pivot rows are final: zero the rest of their L row
        for (int j = k0 + w + lane; j < n; j += 32) Lrow[j] = 0.f;
    }
  } else if (MODE == PM_CHOL) {
    float* R = a.R + mat_off(b, n);
    for (int c = 0; c < w; ++c) {
      const float sd = sqrtf(dpiv[c]);
      float* Rrow = R + (int64_t)(k0 + c) * n + k0;
      for (int p = c + tid; p < m; p += 256)
        Rrow[p] = (p == c) ? sd : sd * P[p * ldp + c];
    }
    for (int c = tid; c < w; c += 256) a.D[b * n + k0 + c] = dpiv[c];
    // raw panel rows of L_G^{-1} before this panel (identity block included), columns < k1
    for (int c = warp; c < w; c += 8) {
      float* bp = a.Bp + ((int64_t)b * a.ldw + c) * n;
      const float* rl = R + (int64_t)(k0 + c) * n;
      for (int j = (a.bp_ready ? k0 : 0) + lane; j < k0 + w; j += 32)
        bp[j] = (j < k0) ? rl[j] : ((j == k0 + c) ? 1.f : 0.f);
    }
    // L11^{-1} (unit lower) into rows [k0, k0+w) of the W buffer
    if (tid < w) {
      const int c = tid;
      float* Wl = a.W + (int64_t)b * n * a.ldw;
      float x[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float v = (i == c) ? 1.f : 0.f;
        if (i > c && i < w) {
#pragma unroll
          for (int l = 0; l < 32; ++l)
            if (l >= c && l < i) v = fmaf(-P[i * ldp + l], x[l], v);
        }
        x[i] = v;
        if (i < w) Wl[(int64_t)(k0 + i) * a.ldw + c] = v;
      }
    }
    // L21 D^{1/2} (rows [k0+w, n)) for the Cholesky trailing update
    if (k0 + w < n) {
      float* Wc = a.Wc + (int64_t)b * n * a.ldw;
      for (int p = w + warp; p < m; p += 8)
        for (int c = lane; c < w; c += 32)
          Wc[(int64_t)(k0 + p) * a.ldw + c] = P[p * ldp + c] * sqrtf(dpiv[c]);
    }
  } else {  // PM_CHART
    TOut* H = reinterpret_cast<TOut*>(a.H) + mat_off(b, n);
    for (int p = warp; p < m; p += 8) {
      TOut* Hrow = H + (int64_t)(k0 + p) * n + k0;
      for (int c = lane; c < w && c < p; c += 32) Hrow[c] = from_f32<TOut>(P[p * ldp + c]);
    }
    TOut* tau = reinterpret_cast<TOut*>(a.tau) + b * n;
    for (int c = warp; c < w; c += 8) {
      float acc = 0.f;
      for (int p = c + 1 + lane; p < m; p += 32) {
        const float y = P[p * ldp + c];
        acc = fmaf(y, y, acc);
      }
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        tau[k0 + c] = from_f32<TOut>(2.f / (acc + 1.f));
        a.s[b * n + k0 + c] = dpiv[c];
      }
    }
  }

  QRB_PT(3);
  // ---- W = L21 * L11^{-1} for the trailing update (PIVOT, CHART; CHOL: of L_G^{-1}) ----
  if (k0 + w < n) {
    __syncthreads();
    for (int p = w + tid; p < m; p += 256) {
      float* row = P + p * ldp;
      for (int j = w - 1; j >= 0; --j) {
        float acc = row[j];
        for (int i = j + 1; i < w; ++i) acc = fmaf(-row[i], P[i * ldp + j], acc);
        row[j] = acc;
      }
    }
    __syncthreads();
    float* W = a.W + (int64_t)b * n * a.ldw;
    for (int p = w + warp; p < m; p += 8)
      for (int c = lane; c < w; c += 32) W[(int64_t)(k0 + p) * a.ldw + c] = P[p * ldp + c];
  }

  QRB_PT(4);
  __syncthreads();
  if (tid == 0 && s_flags) atomicOr(info, s_flags);
}

}  // namespace qrb
