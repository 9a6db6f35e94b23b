// qrb200 -- warp-per-matrix QR for n <= 32: the whole pipeline of one matrix in one warp's
// registers.
//
// Lane r holds row r of the working matrix in 32 registers (rows >= n are idle lanes).  Every
// loop over columns is unrolled with rectangular bounds and a guard (triangular bounds keep
// nvcc from unrolling the nest fully, which moves a row array to local memory), so all
// register indices are static.  Column broadcasts are warp shuffles, the pivot search is two
// redux.sync reductions, and there is no CTA barrier anywhere: the warps of a CTA are
// independent matrices (kWarpWPB per CTA).  Each warp also owns two 32 x 33 float32
// shared-memory tiles for the stages that read columns: the Gram, the triangular solve and
// the closure.
//
// Same stages and the same float32 operation order as the one-CTA-per-matrix kernel
// (qrb_small.cuh), per reflection_no_reflectors.py:
//   I-a  LU with partial pivoting (:66, getrf): pivot = the live row with the largest |a|,
//        ties to the lowest current position (rows are pivoted logically: each lane tracks the
//        position its row would hold after getrf's swaps); multipliers a * (1 / pivot)
//   I-b  CholeskyQR2 on P*L (:68-81): G = X^T X summed over rows in order, mu = 1e-7 mean
//        diag(G) added to each pivot, right-looking Cholesky on the lower triangle, then
//        X <- X R^{-1} by forward substitution with the reciprocal diagonal
//   III  chart (:86-176): sign rule s_k = +1 iff |1 - d| >= |1 + d|, multipliers
//        -s_k m / (1 + |d|) stored below the diagonal, tau_k = 2 / (1 + sum y^2) (:192)
//   II   closure (:186, :195): H_ij = s_i (Q^T A)_ij for j >= i
// Optional explicit Q = frame * diag(s) (householder_product(H, tau)).
#pragma once
#include "qrb_common.cuh"

namespace qrb {

constexpr int kWarpMaxN = 32;
constexpr int kWarpWPB = 4;               // matrices (warps) per CTA
constexpr int kWarpLD = kWarpMaxN + 1;    // padded shared-memory row
constexpr int kWarpTile = kWarpMaxN * kWarpLD;

template <typename T>
__global__ void __launch_bounds__(32 * kWarpWPB)
    warp_qr_kernel(const T* __restrict__ Ag, T* __restrict__ Hg, T* __restrict__ taug,
                   int* __restrict__ info, int n, int64_t batch, T* __restrict__ Qg,
                   int nmu) {
  constexpr int N = kWarpMaxN, LD = kWarpLD;
  constexpr unsigned FULL = 0xffffffffu;
  __shared__ float tiles[kWarpWPB][2][kWarpTile];
  __shared__ float sgn_s[kWarpWPB][N];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t b = (int64_t)blockIdx.x * kWarpWPB + w;
  if (b >= batch) return;  // whole warps only: no CTA-wide barrier follows
  float* S0 = tiles[w][0];
  float* S1 = tiles[w][1];
  float* sg = sgn_s[w];
  const T* A = Ag + mat_off(b, n);
  const bool act = lane < n;
  int flags = 0;

  // ---- load A coalesced into S1 (row-major, padded), then each lane takes its row ----
  for (int r = 0; r < n; ++r)
    if (act) S1[r * LD + lane] = to_f32(A[(int64_t)r * n + lane]);
  __syncwarp();
  float a[N];
#pragma unroll
  for (int c = 0; c < N; ++c) a[c] = (act && c < n) ? S1[lane * LD + c] : 0.f;

  // ---- I-a: LU with partial pivoting, rows pivoted logically ----
  bool live = act;
  int pos = lane;   // position of this row in getrf's swapped order
  int step = N;     // the elimination step at which this row became the pivot row
#pragma unroll
  for (int k = 0; k < N; ++k) {
    if (k < n) {
      const float v = a[k];
      if (live && !isfinite(v)) flags |= INFO_NONFINITE_INPUT;
      // largest |a| among live rows (NaN counts as 0, as a NaN never wins a > compare)
      const unsigned key = (live && !isnan(v)) ? (__float_as_uint(v) & 0x7fffffffu) : 0u;
      const unsigned kmax = __reduce_max_sync(FULL, key);
      const bool cand = live && key == kmax;
      const unsigned pmin = __reduce_min_sync(FULL, cand ? (unsigned)pos : 0xffffffffu);
      const int p = __ffs(__ballot_sync(FULL, cand && (unsigned)pos == pmin)) - 1;
      // the row at position k moves to the pivot's old position (getrf's swap)
      if (live && pos == k) pos = (int)pmin;
      const float pv = __shfl_sync(FULL, v, p);
      if (lane == p) { live = false; pos = k; step = k; }
      if (pv == 0.f) flags |= INFO_LU_ZERO_PIVOT;
      const float inv = (pv != 0.f) ? 1.f / pv : 1.f;
      const float l = v * inv;
#pragma unroll
      for (int c = 0; c < N; ++c) {
        if (c > k && c < n) {
          const float pc = __shfl_sync(FULL, a[c], p);
          if (live) a[c] = fmaf(-l, pc, a[c]);
        }
      }
      if (live) a[k] = l;
    }
  }
  // P*L in original row order: this lane's row of L
  float x[N];
#pragma unroll
  for (int c = 0; c < N; ++c) x[c] = !act ? 0.f : (c < step ? a[c] : (c == step ? 1.f : 0.f));

  // ---- I-b..d: two CholeskyQR passes, X <- X R^{-1} ----
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
    // stage X (rows) in S0; lane i builds row i of G = X^T X (lower part, c <= i)
#pragma unroll
    for (int c = 0; c < N; ++c)
      if (c < n && act) S0[lane * LD + c] = x[c];
    __syncwarp();
    float g[N];
#pragma unroll
    for (int c = 0; c < N; ++c) g[c] = 0.f;
    for (int r = 0; r < n; ++r) {
      const float xi = S0[r * LD + lane];
#pragma unroll
      for (int c = 0; c < N; ++c)
        if (c <= lane) g[c] = fmaf(xi, S0[r * LD + c], g[c]);
    }
    // mu = 1e-7 mean(diag G) (:74) over the first nmu diagonal entries (all n unless the
    // rectangular entry point padded the matrix with zero columns)
    float dsum = 0.f;
#pragma unroll
    for (int c = 0; c < N; ++c)
      if (c == lane && lane < nmu) dsum = g[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dsum += __shfl_down_sync(FULL, dsum, o);
    const float mu = 1e-7f * (__shfl_sync(FULL, dsum, 0) / (float)nmu);
    // right-looking Cholesky on the lower triangle: after step k, lane i > k holds
    // R[k][i] in g[k]; the diagonal's reciprocal goes to rinv_own of lane k
    float rinv_own = 0.f;
#pragma unroll
    for (int k = 0; k < N; ++k) {
      if (k < n) {
        float d = __shfl_sync(FULL, g[k], k) + mu;
        if (!(d > 0.f)) {
          flags |= (pass == 0 ? INFO_CHOL1_NOT_PD : INFO_CHOL2_NOT_PD);
          d = 1.f;
        }
        const float rinv = 1.f / sqrtf(d);
        if (lane == k) rinv_own = rinv;
        const float li = g[k] * rinv;  // lane i > k: R[k][i]
#pragma unroll
        for (int j = 0; j < N; ++j) {
          if (j > k && j < n) {
            const float cj = __shfl_sync(FULL, li, j);
            if (lane > k && j <= lane) g[j] = fmaf(-li, cj, g[j]);
          }
        }
        if (lane > k) g[k] = li;
      }
    }
    // stage R for the solve: S0[c][k] = R[k][c] (c > k), S0[k][k] = 1 / R[k][k]
    __syncwarp();
#pragma unroll
    for (int k = 0; k < N; ++k)
      if (k < n && act && k <= lane) S0[lane * LD + k] = (k == lane) ? rinv_own : g[k];
    __syncwarp();
    // X <- X R^{-1}, one row per lane
#pragma unroll
    for (int k = 0; k < N; ++k) {
      if (k < n) {
        const float xk = x[k] * S0[k * LD + k];
#pragma unroll
        for (int c = 0; c < N; ++c)
          if (c > k && c < n) x[c] = fmaf(-xk, S0[c * LD + k], x[c]);
        x[k] = xk;
      }
    }
    __syncwarp();
  }

  // ---- III: chart on a copy of the frame, one row per lane ----
  float m[N];
#pragma unroll
  for (int c = 0; c < N; ++c) m[c] = x[c];
#pragma unroll
  for (int k = 0; k < N; ++k) {
    if (k < n) {
      const float dk = __shfl_sync(FULL, m[k], k);
      const float pp = 1.f - dk, pm = 1.f + dk;
      const float sk = (fabsf(pp) >= fabsf(pm)) ? 1.f : -1.f;
      const float piv = (sk > 0.f) ? pp : pm;
      if (lane == 0) sg[k] = sk;
      const bool below = act && lane > k;
      const float y = (-sk * m[k]) / piv;  // Y[lane][k] (:158)
#pragma unroll
      for (int c = 0; c < N; ++c) {
        if (c > k && c < n) {
          const float gk = __shfl_sync(FULL, m[c], k);
          if (below) m[c] = fmaf(-y, gk, m[c]);
        }
      }
      if (below) m[k] = y;
    }
  }

  // ---- II: closure H_ij = s_i (Q^T A)_ij, j >= i; Y below the diagonal; tau ----
  // S0 <- frame rows; S1 still holds A.  Lane j builds column j of Q^T A.
#pragma unroll
  for (int c = 0; c < N; ++c)
    if (c < n && act) S0[lane * LD + c] = x[c];
  __syncwarp();
  float acc[N];
#pragma unroll
  for (int i = 0; i < N; ++i) acc[i] = 0.f;
  for (int r = 0; r < n; ++r) {
    const float arj = act ? S1[r * LD + lane] : 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i <= lane) acc[i] = fmaf(S0[r * LD + i], arj, acc[i]);
  }
  __syncwarp();
  // S1 <- Y (rows, strictly lower part); lane k sums column k for tau
#pragma unroll
  for (int c = 0; c < N; ++c)
    if (c < n && act) S1[lane * LD + c] = (c < lane) ? m[c] : 0.f;
  __syncwarp();
  T* H = Hg + mat_off(b, n);
  float tsum = 0.f;
  for (int r = 0; r < n; ++r) {
    const float yv = act ? S1[r * LD + lane] : 0.f;
    tsum = fmaf(yv, yv, tsum);
  }
  if (act) taug[b * n + lane] = from_f32<T>(2.f / (tsum + 1.f));
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n && act)
      H[(int64_t)i * n + lane] = from_f32<T>(lane >= i ? sg[i] * acc[i] : S1[i * LD + lane]);
  if (Qg) {  // explicit Q = frame * diag(s); the frame is still in S0
    T* Q = Qg + mat_off(b, n);
    const float sj = act ? sg[lane] : 0.f;
    for (int r = 0; r < n; ++r)
      if (act) Q[(int64_t)r * n + lane] = from_f32<T>(S0[r * LD + lane] * sj);
  }
  flags = __reduce_or_sync(FULL, flags);
  if (lane == 0) info[b] = flags;
}

}  // namespace qrb
