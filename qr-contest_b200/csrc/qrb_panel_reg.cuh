// qrb200 -- register-resident panel elimination (panels of at most 512 rows x 32 columns).
//
// Same contract and outputs as panel_kernel (qrb_panel.cuh) -- PM_PIVOT / PM_CHOL / PM_CHART --
// but each thread keeps RPT whole panel rows in registers (row r = tid + 256 q), so a column
// step costs a few shuffles and one or two barriers instead of shared-memory round trips:
//   PM_PIVOT : the pivot is chosen among the live rows by (max |a|, then lowest CURRENT
//              position), exactly getrf's choice.  Rows never move: a position <-> row map in
//              shared memory replays getrf's row swaps, so ties and the final row order match
//              the swapping algorithm.  The winner publishes its row; 2 barriers per column.
//   PM_CHOL  : the pivot row's entries right of the diagonal are read from the symmetric
//              column (U[c][j] = S[j][c]), so only the lower triangle of G is ever used and
//              each row owner publishes one value; 1 barrier per column.
//   PM_CHART : the owner of row c publishes it; 1 barrier per column.
// W = L21 L11^{-1} and L11^{-1} are computed in registers (right-looking substitution).
#pragma once
#include <type_traits>

#include "qrb_panel.cuh"

namespace qrb {

constexpr int PR_W = 32;  // maximum panel width handled here

template <typename T>
__device__ __forceinline__ void load_row32(const T* p, int w, bool vec, float (&x)[PR_W]) {
  if (vec && w == PR_W) {
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int c = 0; c < PR_W; c += 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p + c));
        x[c] = t.x; x[c + 1] = t.y; x[c + 2] = t.z; x[c + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < PR_W; c += 4) {
        const uint2 t = __ldg(reinterpret_cast<const uint2*>(p + c));
        const T* h = reinterpret_cast<const T*>(&t);
        x[c] = to_f32(h[0]); x[c + 1] = to_f32(h[1]); x[c + 2] = to_f32(h[2]); x[c + 3] = to_f32(h[3]);
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < PR_W; ++c) x[c] = (c < w) ? to_f32(p[c]) : 0.f;
  }
}

__device__ __forceinline__ void store_row32(float* p, int w, bool vec, const float (&x)[PR_W]) {
  if (vec && w == PR_W) {
#pragma unroll
    for (int c = 0; c < PR_W; c += 4)
      *reinterpret_cast<float4*>(p + c) = make_float4(x[c], x[c + 1], x[c + 2], x[c + 3]);
  } else {
#pragma unroll
    for (int c = 0; c < PR_W; ++c)
      if (c < w) p[c] = x[c];
  }
}

// x <- x * L11^{-1}  (L11 unit lower, L11[i][j] = Ls[i][j] for j < i), in registers.
__device__ __forceinline__ void times_l11_inv(float (&x)[PR_W], const float (*Ls)[PR_W + 1],
                                              int w) {
#pragma unroll
  for (int i = PR_W - 1; i >= 1; --i) {
    if (i < w) {
      const float wi = x[i];
#pragma unroll
      for (int j = 0; j < i; ++j) x[j] = fmaf(-wi, Ls[i][j], x[j]);
    }
  }
}

// x[q][i] <- x[q][i + 1], x[q][31] <- x[q][0] for every row (register moves only)
template <int RPT>
__device__ __forceinline__ void rotate_left(float (&x)[RPT][PR_W]) {
#pragma unroll
  for (int q = 0; q < RPT; ++q) {
    const float t = x[q][0];
#pragma unroll
    for (int i = 0; i < PR_W - 1; ++i) x[q][i] = x[q][i + 1];
    x[q][PR_W - 1] = t;
  }
}

// The finished multipliers a pivot row holds, by column (Ls[j] = multiplier of column j < c),
// from a row's registers in the rotated layout of the column loop (see panel_reg_kernel).
template <int RING>
__device__ __forceinline__ void publish_multipliers(const float (&xr)[PR_W], float* Ls_c, int nr) {
  if constexpr (RING == 16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) Ls_c[j] = xr[16 + j];
  }
#pragma unroll
  for (int i = 1; i < RING; ++i)
    if (i >= nr) Ls_c[i - nr + (PR_W - RING)] = xr[i];
}

// NT threads per CTA (256; 128 for panels of at most 128 rows, which then fit twice as many
// CTAs per SM).
template <int MODE, typename TIn, typename TOut, int RPT, int NT = 256, bool ROT = true>
__global__ void __launch_bounds__(NT, (RPT == 1 ? (NT == 128 ? 6 : 3) : (NT == 64 ? 8 : NT == 128 ? 4 : 2)))
    panel_reg_kernel(PanelArgs a) {
  constexpr int NWARP = NT / 32;
  const int n = a.n, k0 = a.k0, w = a.w, m = n - k0;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  __shared__ __align__(16) float prow[2][PR_W];
  __shared__ float Ls[PR_W][PR_W + 1];   // multipliers of the pivot rows, by position
  __shared__ float dpiv[PR_W];
  __shared__ float red_v[2][NWARP];
  __shared__ int red_p[2][NWARP], red_r[2][NWARP];
  __shared__ int rowpos[NT * RPT], posrow[NT * RPT];  // PIVOT: local row <-> position
  __shared__ int oids[NT * RPT];
  __shared__ float tpart[NWARP][PR_W];
  __shared__ int s_flags;
  __shared__ float s_mu;

  const TIn* src = reinterpret_cast<const TIn*>(a.src) + mat_off(b, n);
  const bool vec = ((n & 3) == 0) && ((k0 & 3) == 0);
  if (tid == 0) s_flags = 0;

  // ---- jitter (CHOL, reflection_no_reflectors.py:74) ----
  if (MODE == PM_CHOL) {
    if (k0 == 0) {
      float acc = 0.f;
      for (int i = tid; i < (a.nmu > 0 ? a.nmu : n); i += NT) acc += to_f32(src[(int64_t)i * n + i]);
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (lane == 0) red_v[0][warp] = acc;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < NWARP; ++i) t += red_v[0][i];
        s_mu = 1e-7f * (t / (float)(a.nmu > 0 ? a.nmu : n));
        a.mu[b] = s_mu;
      }
    } else if (tid == 0) {
      s_mu = a.mu[b];
    }
  }

  QRB_PT(0);
  // ---- load the rows ----
  float x[RPT][PR_W];
  bool live[RPT];
#pragma unroll
  for (int q = 0; q < RPT; ++q) {
    const int r = tid + NT * q;
    live[q] = r < m;
    if (r < m) load_row32(src + (int64_t)(k0 + r) * n + k0, w, vec, x[q]);
    else {
#pragma unroll
      for (int c = 0; c < PR_W; ++c) x[q][c] = 0.f;
    }
    if (MODE == PM_PIVOT && r < NT * RPT) { rowpos[r] = r; posrow[r] = r; }
  }
  __syncthreads();

  QRB_PT(1);
  if constexpr (ROT) {
  // ---- column-by-column elimination ----
  // The column loop is NOT unrolled: fully unrolled, 32 column steps of straight-line code
  // overflow the instruction cache (ncu: "no instruction" was the top stall, 9 cycles per issue,
  // with issue slots 12 % busy).  To keep register indices compile-time constants in a runtime
  // loop, every row rotates a ring of its registers left by one in each step, so the pivot
  // column is always x[q][0].  Full-width panels use a 32-register ring for columns 0-15
  // (before step c, x[q][i] holds column c + i for i < 32 - c and the finished multiplier of
  // column i - (32 - c) above that) and a 16-register ring for columns 16-31 (the multipliers
  // of columns 0-15 rest in x[q][16..31]; before step c, x[q][i] holds column c + i for
  // i < 32 - c and the multiplier of column i + c - 16 for 32 - c <= i < 16), which halves the
  // update work of the second half.  The pivot row is published in the same rotated order
  // (prow[i] = column c + i, zero past the panel), so one branch-free pass
  // x[i-1] <- x[i] - l prow[i] both updates and rotates a ring; rows that take no update use
  // l = 0 (adding -0 * prow leaves them unchanged).  Narrower panels use the 32-register ring
  // for all w steps and 32 - w idle rotations.  At the end every value is back at its column.
  auto col_step = [&](const int c, auto ring_c) {
    constexpr int RING = decltype(ring_c)::value;  // 32 or 16 registers rotate
    const int par = c & 1;
    const int nr = PR_W - c;  // ring positions [0, nr) hold the live columns c .. 31
    float4* pr4 = reinterpret_cast<float4*>(prow[par]);
    bool upd[RPT];
    float l[RPT];
    if (MODE == PM_PIVOT) {
      // candidate key: |a| bits (monotone for non-negative floats; NaN counts as 0 and is
      // flagged), then the lowest current position.  Warp reductions with redux.sync.
      unsigned bv = 0u;
      int bp = INT_MAX, br = -1;
      bool bad = false;
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        if (live[q]) {
          const int r = tid + NT * q;
          const float xv = x[q][0];
          bad |= !isfinite(xv);
          const unsigned v = isnan(xv) ? 0u : __float_as_uint(fabsf(xv));
          const int p = rowpos[r];
          if (v > bv || (v == bv && p < bp)) { bv = v; bp = p; br = r; }
        }
      }
      if (bad) atomicOr(&s_flags, INFO_NONFINITE_INPUT);
      const unsigned wv = __reduce_max_sync(0xffffffffu, bv);
      const int wp = (int)__reduce_min_sync(0xffffffffu, (bv == wv) ? (unsigned)bp : 0xffffffffu);
      const unsigned own = __ballot_sync(0xffffffffu, bv == wv && bp == wp);
      const int wr = __shfl_sync(0xffffffffu, br, own ? (__ffs(own) - 1) : 0);
      if (lane == 0) {
        red_v[par][warp] = __uint_as_float(wv);
        red_p[par][warp] = wp;
        red_r[par][warp] = wr;
      }
      __syncthreads();
      unsigned V = __float_as_uint(red_v[par][0]);
      int Pp = red_p[par][0], Rw = red_r[par][0];
#pragma unroll
      for (int i = 1; i < NWARP; ++i) {
        const unsigned vi = __float_as_uint(red_v[par][i]);
        const int pi = red_p[par][i];
        if (vi > V || (vi == V && pi < Pp)) { V = vi; Pp = pi; Rw = red_r[par][i]; }
      }
      // the winner publishes its row (U row c, rotated, and its multipliers for columns < c)
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        if (tid + NT * q == Rw) {
#pragma unroll
          for (int i = 0; i < RING; i += 4)
            pr4[i / 4] = make_float4((c + i < w) ? x[q][i] : 0.f, (c + i + 1 < w) ? x[q][i + 1] : 0.f,
                                     (c + i + 2 < w) ? x[q][i + 2] : 0.f,
                                     (c + i + 3 < w) ? x[q][i + 3] : 0.f);
          publish_multipliers<RING>(x[q], Ls[c], nr);
          live[q] = false;
        }
      }
      if (tid == 0 && Pp != c) {  // replay getrf's swap of positions c and Pp
        const int rc = posrow[c];
        posrow[c] = Rw; posrow[Pp] = rc;
        rowpos[Rw] = c; rowpos[rc] = Pp;
      }
      __syncthreads();
      const float pv = prow[par][0];
      const float scale = (pv != 0.f) ? 1.f / pv : 1.f;
      if (tid == 0) {
        dpiv[c] = pv;
        if (pv == 0.f) atomicOr(&s_flags, INFO_LU_ZERO_PIVOT);
      }
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        upd[q] = live[q];
        l[q] = upd[q] ? x[q][0] * scale : 0.f;
      }
    } else {
      // row c is the pivot row (no pivoting); rows c .. w-1 live in threads c .. w-1, q = 0
      if (MODE == PM_CHOL) {
        if (tid >= c && tid < w) prow[par][tid - c] = x[0][0];  // U[c][j] = S[j][c]
        if (tid >= w - c && tid < PR_W) prow[par][tid] = 0.f;
      } else {
        if (tid == c) {
#pragma unroll
          for (int i = 0; i < RING; i += 4)
            pr4[i / 4] = make_float4((c + i < w) ? x[0][i] : 0.f, (c + i + 1 < w) ? x[0][i + 1] : 0.f,
                                     (c + i + 2 < w) ? x[0][i + 2] : 0.f,
                                     (c + i + 3 < w) ? x[0][i + 3] : 0.f);
        }
      }
      if (tid == c) {
        publish_multipliers<RING>(x[0], Ls[c], nr);
      }
      __syncthreads();
      // CHOL: the jitter enters with the diagonal entry when it becomes the pivot (adding it
      // before or after the earlier updates of that entry differs only by rounding)
      const float pv = prow[par][0] + ((MODE == PM_CHOL) ? s_mu : 0.f);
      float piv = pv, sgn = 1.f, rpiv = 1.f;
      if (MODE == PM_CHOL) {
        if (!(pv > 0.f)) {
          if (tid == 0) atomicOr(&s_flags, a.info_bit);
          piv = 1.f;  // keep the arithmetic finite; the host reports the failure
        }
        rpiv = __frcp_rn(piv);
        if (tid == 0) dpiv[c] = piv;
      } else {
        const float pp = 1.f - pv, pm = 1.f + pv;
        sgn = (fabsf(pp) >= fabsf(pm)) ? 1.f : -1.f;
        piv = (sgn > 0.f) ? pp : pm;
        if (tid == 0) dpiv[c] = sgn;
      }
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        const int r = tid + NT * q;
        upd[q] = r > c && r < m;
        // Cholesky scales by the reciprocal pivot (as potf2 does); the chart divides (:158)
        l[q] = !upd[q] ? 0.f : (MODE == PM_CHOL) ? x[q][0] * rpiv : (-sgn * x[q][0]) / piv;
      }
    }
    // update and rotate: x[i-1] <- x[i] - l prow[i] (i = 1..31), x[31] <- l or the kept value
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const float x0 = x[q][0];
#pragma unroll
      for (int i4 = 0; i4 < RING / 4; ++i4) {
        const float4 p4 = pr4[i4];
        const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = 4 * i4 + u;
          if (i >= 1) x[q][i - 1] = fmaf(-l[q], pp[u], x[q][i]);
        }
      }
      x[q][RING - 1] = upd[q] ? l[q] : x0;
    }
  };
  using Ring32 = std::integral_constant<int, 32>;
  using Ring16 = std::integral_constant<int, 16>;
  if (w == PR_W) {
#pragma unroll 1
    for (int c = 0; c < 16; ++c) col_step(c, Ring32{});
#pragma unroll 1
    for (int c = 16; c < PR_W; ++c) col_step(c, Ring16{});
#pragma unroll
    for (int q = 0; q < RPT; ++q) {  // x[q][i] holds column 16 + i, x[q][16 + i] column i
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float t = x[q][i];
        x[q][i] = x[q][16 + i];
        x[q][16 + i] = t;
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < w; ++c) col_step(c, Ring32{});
    for (int c = w; c < PR_W; ++c) rotate_left(x);
  }
  } else {
  // fully unrolled column loop (32 straight-line column steps, exact update ranges)
#pragma unroll
  for (int c = 0; c < PR_W; ++c) {
    if (c >= w) break;
    const int par = c & 1;
    if (MODE == PM_PIVOT) {
      // candidate key: |a| bits (monotone for non-negative floats; NaN counts as 0 and is
      // flagged), then the lowest current position.  Warp reductions with redux.sync.
      unsigned bv = 0u;
      int bp = INT_MAX, br = -1;
      bool bad = false;
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        if (live[q]) {
          const int r = tid + NT * q;
          const float xv = x[q][c];
          bad |= !isfinite(xv);
          const unsigned v = isnan(xv) ? 0u : __float_as_uint(fabsf(xv));
          const int p = rowpos[r];
          if (v > bv || (v == bv && p < bp)) { bv = v; bp = p; br = r; }
        }
      }
      if (bad) atomicOr(&s_flags, INFO_NONFINITE_INPUT);
      const unsigned wv = __reduce_max_sync(0xffffffffu, bv);
      const int wp = (int)__reduce_min_sync(0xffffffffu, (bv == wv) ? (unsigned)bp : 0xffffffffu);
      const unsigned own = __ballot_sync(0xffffffffu, bv == wv && bp == wp);
      const int wr = __shfl_sync(0xffffffffu, br, own ? (__ffs(own) - 1) : 0);
      if (lane == 0) {
        red_v[par][warp] = __uint_as_float(wv);
        red_p[par][warp] = wp;
        red_r[par][warp] = wr;
      }
      __syncthreads();
      unsigned V = __float_as_uint(red_v[par][0]);
      int Pp = red_p[par][0], Rw = red_r[par][0];
#pragma unroll
      for (int i = 1; i < NWARP; ++i) {
        const unsigned vi = __float_as_uint(red_v[par][i]);
        const int pi = red_p[par][i];
        if (vi > V || (vi == V && pi < Pp)) { V = vi; Pp = pi; Rw = red_r[par][i]; }
      }
      // the winner publishes its row (U row c and its multipliers for columns < c)
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        if (tid + NT * q == Rw) {
#pragma unroll
          for (int j = 0; j < PR_W; ++j) {
            if (j < w) prow[par][j] = x[q][j];
            if (j < c) Ls[c][j] = x[q][j];
          }
          live[q] = false;
        }
      }
      if (tid == 0 && Pp != c) {  // replay getrf's swap of positions c and Pp
        const int rc = posrow[c];
        posrow[c] = Rw; posrow[Pp] = rc;
        rowpos[Rw] = c; rowpos[rc] = Pp;
      }
      __syncthreads();
      const float pv = prow[par][c];
      const float scale = (pv != 0.f) ? 1.f / pv : 1.f;
      if (tid == 0) {
        dpiv[c] = pv;
        if (pv == 0.f) atomicOr(&s_flags, INFO_LU_ZERO_PIVOT);
      }
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        if (live[q]) {
          const float l = x[q][c] * scale;
          x[q][c] = l;
#pragma unroll
          for (int j = c + 1; j < PR_W; ++j)
            if (j < w) x[q][j] = fmaf(-l, prow[par][j], x[q][j]);
        }
      }
    } else {
      // row c is the pivot row (no pivoting); rows c .. w-1 live in threads c .. w-1, q = 0
      if (MODE == PM_CHOL) {
        if (tid >= c && tid < w) prow[par][tid] = x[0][c];  // U[c][j] = S[j][c]
      } else {
        if (tid == c) {
#pragma unroll
          for (int j = 0; j < PR_W; ++j)
            if (j < w) prow[par][j] = x[0][j];
        }
      }
      if (tid == c) {
#pragma unroll
        for (int j = 0; j < PR_W; ++j)
          if (j < c) Ls[c][j] = x[0][j];
      }
      __syncthreads();
      // CHOL: the jitter enters with the diagonal entry when it becomes the pivot (adding it
      // before or after the earlier updates of that entry differs only by rounding)
      const float pv = prow[par][c] + ((MODE == PM_CHOL) ? s_mu : 0.f);
      float piv = pv, sgn = 1.f, rpiv = 1.f;
      if (MODE == PM_CHOL) {
        if (!(pv > 0.f)) {
          if (tid == 0) atomicOr(&s_flags, a.info_bit);
          piv = 1.f;  // keep the arithmetic finite; the host reports the failure
        }
        rpiv = __frcp_rn(piv);
        if (tid == 0) dpiv[c] = piv;
      } else {
        const float pp = 1.f - pv, pm = 1.f + pv;
        sgn = (fabsf(pp) >= fabsf(pm)) ? 1.f : -1.f;
        piv = (sgn > 0.f) ? pp : pm;
        if (tid == 0) dpiv[c] = sgn;
      }
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        const int r = tid + NT * q;
        if (r > c && r < m) {
          // Cholesky scales by the reciprocal pivot (as potf2 does); the chart divides (:158)
          const float l = (MODE == PM_CHOL) ? x[q][c] * rpiv : (-sgn * x[q][c]) / piv;
          x[q][c] = l;
#pragma unroll
          for (int j = c + 1; j < PR_W; ++j)
            if (j < w) x[q][j] = fmaf(-l, prow[par][j], x[q][j]);
        }
      }
    }
  }
  }
  __syncthreads();

  QRB_PT(2);
  // ---- outputs ----
  int pos[RPT];
#pragma unroll
  for (int q = 0; q < RPT; ++q) {
    const int r = tid + NT * q;
    pos[q] = (MODE == PM_PIVOT && r < m) ? rowpos[r] : r;
  }
  float* Wb = a.W + (int64_t)b * n * a.ldw;

  if (MODE == PM_PIVOT) {
    int* orig = a.orig + b * n;
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = tid + NT * q;
      if (r < m) oids[r] = (k0 == 0) ? r : checked_row(orig[k0 + r], 0, n, a.info + b);
    }
    __syncthreads();
    for (int p = tid; p < m; p += NT) {
      const int r = checked_row(posrow[p], 0, m, a.info + b);
      orig[k0 + p] = oids[r];
      a.srcmap[b * n + k0 + p] = k0 + r;
    }
    float* L = a.L + mat_off(b, n);
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = tid + NT * q;
      if (r >= m) continue;
      float* Lrow = L + (int64_t)oids[r] * n;
      const int p = pos[q];
      if (p < w) {
        float y[PR_W];
#pragma unroll
        for (int c = 0; c < PR_W; ++c) y[c] = (c < p) ? x[q][c] : (c == p ? 1.f : 0.f);
        store_row32(Lrow + k0, w, vec, y);
        // pivot rows are final: zero the rest of the L row
        int j = k0 + w;
        if (vec) for (; j + 4 <= n; j += 4) *reinterpret_cast<float4*>(Lrow + j) = make_float4(0.f, 0.f, 0.f, 0.f);
        for (; j < n; ++j) Lrow[j] = 0.f;
      } else {
        store_row32(Lrow + k0, w, vec, x[q]);
      }
    }
  } else if (MODE == PM_CHOL) {
    float* R = a.R + mat_off(b, n);
    __shared__ float sqd[PR_W];
    if (tid < w) sqd[tid] = __fsqrt_rn(dpiv[tid]);
    __syncthreads();
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = tid + NT * q;
      if (r >= m) continue;
#pragma unroll
      for (int c = 0; c < PR_W; ++c)
        if (c < w && c <= r) R[(int64_t)(k0 + c) * n + k0 + r] = (c == r) ? sqd[c] : sqd[c] * x[q][c];
      if (r >= w) {  // L21 D^{1/2} for the Cholesky trailing update
        float* wc = a.Wc + ((int64_t)b * n + k0 + r) * a.ldw;
        if (w == PR_W && (a.ldw & 3) == 0) {
#pragma unroll
          for (int c = 0; c < PR_W; c += 4)
            *reinterpret_cast<float4*>(wc + c) =
                make_float4(x[q][c] * sqd[c], x[q][c + 1] * sqd[c + 1], x[q][c + 2] * sqd[c + 2],
                            x[q][c + 3] * sqd[c + 3]);
        } else {
#pragma unroll
          for (int c = 0; c < PR_W; ++c)
            if (c < w) wc[c] = x[q][c] * sqd[c];
        }
      }
    }
    QRB_PT(5);
    if (tid < w) a.D[b * n + k0 + tid] = dpiv[tid];
    // rows [k0, k0+w) of L_G^{-1} before this panel (identity block included), columns < k1;
    // one flat float4 copy over all threads (k0 % 4 == 0 here since n % 4 == 0 or k0 == 0)
    {
      // columns [j0, k0 + w): with bp_ready the previous update already stored columns < k0
      const int j0 = a.bp_ready ? k0 : 0;
      const int cols = k0 + w - j0;
      if (vec && (cols & 3) == 0) {
        const int per = cols >> 2;
#pragma unroll 4
        for (int idx = tid; idx < w * per; idx += NT) {
          const int c = idx / per, j = j0 + (idx - c * per) * 4;
          float4 v;
          if (j + 3 < k0) {
            v = *reinterpret_cast<const float4*>(R + (int64_t)(k0 + c) * n + j);
          } else {
            float t[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              t[u] = (j + u < k0) ? R[(int64_t)(k0 + c) * n + j + u] : ((j + u == k0 + c) ? 1.f : 0.f);
            v = make_float4(t[0], t[1], t[2], t[3]);
          }
          *reinterpret_cast<float4*>(a.Bp + ((int64_t)b * a.ldw + c) * n + j) = v;
        }
      } else {
        for (int idx = tid; idx < w * cols; idx += NT) {
          const int c = idx / cols, j = j0 + idx - c * cols;
          a.Bp[((int64_t)b * a.ldw + c) * n + j] =
              (j < k0) ? R[(int64_t)(k0 + c) * n + j] : ((j == k0 + c) ? 1.f : 0.f);
        }
      }
    }
    QRB_PT(6);
    // L11^{-1} (unit lower) into rows [k0, k0+w) of the W buffer: row i of L11^{-1} is
    // e_i^T L11^{-1}, computed by thread i in the registers of its (pivot) row, which is done
    if (tid < w) {
#pragma unroll
      for (int c = 0; c < PR_W; ++c) x[0][c] = (c == tid) ? 1.f : 0.f;
      times_l11_inv(x[0], Ls, w);
      store_row32(Wb + (int64_t)(k0 + tid) * a.ldw, w, (a.ldw & 3) == 0, x[0]);
    }
  } else {  // PM_CHART
    TOut* H = reinterpret_cast<TOut*>(a.H) + mat_off(b, n);
    float part[PR_W];
#pragma unroll
    for (int c = 0; c < PR_W; ++c) part[c] = 0.f;
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = tid + NT * q;
      if (r >= m) continue;
      TOut* Hrow = H + (int64_t)(k0 + r) * n + k0;
      if (r >= PR_W && w == PR_W && vec) {  // whole row below the panel: vector stores
#pragma unroll
        for (int c = 0; c < PR_W; c += 4) {
          if constexpr (sizeof(TOut) == 4) {
            *reinterpret_cast<float4*>(Hrow + c) =
                make_float4(x[q][c], x[q][c + 1], x[q][c + 2], x[q][c + 3]);
          } else {
            TOut t[4] = {from_f32<TOut>(x[q][c]), from_f32<TOut>(x[q][c + 1]),
                         from_f32<TOut>(x[q][c + 2]), from_f32<TOut>(x[q][c + 3])};
            *reinterpret_cast<uint2*>(Hrow + c) = *reinterpret_cast<const uint2*>(t);
          }
        }
#pragma unroll
        for (int c = 0; c < PR_W; ++c) part[c] = fmaf(x[q][c], x[q][c], part[c]);
      } else {
#pragma unroll
        for (int c = 0; c < PR_W; ++c) {
          if (c < w && c < r) {
            Hrow[c] = from_f32<TOut>(x[q][c]);
            part[c] = fmaf(x[q][c], x[q][c], part[c]);
          }
        }
      }
    }
#pragma unroll
    for (int c = 0; c < PR_W; ++c) {
      float v = part[c];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
      if (lane == 0) tpart[warp][c] = v;
    }
    __syncthreads();
    if (tid < w) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NWARP; ++i) acc += tpart[i][tid];
      reinterpret_cast<TOut*>(a.tau)[b * n + k0 + tid] = from_f32<TOut>(2.f / (acc + 1.f));
      a.s[b * n + k0 + tid] = dpiv[tid];
    }
  }

  QRB_PT(3);
  // ---- W = L21 L11^{-1} for the rows below the panel (positions >= w) ----
  if (k0 + w < n) {
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = tid + NT * q;
      if (r < m && pos[q] >= w) {
        times_l11_inv(x[q], Ls, w);
        store_row32(Wb + (int64_t)(k0 + pos[q]) * a.ldw, w, (a.ldw & 3) == 0, x[q]);
      }
    }
  }

  QRB_PT(4);
  __syncthreads();
  if (tid == 0 && s_flags) atomicOr(a.info + b, s_flags);
}

}  // namespace qrb
