// qrb200 -- panel elimination over a thread-block cluster, for panels of 513 .. CL * 512 rows.
//
// Same contract and outputs as panel_reg_kernel (qrb_panel_reg.cuh): PM_PIVOT / PM_CHOL /
// PM_CHART on an m x w panel (w <= 32), but the rows are spread over the CL CTAs of a cluster
// (CTA `rank` keeps rows rank * 512 + tid + 256 q, q < 2, in registers), so an n = 2048 matrix
// keeps 32-wide panels in registers and one matrix occupies CL SMs (the large-n batch has fewer
// matrices than the GPU has SMs).  The CTAs talk through distributed shared memory only:
//   PM_PIVOT : each CTA reduces its rows to one candidate (max |a|, then the lowest current
//              position) and exposes it in its shared memory; after a cluster barrier every
//              CTA reads all CL candidates and picks the same winner.  The winner's owner
//              stores the pivot row and its multipliers into every CTA's shared memory
//              (st.shared::cluster through mapped addresses) before a second cluster barrier.
//              Every CTA replays getrf's position swaps on its own copy of the
//              position <-> row maps, so all copies agree.
//   PM_CHOL / PM_CHART : rows c .. w-1 of the panel live in CTA 0, which stores the pivot
//              values into every CTA's shared memory; one cluster barrier per column.
// tau's column sums are reduced over the cluster through shared memory as well.  Every CTA
// runs the same column loop (no early exit), and a final cluster barrier keeps each CTA's
// shared memory alive until the others stopped reading it.  No TMA, no multicast.
#pragma once
#include <cooperative_groups.h>

#include "qrb_panel_reg.cuh"

namespace qrb {

constexpr int kClRows = 512;  // rows per CTA (2 per thread)

template <int MODE, typename TIn, typename TOut, int CL>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(256, 2)
    panel_cl_kernel(PanelArgs a) {
  namespace cg = cooperative_groups;
  constexpr int RPT = 2;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int n = a.n, k0 = a.k0, w = a.w, m = n - k0;
  const int64_t b = blockIdx.x / CL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rbase = rank * kClRows;

  __shared__ float prow[2][PR_W];
  __shared__ float Ls[PR_W][PR_W + 1];
  __shared__ float dpiv[PR_W];
  __shared__ float red_v[2][8];
  __shared__ int red_p[2][8], red_r[2][8];
  __shared__ float cand_v[2];          // this CTA's candidate for the cluster-wide pivot
  __shared__ int cand_p[2], cand_r[2];
  __shared__ int rowpos[CL * kClRows], posrow[CL * kClRows];  // PIVOT, replicated per CTA
  __shared__ int oids[kClRows];        // PIVOT: original ids of this CTA's rows
  __shared__ float tpart[8][PR_W];
  __shared__ float colsum[PR_W];       // CHART: this CTA's tau partial per column
  __shared__ int s_flags;
  __shared__ float s_mu;

  const TIn* src = reinterpret_cast<const TIn*>(a.src) + mat_off(b, n);
  const bool vec = ((n & 3) == 0) && ((k0 & 3) == 0);
  if (tid == 0) s_flags = 0;

  // ---- jitter (CHOL, reflection_no_reflectors.py:74): every CTA computes the same value ----
  if (MODE == PM_CHOL) {
    if (k0 == 0) {
      float acc = 0.f;
      for (int i = tid; i < (a.nmu > 0 ? a.nmu : n); i += 256) acc += to_f32(src[(int64_t)i * n + i]);
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
      if (lane == 0) red_v[0][warp] = acc;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < 8; ++i) t += red_v[0][i];
        s_mu = 1e-7f * (t / (float)(a.nmu > 0 ? a.nmu : n));
        if (rank == 0) a.mu[b] = s_mu;
      }
    } else if (tid == 0) {
      s_mu = a.mu[b];
    }
  }

  // ---- load this CTA's rows ----
  float x[RPT][PR_W];
  bool live[RPT];
#pragma unroll
  for (int q = 0; q < RPT; ++q) {
    const int r = rbase + tid + 256 * q;
    live[q] = r < m;
    if (r < m) load_row32(src + (int64_t)(k0 + r) * n + k0, w, vec, x[q]);
    else {
#pragma unroll
      for (int c = 0; c < PR_W; ++c) x[q][c] = 0.f;
    }
  }
  if (MODE == PM_PIVOT)
    for (int r = tid; r < CL * kClRows; r += 256) { rowpos[r] = r; posrow[r] = r; }
  __syncthreads();

  // ---- column-by-column elimination ----
#pragma unroll
  for (int c = 0; c < PR_W; ++c) {
    if (c >= w) break;
    const int par = c & 1;
    if (MODE == PM_PIVOT) {
      unsigned bv = 0u;
      int bp = INT_MAX, br = -1;
      bool bad = false;
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        if (live[q]) {
          const int r = rbase + tid + 256 * q;
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
      if (tid == 0) {
        unsigned V = __float_as_uint(red_v[par][0]);
        int Pp = red_p[par][0], Rw = red_r[par][0];
        for (int i = 1; i < 8; ++i) {
          const unsigned vi = __float_as_uint(red_v[par][i]);
          const int pi = red_p[par][i];
          if (vi > V || (vi == V && pi < Pp)) { V = vi; Pp = pi; Rw = red_r[par][i]; }
        }
        cand_v[par] = __uint_as_float(V);
        cand_p[par] = Pp;
        cand_r[par] = Rw;
      }
      cluster.sync();  // every CTA's candidate is visible
      unsigned V = 0u;
      int Pp = INT_MAX, Rw = -1;
#pragma unroll
      for (int k = 0; k < CL; ++k) {
        const unsigned vk = __float_as_uint(*cluster.map_shared_rank(&cand_v[par], k));
        const int pk = *cluster.map_shared_rank(&cand_p[par], k);
        if (pk != INT_MAX && (vk > V || (vk == V && pk < Pp))) {
          V = vk; Pp = pk; Rw = *cluster.map_shared_rank(&cand_r[par], k);
        }
      }
      // the owner publishes the pivot row and its multipliers into every CTA
#pragma unroll
      for (int q = 0; q < RPT; ++q) {
        if (rbase + tid + 256 * q == Rw) {
          for (int k = 0; k < CL; ++k) {
            float* pr = cluster.map_shared_rank(&prow[par][0], k);
            float* lr = cluster.map_shared_rank(&Ls[c][0], k);
#pragma unroll
            for (int j = 0; j < PR_W; ++j) {
              if (j < w) pr[j] = x[q][j];
              if (j < c) lr[j] = x[q][j];
            }
          }
          live[q] = false;
        }
      }
      if (tid == 0 && Pp != c) {  // replay getrf's swap of positions c and Pp
        const int rc = posrow[c];
        posrow[c] = Rw; posrow[Pp] = rc;
        rowpos[Rw] = c; rowpos[rc] = Pp;
      }
      cluster.sync();  // the pivot row reached every CTA; the maps are updated
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
          for (int j = 0; j < PR_W; ++j)
            if (j > c && j < w) x[q][j] = fmaf(-l, prow[par][j], x[q][j]);
        }
      }
    } else {
      // row c is the pivot row: rows c .. w-1 sit in CTA 0, threads c .. w-1, q = 0
      if (rank == 0) {
        if (MODE == PM_CHOL) {
          if (tid >= c && tid < w)
            for (int k = 0; k < CL; ++k) *cluster.map_shared_rank(&prow[par][tid], k) = x[0][c];
        } else if (tid == c) {
          for (int k = 0; k < CL; ++k) {
            float* pr = cluster.map_shared_rank(&prow[par][0], k);
#pragma unroll
            for (int j = 0; j < PR_W; ++j)
              if (j < w) pr[j] = x[0][j];
          }
        }
        if (tid == c)
          for (int k = 0; k < CL; ++k) {
            float* lr = cluster.map_shared_rank(&Ls[c][0], k);
#pragma unroll
            for (int j = 0; j < PR_W; ++j)
              if (j < c) lr[j] = x[0][j];
          }
      }
      cluster.sync();
      const float pv = prow[par][c] + ((MODE == PM_CHOL) ? s_mu : 0.f);
      float piv = pv, sgn = 1.f, rpiv = 1.f;
      if (MODE == PM_CHOL) {
        if (!(pv > 0.f)) {
          if (tid == 0) atomicOr(&s_flags, a.info_bit);
          piv = 1.f;
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
        const int r = rbase + tid + 256 * q;
        if (r > c && r < m) {
          const float l = (MODE == PM_CHOL) ? x[q][c] * rpiv : (-sgn * x[q][c]) / piv;
          x[q][c] = l;
#pragma unroll
          for (int j = 0; j < PR_W; ++j)
            if (j > c && j < w) x[q][j] = fmaf(-l, prow[par][j], x[q][j]);
        }
      }
    }
  }
  __syncthreads();

  // ---- outputs ----
  int pos[RPT];
#pragma unroll
  for (int q = 0; q < RPT; ++q) {
    const int r = rbase + tid + 256 * q;
    pos[q] = (MODE == PM_PIVOT && r < m) ? rowpos[r] : r;
  }
  float* Wb = a.W + (int64_t)b * n * a.ldw;

  if (MODE == PM_PIVOT) {
    int* orig = a.orig + b * n;
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = rbase + tid + 256 * q;
      if (r < m) oids[tid + 256 * q] = (k0 == 0) ? r : checked_row(orig[k0 + r], 0, n, a.info + b);
    }
    cluster.sync();  // every CTA read its original ids before any is overwritten
    for (int p = rbase + tid; p < m && p < rbase + kClRows; p += 256) {
      const int r = checked_row(posrow[p], 0, m, a.info + b);
      orig[k0 + p] = *cluster.map_shared_rank(&oids[r % kClRows], r / kClRows);
      a.srcmap[b * n + k0 + p] = k0 + r;
    }
    float* L = a.L + mat_off(b, n);
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = rbase + tid + 256 * q;
      if (r >= m) continue;
      float* Lrow = L + (int64_t)oids[tid + 256 * q] * n;
      const int p = pos[q];
      if (p < w) {
        float y[PR_W];
#pragma unroll
        for (int c = 0; c < PR_W; ++c) y[c] = (c < p) ? x[q][c] : (c == p ? 1.f : 0.f);
        store_row32(Lrow + k0, w, vec, y);
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
      const int r = rbase + tid + 256 * q;
      if (r >= m) continue;
#pragma unroll
      for (int c = 0; c < PR_W; ++c)
        if (c < w && c <= r) R[(int64_t)(k0 + c) * n + k0 + r] = (c == r) ? sqd[c] : sqd[c] * x[q][c];
      if (r >= w) {
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
    if (rank == 0) {
      if (tid < w) a.D[b * n + k0 + tid] = dpiv[tid];
      // rows [k0, k0+w) of L_G^{-1} before this panel (identity block included), cols < k1
      const int j0 = a.bp_ready ? k0 : 0;  // columns < k0 already stored by the update
      const int cols = k0 + w - j0;
      for (int idx = tid; idx < w * cols; idx += 256) {
        const int c = idx / cols, j = j0 + idx - c * cols;
        a.Bp[((int64_t)b * a.ldw + c) * n + j] =
            (j < k0) ? R[(int64_t)(k0 + c) * n + j] : ((j == k0 + c) ? 1.f : 0.f);
      }
      if (tid < w) {
#pragma unroll
        for (int c = 0; c < PR_W; ++c) x[0][c] = (c == tid) ? 1.f : 0.f;
        times_l11_inv(x[0], Ls, w);
        store_row32(Wb + (int64_t)(k0 + tid) * a.ldw, w, (a.ldw & 3) == 0, x[0]);
      }
    }
  } else {  // PM_CHART
    TOut* H = reinterpret_cast<TOut*>(a.H) + mat_off(b, n);
    float part[PR_W];
#pragma unroll
    for (int c = 0; c < PR_W; ++c) part[c] = 0.f;
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = rbase + tid + 256 * q;
      if (r >= m) continue;
      TOut* Hrow = H + (int64_t)(k0 + r) * n + k0;
#pragma unroll
      for (int c = 0; c < PR_W; ++c) {
        if (c < w && c < r) {
          Hrow[c] = from_f32<TOut>(x[q][c]);
          part[c] = fmaf(x[q][c], x[q][c], part[c]);
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
    if (tid < PR_W) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc += tpart[i][tid];
      colsum[tid] = acc;
    }
    cluster.sync();
    if (rank == 0 && tid < w) {
      float acc = 0.f;
      for (int k = 0; k < CL; ++k) acc += *cluster.map_shared_rank(&colsum[tid], k);
      reinterpret_cast<TOut*>(a.tau)[b * n + k0 + tid] = from_f32<TOut>(2.f / (acc + 1.f));
      a.s[b * n + k0 + tid] = dpiv[tid];
    }
  }

  // ---- W = L21 L11^{-1} for the rows below the panel (positions >= w) ----
  if (k0 + w < n) {
#pragma unroll
    for (int q = 0; q < RPT; ++q) {
      const int r = rbase + tid + 256 * q;
      if (r < m && pos[q] >= w) {
        times_l11_inv(x[q], Ls, w);
        store_row32(Wb + (int64_t)(k0 + pos[q]) * a.ldw, w, (a.ldw & 3) == 0, x[q]);
      }
    }
  }
  __syncthreads();
  if (tid == 0 && s_flags) atomicOr(a.info + b, s_flags);
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

}  // namespace qrb
