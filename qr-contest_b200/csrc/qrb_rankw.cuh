// qrb200 -- rank-w trailing updates as one memory-streaming pass per update (K = the panel
// width 32, or K = 128 for the chart's block update: K is consumed in slices of 32).
//
// Every blocked elimination of the pipeline ends a panel with C' = C - A B where K = w is
// the panel width: the LU and chart trailing updates (reflection_no_reflectors.py:66 via
// getrf, :174), the Cholesky trailing update (:76 via potrf) and the L_G^{-1} update of the
// CholeskyQR passes.  With K = 32 the update does 64 flops per 8 bytes of C streamed, so it
// is bound by HBM bandwidth, not arithmetic: the kernel is built for streaming -- float4
// loads of whole rows, the gathered row pointer resolved once per row, the K-slice of A
// and B staged once in shared memory, and a 64 x 128 tile per CTA (4 x 8 outputs per
// thread) so each thread keeps 8 independent row segments in flight.
//
// Policy Pb supplies: Args; dims(a, M, N, K); live(a, m0, n0);
//   a_ptr(a, b, m)  -> const float*  row m of A (K contiguous floats, 16-byte aligned)
//   b_ptr(a, b, k)  -> const TB*     row k of B (B(k, j) = p[j], j < N, 16-byte aligned)
//   c_load4(a, b, m, j) -> float4    C_in of columns j .. j+3 of row m (j % 4 == 0)
//   store4(a, b, m, j, C_in - acc)   the result of the same 4 columns
// Requires n % 4 == 0 (callers fall back to the scalar tiles otherwise).
#pragma once
#include "qrb_common.cuh"

namespace qrb {

constexpr int RW_M = 64, RW_N = 128, RW_K = 32;

template <typename T>
__device__ __forceinline__ float4 ld4v(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return __ldg(reinterpret_cast<const float4*>(p));
  } else {
    const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
    const T* h = reinterpret_cast<const T*>(&t);
    return make_float4(to_f32(h[0]), to_f32(h[1]), to_f32(h[2]), to_f32(h[3]));
  }
}
// non-cached variant for buffers the same kernel also writes
__device__ __forceinline__ float4 ld4rw(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

template <class Pb>
__global__ void __launch_bounds__(256) rankw_kernel(typename Pb::Args a) {
  __shared__ __align__(16) float As[RW_K][RW_M + 4];
  __shared__ __align__(16) float Bs[RW_K][RW_N + 4];
  const int64_t b = blockIdx.z;
  const int m0 = blockIdx.y * RW_M, n0 = blockIdx.x * RW_N;
  int M, N, K;
  Pb::dims(a, M, N, K);
  if (m0 >= M || n0 >= N || !Pb::live(a, m0, n0)) return;
  const int tid = threadIdx.x;
  // the C tile (64 rows x 4 lines of 128 bytes) starts towards L2 before the K loop
  {
    const int row = tid >> 2, j = n0 + 32 * (tid & 3);
    if (m0 + row < M && j < N) {
      const void* p = Pb::c_addr(a, b, m0 + row, j);
      if (p) asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    }
  }

  const int tn = tid & 15, tm = tid >> 4;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  // K is consumed in slices of RW_K = 32 (a single slice for the rank-32 panel updates)
  for (int kb = 0; kb < K; kb += RW_K) {
    const int Kc = (K - kb < RW_K) ? K - kb : RW_K;
    if (kb > 0) __syncthreads();  // the previous slice has been read
    // A: 64 rows x Kc -> As[k][m]
#pragma unroll
    for (int rep = 0; rep < 2; ++rep) {
      const int mm = (tid >> 3) + 32 * rep, kc = tid & 7;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m0 + mm < M && 4 * kc < Kc)
        v = __ldg(reinterpret_cast<const float4*>(Pb::a_ptr(a, b, m0 + mm) + kb + 4 * kc));
      As[4 * kc + 0][mm] = v.x;
      As[4 * kc + 1][mm] = v.y;
      As[4 * kc + 2][mm] = v.z;
      As[4 * kc + 3][mm] = v.w;
    }
    // B: Kc rows x 128 columns -> Bs[k][j]
#pragma unroll
    for (int rep = 0; rep < 4; ++rep) {
      const int k = (tid >> 5) + 8 * rep, c4 = (tid & 31) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < Kc && n0 + c4 < N) v = ld4v(Pb::b_ptr(a, b, kb + k) + n0 + c4);
      st4(&Bs[k][c4], v);
    }
    __syncthreads();
    for (int k = 0; k < Kc; ++k) {
      const float4 av = *reinterpret_cast<const float4*>(&As[k][tm * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[k][tn * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[k][tn * 8 + 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w};
      const float br[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
  }
  // all C loads of the thread first, then the stores (C may be updated in place: a load after
  // a store would wait for its own round trip)
  float4 xs[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tm * 4 + i;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = n0 + tn * 8 + 4 * h;
      if (m < M && j < N) xs[i][h] = Pb::c_load4(a, b, m, j);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tm * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = n0 + tn * 8 + 4 * h;
      if (j < N) {
        float4 x = xs[i][h];
        x.x -= acc[i][4 * h]; x.y -= acc[i][4 * h + 1];
        x.z -= acc[i][4 * h + 2]; x.w -= acc[i][4 * h + 3];
        Pb::store4(a, b, m, j, x);
      }
    }
  }
}

// ---- LU / chart trailing update: C'[k1+m][k1+j] = C[src(k1+m)][k1+j] - (W C[src(k0:k1)])
struct RWTrailArgs {
  int n, k0, k1, ldw;
  const void* Cold;
  float* Cnew;
  const float* W;
  const int* srcmap;  // nullptr -> identity
  int* info;
};
template <typename T>
struct RWTrail {
  using Args = RWTrailArgs;
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = N = a.n - a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(const Args&, int, int) { return true; }
  __device__ static int srow(const Args& a, int64_t b, int r) {
    return a.srcmap ? checked_row(a.srcmap[b * a.n + r], 0, a.n, a.info + b) : r;
  }
  __device__ static const float* a_ptr(const Args& a, int64_t b, int m) {
    return a.W + ((int64_t)b * a.n + a.k1 + m) * a.ldw;
  }
  __device__ static const T* b_ptr(const Args& a, int64_t b, int k) {
    return reinterpret_cast<const T*>(a.Cold) + mat_off(b, a.n) +
           (int64_t)srow(a, b, a.k0 + k) * a.n + a.k1;
  }
  // address of C_in at row m, column j (an L2 prefetch target), nullptr if it is never read
  __device__ static const void* c_addr(const Args& a, int64_t b, int m, int j) {
    return reinterpret_cast<const T*>(a.Cold) + mat_off(b, a.n) +
           (int64_t)srow(a, b, a.k1 + m) * a.n + a.k1 + j;
  }
  __device__ static float4 c_load4(const Args& a, int64_t b, int m, int j) {
    const T* c = reinterpret_cast<const T*>(a.Cold) + mat_off(b, a.n) +
                 (int64_t)srow(a, b, a.k1 + m) * a.n + a.k1 + j;
    // the chart updates in place: plain loads for a buffer this kernel also writes
    return (a.Cold == static_cast<const void*>(a.Cnew)) ? ld4rw(reinterpret_cast<const float*>(c))
                                                        : ld4v(c);
  }
  __device__ static void store4(const Args& a, int64_t b, int m, int j, float4 x) {
    st4(a.Cnew + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j, x);
  }
};

// ---- Cholesky trailing update on the lower triangle: G22 -= (L21 D^{1/2}) R12 -----------
struct RWSyrkArgs {
  int n, k0, k1, ldw;
  float* G;
  const float* R;   // rows [k0, k1): R12 = D^{1/2} L21^T
  const float* Wc;  // rows [k1, n): L21 D^{1/2}
  int* info;
  int lim;          // columns [k1, lim) are updated (n: the whole trailing triangle)
};
struct RWSyrk {
  using Args = RWSyrkArgs;
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = a.n - a.k1;
    N = a.lim - a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(const Args&, int m0, int n0) { return n0 < m0 + RW_M; }
  __device__ static const float* a_ptr(const Args& a, int64_t b, int m) {
    return a.Wc + ((int64_t)b * a.n + a.k1 + m) * a.ldw;
  }
  __device__ static const float* b_ptr(const Args& a, int64_t b, int k) {
    return a.R + mat_off(b, a.n) + (int64_t)(a.k0 + k) * a.n + a.k1;
  }
  __device__ static const void* c_addr(const Args& a, int64_t b, int m, int j) {
    if (j > m + 3) return nullptr;
    return a.G + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j;
  }
  __device__ static float4 c_load4(const Args& a, int64_t b, int m, int j) {
    if (j > m + 3) return make_float4(0.f, 0.f, 0.f, 0.f);  // strictly upper: never read
    return ld4rw(a.G + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j);
  }
  __device__ static void store4(const Args& a, int64_t b, int m, int j, float4 x) {
    if (j > m + 3) return;
    st4(a.G + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j, x);
  }
};

// ---- L_G^{-1} update of one Cholesky panel (strict lower triangle of RL) -----------------
//   rows r in [k0, k1):  Linv[r][j] = (L11^{-1} B)[r - k0][j],           j < r
//   rows r in [k1, n):   Linv[r][j] = C_in[r][j] - (W B)[r - k1][j],       j < k1
// with B = the panel rows of L_G^{-1} before the panel (Bp, identity block included),
// A rows = [L11^{-1}; W] (W = L21 L11^{-1}), C_in = Linv[r][j] for j < k0 and 0 on the
// panel's own columns.  B lives in its own buffer, so the panel rows can be overwritten.
struct RWLinvArgs {
  int n, k0, k1, ldw;
  float* RL;
  const float* Wl;  // rows [k0, n): L11^{-1} then W
  const float* Bp;  // [ldw][n] per matrix: raw panel rows, columns [0, k1)
  int* info;
  int lim;          // rows [k0, lim) are updated (n: every row below the panel)
  // Next panel's snapshot slot ([ldw][n] per matrix, like Bp) or nullptr: rows [k1, k1 + wn)
  // of the result, columns < k1, are the next panel's rows of L_G^{-1} "before the panel"; they
  // are stored there as well, so the next panel does not copy them back out of RL.
  float* Bn = nullptr;
  int wn = 0;
};
struct RWLinv {
  using Args = RWLinvArgs;
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = a.lim - a.k0;
    N = a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(const Args&, int, int) { return true; }
  __device__ static const float* a_ptr(const Args& a, int64_t b, int m) {
    return a.Wl + ((int64_t)b * a.n + a.k0 + m) * a.ldw;
  }
  __device__ static const float* b_ptr(const Args& a, int64_t b, int k) {
    return a.Bp + ((int64_t)b * a.ldw + k) * a.n;
  }
  // C_in: L_G^{-1}[r][j] for j < k0 on rows below the panel; 0 on the panel's own columns
  // (identity block) and on the panel rows, which are replaced outright (k0 % 4 == 0).
  __device__ static const void* c_addr(const Args& a, int64_t b, int m, int j) {
    const int r = a.k0 + m;
    if (r < a.k1 || j >= a.k0) return nullptr;
    return a.RL + mat_off(b, a.n) + (int64_t)r * a.n + j;
  }
  __device__ static float4 c_load4(const Args& a, int64_t b, int m, int j) {
    const int r = a.k0 + m;
    if (r < a.k1 || j >= a.k0) return make_float4(0.f, 0.f, 0.f, 0.f);
    return ld4rw(a.RL + mat_off(b, a.n) + (int64_t)r * a.n + j);
  }
  __device__ static void store4(const Args& a, int64_t b, int m, int j, float4 x) {
    const int r = a.k0 + m;
    float* p = a.RL + mat_off(b, a.n) + (int64_t)r * a.n + j;
    if (r < a.k1) {  // panel row: result is +L11^{-1} B (the kernel computed 0 - acc)
      const float t[4] = {-x.x, -x.y, -x.z, -x.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (j + q < r) p[q] = t[q];
    } else {
      st4(p, x);
      if (a.Bn && r < a.k1 + a.wn) st4(a.Bn + ((int64_t)b * a.ldw + (r - a.k1)) * a.n + j, x);
    }
  }
};

// ---- the same update for long K (the chart's K = 128 block update), SGEMM-shaped -----------
// 128 x 128 output tile per CTA, 8 x 8 outputs per thread (rows ty*4 + i and 64 + ty*4 + i,
// columns tx*4 + j and 64 + tx*4 + j, so a warp's shared-memory fragment reads are
// conflict-free), K consumed in slices of 16 that are double-buffered: the global loads of
// slice s+1 are in flight while slice s is multiplied out of shared memory.  Each output
// accumulates its K products in order k = 0, 1, ... with fmaf, exactly like rankw_kernel, so
// both give bit-identical results; this one issues ~4x fewer shared-memory loads per FMA.
constexpr int RWB_T = 128, RWB_K = 16, RWB_LD = RWB_T + 4;

template <class Pb>
__global__ void __launch_bounds__(256, 2) rankw_big_kernel(typename Pb::Args a) {
  __shared__ __align__(16) float As[2][RWB_K][RWB_LD];
  __shared__ __align__(16) float Bs[2][RWB_K][RWB_LD];
  const int64_t b = blockIdx.z;
  const int m0 = blockIdx.y * RWB_T, n0 = blockIdx.x * RWB_T;
  int M, N, K;
  Pb::dims(a, M, N, K);
  if (m0 >= M || n0 >= N || !Pb::live(a, m0, n0)) return;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  // the C tile (128 rows x 4 lines of 128 bytes) starts towards L2 before the K loop
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int idx = tid + 256 * h, row = idx >> 2, j = n0 + 32 * (idx & 3);
    if (m0 + row < M && j < N) {
      const void* p = Pb::c_addr(a, b, m0 + row, j);
      if (p) asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    }
  }
  // loaders: A slice = 128 rows x 16 k (two float4 per thread), B slice = 16 k x 128 columns
  const int am = tid >> 2, akc = tid & 3;        // rows am and am + 64, k 4*akc .. +3
  const int bk = tid >> 5, bc = (tid & 31) * 4;  // k rows bk and bk + 8, columns bc .. +3
  float4 ra[2], rb[2];
  auto fetch = [&](int kb) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = am + 64 * h, k = kb + 4 * akc;
      ra[h] = (m0 + m < M && k < K)
                  ? __ldg(reinterpret_cast<const float4*>(Pb::a_ptr(a, b, m0 + m) + k))
                  : make_float4(0.f, 0.f, 0.f, 0.f);
      const int kk = kb + bk + 8 * h;
      rb[h] = (kk < K && n0 + bc < N) ? ld4v(Pb::b_ptr(a, b, kk) + n0 + bc)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto put = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = am + 64 * h;
      As[buf][4 * akc + 0][m] = ra[h].x;
      As[buf][4 * akc + 1][m] = ra[h].y;
      As[buf][4 * akc + 2][m] = ra[h].z;
      As[buf][4 * akc + 3][m] = ra[h].w;
      st4(&Bs[buf][bk + 8 * h][bc], rb[h]);
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const int ns = (K + RWB_K - 1) / RWB_K;
  fetch(0);
  put(0);
  __syncthreads();
  for (int s = 0; s < ns; ++s) {
    const int buf = s & 1;
    if (s + 1 < ns) fetch((s + 1) * RWB_K);
#pragma unroll
    for (int k = 0; k < RWB_K; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
      const float ar[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float br[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    if (s + 1 < ns) {
      put(buf ^ 1);  // the other buffer was last read in slice s - 1, before the barrier
      __syncthreads();
    }
  }
  // C loads of four rows issued before their stores (C may be updated in place)
#pragma unroll
  for (int i0 = 0; i0 < 8; i0 += 4) {
    float4 xs[4][2];
#pragma unroll
    for (int i = i0; i < i0 + 4; ++i) {
      const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = n0 + (h ? 64 : 0) + tx * 4;
        if (m < M && j < N) xs[i - i0][h] = Pb::c_load4(a, b, m, j);
      }
    }
#pragma unroll
    for (int i = i0; i < i0 + 4; ++i) {
      const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
      if (m >= M) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = n0 + (h ? 64 : 0) + tx * 4;
        if (j < N) {
          float4 x = xs[i - i0][h];
          x.x -= acc[i][4 * h]; x.y -= acc[i][4 * h + 1];
          x.z -= acc[i][4 * h + 2]; x.w -= acc[i][4 * h + 3];
          Pb::store4(a, b, m, j, x);
        }
      }
    }
  }
}

// ---- general in-place rank-K update of a block of each matrix (K may exceed 32) ----------
//   C[r0 + m][c0 + j] -= sum_k W[r0 + m][k] * C[kb + k][c0 + j],  m < M, j < N, k < K
// W rows have ldw columns (the pointer already at the first column used).  The B rows
// [kb, kb + K) must not overlap the updated rows [r0, r0 + M) (they are read while others
// are written).  Used by the two-level chart elimination.
struct RWGenArgs {
  int n, r0, c0, M, N, K, kb, ldw;
  float* C;
  const float* W;
  int* info;
};
struct RWGen {
  using Args = RWGenArgs;
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = a.M;
    N = a.N;
    K = a.K;
  }
  __device__ static bool live(const Args&, int, int) { return true; }
  __device__ static const float* a_ptr(const Args& a, int64_t b, int m) {
    return a.W + ((int64_t)b * a.n + a.r0 + m) * a.ldw;
  }
  __device__ static const float* b_ptr(const Args& a, int64_t b, int k) {
    return a.C + mat_off(b, a.n) + (int64_t)(a.kb + k) * a.n + a.c0;
  }
  __device__ static const void* c_addr(const Args& a, int64_t b, int m, int j) {
    return a.C + mat_off(b, a.n) + (int64_t)(a.r0 + m) * a.n + a.c0 + j;
  }
  __device__ static float4 c_load4(const Args& a, int64_t b, int m, int j) {
    return ld4rw(a.C + mat_off(b, a.n) + (int64_t)(a.r0 + m) * a.n + a.c0 + j);
  }
  __device__ static void store4(const Args& a, int64_t b, int m, int j, float4 x) {
    st4(a.C + mat_off(b, a.n) + (int64_t)(a.r0 + m) * a.n + a.c0 + j, x);
  }
};

}  // namespace qrb
