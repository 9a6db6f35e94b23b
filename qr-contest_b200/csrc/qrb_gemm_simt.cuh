// qrb200 -- batched fp32 SIMT GEMM tiles for the trailing updates, Grams and the closure.
//
// One 64x64 output tile per CTA (256 threads, 4x4 register micro-tile, BK = 32 staged in
// shared memory).  grid = (tiles_n, tiles_m, batch); the problem policy decides which
// tiles are live (triangular skip), how A/B tiles are fetched (row gathers, transposed
// operands, input dtype) and what the epilogue writes.
//
// Policies (all per matrix, n x n row-major):
//   TrailW     C'[k1+q][k1+j] = C[src(k1+q)][k1+j] - sum_i W[k1+q][i] * C[src(k0+i)][k1+j]
//              (LU and chart trailing update; src = row gather of the pivoted LU, identity
//              for the chart)
//   TrailSyrk  G[k1+q][k1+j] -= sum_i R[k0+i][k1+q] * R[k0+i][k1+j]   (lower tiles; Cholesky)
//   Gram       G = X^T X                                               (lower tiles)
//   Closure    H[i][j] = s_i * (Q^T A)[i][j], j >= i                    (upper tiles)
#pragma once
#include "qrb_common.cuh"

namespace qrb {

constexpr int GT = 64;   // tile edge
constexpr int GBK = 32;  // k-step

struct TrailWArgs {
  int n, k0, k1, ldw;
  const void* Cold;   // TIn
  float* Cnew;
  const float* W;
  const int* srcmap;  // nullptr -> identity
};

template <typename TIn>
struct TrailW {
  using Args = TrailWArgs;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = N = a.n - a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(int, int) { return true; }
  __device__ static int srow(const Args& a, int64_t b, int r) {
    return a.srcmap ? checked_row(a.srcmap[b * a.n + r], 0, a.n, nullptr) : r;
  }
  // A(m, k) = W[k1+m][k]
  __device__ static float ldA(const Args& a, int64_t b, int k, int m) {
    return a.W[((int64_t)b * a.n + a.k1 + m) * a.ldw + k];
  }
  // B(k, j) = C[src(k0+k)][k1+j]
  __device__ static float ldB(const Args& a, int64_t b, int k, int j) {
    const TIn* C = reinterpret_cast<const TIn*>(a.Cold) + mat_off(b, a.n);
    return to_f32(C[(int64_t)srow(a, b, a.k0 + k) * a.n + a.k1 + j]);
  }
  __device__ static void epi(const Args& a, int64_t b, int m, int j, float v) {
    const TIn* C = reinterpret_cast<const TIn*>(a.Cold) + mat_off(b, a.n);
    const int r = srow(a, b, a.k1 + m);
    a.Cnew[mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j] =
        to_f32(C[(int64_t)r * a.n + a.k1 + j]) - v;
  }
};

struct TrailSyrkArgs {
  int n, k0, k1;
  float* G;
  const float* R;
};

struct TrailSyrk {
  using Args = TrailSyrkArgs;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = N = a.n - a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(int tm, int tn) { return tm >= tn; }
  __device__ static float ldA(const Args& a, int64_t b, int k, int m) {
    return a.R[mat_off(b, a.n) + (int64_t)(a.k0 + k) * a.n + a.k1 + m];
  }
  __device__ static float ldB(const Args& a, int64_t b, int k, int j) {
    return a.R[mat_off(b, a.n) + (int64_t)(a.k0 + k) * a.n + a.k1 + j];
  }
  __device__ static void epi(const Args& a, int64_t b, int m, int j, float v) {
    float* g = a.G + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j;
    *g = *g - v;
  }
};

struct GramArgs {
  int n;
  const float* X;
  float* G;
};

struct Gram {
  using Args = GramArgs;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) { M = N = K = a.n; }
  __device__ static bool live(int tm, int tn) { return tm >= tn; }
  __device__ static float ldA(const Args& a, int64_t b, int k, int m) {
    return a.X[mat_off(b, a.n) + (int64_t)k * a.n + m];
  }
  __device__ static float ldB(const Args& a, int64_t b, int k, int j) {
    return a.X[mat_off(b, a.n) + (int64_t)k * a.n + j];
  }
  __device__ static void epi(const Args& a, int64_t b, int m, int j, float v) {
    a.G[mat_off(b, a.n) + (int64_t)m * a.n + j] = v;
  }
};

struct ClosureArgs {
  int n;
  const float* Q;
  const void* A;   // TIn
  const float* s;
  void* H;         // TIn (output dtype == input dtype)
};

template <typename TIn>
struct Closure {
  using Args = ClosureArgs;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) { M = N = K = a.n; }
  __device__ static bool live(int tm, int tn) { return tn >= tm; }
  __device__ static float ldA(const Args& a, int64_t b, int k, int m) {
    return a.Q[mat_off(b, a.n) + (int64_t)k * a.n + m];
  }
  __device__ static float ldB(const Args& a, int64_t b, int k, int j) {
    const TIn* A = reinterpret_cast<const TIn*>(a.A) + mat_off(b, a.n);
    return to_f32(A[(int64_t)k * a.n + j]);
  }
  __device__ static void epi(const Args& a, int64_t b, int m, int j, float v) {
    if (j < m) return;
    TIn* H = reinterpret_cast<TIn*>(a.H) + mat_off(b, a.n);
    H[(int64_t)m * a.n + j] = from_f32<TIn>(a.s[b * a.n + m] * v);
  }
};

template <class Pb>
__global__ void __launch_bounds__(256) simt_gemm_kernel(typename Pb::Args a) {
  __shared__ __align__(16) float As[GBK][GT + 4];
  __shared__ __align__(16) float Bs[GBK][GT + 4];
  const int64_t b = blockIdx.z;
  const int tmi = blockIdx.y, tni = blockIdx.x;
  if (!Pb::live(tmi, tni)) return;
  int M, N, K;
  Pb::dims(a, M, N, K);
  const int m0 = tmi * GT, n0 = tni * GT;
  if (m0 >= M || n0 >= N) return;
  const int tid = threadIdx.x;
  const int tn = tid & 15, tm = tid >> 4;

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int kb = 0; kb < K; kb += GBK) {
#pragma unroll
    for (int t = 0; t < (GBK * GT) / 256; ++t) {
      const int idx = tid + 256 * t;
      const int kk = idx / GT, mm = idx - kk * GT;
      const int k = kb + kk;
      As[kk][mm] = (k < K && m0 + mm < M) ? Pb::ldA(a, b, k, m0 + mm) : 0.f;
      Bs[kk][mm] = (k < K && n0 + mm < N) ? Pb::ldB(a, b, k, n0 + mm) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < GBK; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&As[kk][tm * 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk][tn * 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w};
      const float br[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tm * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tn * 4 + j;
      if (c < N) Pb::epi(a, b, m, c, acc[i][j]);
    }
  }
}

}  // namespace qrb

namespace qrb {

// ---- CholeskyQR without a triangular solve ----------------------------------------------
// The Cholesky elimination leaves L_G^{-1} (strict lower triangle of the RL buffer, unit
// diagonal implicit) and D, with R^{-1} = L_G^{-T} D^{-1/2}.  These policies build
// L_G^{-1} panel by panel and apply R^{-1}.

// L_G^{-1} update of one Cholesky panel, scalar tiles (any n); same contract as RWLinv in
// qrb_rankw.cuh: rows [k0, k1) get L11^{-1} B, rows [k1, n) get C_in - W B (j < k1), with
// A rows = [L11^{-1}; W] and B = the panel rows of L_G^{-1} before the panel.
struct LinvTrailArgs {
  int n, k0, k1, ldw;
  float* RL;
  const float* Wl;
  const float* Bp;
};
struct LinvTrail {
  using Args = LinvTrailArgs;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = a.n - a.k0;
    N = a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(int, int) { return true; }
  __device__ static float ldA(const Args& a, int64_t b, int k, int m) {
    return a.Wl[((int64_t)b * a.n + a.k0 + m) * a.ldw + k];
  }
  __device__ static float ldB(const Args& a, int64_t b, int k, int j) {
    return a.Bp[((int64_t)b * a.ldw + k) * a.n + j];
  }
  __device__ static void epi(const Args& a, int64_t b, int m, int j, float v) {
    const int r = a.k0 + m;
    float* p = a.RL + mat_off(b, a.n) + (int64_t)r * a.n + j;
    if (r < a.k1) {
      if (j < r) *p = v;
    } else {
      *p = ((j < a.k0) ? *p : 0.f) - v;
    }
  }
};

// R^{-1}(k, j) of one CholeskyQR pass, and its use:
//   pass 1: Q[m][j] = sum_k X[m][k] R^{-1}[k][j]
//   pass 2: Q[m][j] = X[m][j] - sum_k X[m][k] F[k][j],  F = I - R^{-1}  (small: the tensor
//           cores / accumulators only see the correction, float32 does the subtraction)
struct QApplyArgs {
  int n;
  int pass2;
  const float* X;
  const float* RL;
  const float* D;
  float* Q;
  int* info;
};
__device__ __forceinline__ float rinv_entry(const QApplyArgs& a, int64_t b, int k, int j) {
  if (k > j) return 0.f;
  const float rs = 1.f / sqrtf(a.D[b * a.n + j]);
  if (k == j) return a.pass2 ? (1.f - rs) : rs;
  const float l = a.RL[mat_off(b, a.n) + (int64_t)j * a.n + k];
  return a.pass2 ? -(l * rs) : l * rs;
}
struct QApply {
  using Args = QApplyArgs;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) { M = N = K = a.n; }
  __device__ static bool live(int, int) { return true; }
  __device__ static float ldA(const Args& a, int64_t b, int k, int m) {
    return a.X[mat_off(b, a.n) + (int64_t)m * a.n + k];
  }
  __device__ static float ldB(const Args& a, int64_t b, int k, int j) {
    return rinv_entry(a, b, k, j);
  }
  __device__ static void epi(const Args& a, int64_t b, int m, int j, float v) {
    const int64_t o = mat_off(b, a.n) + (int64_t)m * a.n + j;
    a.Q[o] = a.pass2 ? a.X[o] - v : v;
  }
};

// G[j][j] = sum_k X[k][j]^2 in float32 (fixed order): exact diagonals for the second Gram.
__global__ void __launch_bounds__(256) colnorm2_kernel(const float* __restrict__ X,
                                                       float* __restrict__ G, int n) {
  const int64_t b = blockIdx.y;
  const int j = blockIdx.x * 256 + threadIdx.x;
  if (j >= n) return;
  const float* x = X + mat_off(b, n) + j;
  float acc = 0.f;
  for (int k = 0; k < n; ++k) {
    const float v = x[(int64_t)k * n];
    acc = fmaf(v, v, acc);
  }
  G[mat_off(b, n) + (int64_t)j * n + j] = acc;
}

}  // namespace qrb
