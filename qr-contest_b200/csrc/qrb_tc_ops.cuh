// qrb200 -- the pipeline's GEMM-shaped stages as policies of the tcgen05 3xTF32 tile kernel.
//
//   GramTC      G = X^T X                      lower tiles   (reflection_no_reflectors.py:73)
//   ClosureTC   H_ij = s_i (Q^T A)_ij, j >= i  upper tiles   (:186, :195)
//   TrailWTC    C'[k1+q] = C[src(k1+q)] - W[k1+q] * C[src(k0:k1)]   (LU trailing update,
//               :66 via getrf; src = pivot gather)
//   SyrkTC      G22 -= R12^T R12               lower tiles   (Cholesky trailing update, :76)
//   QApplyTC    Q = X R^{-1} / Q = X - X (I - R^{-1})        (solve_triangular, :77)
#pragma once
#include "qrb_gemm_simt.cuh"
#include "qrb_tc.cuh"

namespace qrb {
namespace tc {

// 4 consecutive elements starting at p, `valid` of them in range; vector load when allowed.
template <typename T>
__device__ __forceinline__ void ld4(const T* p, int valid, bool vec, float (&o)[4]) {
  if (vec && valid >= 4) {
    if constexpr (sizeof(T) == 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p));
      o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
    } else {
      const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
      const T* h = reinterpret_cast<const T*>(&t);
      o[0] = to_f32(h[0]); o[1] = to_f32(h[1]); o[2] = to_f32(h[2]); o[3] = to_f32(h[3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = (i < valid) ? to_f32(p[i]) : 0.f;
  }
}

__device__ __forceinline__ int clamp4(int x) { return x < 0 ? 0 : (x > 4 ? 4 : x); }

// v[i][kk] = S[(k0+kk) * ld + c0 + i]  (source contiguous along the tile-row index)
template <typename T>
__device__ __forceinline__ void ld_rows_k(const T* S, int64_t ld, int c0, int cvalid, int k0,
                                          int kvalid, bool vec, float (&v)[4][4]) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    if (kk < kvalid) ld4(S + (int64_t)(k0 + kk) * ld + c0, cvalid, vec, o);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i][kk] = o[i];
  }
}

__device__ __forceinline__ void st_row32(float* dst, const float* v, int valid, bool vec) {
  if (vec && valid >= 32) {
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = v[i];
  }
}

// dst[0..31] = src[0..31] - v[0..31] (src may alias dst), `valid` columns in range
template <typename T>
__device__ __forceinline__ void sub_row32(const T* src, float* dst, const float* v, int valid,
                                          bool vec) {
  float o[32];
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    float t[4];
    ld4(src + i, clamp4(valid - i), vec, t);
    o[i] = t[0] - v[i]; o[i + 1] = t[1] - v[i + 1];
    o[i + 2] = t[2] - v[i + 2]; o[i + 3] = t[3] - v[i + 3];
  }
  st_row32(dst, o, valid, vec);
}

// ---------------------------------------------------------------------------------------
struct GramTCArgs {
  int n;
  const float* X;
  float* G;
  int* info;
};
struct GramTC {
  // the epilogue reads nothing from global memory (no early L2 prefetch)
  __device__ static const void* c_addr(const GramTCArgs&, int64_t, int, int) { return nullptr; }
  using Args = GramTCArgs;
  static constexpr bool A_ALONG_K = false, B_ALONG_K = false;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) { M = N = K = a.n; }
  __device__ static bool live(int m0, int n0, int bm, int) { return n0 < m0 + bm; }
  __device__ static void krange(const Args& a, int, int, int& kb, int& ke) { kb = 0; ke = a.n; }
  __device__ static void loadA(const Args& a, int64_t b, int m0, int k0, float (&v)[4][4]) {
    ld_rows_k(a.X + mat_off(b, a.n), a.n, m0, clamp4(a.n - m0), k0, clamp4(a.n - k0),
              (a.n & 3) == 0, v);
  }
  __device__ static void loadB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
    loadA(a, b, j0, k0, v);
  }
  __device__ static void store(const Args& a, int64_t b, int m, int j0, const float* v, int,
                               int N) {
    st_row32(a.G + mat_off(b, a.n) + (int64_t)m * a.n + j0, v, N - j0, (a.n & 3) == 0);
  }
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void fixB(const Args&, int64_t, int, int, float (&)[4][4]) {}
};

// ---------------------------------------------------------------------------------------
struct ClosureTCArgs {
  int n;
  const float* Q;
  const void* A;
  const float* s;
  void* H;
  int* info;
};
template <typename T>
struct ClosureTC {
  __device__ static const void* c_addr(const ClosureTCArgs&, int64_t, int, int) { return nullptr; }
  using Args = ClosureTCArgs;
  static constexpr bool A_ALONG_K = false, B_ALONG_K = false;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) { M = N = K = a.n; }
  __device__ static bool live(int m0, int n0, int, int bn) { return n0 + bn > m0; }
  __device__ static void krange(const Args& a, int, int, int& kb, int& ke) { kb = 0; ke = a.n; }
  __device__ static void loadA(const Args& a, int64_t b, int m0, int k0, float (&v)[4][4]) {
    ld_rows_k(a.Q + mat_off(b, a.n), a.n, m0, clamp4(a.n - m0), k0, clamp4(a.n - k0),
              (a.n & 3) == 0, v);
  }
  __device__ static void loadB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
    ld_rows_k(reinterpret_cast<const T*>(a.A) + mat_off(b, a.n), a.n, j0, clamp4(a.n - j0), k0,
              clamp4(a.n - k0), (a.n & 3) == 0, v);
  }
  __device__ static void store(const Args& a, int64_t b, int m, int j0, const float* v, int,
                               int N) {
    T* H = reinterpret_cast<T*>(a.H) + mat_off(b, a.n) + (int64_t)m * a.n;
    const float sm = a.s[b * a.n + m];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int j = j0 + i;
      if (j >= m && j < N) H[j] = from_f32<T>(sm * v[i]);
    }
  }
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void fixB(const Args&, int64_t, int, int, float (&)[4][4]) {}
};

// ---------------------------------------------------------------------------------------
struct TrailWTCArgs {
  int n, k0, k1, ldw;
  const void* Cold;
  float* Cnew;
  const float* W;
  const int* srcmap;
  int* info;
};
template <typename T>
struct TrailWTC {
  using Args = TrailWTCArgs;
  static constexpr bool A_ALONG_K = true, B_ALONG_K = false;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = N = a.n - a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(int, int, int, int) { return true; }
  __device__ static void krange(const Args& a, int, int, int& kb, int& ke) {
    kb = 0;
    ke = a.k1 - a.k0;
  }
  __device__ static int srow(const Args& a, int64_t b, int r) {
    return a.srcmap ? checked_row(a.srcmap[b * a.n + r], 0, a.n, a.info + b) : r;
  }
  __device__ static void loadA(const Args& a, int64_t b, int m0, int k0, float (&v)[4][4]) {
    const int M = a.n - a.k1, K = a.k1 - a.k0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (m0 + i < M)
        ld4(a.W + ((int64_t)b * a.n + a.k1 + m0 + i) * a.ldw + k0, clamp4(K - k0),
            (a.ldw & 3) == 0, o);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) v[i][kk] = o[kk];
    }
  }
  __device__ static void loadB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
    const int N = a.n - a.k1, K = a.k1 - a.k0;
    const T* C = reinterpret_cast<const T*>(a.Cold) + mat_off(b, a.n);
    const bool vec = ((a.n & 3) == 0) && ((a.k1 & 3) == 0);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (k0 + kk < K)
        ld4(C + (int64_t)srow(a, b, a.k0 + k0 + kk) * a.n + a.k1 + j0, clamp4(N - j0), vec, o);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i][kk] = o[i];
    }
  }
  __device__ static void store(const Args& a, int64_t b, int m, int j0, const float* v, int,
                               int N) {
    const T* C = reinterpret_cast<const T*>(a.Cold) + mat_off(b, a.n) +
                 (int64_t)srow(a, b, a.k1 + m) * a.n + a.k1 + j0;
    float* D = a.Cnew + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j0;
    sub_row32(C, D, v, N - j0, ((a.n & 3) == 0) && ((a.k1 & 3) == 0));
  }
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void fixB(const Args&, int64_t, int, int, float (&)[4][4]) {}
};

// ---------------------------------------------------------------------------------------
struct SyrkTCArgs {
  int n, k0, k1;
  float* G;
  const float* R;
  int* info;
};
struct SyrkTC {
  using Args = SyrkTCArgs;
  static constexpr bool A_ALONG_K = false, B_ALONG_K = false;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = N = a.n - a.k1;
    K = a.k1 - a.k0;
  }
  __device__ static bool live(int m0, int n0, int bm, int) { return n0 < m0 + bm; }
  __device__ static void krange(const Args& a, int, int, int& kb, int& ke) {
    kb = 0;
    ke = a.k1 - a.k0;
  }
  __device__ static void loadA(const Args& a, int64_t b, int m0, int k0, float (&v)[4][4]) {
    const int M = a.n - a.k1, K = a.k1 - a.k0;
    ld_rows_k(a.R + mat_off(b, a.n) + (int64_t)a.k0 * a.n + a.k1, a.n, m0, clamp4(M - m0), k0,
              clamp4(K - k0), ((a.n & 3) == 0) && ((a.k1 & 3) == 0), v);
  }
  __device__ static void loadB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
    loadA(a, b, j0, k0, v);
  }
  // address the epilogue reads at (row m, column j) of the tile, for an early L2 prefetch
  __device__ static const void* c_addr(const Args& a, int64_t b, int m, int j) {
    return a.G + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j;
  }
  __device__ static void store(const Args& a, int64_t b, int m, int j0, const float* v, int,
                               int N) {
    float* g = a.G + mat_off(b, a.n) + (int64_t)(a.k1 + m) * a.n + a.k1 + j0;
    sub_row32(g, g, v, N - j0, ((a.n & 3) == 0) && ((a.k1 & 3) == 0));
  }
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void fixB(const Args&, int64_t, int, int, float (&)[4][4]) {}
};

// ---------------------------------------------------------------------------------------
// L_G^{-1} update of a whole column block [kb, ke) of the Cholesky elimination, for the rows
// below the block (the block's panels updated only the rows inside it):
//   Linv[r][j] = C_in[r][j] - sum_p W_p[r] B_p[j],   r in [ke, n), j < ke,
// with W_p = L21 L11^{-1} of panel p (column block [kb + 32p, kb + 32p + 32) of the W buffer)
// and B_p = the panel's rows of L_G^{-1} just before that panel (rows [32p, 32p + 32) of the Bp
// buffer, identity block included, zero from the panel's end column on).  C_in is Linv[r][j]
// for j < kb and 0 on the block's own columns.  The sum over the block's panels is the product
// of the stacked operands, one GEMM with K = ke - kb.
struct LinvBlkArgs {
  int n, kb, ke, ldw;
  float* RL;
  const float* W;   // [n][ldw] per matrix
  const float* Bp;  // [ldw][n] per matrix
  int* info;
};
struct LinvBlkTC {
  using Args = LinvBlkArgs;
  static constexpr bool A_ALONG_K = true, B_ALONG_K = false;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = a.n - a.ke;
    N = a.ke;
    K = a.ke - a.kb;
  }
  __device__ static bool live(int, int, int, int) { return true; }
  __device__ static void krange(const Args& a, int, int, int& kb, int& ke) {
    kb = 0;
    ke = a.ke - a.kb;
  }
  __device__ static void loadA(const Args& a, int64_t b, int m0, int k0, float (&v)[4][4]) {
    const int M = a.n - a.ke, K = a.ke - a.kb;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (m0 + i < M)
        ld4(a.W + ((int64_t)b * a.n + a.ke + m0 + i) * a.ldw + k0, clamp4(K - k0),
            (a.ldw & 3) == 0, o);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) v[i][kk] = o[kk];
    }
  }
  __device__ static void loadB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
    ld_rows_k(a.Bp + (int64_t)b * a.ldw * a.n, a.n, j0, clamp4(a.ke - j0), k0,
              clamp4(a.ke - a.kb - k0), (a.n & 3) == 0, v);
  }
  // row k of B belongs to panel k / 32, whose snapshot ends at column kb + 32 (k / 32 + 1)
  __device__ static void fixB(const Args& a, int64_t, int j0, int k0, float (&v)[4][4]) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int jend = a.kb + 32 * ((k0 + kk) / 32 + 1);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (j0 + i >= jend) v[i][kk] = 0.f;
    }
  }
  __device__ static const void* c_addr(const Args& a, int64_t b, int m, int j) {
    return j < a.kb ? a.RL + mat_off(b, a.n) + (int64_t)(a.ke + m) * a.n + j : nullptr;
  }
  __device__ static void store(const Args& a, int64_t b, int m, int j0, const float* v, int,
                               int N) {
    float* row = a.RL + mat_off(b, a.n) + (int64_t)(a.ke + m) * a.n;
    float o[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const int j = j0 + i;
      float t[4] = {0.f, 0.f, 0.f, 0.f};
      if (j + 3 < a.kb && (a.n & 3) == 0) {
        const float4 c = *reinterpret_cast<const float4*>(row + j);
        t[0] = c.x; t[1] = c.y; t[2] = c.z; t[3] = c.w;
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j + u < a.kb) t[u] = row[j + u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) o[i + u] = t[u] - v[i + u];
    }
    st_row32(row + j0, o, N - j0, (a.n & 3) == 0);
  }
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
};

// ---------------------------------------------------------------------------------------
// R^{-1} application of one CholeskyQR pass (see QApply in qrb_gemm_simt.cuh):
// B(k, j) = R^{-1}[k][j] (pass 1) or (I - R^{-1})[k][j] (pass 2), built in the loader from
// row j of L_G^{-1} (contiguous in k) and d_j; the k range of column tile [n0, n0+BN) stops
// at the tile's last column because R^{-1} is upper triangular.  Needs n % 4 == 0.
struct QApplyTC {
  using Args = QApplyArgs;
  static constexpr bool A_ALONG_K = true, B_ALONG_K = true;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) { M = N = K = a.n; }
  __device__ static bool live(int, int, int, int) { return true; }
  __device__ static void krange(const Args& a, int, int n0, int& kb, int& ke) {
    kb = 0;
    ke = min(a.n, n0 + 128);
  }
  __device__ static void loadA(const Args& a, int64_t b, int m0, int k0, float (&v)[4][4]) {
    const float* X = a.X + mat_off(b, a.n);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (m0 + i < a.n) ld4(X + (int64_t)(m0 + i) * a.n + k0, clamp4(a.n - k0), true, o);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) v[i][kk] = o[kk];
    }
  }
  __device__ static void loadB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
    const float* RL = a.RL + mat_off(b, a.n);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = j0 + i;
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (j < a.n && k0 <= j) ld4(RL + (int64_t)j * a.n + k0, clamp4(a.n - k0), true, o);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) v[i][kk] = o[kk];
    }
  }
  // raw row j of the R buffer (strict lower = L_G^{-1}) -> R^{-1} or I - R^{-1}
  __device__ static void fixB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = j0 + i;
      const float rs = (j < a.n) ? 1.f / sqrtf(a.D[b * a.n + j]) : 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int k = k0 + kk;
        float r;
        if (j >= a.n || k > j) r = 0.f;
        else if (k < j) r = a.pass2 ? -(v[i][kk] * rs) : v[i][kk] * rs;
        else r = a.pass2 ? (1.f - rs) : rs;
        v[i][kk] = r;
      }
    }
  }
  __device__ static const void* c_addr(const Args& a, int64_t b, int m, int j) {
    return a.pass2 ? a.X + mat_off(b, a.n) + (int64_t)m * a.n + j : nullptr;
  }
  __device__ static void store(const Args& a, int64_t b, int m, int j0, const float* v, int,
                               int N) {
    const int64_t o = mat_off(b, a.n) + (int64_t)m * a.n + j0;
    if (a.pass2) {
      sub_row32(a.X + o, a.Q + o, v, N - j0, true);
    } else {
      st_row32(a.Q + o, v, N - j0, true);
    }
  }
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
};

}  // namespace tc
}  // namespace qrb
