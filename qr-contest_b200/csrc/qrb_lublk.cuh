// qrb200 -- the block update of the two-level LU (reflection_no_reflectors.py:66, getrf's
// right-looking blocked form).
//
// Inside a block of KB = 128 columns the 32-wide panels (with their pivot search over every live
// row) update only the block's columns.  After the block, ONE update with K = 128 brings the rest
// of the trailing matrix up to date:
//     C22' = C22 - W A12,   W = L21 L11^{-1},
// where A12 are the block's pivot rows as they were at block start, L11 the block's unit-lower
// multipliers among its pivot rows and L21 those of the rows below.  Rows are never moved: the
// trailing buffers hold rows in getrf's position order, each panel records where its positions
// came from (its row map, one slot per panel of the block), and the update gathers block-start
// rows through the composition of the block's maps.
//   lu_blk_prep_kernel : per matrix, the composite map and L11^{-1} (128 x 128, shared memory)
//   WBlkTC             : W = L21 L11^{-1} as a tcgen05 3xTF32 tile (L21 gathered from P*L)
// The update itself is tc_gemm_kernel<TrailWTC> with K = 128 and the composite map.
#pragma once
#include "qrb_tc_ops.cuh"

namespace qrb {

constexpr int kLuBlock = 128;  // columns per block of the two-level LU
constexpr int kLuPanel = 32;   // panel width inside a block

struct LuBlkArgs {
  int n, kb, ke, npan;     // block columns [kb, ke); its npan panels start at kb + 32 j
  const int* slots;        // per-panel row maps: slot j at slots + j * slot_stride, [b][n] each
  int64_t slot_stride;
  const int* orig;         // [b][n] original row id at each position (block end)
  const float* L;          // [b][n][n] P*L in original row order
  int* comp;               // [b][n] out: block-start position of the row at position p >= kb
  float* Linv;             // [b][KB][KB] out: L11^{-1}, unit lower, row-major
  int* info;
};

constexpr int kLuPrepThreads = 512;
constexpr int kLuLD = kLuBlock + 1;
__host__ __device__ constexpr size_t lu_prep_smem() { return 2 * (size_t)kLuBlock * kLuLD * 4; }

__global__ void __launch_bounds__(kLuPrepThreads) lu_blk_prep_kernel(LuBlkArgs a) {
  extern __shared__ float lsm[];
  float* Ls = lsm;                    // [KB][KB + 1] L11 (strictly lower part)
  float* X = lsm + kLuBlock * kLuLD;  // [KB][KB + 1] L11^{-1}
  const int64_t b = blockIdx.x;
  const int n = a.n, kb = a.kb, KB = a.ke - a.kb, tid = threadIdx.x;
  int* info = a.info + b;
  // composite map: undo the block's panels, last one first (a panel leaves positions before
  // its own first column alone)
  for (int p = kb + tid; p < n; p += kLuPrepThreads) {
    int q = p;
    for (int j = a.npan - 1; j >= 0; --j)
      if (q >= kb + kLuPanel * j) q = checked_row(a.slots[j * a.slot_stride + b * n + q], 0, n, info);
    a.comp[b * n + p] = q;
  }
  // L11[i][t] = multiplier of the pivot row at position kb + i for column kb + t (t < i)
  const float* Lb = a.L + mat_off(b, n);
  for (int idx = tid; idx < KB * KB; idx += kLuPrepThreads) {
    const int i = idx / KB, t = idx - i * KB;
    const int o = checked_row(a.orig[b * n + kb + i], 0, n, info);
    Ls[i * kLuLD + t] = (t < i) ? Lb[(int64_t)o * n + kb + t] : 0.f;
    X[i * kLuLD + t] = (i == t) ? 1.f : 0.f;
  }
  __syncthreads();
  // column j of L11^{-1} by forward substitution, four lanes per column (t = j + g mod 4):
  //   X[i][j] = -sum_{t = j}^{i - 1} L11[i][t] X[t][j]
  // the loop over i is uniform across the warp (guards inside), so the shuffles and warp
  // barriers see every lane
  const int j = tid >> 2, g = tid & 3;
  for (int i = 1; i < kLuBlock; ++i) {
    float acc = 0.f;
    if (j < KB && i < KB && i > j)
      for (int t = j + g; t < i; t += 4) acc = fmaf(Ls[i * kLuLD + t], X[t * kLuLD + j], acc);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (g == 0 && j < KB && i < KB && i > j) X[i * kLuLD + j] = -acc;
    __syncwarp();
  }
  __syncthreads();
  float* Li = a.Linv + b * (int64_t)KB * KB;
  for (int idx = tid; idx < KB * KB; idx += kLuPrepThreads) {
    const int i = idx / KB, t = idx - i * KB;
    Li[idx] = X[i * kLuLD + t];
  }
}

// W[p][j] = sum_k L21[p][k] L11^{-1}[k][j] for the rows below the block (positions p >= ke):
// L21[p][k] = P*L[orig[p]][kb + k].  W is written at rows p of a [b][n][ldw] buffer.
struct WBlkArgs {
  int n, kb, ke, ldw;
  const int* orig;
  const float* L;
  const float* Linv;
  float* W;
  int* info;
};
struct WBlkTC {
  using Args = WBlkArgs;
  static constexpr bool A_ALONG_K = true, B_ALONG_K = false;
  __device__ static void dims(const Args& a, int& M, int& N, int& K) {
    M = a.n - a.ke;
    N = K = a.ke - a.kb;
  }
  __device__ static bool live(int, int, int, int) { return true; }
  __device__ static void krange(const Args& a, int, int n0, int& kb, int& ke) {
    kb = n0 & ~31;  // L11^{-1} is lower triangular: rows k < j contribute nothing to column j
    ke = a.ke - a.kb;
  }
  __device__ static void loadA(const Args& a, int64_t b, int m0, int k0, float (&v)[4][4]) {
    const int M = a.n - a.ke, K = a.ke - a.kb;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (m0 + i < M) {
        const int r = checked_row(a.orig[b * a.n + a.ke + m0 + i], 0, a.n, a.info + b);
        tc::ld4(a.L + mat_off(b, a.n) + (int64_t)r * a.n + a.kb + k0, tc::clamp4(K - k0), true, o);
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) v[i][kk] = o[kk];
    }
  }
  __device__ static void loadB(const Args& a, int64_t b, int j0, int k0, float (&v)[4][4]) {
    const int K = a.ke - a.kb;
    const float* Li = a.Linv + b * (int64_t)K * K;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (k0 + kk < K) tc::ld4(Li + (int64_t)(k0 + kk) * K + j0, tc::clamp4(K - j0), true, o);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i][kk] = o[i];
    }
  }
  __device__ static void store(const Args& a, int64_t b, int m, int j0, const float* v, int,
                               int N) {
    float* D = a.W + ((int64_t)b * a.n + a.ke + m) * a.ldw + j0;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (j0 + i < N) D[i] = v[i];
  }
  __device__ static int* info(const Args& a, int64_t b) { return a.info + b; }
  __device__ static void fixB(const Args&, int64_t, int, int, float (&)[4][4]) {}
};

}  // namespace qrb
