// qrb200 -- C ABI and stage orchestration for the batched square QR (sm_100a).
//
// Pipeline per matrix (reflection_no_reflectors.py):
//   I   frame    : A = P L U (PM_PIVOT panels + TrailW)          -> P*L       (:66)
//                  CholeskyQR pass 1: G = (PL)^T(PL) (Gram), G + mu I = L_G D L_G^T
//                  (PM_CHOL panels + TrailSyrk + LinvTrail), Q1 = PL R1^{-1} with
//                  R1^{-1} = L_G^{-T} D^{-1/2} (QApply, one GEMM)               (:68-79)
//                  CholeskyQR pass 2 on Q1 -> Q = P Q_L  (row order of A)      (:80-81)
//   III chart    : elimination of I - QS on a copy of Q (PM_CHART panels + TrailW)
//                  -> strict lower H, s, tau                               (:86-176,:192)
//   II  closure  : H_upper = s_i * triu(Q^T A)_ij                         (:186,:195)
// The batch is processed in chunks so that the float32 working set stays bounded.
#include "../../include/qrb200.h"
#include "qrb_common.cuh"
#include "qrb_gemm_simt.cuh"
#include "qrb_panel.cuh"
#include "qrb_panel_reg.cuh"
#include "qrb_panel_cl.cuh"
#include "qrb_tc_ops.cuh"
#include "qrb_rankw.cuh"
#include "qrb_tc_rankw.cuh"
#include "qrb_tcx.cuh"
#include "qrb_tmap.cuh"
#include "qrb_small.cuh"
#include "qrb_warp.cuh"

#include <atomic>
#include <type_traits>
#include <mutex>
#include <utility>
#include <vector>

namespace qrb {

// Kernel families, in the order of the per-family timings qrb200_geqrf_batched_timed returns.
enum Family : int {
  F_LU_PANEL = 0, F_LU_TRAIL, F_GRAM, F_CHOL_PANEL, F_CHOL_TRAIL, F_QAPPLY, F_CHART_PANEL,
  F_CHART_TRAIL, F_CLOSURE, F_SMALL, F_COUNT
};

static std::atomic<long long> g_launches{0};
static std::atomic<int> g_gemm_path{0};  // 0 auto, 1 SIMT only, 2 tcgen05 wherever legal
static thread_local cudaError_t g_last_cuda_error = cudaSuccess;

static inline cudaError_t note(cudaError_t e) {
  if (e != cudaSuccess) g_last_cuda_error = e;
  return e;
}

// Optional per-launch CUDA-event bracketing (only for the timed entry point).
struct Prof {
  cudaStream_t st;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> rec;
  cudaEvent_t pending = nullptr;
  int fam = 0;
  void begin(int f) {
    fam = f;
    cudaEventCreate(&pending);
    cudaEventRecord(pending, st);
  }
  void end() {
    cudaEvent_t e1;
    cudaEventCreate(&e1);
    cudaEventRecord(e1, st);
    rec.push_back({fam, {pending, e1}});
  }
  cudaError_t collect(float* ms) {
    cudaError_t e = cudaStreamSynchronize(st);
    for (int i = 0; i < F_COUNT; ++i) ms[i] = 0.f;
    for (auto& r : rec) {
      float t = 0.f;
      if (e == cudaSuccess) e = cudaEventElapsedTime(&t, r.second.first, r.second.second);
      ms[r.first] += t;
      cudaEventDestroy(r.second.first);
      cudaEventDestroy(r.second.second);
    }
    rec.clear();
    return e;
  }
};

#define QRB_LAUNCH(prof, fam, ...)        \
  do {                                   \
    if (prof) (prof)->begin(fam);        \
    __VA_ARGS__;                         \
    if (prof) (prof)->end();             \
    g_launches.fetch_add(1, std::memory_order_relaxed); \
  } while (0)

constexpr int kMaxN = 4096;
constexpr int kSmallMax = 128;   // largest order the fused one-CTA-per-matrix kernel supports
static std::atomic<int> g_small_n{64};  // n <= g_small_n: fused kernel, no workspace
#ifndef QRB_CHUNK_GIB
#define QRB_CHUNK_GIB 24
#endif
constexpr size_t kChunkBudget = size_t(QRB_CHUNK_GIB) << 30;  // float32 working set per chunk
constexpr int64_t kMaxChunk = 65535;              // grid.y / grid.z limit
constexpr size_t kPanelSmemCap = 200 * 1024;
// column block of the two-level Cholesky elimination (QRB200_OPT_CHOL_BLOCK; 0 = one level)
static std::atomic<int> g_chol_block{128};

// Panels taller than 512 rows run over a CTA cluster (qrb_panel_cl.cuh) when the rows are
// float4-aligned, up to 4 x 512 rows, so those orders keep 32-wide panels too.
constexpr int kClusterPanelMaxM = 4 * kClRows;
static inline bool cluster_panel(int n) { return (n & 3) == 0 && n <= kClusterPanelMaxM; }

static int pick_nb(int n) {
  if (cluster_panel(n)) return 32;
  for (int w = 32; w >= 8; w >>= 1)
    if (panel_smem_bytes(n, w) <= kPanelSmemCap) return w;
  return 0;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// Carving the workspace into per-lane parts costs at most 13 x 256 bytes of alignment each.
constexpr size_t kLaneSlack = 4 * 13 * 256;

// Columns of the W / Wc panel buffers (rows of Bp): the panels of one Cholesky column block
// keep theirs side by side when the two-level elimination runs (nb = 32, n > kCholBlock).
static std::atomic<int> g_chart_block{128};  // QRB200_OPT_CHART_BLOCK (0 = one level)
static int ws_cols(int n) {
  const int nb = pick_nb(n);
  int c = nb;
  const int cb = g_chol_block.load(std::memory_order_relaxed);
  const int hb = g_chart_block.load(std::memory_order_relaxed);
  if (nb == 32 && cb > 0 && n > cb && cb > c) c = cb;
  if (nb == 32 && hb > 0 && n > hb && hb > c) c = hb;
  return c;
}

struct Ws {
  float *T0, *T1, *L, *R, *Q1, *W, *s, *mu, *D, *Wc, *Bp;
  int *orig, *srcmap;
};

static size_t per_chunk_bytes(int64_t cb, int n, int nbmax) {
  const size_t nn = (size_t)n * n;
  size_t t = 0;
  t += 5 * align256(cb * nn * sizeof(float));
  t += 3 * align256(cb * (size_t)n * nbmax * sizeof(float));  // W, Wc, Bp
  t += align256(cb * (size_t)n * sizeof(float));  // s
  t += align256(cb * sizeof(float));              // mu
  t += align256(cb * (size_t)n * sizeof(float));  // D
  t += 2 * align256(cb * (size_t)n * sizeof(int));
  return t;
}

static int64_t chunk_of(int64_t batch, int n) {
  const size_t per = per_chunk_bytes(1, n, ws_cols(n));
  int64_t c = (int64_t)(kChunkBudget / per);
  if (c < 1) c = 1;
  if (c > kMaxChunk) c = kMaxChunk;
  return batch < c ? batch : c;
}

static Ws carve(void* base, int64_t cb, int n, int nbmax) {
  const size_t nn = (size_t)n * n;
  char* p = static_cast<char*>(base);
  Ws w;
  auto take = [&](size_t bytes) { char* q = p; p += align256(bytes); return q; };
  w.T0 = (float*)take(cb * nn * sizeof(float));
  w.T1 = (float*)take(cb * nn * sizeof(float));
  w.L = (float*)take(cb * nn * sizeof(float));
  w.R = (float*)take(cb * nn * sizeof(float));
  w.Q1 = (float*)take(cb * nn * sizeof(float));
  w.W = (float*)take(cb * (size_t)n * nbmax * sizeof(float));
  w.Wc = (float*)take(cb * (size_t)n * nbmax * sizeof(float));
  w.Bp = (float*)take(cb * (size_t)n * nbmax * sizeof(float));
  w.s = (float*)take(cb * (size_t)n * sizeof(float));
  w.mu = (float*)take(cb * sizeof(float));
  w.D = (float*)take(cb * (size_t)n * sizeof(float));
  w.orig = (int*)take(cb * (size_t)n * sizeof(int));
  w.srcmap = (int*)take(cb * (size_t)n * sizeof(int));
  return w;
}

static inline dim3 tiles_grid(int M, int N, int64_t cb) {
  return dim3((N + GT - 1) / GT, (M + GT - 1) / GT, (unsigned)cb);
}
static inline dim3 rwt_grid(int M, int N, int64_t cb) {
  return dim3((N + 127) / 128, (M + 127) / 128, (unsigned)cb);
}
static inline dim3 rw_grid(int M, int N, int64_t cb) {
  return dim3((N + RW_N - 1) / RW_N, (M + RW_M - 1) / RW_M, (unsigned)cb);
}

// tcgen05 tiles need float4-aligned rows; small orders stay on the SIMT tiles.
static inline bool use_tc(int n) {
  const int p = g_gemm_path.load(std::memory_order_relaxed);
  if (p == 1) return false;
  if (p == 2) return (n & 3) == 0;
  return (n & 3) == 0 && n >= 128;
}

// Rank-w trailing updates stream on float4 rows (n % 4 == 0); QRB200_OPT_GEMM_PATH = 2 sends
// the LU trailing update through the tcgen05 tiles instead (comparison runs).
static inline bool use_rankw(int n) {
  return (n & 3) == 0 && g_gemm_path.load(std::memory_order_relaxed) != 2;
}

// Output tile of the tcgen05 GEMMs: 128 x kTcBN (64 was measured slower: twice the loader work per flop).
constexpr int kTcBN = 128;

template <typename T>
static cudaError_t small_attr() {
  cudaError_t e = cudaFuncSetAttribute(small_qr_kernel<64, 256, T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)small_smem_bytes<64, 256>());
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(small_qr_kernel<128, 256, T>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)small_smem_bytes<128, 256>());
}

template <class Pb>
static cudaError_t tcx_attr() {
  cudaError_t e = cudaFuncSetAttribute(tcx::tcx_gemm_kernel<Pb, tcx::CfgWide>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       tcx::smem_bytes<Pb, tcx::CfgWide>());
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(tcx::tcx_gemm_kernel<Pb, tcx::CfgDual>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              tcx::smem_bytes<Pb, tcx::CfgDual>());
}

// TMA-fed tile launch: reductions of K <= 512 run two CTAs per SM (tcx::CfgDual), longer ones
// the one-CTA shape that drains TMEM into registers (tcx::CfgWide).
template <class Pb>
static void launch_tcx(dim3 grid, const tcx::Maps& mp, const typename Pb::Args& args, int K,
                       cudaStream_t st) {
  if (K <= tcx::kDualMaxK)
    tcx::tcx_gemm_kernel<Pb, tcx::CfgDual>
        <<<grid, tcx::XTHREADS, tcx::smem_bytes<Pb, tcx::CfgDual>(), st>>>(mp, args);
  else
    tcx::tcx_gemm_kernel<Pb, tcx::CfgWide>
        <<<grid, tcx::XTHREADS, tcx::smem_bytes<Pb, tcx::CfgWide>(), st>>>(mp, args);
}

// TMA maps for a tcx launch: operands stored k-major use 128-row boxes, m-major 32-row boxes.
static bool tcx_maps(tcx::Maps& mp, const void* a, bool a_kmajor, const void* b, bool b_kmajor,
                     int n, int64_t cb) {
  return (a_kmajor ? encode_batched(&mp.a, a, n, cb, 128) : encode_batched_wide(&mp.a, a, n, cb)) &&
         (b_kmajor ? encode_batched(&mp.b, b, n, cb, 128) : encode_batched_wide(&mp.b, b, n, cb));
}

template <class Pb>
static cudaError_t rwt_attr() {
  return cudaFuncSetAttribute(tc::tc_rankw_kernel<Pb>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              tc::RWT_SMEM);
}

template <class Pb>
static cudaError_t tc_attr() {
  return cudaFuncSetAttribute(tc::tc_gemm_kernel<Pb, kTcBN>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              tc::SmemLayout<kTcBN>::TOTAL);
}
static inline dim3 tc_grid(int M, int N, int64_t cb) {
  return dim3((N + kTcBN - 1) / kTcBN, (M + tc::BM - 1) / tc::BM, (unsigned)cb);
}
constexpr size_t kTcSmem = tc::SmemLayout<kTcBN>::TOTAL;

// Raise the dynamic shared-memory limit of every big-smem kernel once per device.
template <typename TIn>
static cudaError_t set_smem_attrs() {
  const int big = 225 * 1024;  // leaves room for the kernels' static shared memory
  cudaError_t e;
  e = cudaFuncSetAttribute(panel_kernel<PM_PIVOT, TIn, float>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(panel_kernel<PM_CHART, float, TIn>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  return e;
}

static cudaError_t set_common_attrs() {
  const int big = 225 * 1024;  // leaves room for the kernels' static shared memory
  cudaError_t e;
  e = cudaFuncSetAttribute(panel_kernel<PM_PIVOT, float, float>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(panel_kernel<PM_CHOL, float, float>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (e != cudaSuccess) return e;
  e = set_smem_attrs<float>();
  if (e != cudaSuccess) return e;
  e = set_smem_attrs<__nv_bfloat16>();
  if (e != cudaSuccess) return e;
  e = set_smem_attrs<__half>();
  if (e != cudaSuccess) return e;
  if ((e = tc_attr<tc::GramTC>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::QApplyTC>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::SyrkTC>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::LinvBlkTC>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::ClosureTC<float>>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::ClosureTC<__nv_bfloat16>>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::ClosureTC<__half>>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::TrailWTC<float>>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::TrailWTC<__nv_bfloat16>>()) != cudaSuccess) return e;
  if ((e = tc_attr<tc::TrailWTC<__half>>()) != cudaSuccess) return e;
  if ((e = rwt_attr<RWSyrk>()) != cudaSuccess) return e;
  if ((e = rwt_attr<RWLinv>()) != cudaSuccess) return e;
  if ((e = rwt_attr<RWTrail<float>>()) != cudaSuccess) return e;
  if ((e = rwt_attr<RWTrail<__nv_bfloat16>>()) != cudaSuccess) return e;
  if ((e = rwt_attr<RWTrail<__half>>()) != cudaSuccess) return e;
  if ((e = small_attr<float>()) != cudaSuccess) return e;
  if ((e = small_attr<__nv_bfloat16>()) != cudaSuccess) return e;
  if ((e = small_attr<__half>()) != cudaSuccess) return e;
  if ((e = tcx_attr<tcx::GramX>()) != cudaSuccess) return e;
  if ((e = tcx_attr<tcx::SyrkX>()) != cudaSuccess) return e;
  if ((e = tcx_attr<tcx::LinvBlkX>()) != cudaSuccess) return e;
  if ((e = tcx_attr<tcx::QApplyX>()) != cudaSuccess) return e;
  if ((e = tcx_attr<tcx::ClosureXT<__nv_bfloat16>>()) != cudaSuccess) return e;
  if ((e = tcx_attr<tcx::ClosureXT<__half>>()) != cudaSuccess) return e;
  return tcx_attr<tcx::ClosureX>();
}

// Identity of the CUDA context current on this thread, making the device's primary context
// current first when none is.  Per-device caches (kernel attributes, internal streams, the
// allocation-free scratch address, the host-path staging buffers) are keyed on it as well as
// on the device index: after cudaDeviceReset the primary context is created again, module
// globals may move, and streams and allocations of the old context are gone.
static cudaError_t current_ctx(int* dev_out, unsigned long long* id_out) {
  using GetCur = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCur get_cur = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<GetCur>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  CUcontext c = nullptr;
  if (!get_cur || get_cur(&c) != CUDA_SUCCESS) return cudaErrorNotSupported;
  if (!c) {  // no context yet: cudaSetDevice initializes the primary context (CUDA 12+)
    if ((e = cudaSetDevice(dev)) != cudaSuccess) return e;
    if (get_cur(&c) != CUDA_SUCCESS || !c) return cudaErrorDeviceUninitialized;
  }
  unsigned long long id = 0;
  if (!get_id || get_id(c, &id) != CUDA_SUCCESS) return cudaErrorNotSupported;
  *dev_out = dev;
  *id_out = id;
  return cudaSuccess;
}

static cudaError_t ensure_attrs() {
  static std::mutex mu;
  static unsigned long long done_ctx[128] = {0};  // context whose attributes are set
  int dev = 0;
  unsigned long long ctx = 0;
  cudaError_t e = current_ctx(&dev, &ctx);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(mu);
  if (done_ctx[dev] == ctx) return cudaSuccess;
  e = set_common_attrs();
  if (e == cudaSuccess) done_ctx[dev] = ctx;
  return e;
}

// Panels of at most 512 rows run register-resident (qrb_panel_reg.cuh); taller panels keep
// the shared-memory panel kernel.
// QRB200_OPT_CLOSURE_DUAL_N: largest n whose closure runs the two-CTAs-per-SM tile shape
static std::atomic<int> g_closure_dual_n{256};
// QRB200_OPT_PANEL_LOOP: 0 automatic, 1 unrolled column loop everywhere, 2 rotating loop
static std::atomic<int> g_panel_loop{0};
template <int MODE, typename TIn, typename TOut>
static void launch_panel(const PanelArgs& pa, int64_t cb, cudaStream_t st) {
  const int m = pa.n - pa.k0;
  const int pl = g_panel_loop.load(std::memory_order_relaxed);
  // automatic: the rotating (not unrolled) column loop for two rows per thread, whose
  // unrolled code overflows the instruction cache, and for LU panels; Cholesky and chart
  // panels of one row per thread keep the unrolled loop (exact update ranges: about half the
  // FMAs).  Measured per 1536 matrices at n = 512 (rotating vs unrolled): lu_panel 3.26 vs
  // 4.17 ms, chol_panel 4.86 vs 6.04, chart_panel 2.37 vs 2.63; per 8192 bf16 matrices at
  // n = 256: lu_panel 4.62 vs 4.78, chol_panel 6.44 vs 5.88, chart_panel 3.31 vs 3.04.
  const bool rot1 = pl == 2 || (pl == 0 && MODE == PM_PIVOT), rot2 = pl != 1;
  if (m <= 128) {
    // automatic, LU and chart: two rows per thread of 64 (rotating loop, eight CTAs per SM).
    // Measured per 16384 matrices at n = 128 (2 x 64 vs 1 x 128 threads): lu_panel 2.37 vs
    // 2.70 ms, chart_panel 1.74 vs 1.87; the Cholesky panel was slower (4.12 vs 3.95).
    if (pl == 0 && MODE != PM_CHOL)
      panel_reg_kernel<MODE, TIn, TOut, 2, 64, true><<<(unsigned)cb, 64, 0, st>>>(pa);
    else if (rot1) panel_reg_kernel<MODE, TIn, TOut, 1, 128, true><<<(unsigned)cb, 128, 0, st>>>(pa);
    else panel_reg_kernel<MODE, TIn, TOut, 1, 128, false><<<(unsigned)cb, 128, 0, st>>>(pa);
  } else if (m <= 256) {
    // automatic: two rows per thread of 128 (rotating loop; four CTAs per SM instead of three).
    // Measured per 8192 bf16 matrices at n = 256 (2 x 128 vs 1 x 256 threads): lu_panel 3.95
    // vs 4.61 ms, chart_panel 2.92 vs 3.05, chol_panel 5.85 vs 5.92.
    if (pl == 0) panel_reg_kernel<MODE, TIn, TOut, 2, 128, true><<<(unsigned)cb, 128, 0, st>>>(pa);
    else if (rot1) panel_reg_kernel<MODE, TIn, TOut, 1, 256, true><<<(unsigned)cb, 256, 0, st>>>(pa);
    else panel_reg_kernel<MODE, TIn, TOut, 1, 256, false><<<(unsigned)cb, 256, 0, st>>>(pa);
  } else if (m <= 512) {
    if (rot2) panel_reg_kernel<MODE, TIn, TOut, 2, 256, true><<<(unsigned)cb, 256, 0, st>>>(pa);
    else panel_reg_kernel<MODE, TIn, TOut, 2, 256, false><<<(unsigned)cb, 256, 0, st>>>(pa);
  }
  else if (cluster_panel(pa.n) && m <= 2 * kClRows)
    panel_cl_kernel<MODE, TIn, TOut, 2><<<(unsigned)(2 * cb), 256, 0, st>>>(pa);
  else if (cluster_panel(pa.n))
    panel_cl_kernel<MODE, TIn, TOut, 4><<<(unsigned)(4 * cb), 256, 0, st>>>(pa);
  else panel_kernel<MODE, TIn, TOut><<<(unsigned)cb, 256, panel_smem_bytes(m, pa.w), st>>>(pa);
}

// One CholeskyQR pass (reflection_no_reflectors.py:68-77): G = X^T X (+ mu I),
// G = L_G D L_G^T by panels, then Q = X R^{-1} with R^{-1} = L_G^{-T} D^{-1/2}.
//   pass 1: Q = X R^{-1};  pass 2: Q = X - X (I - R^{-1}) (only the small correction goes
//   through the tensor cores; the subtraction is float32).
// The second pass sets the frame's final orthogonality (|q_k|^2 - 1 shows up one-for-one in
// tau_k = 2/(1+|y_k|^2) when d_k ~ 0), so its Gram diagonal is recomputed in exact float32
// column sums.  G lives in ws.T0; R (upper) and L_G^{-1} (strict lower) share ws.R.
static void cholqr_pass(const float* X, float* Q, int n, int64_t cb, int nb, const Ws& ws,
                        int* info, int info_bit, cudaStream_t st, Prof* prof, int nmu) {
  const bool tcp = use_tc(n);
  const bool rw = use_rankw(n);
  const bool pass2 = (info_bit == INFO_CHOL2_NOT_PD);
  tcx::Maps gm;
  const bool gx = tcp && tcx_maps(gm, X, false, X, false, n, cb);
  QRB_LAUNCH(prof, F_GRAM,
             if (gx) launch_tcx<tcx::GramX>(tc_grid(n, n, cb), gm, tc::GramTCArgs{n, X, ws.T0, info},
                                            n, st);
             else if (tcp) tc::tc_gemm_kernel<tc::GramTC, kTcBN><<<tc_grid(n, n, cb), tc::NTHREADS,
                                                               kTcSmem, st>>>(
                 tc::GramTCArgs{n, X, ws.T0, info});
             else simt_gemm_kernel<Gram><<<tiles_grid(n, n, cb), 256, 0, st>>>(
                 GramArgs{n, X, ws.T0}));
  if (tcp && pass2)
    QRB_LAUNCH(prof, F_GRAM,
               colnorm2_kernel<<<dim3((n + 255) / 256, (unsigned)cb), 256, 0, st>>>(X, ws.T0, n));
  // Two-level blocking: the 32-wide panels of a column block [kb, ke) update only the block
  // (its columns for every row below, and the L_G^{-1} rows inside it); the rest of the
  // trailing triangle and the L_G^{-1} rows below the block then take one update with
  // K = ke - kb (SyrkTC and LinvBlkTC), which moves the trailing matrix once per block
  // instead of once per panel.  The panels of a block keep their W / Wc columns and their
  // L_G^{-1} row snapshots side by side (ldw = the block width).
  const int cblk = g_chol_block.load(std::memory_order_relaxed);
  const bool blk = tcp && rw && nb == 32 && cblk > 0 && n > cblk;
  const int ldw = blk ? cblk : nb;
  for (int kb = 0; kb < n; kb += (blk ? cblk : n)) {
    const int ke = blk ? (n - kb < cblk ? n : kb + cblk) : n;
    for (int k0 = kb; k0 < ke; k0 += nb) {
      const int w = (n - k0 < nb) ? n - k0 : nb;
      const int jo = blk ? k0 - kb : 0;  // this panel's column / row offset in W, Wc, Bp
      float* Wp = ws.W + jo;
      float* Wcp = ws.Wc + jo;
      float* Bpp = ws.Bp + (size_t)jo * n;
      PanelArgs pa{};
      pa.n = n; pa.k0 = k0; pa.w = w; pa.ldw = ldw;
      pa.src = ws.T0; pa.R = ws.R; pa.D = ws.D; pa.W = Wp; pa.Wc = Wcp; pa.Bp = Bpp;
      pa.mu = ws.mu; pa.nmu = nmu; pa.info = info; pa.info_bit = info_bit;
      pa.bp_ready = blk && k0 > kb;  // stored by the previous panel's L_G^{-1} update
      QRB_LAUNCH(prof, F_CHOL_PANEL,
                 (launch_panel<PM_CHOL, float, float>(pa, cb, st)));
      const int k1 = k0 + w;
      if (k1 < ke)
        QRB_LAUNCH(prof, F_CHOL_TRAIL,
                   if (tcp && rw) tc::tc_rankw_kernel<RWSyrk>
                       <<<rwt_grid(n - k1, ke - k1, cb), 256, tc::RWT_SMEM, st>>>(
                           RWSyrkArgs{n, k0, k1, ldw, ws.T0, ws.R, Wcp, info, ke});
                   else if (rw) rankw_kernel<RWSyrk><<<rw_grid(n - k1, n - k1, cb), 256, 0, st>>>(
                       RWSyrkArgs{n, k0, k1, ldw, ws.T0, ws.R, Wcp, info, n});
                   else simt_gemm_kernel<TrailSyrk><<<tiles_grid(n - k1, n - k1, cb), 256, 0, st>>>(
                       TrailSyrkArgs{n, k0, k1, ws.T0, ws.R}));
      RWLinvArgs lv{n, k0, k1, ldw, ws.R, Wp, Bpp, info, ke};
      if (blk && k1 < ke) {  // the next panel of this block takes its snapshot from here
        lv.Bn = Bpp + (size_t)w * n;
        lv.wn = (n - k1 < nb) ? n - k1 : nb;
      }
      QRB_LAUNCH(prof, F_CHOL_TRAIL,
                 if (tcp && rw) tc::tc_rankw_kernel<RWLinv>
                     <<<rwt_grid(ke - k0, k1, cb), 256, tc::RWT_SMEM, st>>>(lv);
                 else if (rw) rankw_kernel<RWLinv><<<rw_grid(n - k0, k1, cb), 256, 0, st>>>(
                     RWLinvArgs{n, k0, k1, ldw, ws.R, Wp, Bpp, info, n});
                 else simt_gemm_kernel<LinvTrail><<<tiles_grid(n - k0, k1, cb), 256, 0, st>>>(
                     LinvTrailArgs{n, k0, k1, nb, ws.R, ws.W, ws.Bp}));
    }
    if (ke < n) {
      // TMA-fed tiles when the maps encode (16-byte aligned buffers), else the register-fed ones
      const uint64_t un = (uint64_t)n, ul = (uint64_t)ldw;
      tcx::Maps sm_, lm_;
      const bool sx = encode_batched_wide(&sm_.a, ws.R, n, cb) && encode_batched_wide(&sm_.b, ws.R, n, cb);
      const bool lx = encode_3d(&lm_.a, ws.W, ul, un, cb, ul * 4, un * ul * 4, 32, 128) &&
                      encode_3d(&lm_.b, ws.Bp, un, ul, cb, un * 4, ul * un * 4, 128, 32);
      const tc::SyrkTCArgs sa{n, kb, ke, ws.T0, ws.R, info};
      const tc::LinvBlkArgs la{n, kb, ke, ldw, ws.R, ws.W, ws.Bp, info};
      QRB_LAUNCH(prof, F_CHOL_TRAIL,
                 if (sx) launch_tcx<tcx::SyrkX>(tc_grid(n - ke, n - ke, cb), sm_, sa, ke - kb, st);
                 else tc::tc_gemm_kernel<tc::SyrkTC, kTcBN><<<tc_grid(n - ke, n - ke, cb), tc::NTHREADS,
                                                              kTcSmem, st>>>(sa));
      QRB_LAUNCH(prof, F_CHOL_TRAIL,
                 if (lx) launch_tcx<tcx::LinvBlkX>(tc_grid(n - ke, ke, cb), lm_, la, ke - kb, st);
                 else tc::tc_gemm_kernel<tc::LinvBlkTC, kTcBN><<<tc_grid(n - ke, ke, cb), tc::NTHREADS,
                                                                kTcSmem, st>>>(la));
    }
  }
  const QApplyArgs qa{n, pass2 ? 1 : 0, X, ws.R, ws.D, Q, info};
  tcx::Maps qm;
  const bool qx = tcp && tcx_maps(qm, X, true, ws.R, true, n, cb);
  QRB_LAUNCH(prof, F_QAPPLY,
             if (qx) launch_tcx<tcx::QApplyX>(tc_grid(n, n, cb), qm, qa, n, st);
             else if (tcp) tc::tc_gemm_kernel<tc::QApplyTC, kTcBN><<<tc_grid(n, n, cb), tc::NTHREADS,
                                                                kTcSmem, st>>>(qa);
             else simt_gemm_kernel<QApply><<<tiles_grid(n, n, cb), 256, 0, st>>>(qa));
}

template <typename T>
static void launch_small(const T* A, T* H, T* tau, int* info, int64_t cb, int n, cudaStream_t st,
                         Prof* prof, T* Q, int nmu) {
  QRB_LAUNCH(prof, F_SMALL,
             if (n <= kWarpMaxN) warp_qr_kernel<T>
                 <<<(unsigned)((cb + kWarpWPB - 1) / kWarpWPB), 32 * kWarpWPB, 0, st>>>(
                     A, H, tau, info, n, cb, Q, nmu > 0 ? nmu : n);
             else if (n <= 64) small_qr_kernel<64, 256, T>
                 <<<(unsigned)cb, 256, small_smem_bytes<64, 256>(), st>>>(A, H, tau, info, n, Q, nmu);
             else small_qr_kernel<128, 256, T>
                 <<<(unsigned)cb, 256, small_smem_bytes<128, 256>(), st>>>(A, H, tau, info, n, Q, nmu));
}

// Explicit Q (optional output): householder_product(H, tau) = (I - Y T Y^T) = Q_frame * S,
// because the chart factors I - Q_frame S = Y (T Y^T) (reflection_no_reflectors.py:86-176).
// 16-bit input widened to float32 (n % 4 == 0, so the batch holds a multiple of 16 elements:
// eight elements per thread and step, one 16-byte load and two 16-byte stores), the B operand
// of the TMA-fed closure tile.
template <typename T>
__global__ void widen_kernel(const T* __restrict__ A, float* __restrict__ X, int64_t count8) {
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < count8;
       q += (int64_t)gridDim.x * blockDim.x) {
    const uint4 t = __ldg(reinterpret_cast<const uint4*>(A) + q);
    const T* h = reinterpret_cast<const T*>(&t);
    float4* o = reinterpret_cast<float4*>(X) + 2 * q;
    o[0] = make_float4(to_f32(h[0]), to_f32(h[1]), to_f32(h[2]), to_f32(h[3]));
    o[1] = make_float4(to_f32(h[4]), to_f32(h[5]), to_f32(h[6]), to_f32(h[7]));
  }
}

// One float4 of Q per thread: Q[r][c] = frame[r][c] * s_c, in the output dtype.
template <typename T>
__global__ void explicit_q_kernel(const float* __restrict__ F, const float* __restrict__ s,
                                  T* __restrict__ Q, int n) {
  const int64_t b = blockIdx.y;
  const int nn4 = (n * n) >> 2;
  const float4* F4 = reinterpret_cast<const float4*>(F + mat_off(b, n));
  const float* sb = s + b * n;
  T* Qb = Q + mat_off(b, n);
  for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < nn4; q += gridDim.x * blockDim.x) {
    const float4 v = F4[q];
    const int c = (q << 2) % n;  // n % 4 == 0: the four elements share a row
    Qb[4 * (int64_t)q] = from_f32<T>(v.x * sb[c]);
    Qb[4 * (int64_t)q + 1] = from_f32<T>(v.y * sb[c + 1]);
    Qb[4 * (int64_t)q + 2] = from_f32<T>(v.z * sb[c + 2]);
    Qb[4 * (int64_t)q + 3] = from_f32<T>(v.w * sb[c + 3]);
  }
}
template <typename T>
__global__ void explicit_q_kernel_any(const float* __restrict__ F, const float* __restrict__ s,
                                      T* __restrict__ Q, int n) {
  const int64_t b = blockIdx.y;
  const int nn = n * n;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nn; e += gridDim.x * blockDim.x)
    Q[mat_off(b, n) + e] = from_f32<T>(F[mat_off(b, n) + e] * s[b * n + e % n]);
}

template <typename T>
static cudaError_t run_chunk(const T* A, T* H, T* tau, int* info, int64_t cb, int n,
                             const Ws& ws, cudaStream_t st, Prof* prof, T* Q = nullptr,
                             int nmu = 0) {
  if (n <= g_small_n.load(std::memory_order_relaxed)) {  // whole pipeline, one CTA per matrix
    launch_small<T>(A, H, tau, info, cb, n, st, prof, Q, nmu);
    return cudaGetLastError();
  }
  const int nb = pick_nb(n);
  const bool tcp = use_tc(n);
  const bool rw = use_rankw(n);  // streaming rank-w tiles for every trailing update
  cudaError_t e = cudaMemsetAsync(info, 0, cb * sizeof(int), st);
  if (e != cudaSuccess) return e;

  // ---- I-a: partial-pivot LU; P*L lands in ws.L ----
  {
    const void* cur = A;
    bool cur_in = true;
    float* Tb[2] = {ws.T0, ws.T1};
    int ti = 0;
    for (int k0 = 0; k0 < n; k0 += nb) {
      const int w = (n - k0 < nb) ? n - k0 : nb;
      PanelArgs pa{};
      pa.n = n; pa.k0 = k0; pa.w = w; pa.ldw = nb;
      pa.src = cur; pa.orig = ws.orig; pa.srcmap = ws.srcmap; pa.W = ws.W; pa.L = ws.L;
      pa.info = info;
      const size_t smem = panel_smem_bytes(n - k0, w);
      QRB_LAUNCH(prof, F_LU_PANEL,
                 if (cur_in) launch_panel<PM_PIVOT, T, float>(pa, cb, st);
                 else launch_panel<PM_PIVOT, float, float>(pa, cb, st));
      const int k1 = k0 + w;
      if (k1 < n) {
        TrailWArgs ta{n, k0, k1, nb, cur, Tb[ti], ws.W, ws.srcmap};
        const dim3 g = tiles_grid(n - k1, n - k1, cb);
        const tc::TrailWTCArgs tca{n, k0, k1, nb, cur, Tb[ti], ws.W, ws.srcmap, info};
        const dim3 gt = tc_grid(n - k1, n - k1, cb);
        const RWTrailArgs rwa{n, k0, k1, nb, cur, Tb[ti], ws.W, ws.srcmap, info};
        const dim3 gr = rw_grid(n - k1, n - k1, cb);
        QRB_LAUNCH(prof, F_LU_TRAIL,
                   if (tcp && rw && cur_in) tc::tc_rankw_kernel<RWTrail<T>>
                       <<<rwt_grid(n - k1, n - k1, cb), 256, tc::RWT_SMEM, st>>>(rwa);
                   else if (tcp && rw) tc::tc_rankw_kernel<RWTrail<float>>
                       <<<rwt_grid(n - k1, n - k1, cb), 256, tc::RWT_SMEM, st>>>(rwa);
                   else if (rw && cur_in) rankw_kernel<RWTrail<T>><<<gr, 256, 0, st>>>(rwa);
                   else if (rw) rankw_kernel<RWTrail<float>><<<gr, 256, 0, st>>>(rwa);
                   else if (tcp && cur_in) tc::tc_gemm_kernel<tc::TrailWTC<T>, kTcBN>
                       <<<gt, tc::NTHREADS, kTcSmem, st>>>(tca);
                   else if (tcp) tc::tc_gemm_kernel<tc::TrailWTC<float>, kTcBN>
                       <<<gt, tc::NTHREADS, kTcSmem, st>>>(tca);
                   else if (cur_in) simt_gemm_kernel<TrailW<T>><<<g, 256, 0, st>>>(ta);
                   else simt_gemm_kernel<TrailW<float>><<<g, 256, 0, st>>>(ta));
        cur = Tb[ti];
        ti ^= 1;
        cur_in = false;
      }
    }
  }
  // ---- I-b..d: CholeskyQR2 on P*L; the frame Q = P Q_L lands in ws.L ----
  cholqr_pass(ws.L, ws.Q1, n, cb, nb, ws, info, INFO_CHOL1_NOT_PD, st, prof, nmu);
  cholqr_pass(ws.Q1, ws.L, n, cb, nb, ws, info, INFO_CHOL2_NOT_PD, st, prof, nmu);

  // ---- III: chart on a copy of Q (working copy in ws.T0) ----
  // The chart's trailing updates stay on float32 FMA tiles: tau_k = 2/(1+|y_k|^2) sits at 1
  // when d_k = 0, and the 2^-21 products of 3xTF32 would push it below the tau >= 1 - 1e-6 gate.
  const int hblk = g_chart_block.load(std::memory_order_relaxed);
  if (rw && nb == 32 && hblk > 0 && n > hblk) {
    // Two-level: the 32-wide panels of a column block [kb, ke) update the block's columns for
    // every row below and the block's rows for the columns right of it; the rest takes one
    // K = ke - kb update per block (the panels' W column groups side by side, ldw = hblk).
    // Everything runs in place on a copy of the frame.
    e = cudaMemcpyAsync(ws.T0, ws.L, (size_t)cb * n * n * sizeof(float), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return e;
    for (int kb = 0; kb < n; kb += hblk) {
      const int ke = (n - kb < hblk) ? n : kb + hblk;
      for (int k0 = kb; k0 < ke; k0 += nb) {
        const int w = (n - k0 < nb) ? n - k0 : nb;
        const int k1 = k0 + w;
        float* Wp = ws.W + (k0 - kb);
        PanelArgs pa{};
        pa.n = n; pa.k0 = k0; pa.w = w; pa.ldw = hblk;
        pa.src = ws.T0; pa.W = Wp; pa.H = H; pa.tau = tau; pa.s = ws.s; pa.info = info;
        QRB_LAUNCH(prof, F_CHART_PANEL, (launch_panel<PM_CHART, float, T>(pa, cb, st)));
        if (k1 < ke) {
          const RWGenArgs col{n, k1, k1, n - k1, ke - k1, w, k0, hblk, ws.T0, Wp, info};
          QRB_LAUNCH(prof, F_CHART_TRAIL,
                     rankw_kernel<RWGen><<<rw_grid(n - k1, ke - k1, cb), 256, 0, st>>>(col));
          if (ke < n) {
            const RWGenArgs row{n, k1, ke, ke - k1, n - ke, w, k0, hblk, ws.T0, Wp, info};
            QRB_LAUNCH(prof, F_CHART_TRAIL,
                       rankw_kernel<RWGen><<<rw_grid(ke - k1, n - ke, cb), 256, 0, st>>>(row));
          }
        }
      }
      if (ke < n) {
        const RWGenArgs blk{n, ke, ke, n - ke, n - ke, ke - kb, kb, hblk, ws.T0, ws.W, info};
        QRB_LAUNCH(prof, F_CHART_TRAIL,
                   rankw_big_kernel<RWGen><<<dim3((n - ke + RWB_T - 1) / RWB_T,
                                                  (n - ke + RWB_T - 1) / RWB_T, (unsigned)cb),
                                             256, 0, st>>>(blk));
      }
    }
  } else {
    for (int k0 = 0; k0 < n; k0 += nb) {
      const int w = (n - k0 < nb) ? n - k0 : nb;
      const float* cur = (k0 == 0) ? ws.L : ws.T0;
      PanelArgs pa{};
      pa.n = n; pa.k0 = k0; pa.w = w; pa.ldw = nb;
      pa.src = cur; pa.W = ws.W; pa.H = H; pa.tau = tau; pa.s = ws.s; pa.info = info;
      QRB_LAUNCH(prof, F_CHART_PANEL,
                 (launch_panel<PM_CHART, float, T>(pa, cb, st)));
      const int k1 = k0 + w;
      if (k1 < n)
        QRB_LAUNCH(prof, F_CHART_TRAIL,
                   if (rw) rankw_kernel<RWTrail<float>><<<rw_grid(n - k1, n - k1, cb), 256, 0, st>>>(
                       RWTrailArgs{n, k0, k1, nb, cur, ws.T0, ws.W, nullptr, info});
                   else simt_gemm_kernel<TrailW<float>><<<tiles_grid(n - k1, n - k1, cb), 256, 0, st>>>(
                       TrailWArgs{n, k0, k1, nb, cur, ws.T0, ws.W, nullptr}));
    }
  }
  // ---- II: closure, H_upper = s * triu(Q^T A) ----
  // float32 input: A is the closure tile's B operand; 16-bit input is widened into ws.T1 (free
  // after the LU) first, so that the TMA-fed tile serves every dtype (measured at n = 256, 8192
  // bf16 matrices: closure 7.3 ms on the register-fed tile)
  tcx::Maps cm;
  constexpr bool f32 = std::is_same<T, float>::value;
  const bool cx = tcp && (f32 || (reinterpret_cast<uintptr_t>(A) & 15) == 0) &&
                  tcx_maps(cm, ws.L, false, f32 ? static_cast<const void*>(A) : ws.T1, false, n, cb);
  if (cx && !f32) {
    const int64_t c8 = cb * (int64_t)n * n / 8;
    const unsigned gw = (unsigned)((c8 + 255) / 256 < 148 * 32 ? (c8 + 255) / 256 : 148 * 32);
    QRB_LAUNCH(prof, F_CLOSURE, (widen_kernel<T><<<gw, 256, 0, st>>>(A, ws.T1, c8)));
  }
  QRB_LAUNCH(prof, F_CLOSURE,
             // n <= 256 (QRB200_OPT_CLOSURE_DUAL_N) runs two CTAs per SM, larger n the one-CTA
             // shape.  Closure ms, two vs one CTA per SM: n = 512 (1536) 2.63 vs 2.55; n = 256
             // (8192) 2.69 vs 2.77, bf16 4.00 vs 4.32; n = 128 (16384) 1.19 vs 1.32.
             if (cx) launch_tcx<tcx::ClosureXT<T>>(tc_grid(n, n, cb), cm,
                                               tc::ClosureTCArgs{n, ws.L, A, ws.s, H, info},
                                               g_closure_dual_n.load() >= n ? n : tcx::kDualMaxK + 1, st);
             else if (tcp) tc::tc_gemm_kernel<tc::ClosureTC<T>, kTcBN>
                 <<<tc_grid(n, n, cb), tc::NTHREADS, kTcSmem, st>>>(
                     tc::ClosureTCArgs{n, ws.L, A, ws.s, H, info});
             else simt_gemm_kernel<Closure<T>><<<tiles_grid(n, n, cb), 256, 0, st>>>(
                 ClosureArgs{n, ws.L, A, ws.s, H}));
  if (Q) {
    const unsigned gx = (unsigned)((n * n / 4 + 255) / 256 < 64 ? (n * n / 4 + 255) / 256 : 64);
    QRB_LAUNCH(prof, F_CLOSURE,
               if ((n & 3) == 0) explicit_q_kernel<T><<<dim3(gx, (unsigned)cb), 256, 0, st>>>(
                   ws.L, ws.s, Q, n);
               else explicit_q_kernel_any<T><<<dim3(gx, (unsigned)cb), 256, 0, st>>>(
                   ws.L, ws.s, Q, n));
  }
  return cudaGetLastError();
}

// Internal streams of the lane split (created once per device, never destroyed).
constexpr int kMaxLanes = 4;
static std::atomic<int> g_lanes{2};  // QRB200_OPT_LANES
static cudaStream_t* lane_streams() {
  static std::mutex mu;
  static cudaStream_t lanes[128][kMaxLanes];
  static unsigned long long made_ctx[128] = {0};  // context the streams belong to
  int dev = 0;
  unsigned long long ctx = 0;
  if (note(current_ctx(&dev, &ctx)) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (made_ctx[dev] != ctx) {  // streams of a context that was reset are gone with it
    for (int l = 0; l < kMaxLanes; ++l)
      if (note(cudaStreamCreateWithFlags(&lanes[dev][l], cudaStreamNonBlocking)) != cudaSuccess)
        return nullptr;
    made_ctx[dev] = ctx;
  }
  return lanes[dev];
}

template <typename T>
static int run_all(const void* A, void* H, void* tau, int32_t* info, int64_t batch, int n,
                   void* workspace, cudaStream_t st, Prof* prof, void* Qv = nullptr,
                   int nmu = 0) {
  T* Qo = static_cast<T*>(Qv);
  auto qoff = [&](int64_t o) { return Qo ? Qo + o * (int64_t)n * n : nullptr; };
  if (n <= g_small_n.load(std::memory_order_relaxed)) {
    const Ws none{};
    for (int64_t b0 = 0; b0 < batch; b0 += (int64_t(1) << 30)) {
      const int64_t cnt = (batch - b0 < (int64_t(1) << 30)) ? batch - b0 : (int64_t(1) << 30);
      const size_t nn = (size_t)n * n;
      cudaError_t e = run_chunk<T>(static_cast<const T*>(A) + b0 * nn,
                                   static_cast<T*>(H) + b0 * nn, static_cast<T*>(tau) + b0 * n,
                                   info + b0, cnt, n, none, st, prof, qoff(b0), nmu);
      if (note(e) != cudaSuccess) return QRB200_ERR_CUDA;
    }
    return QRB200_OK;
  }
  const int64_t cb = chunk_of(batch, n);
  const int nb = pick_nb(n);
  const size_t need = per_chunk_bytes(cb, n, ws_cols(n)) + kLaneSlack;
  void* ws = workspace;
  bool owned = false;
  if (!ws) {
    if (note(cudaMallocAsync(&ws, need, st)) != cudaSuccess) return QRB200_ERR_CUDA;
    owned = true;
  }
  int rc = QRB200_OK;
  const size_t nn = (size_t)n * n;
  const int cols = ws_cols(n);
  const int L = prof ? 1 : g_lanes.load(std::memory_order_relaxed);
  cudaStream_t* lane = (L > 1) ? lane_streams() : nullptr;
  for (int64_t b0 = 0; b0 < batch; b0 += cb) {
    const int64_t cnt = (batch - b0 < cb) ? batch - b0 : cb;
    if (!lane || cnt < 2 * L) {
      const Ws w = carve(ws, cnt, n, cols);
      cudaError_t e = run_chunk<T>(static_cast<const T*>(A) + b0 * nn, static_cast<T*>(H) + b0 * nn,
                                   static_cast<T*>(tau) + b0 * n, info + b0, cnt, n, w, st, prof,
                                   qoff(b0), nmu);
      if (note(e) != cudaSuccess) { rc = QRB200_ERR_CUDA; break; }
      continue;
    }
    // Lanes: the chunk's matrices are independent, so sub-batches run on L internal streams
    // forked from and joined back to the caller's stream.  The latency-bound panels of one
    // sub-batch then overlap the bandwidth-bound trailing updates of another.
    cudaEvent_t fork = nullptr, join[kMaxLanes] = {};
    cudaError_t e = cudaEventCreateWithFlags(&fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(fork, st);
    char* p = static_cast<char*>(ws);
    const int64_t per = (cnt + L - 1) / L;
    for (int l = 0; l < L && e == cudaSuccess; ++l) {
      const int64_t s0 = l * per, c = (cnt - s0 < per) ? cnt - s0 : per;
      if (c <= 0) break;
      e = cudaStreamWaitEvent(lane[l], fork, 0);
      if (e != cudaSuccess) break;
      const Ws w = carve(p, c, n, cols);
      p += per_chunk_bytes(c, n, cols);
      const int64_t o = b0 + s0;
      e = run_chunk<T>(static_cast<const T*>(A) + o * nn, static_cast<T*>(H) + o * nn,
                       static_cast<T*>(tau) + o * n, info + o, c, n, w, lane[l], nullptr, qoff(o),
                       nmu);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&join[l], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventRecord(join[l], lane[l]);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(st, join[l], 0);
    }
    if (fork) cudaEventDestroy(fork);
    for (int l = 0; l < L; ++l)
      if (join[l]) cudaEventDestroy(join[l]);
    if (note(e) != cudaSuccess) { rc = QRB200_ERR_CUDA; break; }
  }
  if (owned && note(cudaFreeAsync(ws, st)) != cudaSuccess) rc = QRB200_ERR_CUDA;
  return rc;
}

}  // namespace qrb

extern "C" {

int qrb200_version(void) { return 100; }

const char* qrb200_status_string(int status) {
  switch (status) {
    case QRB200_OK: return "ok";
    case QRB200_ERR_INVALID_ARG: return "invalid argument";
    case QRB200_ERR_UNSUPPORTED_N: return "unsupported matrix order n";
    case QRB200_ERR_WORKSPACE: return "workspace too small";
    case QRB200_ERR_CUDA: return "CUDA runtime error";
    case QRB200_ERR_SCRATCH_LIMIT:
      return "one matrix of this order needs more than the allocation-free entry point's "
             "built-in scratch (QRB200_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown status";
  }
}

int32_t qrb200_max_n(void) { return qrb::kMaxN; }

int qrb200_workspace_bytes(int64_t batch, int32_t n, size_t* bytes) {
  if (!bytes || batch < 0) return QRB200_ERR_INVALID_ARG;
  if (n < 0 || n > qrb::kMaxN) return QRB200_ERR_UNSUPPORTED_N;
  if (batch == 0 || n == 0 || n <= qrb::g_small_n.load()) { *bytes = 0; return QRB200_OK; }
  const int64_t cb = qrb::chunk_of(batch, n);
  *bytes = qrb::per_chunk_bytes(cb, n, qrb::ws_cols(n)) + qrb::kLaneSlack;
  return QRB200_OK;
}

static int geqrf_impl(const void* A, void* H, void* tau, int32_t* info, int64_t batch,
                      int32_t n, int32_t dtype, void* workspace, size_t workspace_bytes,
                      void* stream, qrb::Prof* prof, void* Q = nullptr, int nmu = 0) {
  if (batch < 0) return QRB200_ERR_INVALID_ARG;
  if (n < 0 || n > qrb::kMaxN) return QRB200_ERR_UNSUPPORTED_N;
  if (dtype != QRB200_F32 && dtype != QRB200_BF16 && dtype != QRB200_F16)
    return QRB200_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB200_OK;
  if (!A || !H || !tau || !info) return QRB200_ERR_INVALID_ARG;
  if (workspace) {
    size_t need = 0;
    qrb200_workspace_bytes(batch, n, &need);
    if (workspace_bytes < need) return QRB200_ERR_WORKSPACE;
  }
  if (qrb::note(qrb::ensure_attrs()) != cudaSuccess) return QRB200_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case QRB200_F32:
      return qrb::run_all<float>(A, H, tau, info, batch, n, workspace, st, prof, Q, nmu);
    case QRB200_BF16:
      return qrb::run_all<__nv_bfloat16>(A, H, tau, info, batch, n, workspace, st, prof, Q, nmu);
    default: return qrb::run_all<__half>(A, H, tau, info, batch, n, workspace, st, prof, Q, nmu);
  }
}

int qrb200_geqrf_batched_q(const void* A, void* H, void* tau, void* Q, int32_t* info,
                           int64_t batch, int32_t n, int32_t dtype, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!Q && batch > 0 && n > 0) return QRB200_ERR_INVALID_ARG;
  return geqrf_impl(A, H, tau, info, batch, n, dtype, workspace, workspace_bytes, stream,
                    nullptr, Q);
}

int qrb200_geqrf_batched(const void* A, void* H, void* tau, int32_t* info, int64_t batch,
                         int32_t n, int32_t dtype, void* workspace, size_t workspace_bytes,
                         void* stream) {
  return geqrf_impl(A, H, tau, info, batch, n, dtype, workspace, workspace_bytes, stream,
                    nullptr);
}

int qrb200_geqrf_batched_timed(const void* A, void* H, void* tau, int32_t* info,
                               int64_t batch, int32_t n, int32_t dtype, void* workspace,
                               size_t workspace_bytes, void* stream, float* family_ms) {
  if (!family_ms) return QRB200_ERR_INVALID_ARG;
  qrb::Prof prof;
  prof.st = static_cast<cudaStream_t>(stream);
  const int rc = geqrf_impl(A, H, tau, info, batch, n, dtype, workspace, workspace_bytes,
                            stream, &prof);
  const cudaError_t e = prof.collect(family_ms);
  if (rc != QRB200_OK) return rc;
  return e == cudaSuccess ? QRB200_OK : QRB200_ERR_CUDA;
}

int32_t qrb200_num_families(void) { return qrb::F_COUNT; }

const char* qrb200_family_name(int32_t family) {
  static const char* names[qrb::F_COUNT] = {"lu_panel",    "lu_trail",    "gram",
                                            "chol_panel",  "chol_trail",  "q_apply",
                                            "chart_panel", "chart_trail", "closure",
                                            "small_fused"};
  return (family >= 0 && family < qrb::F_COUNT) ? names[family] : "unknown";
}

long long qrb200_launch_count(void) { return qrb::g_launches.load(); }

int qrb200_set_option(int32_t key, int64_t value) {
  if (key == QRB200_OPT_GEMM_PATH) {
    if (value < 0 || value > 2) return QRB200_ERR_INVALID_ARG;
    qrb::g_gemm_path.store((int)value);
    return QRB200_OK;
  }
  if (key == QRB200_OPT_LANES) {
    if (value < 1 || value > qrb::kMaxLanes) return QRB200_ERR_INVALID_ARG;
    qrb::g_lanes.store((int)value);
    return QRB200_OK;
  }
  if (key == QRB200_OPT_CHART_BLOCK) {
    if (value != 0 && value != 64 && value != 128 && value != 256) return QRB200_ERR_INVALID_ARG;
    qrb::g_chart_block.store((int)value);
    return QRB200_OK;
  }
  if (key == QRB200_OPT_CHOL_BLOCK) {
    if (value != 0 && value != 64 && value != 128 && value != 256) return QRB200_ERR_INVALID_ARG;
    qrb::g_chol_block.store((int)value);
    return QRB200_OK;
  }
  if (key == QRB200_OPT_CLOSURE_DUAL_N) {
    if (value < 0 || value > qrb::tcx::kDualMaxK) return QRB200_ERR_INVALID_ARG;
    qrb::g_closure_dual_n.store((int)value);
    return QRB200_OK;
  }
  if (key == QRB200_OPT_PANEL_LOOP) {
    if (value < 0 || value > 2) return QRB200_ERR_INVALID_ARG;
    qrb::g_panel_loop.store((int)value);
    return QRB200_OK;
  }
  if (key == QRB200_OPT_SMALL_N) {
    if (value < 0 || value > qrb::kSmallMax) return QRB200_ERR_INVALID_ARG;
    qrb::g_small_n.store((int)value);
    return QRB200_OK;
  }
  return QRB200_ERR_INVALID_ARG;
}

const char* qrb200_last_cuda_error(void) {
  const cudaError_t e = qrb::g_last_cuda_error;
  return e == cudaSuccess ? "no error" : cudaGetErrorString(e);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory at the point where they factor: code running
// inside a host callback or a custom allocator hook (where cudaMalloc/cudaMallocAsync would
// re-enter the allocator or deadlock), embedders whose memory is fully pre-partitioned, and
// plug-in hosts that forbid allocation after start-up.  For them this file keeps the
// working buffers of the pipeline in one file-scope device array of
// QRB200_NOALLOC_SCRATCH_BYTES bytes, which every GPU that loads this library holds until
// the process exits.  The caller still owns A, H, tau and info.
//
// Host code must not pass the array's name to a kernel: on the host it is only a
// stand-in symbol, not a device address.  The first call on each device (with that device
// current) asks the runtime for the array's device address with cudaGetSymbolAddress and
// caches it; make that first call before any stream capture.
//
// Every call shares the array and it keeps the previous call's contents.  Nothing in it has
// to start at zero: each stage writes every word it later reads (info, which must start at
// zero, is the caller's buffer and is cleared on the stream per chunk).  Calls that overlap
// on the GPU (two streams, or two host threads) race on the array; serialize them.
// ---------------------------------------------------------------------------------------
namespace qrb {

constexpr size_t kNoAllocScratchBytes = QRB200_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[128] = {nullptr};
static unsigned long long g_noalloc_ctx[128] = {0};

// Device address of g_noalloc_scratch in the current context: looked up on the first call in
// each context of each device (a reset device gets a new context, where the array may sit
// elsewhere) and cached.
static cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  unsigned long long ctx = 0;
  cudaError_t e = current_ctx(&dev, &ctx);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[dev] || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

// Largest number of matrices whose working set fits the built-in scratch (0 = none).
static int64_t noalloc_chunk(int n, int nb) {
  int64_t c = (int64_t)(kNoAllocScratchBytes / per_chunk_bytes(1, n, nb)) + 1;
  while (c > 0 && per_chunk_bytes(c, n, nb) > kNoAllocScratchBytes) --c;
  return c < kMaxChunk ? c : kMaxChunk;
}

template <typename T>
static int run_noalloc(const void* A, void* H, void* tau, int32_t* info, int64_t batch, int n,
                       void* scratch, int64_t cb, cudaStream_t st) {
  const int cols = ws_cols(n);
  const size_t nn = (size_t)n * n;
  for (int64_t b0 = 0; b0 < batch; b0 += cb) {
    const int64_t cnt = (batch - b0 < cb) ? batch - b0 : cb;
    const Ws w = carve(scratch, cnt, n, cols);
    cudaError_t e = run_chunk<T>(static_cast<const T*>(A) + b0 * nn, static_cast<T*>(H) + b0 * nn,
                                 static_cast<T*>(tau) + b0 * n, info + b0, cnt, n, w, st,
                                 nullptr);
    if (note(e) != cudaSuccess) return QRB200_ERR_CUDA;
  }
  return QRB200_OK;
}

}  // namespace qrb

extern "C" int qrb200_geqrf_batched_noalloc(const void* A, void* H, void* tau, int32_t* info,
                                            int64_t batch, int32_t n, int32_t dtype,
                                            void* stream) {
  if (batch < 0) return QRB200_ERR_INVALID_ARG;
  if (n < 0 || n > qrb::kMaxN) return QRB200_ERR_UNSUPPORTED_N;
  if (dtype != QRB200_F32 && dtype != QRB200_BF16 && dtype != QRB200_F16)
    return QRB200_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB200_OK;
  // the size check comes first: it needs no device and no valid buffers
  // (orders of the fused kernel use no scratch: one launch covers up to 2^30 matrices)
  const int64_t cb = n <= qrb::g_small_n.load() ? (int64_t(1) << 30)
                                                : qrb::noalloc_chunk(n, qrb::ws_cols(n));
  if (cb < 1) return QRB200_ERR_SCRATCH_LIMIT;
  if (!A || !H || !tau || !info) return QRB200_ERR_INVALID_ARG;
  if (qrb::note(qrb::ensure_attrs()) != cudaSuccess) return QRB200_ERR_CUDA;
  void* scratch = nullptr;
  if (qrb::note(qrb::noalloc_scratch(&scratch)) != cudaSuccess) return QRB200_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case QRB200_F32: return qrb::run_noalloc<float>(A, H, tau, info, batch, n, scratch, cb, st);
    case QRB200_BF16:
      return qrb::run_noalloc<__nv_bfloat16>(A, H, tau, info, batch, n, scratch, cb, st);
    default: return qrb::run_noalloc<__half>(A, H, tau, info, batch, n, scratch, cb, st);
  }
}

// ---------------------------------------------------------------------------------------
// Host-buffer entry point.
//
// A, H, tau and info live in host memory.  The batch is cut into sub-batches that rotate
// over kHostSlots streams; each slot owns device copies of its sub-batch's A/H/tau/info and
// its own workspace, and runs  upload -> factor -> download  in stream order.  Sub-batch i's
// kernels therefore overlap the upload of i+1 and the download of i-1 (the two copy
// directions run on separate copy engines), and kernels of neighbouring slots overlap each
// other, which keeps the one-CTA-per-matrix panel stages busy.  With page-locked host
// buffers the copies are asynchronous; pageable buffers give the same results without the
// overlap.  The device buffers are cached per device and only ever grow; they are released
// by qrb200_release_host_staging.
// ---------------------------------------------------------------------------------------
namespace qrb {

constexpr int kHostSlots = 3;

struct HostStaging {
  void* base = nullptr;
  size_t bytes = 0;
  unsigned long long ctx = 0;  // context the buffer was allocated in
};
static std::mutex g_host_mu;
static HostStaging g_host_staging[128];

static int64_t host_sub_batch(int64_t batch, int n) {
  // six sub-batches keep the exposed first upload / last download at about 1/6 of one copy
  // direction; at least 2 matrices per SM per sub-batch so each stage still fills the GPU
  const int64_t floor_cnt = n <= g_small_n.load() ? 4096 : (n <= 256 ? 1184 : 296);
  int64_t sb = (batch + 5) / 6;
  if (sb < floor_cnt) sb = floor_cnt;
  return sb < batch ? sb : batch;
}

}  // namespace qrb

extern "C" int qrb200_geqrf_batched_host(const void* A, void* H, void* tau, int32_t* info,
                                         int64_t batch, int32_t n, int32_t dtype,
                                         int64_t sub_batch, void* stream) {
  using namespace qrb;
  if (batch < 0 || sub_batch < 0) return QRB200_ERR_INVALID_ARG;
  if (n < 0 || n > kMaxN) return QRB200_ERR_UNSUPPORTED_N;
  if (dtype != QRB200_F32 && dtype != QRB200_BF16 && dtype != QRB200_F16)
    return QRB200_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB200_OK;
  if (!A || !H || !tau || !info) return QRB200_ERR_INVALID_ARG;
  const size_t es = dtype == QRB200_F32 ? 4 : 2;
  const int64_t sb = sub_batch > 0 ? (sub_batch < batch ? sub_batch : batch)
                                   : host_sub_batch(batch, n);
  const size_t nn = (size_t)n * n;
  size_t ws_bytes = 0;
  int rc = qrb200_workspace_bytes(sb, n, &ws_bytes);
  if (rc != QRB200_OK) return rc;
  const size_t a_b = align256(sb * nn * es), t_b = align256(sb * n * es),
               i_b = align256(sb * sizeof(int32_t)), w_b = align256(ws_bytes);
  const size_t slot_bytes = 2 * a_b + t_b + i_b + w_b;

  int dev = 0;
  unsigned long long ctx = 0;
  if (note(current_ctx(&dev, &ctx)) != cudaSuccess) return QRB200_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_host_mu);
  HostStaging& hs = g_host_staging[dev];
  if (hs.base && hs.ctx != ctx) hs = HostStaging{};  // freed with the context it came from
  const size_t need = kHostSlots * slot_bytes;
  if (hs.bytes < need) {
    if (hs.base && note(cudaFree(hs.base)) != cudaSuccess) return QRB200_ERR_CUDA;
    hs.base = nullptr;
    hs.bytes = 0;
    if (note(cudaMalloc(&hs.base, need)) != cudaSuccess) return QRB200_ERR_CUDA;
    hs.bytes = need;
    hs.ctx = ctx;
  }
  cudaStream_t caller = static_cast<cudaStream_t>(stream);
  cudaStream_t st[kHostSlots] = {};
  cudaEvent_t start = nullptr;
  auto cleanup = [&](int r) {
    for (int s = 0; s < kHostSlots; ++s)
      if (st[s]) {
        if (cudaStreamSynchronize(st[s]) != cudaSuccess && r == QRB200_OK) r = QRB200_ERR_CUDA;
        cudaStreamDestroy(st[s]);
      }
    if (start) cudaEventDestroy(start);
    return r;
  };
  if (note(cudaEventCreateWithFlags(&start, cudaEventDisableTiming)) != cudaSuccess ||
      note(cudaEventRecord(start, caller)) != cudaSuccess)
    return cleanup(QRB200_ERR_CUDA);
  for (int s = 0; s < kHostSlots; ++s)
    if (note(cudaStreamCreateWithFlags(&st[s], cudaStreamNonBlocking)) != cudaSuccess ||
        note(cudaStreamWaitEvent(st[s], start, 0)) != cudaSuccess)
      return cleanup(QRB200_ERR_CUDA);

  const char* hA = static_cast<const char*>(A);
  char* hH = static_cast<char*>(H);
  char* hT = static_cast<char*>(tau);
  int64_t j = 0;
  for (int64_t b0 = 0; b0 < batch; b0 += sb, ++j) {
    const int64_t cnt = batch - b0 < sb ? batch - b0 : sb;
    const int s = (int)(j % kHostSlots);
    char* base = static_cast<char*>(hs.base) + s * slot_bytes;
    void* dA = base;
    void* dH = base + a_b;
    void* dT = base + 2 * a_b;
    int32_t* dI = reinterpret_cast<int32_t*>(base + 2 * a_b + t_b);
    void* dW = ws_bytes ? base + 2 * a_b + t_b + i_b : nullptr;
    if (note(cudaMemcpyAsync(dA, hA + b0 * nn * es, cnt * nn * es, cudaMemcpyHostToDevice,
                             st[s])) != cudaSuccess)
      return cleanup(QRB200_ERR_CUDA);
    rc = geqrf_impl(dA, dH, dT, dI, cnt, n, dtype, dW, ws_bytes, st[s], nullptr);
    if (rc != QRB200_OK) return cleanup(rc);
    if (note(cudaMemcpyAsync(hH + b0 * nn * es, dH, cnt * nn * es, cudaMemcpyDeviceToHost,
                             st[s])) != cudaSuccess ||
        note(cudaMemcpyAsync(hT + b0 * n * es, dT, cnt * n * es, cudaMemcpyDeviceToHost,
                             st[s])) != cudaSuccess ||
        note(cudaMemcpyAsync(info + b0, dI, cnt * sizeof(int32_t), cudaMemcpyDeviceToHost,
                             st[s])) != cudaSuccess)
      return cleanup(QRB200_ERR_CUDA);
  }
  return cleanup(QRB200_OK);
}

extern "C" int qrb200_release_host_staging(void) {
  using namespace qrb;
  int dev = 0;
  unsigned long long ctx = 0;
  if (note(current_ctx(&dev, &ctx)) != cudaSuccess) return QRB200_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_host_mu);
  HostStaging& hs = g_host_staging[dev];
  if (hs.base && hs.ctx == ctx && note(cudaFree(hs.base)) != cudaSuccess) return QRB200_ERR_CUDA;
  hs.base = nullptr;
  hs.bytes = 0;
  return QRB200_OK;
}

// ---------------------------------------------------------------------------------------
// Rectangular (tall) entry point.
//
// The pipeline is column-nested: the LU's pivot choices and L's first n columns, the
// Cholesky factor's leading n x n block, the frame's first n columns, the chart's first n
// multipliers, signs and tau, and the closure's first n columns all depend only on A's first
// n columns.  So a tall m x n matrix is factored by the square kernels on the m x m matrix
// [A | 0], with the CholeskyQR jitter's mean taken over the first n diagonal entries only
// (the one quantity that would see the padding), and the first n columns of H and tau are
// returned.  On the zero columns the LU meets zero pivots, which leave L unit lower
// triangular, so the padded frame stays well defined.
// ---------------------------------------------------------------------------------------
namespace qrb {

template <typename E>  // E: an element-sized integer (the copy never converts)
__global__ void pad_cols_kernel(const E* __restrict__ A, E* __restrict__ P, int m, int n) {
  const int64_t b = blockIdx.y;
  const int64_t mm = (int64_t)m * m;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < mm;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / m), c = (int)(e - (int64_t)r * m);
    P[b * mm + e] = (c < n) ? A[b * (int64_t)m * n + (int64_t)r * n + c] : E(0);
  }
}

template <typename E>
__global__ void crop_cols_kernel(const E* __restrict__ P, const E* __restrict__ tp,
                                 E* __restrict__ H, E* __restrict__ tau, int* __restrict__ info,
                                 int m, int n) {
  const int64_t b = blockIdx.y;
  const int64_t mn = (int64_t)m * n;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < mn;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / n), c = (int)(e - (int64_t)r * n);
    H[b * mn + e] = P[b * (int64_t)m * m + (int64_t)r * m + c];
  }
  if (blockIdx.x == 0) {
    for (int k = threadIdx.x; k < n; k += blockDim.x) tau[b * n + k] = tp[b * m + k];
    // zero pivots are expected on the padding columns: the informational bit is not reported
    if (threadIdx.x == 0) info[b] &= ~INFO_LU_ZERO_PIVOT;
  }
}

constexpr size_t kRectBudget = size_t(8) << 30;  // padded A, H, tau per chunk

}  // namespace qrb

extern "C" int qrb200_geqrf_batched_rect(const void* A, void* H, void* tau, int32_t* info,
                                         int64_t batch, int32_t m, int32_t n, int32_t dtype,
                                         void* stream) {
  using namespace qrb;
  if (batch < 0) return QRB200_ERR_INVALID_ARG;
  if (m < 0 || m > kMaxN || n < 0) return QRB200_ERR_UNSUPPORTED_N;
  if (n > m) return QRB200_ERR_INVALID_ARG;  // tall or square only
  if (dtype != QRB200_F32 && dtype != QRB200_BF16 && dtype != QRB200_F16)
    return QRB200_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return QRB200_OK;
  if (!A || !H || !tau || !info) return QRB200_ERR_INVALID_ARG;
  if (n == m)
    return geqrf_impl(A, H, tau, info, batch, n, dtype, nullptr, 0, stream, nullptr);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t es = dtype == QRB200_F32 ? 4 : 2;
  const size_t mm = (size_t)m * m;
  const size_t per = 2 * mm * es + m * es + 3 * 256;
  int64_t cb = (int64_t)(kRectBudget / per);
  if (cb < 1) cb = 1;
  if (cb > kMaxChunk) cb = kMaxChunk;
  if (cb > batch) cb = batch;
  const size_t a_b = align256(cb * mm * es), t_b = align256(cb * m * es);
  void* buf = nullptr;
  if (note(cudaMallocAsync(&buf, 2 * a_b + t_b, st)) != cudaSuccess) return QRB200_ERR_CUDA;
  char* Ap = static_cast<char*>(buf);
  char* Hp = Ap + a_b;
  char* Tp = Hp + a_b;
  int rc = QRB200_OK;
  for (int64_t b0 = 0; b0 < batch && rc == QRB200_OK; b0 += cb) {
    const int64_t cnt = batch - b0 < cb ? batch - b0 : cb;
    const dim3 pg((unsigned)((mm + 255) / 256 < 128 ? (mm + 255) / 256 : 128), (unsigned)cnt);
    const dim3 cg((unsigned)(((size_t)m * n + 255) / 256 < 128 ? ((size_t)m * n + 255) / 256 : 128),
                  (unsigned)cnt);
    const char* Ab = static_cast<const char*>(A) + b0 * (int64_t)m * n * es;
    if (es == 4)
      pad_cols_kernel<uint32_t><<<pg, 256, 0, st>>>((const uint32_t*)Ab, (uint32_t*)Ap, m, n);
    else
      pad_cols_kernel<uint16_t><<<pg, 256, 0, st>>>((const uint16_t*)Ab, (uint16_t*)Ap, m, n);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (note(cudaGetLastError()) != cudaSuccess) { rc = QRB200_ERR_CUDA; break; }
    rc = geqrf_impl(Ap, Hp, Tp, info + b0, cnt, m, dtype, nullptr, 0, stream, nullptr, nullptr, n);
    if (rc != QRB200_OK) break;
    char* Hb = static_cast<char*>(H) + b0 * (int64_t)m * n * es;
    char* tb = static_cast<char*>(tau) + b0 * (int64_t)n * es;
    if (es == 4)
      crop_cols_kernel<uint32_t><<<cg, 256, 0, st>>>((const uint32_t*)Hp, (const uint32_t*)Tp,
                                                     (uint32_t*)Hb, (uint32_t*)tb, info + b0, m, n);
    else
      crop_cols_kernel<uint16_t><<<cg, 256, 0, st>>>((const uint16_t*)Hp, (const uint16_t*)Tp,
                                                     (uint16_t*)Hb, (uint16_t*)tb, info + b0, m, n);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (note(cudaGetLastError()) != cudaSuccess) rc = QRB200_ERR_CUDA;
  }
  if (note(cudaFreeAsync(buf, st)) != cudaSuccess && rc == QRB200_OK) rc = QRB200_ERR_CUDA;
  return rc;
}
