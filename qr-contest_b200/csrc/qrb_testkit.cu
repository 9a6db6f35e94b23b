// qrb200 test kit: single-stage entry points for the GPU unit tests (not part of the
// product ABI).  Each runs one GEMM-shaped stage with either the SIMT tiles (tc = 0) or the
// tcgen05 3xTF32 tiles (tc = 1) on float32 data, so the tests can compare both against a
// float64 product of the same operands.
#include "qrb_common.cuh"
#include "qrb_gemm_simt.cuh"
#include "qrb_tc_ops.cuh"
#include "qrb_tc_rankw.cuh"
#include "qrb_tcx.cuh"
#include "qrb_tmap.cuh"

using namespace qrb;

static dim3 g64(int M, int N, int64_t b) { return dim3((N + 63) / 64, (M + 63) / 64, (unsigned)b); }
static dim3 g128(int M, int N, int64_t b) { return dim3((N + 127) / 128, (M + 127) / 128, (unsigned)b); }
constexpr int kSm = tc::SmemLayout<128>::TOTAL;

template <class Pb>
static int prep() {
  return (int)cudaFuncSetAttribute(tc::tc_gemm_kernel<Pb, 128>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSm);
}

// dual = 1: the two-CTAs-per-SM shape (K <= 512 only), else the one-CTA shape that drains
template <class Pb>
static int tcx_launch(const void* a, bool ak, const void* b, bool bk, int n, int64_t batch,
                      const typename Pb::Args& args, cudaStream_t s, int dual = 0) {
  tcx::Maps mp;
  if (!(ak ? encode_batched(&mp.a, a, n, batch, 128) : encode_batched_wide(&mp.a, a, n, batch)) ||
      !(bk ? encode_batched(&mp.b, b, n, batch, 128) : encode_batched_wide(&mp.b, b, n, batch)))
    return 999;
  if (dual) {
    if (n > tcx::kDualMaxK) return 998;
    cudaFuncSetAttribute(tcx::tcx_gemm_kernel<Pb, tcx::CfgDual>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, tcx::smem_bytes<Pb, tcx::CfgDual>());
    tcx::tcx_gemm_kernel<Pb, tcx::CfgDual>
        <<<g128(n, n, batch), tcx::XTHREADS, tcx::smem_bytes<Pb, tcx::CfgDual>(), s>>>(mp, args);
    return 0;
  }
  cudaFuncSetAttribute(tcx::tcx_gemm_kernel<Pb>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       tcx::smem_bytes<Pb>());
  tcx::tcx_gemm_kernel<Pb><<<g128(n, n, batch), tcx::XTHREADS, tcx::smem_bytes<Pb>(), s>>>(mp, args);
  return 0;
}

extern "C" {

int qrbt_gram(const float* X, float* G, int* info, int64_t batch, int n, int use_tc, void* st) {
  cudaStream_t s = (cudaStream_t)st;
  if (use_tc == 2 || use_tc == 4) {
    if (int e = tcx_launch<tcx::GramX>(X, false, X, false, n, batch, tc::GramTCArgs{n, X, G, info}, s,
                                       use_tc == 4))
      return e;
  } else if (use_tc) {
    if (int e = prep<tc::GramTC>()) return e;
    tc::tc_gemm_kernel<tc::GramTC, 128><<<g128(n, n, batch), tc::NTHREADS, kSm, s>>>(
        tc::GramTCArgs{n, X, G, info});
  } else {
    simt_gemm_kernel<Gram><<<g64(n, n, batch), 256, 0, s>>>(GramArgs{n, X, G});
  }
  return (int)cudaGetLastError();
}

int qrbt_trailw(const float* Cold, float* Cnew, const float* W, const int* srcmap, int* info,
                int64_t batch, int n, int k0, int k1, int ldw, int use_tc, void* st) {
  cudaStream_t s = (cudaStream_t)st;
  // use_tc: 0 scalar tiles, 1 tcgen05 GEMM tile, 2 tcgen05 rank-w tile, 3 streaming rank-w tile
  const RWTrailArgs rwa{n, k0, k1, ldw, Cold, Cnew, W, srcmap, info};
  if (use_tc == 2) {
    cudaFuncSetAttribute(tc::tc_rankw_kernel<RWTrail<float>>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, tc::RWT_SMEM);
    tc::tc_rankw_kernel<RWTrail<float>><<<g128(n - k1, n - k1, batch), 256, tc::RWT_SMEM, s>>>(rwa);
  } else if (use_tc == 3) {
    rankw_kernel<RWTrail<float>><<<dim3((n - k1 + 127) / 128, (n - k1 + 63) / 64, (unsigned)batch),
                                   256, 0, s>>>(rwa);
  } else if (use_tc) {
    if (int e = prep<tc::TrailWTC<float>>()) return e;
    tc::tc_gemm_kernel<tc::TrailWTC<float>, 128><<<g128(n - k1, n - k1, batch), tc::NTHREADS,
                                                   kSm, s>>>(
        tc::TrailWTCArgs{n, k0, k1, ldw, Cold, Cnew, W, srcmap, info});
  } else {
    simt_gemm_kernel<TrailW<float>><<<g64(n - k1, n - k1, batch), 256, 0, s>>>(
        TrailWArgs{n, k0, k1, ldw, Cold, Cnew, W, srcmap});
  }
  return (int)cudaGetLastError();
}

int qrbt_syrk(float* G, const float* R, int* info, int64_t batch, int n, int k0, int k1,
              int use_tc, void* st) {
  cudaStream_t s = (cudaStream_t)st;
  if (use_tc) {
    if (int e = prep<tc::SyrkTC>()) return e;
    tc::tc_gemm_kernel<tc::SyrkTC, 128><<<g128(n - k1, n - k1, batch), tc::NTHREADS, kSm, s>>>(
        tc::SyrkTCArgs{n, k0, k1, G, R, info});
  } else {
    simt_gemm_kernel<TrailSyrk><<<g64(n - k1, n - k1, batch), 256, 0, s>>>(
        TrailSyrkArgs{n, k0, k1, G, R});
  }
  return (int)cudaGetLastError();
}

int qrbt_closure(const float* Q, const float* A, const float* sgn, float* H, int* info,
                 int64_t batch, int n, int use_tc, void* st) {
  cudaStream_t s = (cudaStream_t)st;
  if (use_tc == 2 || use_tc == 4) {
    if (int e = tcx_launch<tcx::ClosureX>(Q, false, A, false, n, batch,
                                          tc::ClosureTCArgs{n, Q, A, sgn, H, info}, s, use_tc == 4))
      return e;
  } else if (use_tc) {
    if (int e = prep<tc::ClosureTC<float>>()) return e;
    tc::tc_gemm_kernel<tc::ClosureTC<float>, 128><<<g128(n, n, batch), tc::NTHREADS, kSm, s>>>(
        tc::ClosureTCArgs{n, Q, A, sgn, H, info});
  } else {
    simt_gemm_kernel<Closure<float>><<<g64(n, n, batch), 256, 0, s>>>(
        ClosureArgs{n, Q, A, sgn, H});
  }
  return (int)cudaGetLastError();
}

// Q = X R^{-1} (pass2 = 0) or X - X (I - R^{-1}) (pass2 = 1), R^{-1}[k][j] = RL[j][k] / sqrt(D[j])
// for k < j and 1 / sqrt(D[j]) on the diagonal.
int qrbt_qapply(const float* X, const float* RL, const float* D, float* Q, int* info,
                int64_t batch, int n, int pass2, int use_tc, void* st) {
  cudaStream_t s = (cudaStream_t)st;
  const QApplyArgs qa{n, pass2, X, RL, D, Q, info};
  if (use_tc == 2 || use_tc == 4) {
    if (int e = tcx_launch<tcx::QApplyX>(X, true, RL, true, n, batch, qa, s, use_tc == 4)) return e;
  } else if (use_tc) {
    if (int e = prep<tc::QApplyTC>()) return e;
    tc::tc_gemm_kernel<tc::QApplyTC, 128><<<g128(n, n, batch), tc::NTHREADS, kSm, s>>>(qa);
  } else {
    simt_gemm_kernel<QApply><<<g64(n, n, batch), 256, 0, s>>>(qa);
  }
  return (int)cudaGetLastError();
}

}  // extern "C"

// ---- panel phase timing (built with QRB_PANEL_TIMERS) ----
#include "qrb_panel_reg.cuh"
#include "qrb_small.cuh"

template <int MODE>
static int panel_timing_impl(const float* src, int64_t batch, int n, int k0, int w, int reg,
                             long long* cycles_out, float* ms_out) {
  const size_t nn = (size_t)n * n;
  float *L, *R, *W, *Wc, *Bp, *D, *mu, *s, *tau, *H;
  int *orig, *srcmap, *info;
  cudaMalloc(&L, batch * nn * 4); cudaMalloc(&R, batch * nn * 4); cudaMalloc(&H, batch * nn * 4);
  cudaMalloc(&W, batch * n * 32 * 4); cudaMalloc(&Wc, batch * n * 32 * 4);
  cudaMalloc(&Bp, batch * n * 32 * 4); cudaMalloc(&D, batch * n * 4); cudaMalloc(&mu, batch * 4);
  cudaMalloc(&s, batch * n * 4); cudaMalloc(&tau, batch * n * 4);
  cudaMalloc(&orig, batch * n * 4); cudaMalloc(&srcmap, batch * n * 4); cudaMalloc(&info, batch * 4);
  cudaMemset(R, 0, batch * nn * 4); cudaMemset(info, 0, batch * 4); cudaMemset(mu, 0, batch * 4);
  PanelArgs pa{};
  pa.n = n; pa.k0 = k0; pa.w = w; pa.ldw = 32; pa.src = src; pa.orig = orig; pa.srcmap = srcmap;
  pa.W = W; pa.L = L; pa.R = R; pa.D = D; pa.Wc = Wc; pa.Bp = Bp; pa.mu = mu; pa.H = H;
  pa.tau = tau; pa.s = s; pa.info = info; pa.info_bit = 2;
  const size_t smem = panel_smem_bytes(n - k0, w);
  cudaFuncSetAttribute(panel_kernel<MODE, float, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       225 * 1024);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0); cudaEventCreate(&e1);
  auto launch = [&]() {
    if (reg && n - k0 <= 256) panel_reg_kernel<MODE, float, float, 1><<<(unsigned)batch, 256>>>(pa);
    else if (reg) panel_reg_kernel<MODE, float, float, 2><<<(unsigned)batch, 256>>>(pa);
    else panel_kernel<MODE, float, float><<<(unsigned)batch, 256, smem>>>(pa);
  };
  launch();  // warm
  cudaEventRecord(e0);
  launch();
  cudaEventRecord(e1);
  cudaEventSynchronize(e1);
  cudaEventElapsedTime(ms_out, e0, e1);
  cudaMemcpyFromSymbol(cycles_out, g_panel_timers, 8 * sizeof(long long));
  int rc = (int)cudaGetLastError();
  cudaFree(L); cudaFree(R); cudaFree(H); cudaFree(W); cudaFree(Wc); cudaFree(Bp); cudaFree(D);
  cudaFree(mu); cudaFree(s); cudaFree(tau); cudaFree(orig); cudaFree(srcmap); cudaFree(info);
  return rc;
}

extern "C" int qrbt_panel_timing(int mode, const float* src, int64_t batch, int n, int k0, int w,
                                 int reg, long long* cycles_out, float* ms_out) {
  if (mode == 0) return panel_timing_impl<PM_PIVOT>(src, batch, n, k0, w, reg, cycles_out, ms_out);
  if (mode == 1) return panel_timing_impl<PM_CHOL>(src, batch, n, k0, w, reg, cycles_out, ms_out);
  return panel_timing_impl<PM_CHART>(src, batch, n, k0, w, reg, cycles_out, ms_out);
}

// fused small-n kernel: one launch over `batch` matrices, CTA 0's phase cycles
extern "C" int qrbt_small_timing(const float* A, float* H, float* tau, int* info, int64_t batch,
                                 int n, long long* cycles_out, float* ms_out) {
  auto launch = [&]() {
    if (n <= 32) small_qr_kernel<32, 128, float><<<(unsigned)batch, 128, small_smem_bytes<32, 128>()>>>(A, H, tau, info, n);
    else if (n <= 64) small_qr_kernel<64, 256, float><<<(unsigned)batch, 256, small_smem_bytes<64, 256>()>>>(A, H, tau, info, n);
    else small_qr_kernel<128, 256, float><<<(unsigned)batch, 256, small_smem_bytes<128, 256>()>>>(A, H, tau, info, n);
  };
  cudaFuncSetAttribute(small_qr_kernel<64, 256, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)small_smem_bytes<64, 256>());
  cudaFuncSetAttribute(small_qr_kernel<128, 256, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)small_smem_bytes<128, 256>());
  launch();
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0); cudaEventCreate(&e1);
  cudaEventRecord(e0);
  launch();
  cudaEventRecord(e1);
  cudaEventSynchronize(e1);
  cudaEventElapsedTime(ms_out, e0, e1);
  cudaMemcpyFromSymbol(cycles_out, g_panel_timers, 8 * sizeof(long long));
  return (int)cudaGetLastError();
}

// Phase cycle sums (thread 0, all CTAs) of the TMA-fed Gram tile over `batch` n x n matrices:
// prologue, wait raw, wait planes free, split, barrier, issue, epilogue; plus the launch time.
extern "C" int qrbt_tcx_timing(const float* X, float* G, int* info, int64_t batch, int n,
                               long long* cycles_out, float* ms_out) {
  cudaStream_t s = 0;
  if (int e = tcx_launch<tcx::GramX>(X, false, X, false, n, batch, tc::GramTCArgs{n, X, G, info}, s))
    return e;
  long long zero[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  cudaMemcpyToSymbol(g_panel_timers, zero, sizeof(zero));
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0); cudaEventCreate(&e1);
  cudaEventRecord(e0);
  tcx_launch<tcx::GramX>(X, false, X, false, n, batch, tc::GramTCArgs{n, X, G, info}, s);
  cudaEventRecord(e1);
  cudaEventSynchronize(e1);
  cudaEventElapsedTime(ms_out, e0, e1);
  cudaEventDestroy(e0); cudaEventDestroy(e1);
  cudaMemcpyFromSymbol(cycles_out, g_panel_timers, 8 * sizeof(long long));
  return (int)cudaGetLastError();
}

// ---- bounded-wait failure path (no GPU fault involved) ----
// Each CTA holds TMEM like the production tiles, then waits with a short limit on an
// mbarrier that no thread arrives at and no copy or MMA targets, so the wait runs out.  The
// CTA takes the production tiles' timeout path: INFO_DEVICE_TIMEOUT into its info word,
// nothing in flight to drain, TMEM freed, normal return.  The host then checks the bits and
// that the context still runs tensor-core work.
__global__ void timeout_probe_kernel(int* info, unsigned limit) {
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  const int tid = threadIdx.x;
  if (tid < 32) {
    tc::tmem_alloc(&slot, 32);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const bool ok = !__syncthreads_or(!tc::mbar_wait_n(&bar, 0, limit));
  if (!ok && tid == 0) atomicOr(&info[blockIdx.x], INFO_DEVICE_TIMEOUT);
  tc::tc_fence_before();
  __syncthreads();
  if (tid < 32) tc::tmem_dealloc(slot, 32);
}

extern "C" int qrbt_timeout_probe(int* info, int blocks, unsigned limit, void* st) {
  if (blocks < 1 || limit < 1 || limit > (1u << 20)) return (int)cudaErrorInvalidValue;
  timeout_probe_kernel<<<blocks, 128, 0, (cudaStream_t)st>>>(info, limit);
  return (int)cudaGetLastError();
}
