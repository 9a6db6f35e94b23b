// qrb200 -- rank-w (w <= 32) trailing updates on tcgen05 (3xTF32), with the policies of
// qrb_rankw.cuh.  Used where 2^-21-relative products are acceptable: the LU, the Cholesky and
// the L_G^{-1} updates (the chart keeps the float32 kernel, see qrb_api.cu).
#pragma once
#include "qrb_rankw.cuh"
#include "qrb_tc.cuh"

namespace qrb {
namespace tc {

// ---- rank-w update tile on tcgen05: C' = C - A B, K = w <= 32 -------------------------------
// One 128 x 128 output tile per CTA and a single K stage: A (128 x K, rows contiguous in k) and
// B (K x 128, rows contiguous in j) are split into hi/lo tf32 planes, 12 MMAs (3 per k-step of
// 8) accumulate in TMEM, and the accumulator is staged through shared memory so that the
// read-modify-write of C is fully coalesced (each warp streams whole 512-byte row segments).
// 64 KB of shared memory -> three CTAs per SM overlap one another's loads, MMAs and epilogues.
// Uses the policies of qrb_rankw.cuh (a_ptr, b_ptr, c_load4, store4, dims, live).
constexpr int RWT_STAGE_LD = 132;  // padded row stride (floats) of the epilogue staging
constexpr int RWT_STAGE_BYTES = 128 * RWT_STAGE_LD * 4;  // >= the 64 KB of operand planes
constexpr int RWT_SMEM = RWT_STAGE_BYTES + 64 + 1024;     // + barrier/slot + alignment

template <class Pb>
__global__ void __launch_bounds__(NTHREADS, 3) tc_rankw_kernel(typename Pb::Args a) {
  extern __shared__ __align__(1024) char smraw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  char* a_hi = sm;
  char* a_lo = sm + 16384;
  char* b_hi = sm + 2 * 16384;
  char* b_lo = sm + 3 * 16384;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + RWT_STAGE_BYTES);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  float* stage = reinterpret_cast<float*>(sm);  // 128 x RWT_STAGE_LD floats after the MMAs

  const int64_t b = blockIdx.z;
  const int m0 = blockIdx.y * 128, n0 = blockIdx.x * 128;
  int M, N, K;
  Pb::dims(a, M, N, K);
  if (m0 >= M || n0 >= N || !Pb::live(a, m0, n0)) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    tmem_alloc(tslot, 128);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Start the C tile on its way to L2 now: the epilogue's read of C (64 KB) then overlaps the
  // operand loads, the split and the MMAs instead of following them.  Two 128-byte lines per
  // thread: row tid / 2, lines (tid % 2) * 2 and +1 of the row's 512-byte segment.
  {
    const int row = tid >> 1;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = n0 + 32 * ((tid & 1) * 2 + h);
      if (m0 + row < M && j < N) {
        const void* p = Pb::c_addr(a, b, m0 + row, j);
        if (p) asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
      }
    }
  }
  // A: micro-block (rows 4*mb.., k 4*kc..), rows contiguous in k
  {
    const int mb = tid >> 3, kc = tid & 7;
    float v[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + 4 * mb + i;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < M && 4 * kc < K) t = __ldg(reinterpret_cast<const float4*>(Pb::a_ptr(a, b, m) + 4 * kc));
      v[i][0] = t.x; v[i][1] = t.y; v[i][2] = t.z; v[i][3] = t.w;
    }
    put4x4(a_hi, a_lo, 4 * mb, kc, v);
  }
  // B: micro-block (columns 4*jb.., k 4*kc..), rows of B contiguous in j
  {
    const int jb = tid & 31, kc = tid >> 5;
    float v[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int k = 4 * kc + kk;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < K && n0 + 4 * jb < N) t = ld4v(Pb::b_ptr(a, b, k) + n0 + 4 * jb);
      v[0][kk] = t.x; v[1][kk] = t.y; v[2][kk] = t.z; v[3][kk] = t.w;
    }
    put4x4(b_hi, b_lo, 4 * jb, kc, v);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    constexpr uint32_t IDESC = idesc_tf32(128, 128);
    const uint32_t ah = smem_u32(a_hi), al = smem_u32(a_lo), bh = smem_u32(b_hi), bl = smem_u32(b_lo);
#pragma unroll
    for (int kk = 0; kk < BK / UK; ++kk) {
      const uint32_t koff = kk * UK * 4;
      const uint64_t dah = sdesc_sw128(ah + koff), dal = sdesc_sw128(al + koff);
      const uint64_t dbh = sdesc_sw128(bh + koff), dbl = sdesc_sw128(bl + koff);
      mma_tf32(tmem, dal, dbh, IDESC, kk > 0 ? 1u : 0u);
      mma_tf32(tmem, dah, dbl, IDESC, 1u);
      mma_tf32(tmem, dah, dbh, IDESC, 1u);
    }
    mma_commit(bar);
  }
  // one commit (phase 0); a thread whose wait timed out makes the whole CTA skip the
  // epilogue, and thread 0 waits once more so that the TMEM is not freed under the MMAs
  bool ok = !__syncthreads_or(!mbar_wait(bar, 0));
  bool drained = true;
  if (!ok && tid == 0) drained = mbar_wait(bar, 0);
  drained = __syncthreads_and(drained);
  tc_fence_after();
  if (ok) {
    // TMEM -> shared staging (row = TMEM lane), the operand planes are free now
    const int lq = warp & 3, half = warp >> 2;
#pragma unroll
    for (int c = 0; c < 64; c += 32) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(32 * lq) << 16) + half * 64 + c, v);
      float* dst = stage + (32 * lq + lane) * RWT_STAGE_LD + half * 64 + c;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (!ok) {
    if (tid == 0) atomicOr(Pb::info(a, b), INFO_DEVICE_TIMEOUT);
  } else {
    // coalesced C read-modify-write: warp-wide 512-byte row segments.  The loads of a group
    // are all issued before its stores: C may be updated in place, so a load placed after a
    // store could not be moved above it and every element would wait out its own round trip.
    constexpr int IT = 128 * 32 / NTHREADS, G = 8;
#pragma unroll
    for (int g = 0; g < IT; g += G) {
      float4 xs[G];
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int idx = tid + (g + u) * NTHREADS;
        const int m = m0 + (idx >> 5), j = n0 + (idx & 31) * 4;
        if (m < M && j < N) xs[u] = Pb::c_load4(a, b, m, j);
      }
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int idx = tid + (g + u) * NTHREADS;
        const int row = idx >> 5, c4 = (idx & 31) * 4;
        const int m = m0 + row, j = n0 + c4;
        if (m < M && j < N) {
          float4 x = xs[u];
          const float4 p = *reinterpret_cast<const float4*>(stage + row * RWT_STAGE_LD + c4);
          x.x -= p.x; x.y -= p.y; x.z -= p.z; x.w -= p.w;
          Pb::store4(a, b, m, j, x);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 0 && drained) tmem_dealloc(tmem, 128);
}

}  // namespace tc
}  // namespace qrb
