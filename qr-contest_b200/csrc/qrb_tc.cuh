// qrb200 -- tcgen05 / TMEM primitives for sm_100a (inline PTX) and a batched 3xTF32 GEMM tile.
//
// Precision: every float32 operand x is split into hi = tf32_rn(x) and lo = tf32_rn(x - hi);
// the tile accumulates hi*hi + hi*lo + lo*hi in float32 in TMEM (3 tcgen05.mma kind::tf32
// per K-step of 8).  Products are accurate to ~2^-21 relative.  The TMEM accumulation itself
// is not round-to-nearest per add, so stages whose result is a sum of order one that must be
// float32-exact (the second CholeskyQR pass) only route small corrections through it.
//
// Shared-memory operand layout: K-major, 128-byte swizzle (the canonical SW128 K-major UMMA
// layout): a tile row (one M or N index) holds BK = 32 consecutive k values = 128 bytes;
// 8 rows form a 1024-byte swizzle atom; the 16-byte chunk c of row r sits at chunk c ^ (r%8).
// The loader threads write the hi/lo planes in that layout from any global layout (row
// gathers, transposed operands, bf16/f16 inputs), so only one descriptor form is needed.
//
// Every wait is bounded: on timeout the kernel raises INFO_DEVICE_TIMEOUT in the matrix's
// info word, stops issuing MMAs and copies, waits (again bounded) for the ones already in
// flight, and frees its TMEM only when that drain completed (a tile whose drain also timed
// out leaves its TMEM allocated rather than free it under a running MMA).
#pragma once
#include "qrb_common.cuh"

namespace qrb {
namespace tc {

constexpr int BM = 128;   // tile rows (UMMA M)
constexpr int BK = 32;    // k per stage (one 128-byte swizzle row)
constexpr int UK = 8;     // k per tcgen05.mma kind::tf32
constexpr int NTHREADS = 256;
constexpr unsigned kSpinLimit = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// Same rounding (to nearest, ties away from zero) on the integer pipe: add half of the 13
// dropped mantissa bits to the bit pattern, then clear them.  A carry out of the mantissa
// bumps the exponent, which is the correctly rounded result.  Finite inputs below the
// largest binade only (all operands here are).
__device__ __forceinline__ float tf32_rn_int(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// ---- mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait; returns false on timeout.
__device__ __forceinline__ bool mbar_wait_n(uint64_t* bar, uint32_t phase, unsigned limit) {
  for (unsigned i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, phase)) return true;
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase) {
  return mbar_wait_n(bar, phase, kSpinLimit);
}

// ---- TMEM ----
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- MMA ----
// Instruction descriptor: D f32, A/B tf32, both K-major, M = m, N = n.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
// Shared-memory matrix descriptor, K-major SWIZZLE_128B, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Same MMA with the A operand read from tensor memory (K-major: lane = row, one tf32 per column).
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive fp32 columns of this thread's TMEM lane <- v (waits for the stores).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Byte offset of 16-byte chunk `kchunk` (k = 4*kchunk..+3) of row r in a K-major SW128 tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int kchunk) {
  return ((uint32_t)(r >> 3) << 10) | ((uint32_t)(r & 7) << 7) |
         ((uint32_t)((kchunk ^ (r & 7)) & 7) << 4);
}

// Store a 4(row) x 4(k) micro-block, split into hi/lo planes.
__device__ __forceinline__ void put4x4(char* hi, char* lo, int r0, int kchunk,
                                       const float (&v)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 h, l;
    h.x = tf32_rn_int(v[i][0]); l.x = tf32_rn_int(v[i][0] - h.x);
    h.y = tf32_rn_int(v[i][1]); l.y = tf32_rn_int(v[i][1] - h.y);
    h.z = tf32_rn_int(v[i][2]); l.z = tf32_rn_int(v[i][2] - h.z);
    h.w = tf32_rn_int(v[i][3]); l.w = tf32_rn_int(v[i][3] - h.w);
    const uint32_t off = sw128_off(r0 + i, kchunk);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = l;
  }
}

// ---- generic batched tile kernel ----
//
// Policy Pb supplies:
//   Args; dims(a, M, N, K); live(m0, n0, BM, BN) (tile needed at all);
//   krange(a, m0, n0, kb, ke) (k range the tile reduces over);
//   A_ALONG_K / B_ALONG_K : the global source of A(m,k) / B(k,j) is contiguous along k
//   loadA(a, b, m0, k0, v[4][4]) : v[i][kk] = A(m0+i, k0+kk), zero outside
//   loadB(a, b, j0, k0, v[4][4]) : v[i][kk] = B(k0+kk, j0+i), zero outside (raw loads)
//   fixB(a, b, j0, k0, v[4][4])  : elementwise transform of a fetched B block, applied when
//                                  it is written to shared memory (keeps loads in flight)
//   store(a, b, m, j0, v[32], M, N) : row m, columns j0 .. j0+31 of the result
//   info(a, b) : int* of the matrix's status word
template <int BN>
struct SmemLayout {
  static constexpr int A_BYTES = BM * BK * 4;   // 16 KB
  static constexpr int B_BYTES = BN * BK * 4;   // 16 KB (BN = 128) / 8 KB (BN = 64)
  static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int STAGES = 2;
  static constexpr int TOTAL = STAGES * STAGE + 1024 /*align*/ + 64 /*barriers + slot*/;
};

template <class Pb, int BN>
__global__ void __launch_bounds__(NTHREADS, BN == 64 ? 2 : 1) tc_gemm_kernel(typename Pb::Args a) {
  using L = SmemLayout<BN>;
  extern __shared__ __align__(1024) char smraw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::STAGES * L::STAGE);  // [STAGES]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + L::STAGES);

  const int64_t b = blockIdx.z;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  if (!Pb::live(m0, n0, BM, BN)) return;
  int M, N, K;
  Pb::dims(a, M, N, K);
  if (m0 >= M || n0 >= N) return;
  int kb, ke;
  Pb::krange(a, m0, n0, kb, ke);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    tmem_alloc(tslot, BN);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < L::STAGES; ++s) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  auto stageA_hi = [&](int s) { return sm + s * L::STAGE; };
  auto stageA_lo = [&](int s) { return sm + s * L::STAGE + L::A_BYTES; };
  auto stageB_hi = [&](int s) { return sm + s * L::STAGE + 2 * L::A_BYTES; };
  auto stageB_lo = [&](int s) { return sm + s * L::STAGE + 2 * L::A_BYTES + L::B_BYTES; };

  // Loader: each thread owns one 4x4 micro-block of A and (if tid < NB) one of B per stage.
  // Global loads for stage it+2 are issued into registers while the MMAs of stage it run;
  // they are split and written to shared memory only once that buffer is free again.
  constexpr int NB = BN * BK / 16;  // B micro-blocks
  int a_mb, a_kc, b_jb, b_kc;
  if (Pb::A_ALONG_K) { a_mb = tid >> 3; a_kc = tid & 7; }
  else { a_mb = tid & 31; a_kc = tid >> 5; }
  if (Pb::B_ALONG_K) { b_jb = tid >> 3; b_kc = tid & 7; }
  else { b_jb = tid % (BN / 4); b_kc = tid / (BN / 4); }
  float va[4][4], vb[4][4];
  auto fetch = [&](int k0) {
    Pb::loadA(a, b, m0 + 4 * a_mb, k0 + 4 * a_kc, va);
    if (tid < NB) Pb::loadB(a, b, n0 + 4 * b_jb, k0 + 4 * b_kc, vb);
  };
  auto put = [&](int s, int k0) {
    put4x4(stageA_hi(s), stageA_lo(s), 4 * a_mb, a_kc, va);
    if (tid < NB) {
      Pb::fixB(a, b, n0 + 4 * b_jb, k0 + 4 * b_kc, vb);
      put4x4(stageB_hi(s), stageB_lo(s), 4 * b_jb, b_kc, vb);
    }
    fence_async_smem();
  };

  constexpr uint32_t IDESC = idesc_tf32(BM, BN);
  const int nk = (ke > kb) ? (ke - kb + BK - 1) / BK : 0;
  bool ok = true;
  int last = nk - 1;       // last iteration whose MMAs were issued and committed
  uint32_t phasebits = 0;  // bit s = parity of the next wait on bars[s]

  if (nk > 0) {
    fetch(kb);
    put(0, kb);
    if (nk > 1) fetch(kb + BK);
  }
  __syncthreads();
  for (int it = 0; it < nk; ++it) {
    const int s = it & 1;
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ah = smem_u32(stageA_hi(s)), al = smem_u32(stageA_lo(s));
      const uint32_t bh = smem_u32(stageB_hi(s)), bl = smem_u32(stageB_lo(s));
#pragma unroll
      for (int kk = 0; kk < BK / UK; ++kk) {
        const uint32_t koff = kk * UK * 4;  // 32 bytes per k-step inside the swizzle row
        const uint64_t dah = sdesc_sw128(ah + koff), dal = sdesc_sw128(al + koff);
        const uint64_t dbh = sdesc_sw128(bh + koff), dbl = sdesc_sw128(bl + koff);
        const uint32_t acc0 = (it > 0 || kk > 0) ? 1u : 0u;
        mma_tf32(tmem, dal, dbh, IDESC, acc0);
        mma_tf32(tmem, dah, dbl, IDESC, 1u);
        mma_tf32(tmem, dah, dbh, IDESC, 1u);
      }
      mma_commit(&bars[s]);
    }
    if (it + 1 < nk) {
      const int s2 = (it + 1) & 1;
      if (it >= 1) {  // the MMAs of iteration it-1 read stage s2
        if (!mbar_wait(&bars[s2], (phasebits >> s2) & 1)) ok = false;
        phasebits ^= 1u << s2;
      }
      if (ok) put(s2, kb + (it + 1) * BK);
      if (it + 2 < nk) fetch(kb + (it + 2) * BK);
      // a timeout anywhere stops the issue of further MMAs for the whole CTA
      if (__syncthreads_or(!ok)) { ok = false; last = it; break; }
    }
  }
  // Commits are cumulative: the last one covers every MMA issued before it.  Commit j
  // completes phase j / 2 of bars[j % 2].  On the timeout path this is also the drain: the
  // TMEM is freed below only when it completed.
  bool drained = true;
  if (last >= 0) {
    if (!mbar_wait(&bars[last & 1], (last >> 1) & 1)) ok = drained = false;
  }
  ok = !__syncthreads_or(!ok);
  drained = __syncthreads_and(drained);
  tc_fence_after();

  // ---- epilogue: warp w reads TMEM lanes 32*(w%4) .. +31, column half w/4 ----
  if (!ok) {
    if (tid == 0) atomicOr(Pb::info(a, b), INFO_DEVICE_TIMEOUT);
  } else {
    const int lq = warp & 3;
    const int m = m0 + 32 * lq + lane;
    constexpr int CPW = BN / 2;  // columns per warp half
    for (int c = 0; c < CPW; c += 32) {
      const int col = (warp >> 2) * CPW + c;
      float v[32];
      if (nk > 0) tmem_ld32(tmem + ((uint32_t)(32 * lq) << 16) + col, v);
      else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      if (m < M && n0 + col < N) Pb::store(a, b, m, n0 + col, v, M, N);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && drained) tmem_dealloc(tmem, BN);
}

}  // namespace tc
}  // namespace qrb

