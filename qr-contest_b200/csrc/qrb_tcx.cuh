// qrb200 -- TMA-fed 3xTF32 tcgen05 GEMM tile for the float32 n^3 stages (Grams, R^{-1} apply,
// float32 closure) and the K = 128 block updates of the two-level Cholesky elimination.
//
// Same mathematics and policies as tc_gemm_kernel (qrb_tc.cuh / qrb_tc_ops.cuh), different
// data movement.  One 128 x 128 output tile per CTA, 9 warps:
//  * one lane of warp 8 brings raw float32 tiles into a 3-deep shared-memory ring with
//    cp.async.bulk.tensor (k-major operands: one {32 k, 128 row} SWIZZLE_128B box; m-major
//    operands: one unswizzled {128 row, 32 k} box), then issues the 12 MMAs of each stage and
//    commits them to an mbarrier;
//  * warps 0-7 split the raw tiles into tf32 hi / lo parts: for A_TMEM policies warps 0-3 write
//    A's rows straight into tensor memory (tcgen05.st; the MMA reads A from TMEM) and all 8
//    warps split B into shared-memory planes (K-major SW128, the UMMA operand layout); other
//    policies split both operands into planes.  Two plane / TMEM sets let the split of stage
//    t+1 overlap the MMAs of stage t.  Hand-offs are mbarriers only (no CTA barrier per stage).
// Out-of-range boxes are zero-filled by the TMA unit.  No multicast: every CTA loads its own
// tiles (the library also runs on 2-8 GPUs).
#pragma once
#include <cuda.h>

#include "qrb_tc_ops.cuh"

namespace qrb {
namespace tcx {

using tc::BK;
using tc::BM;
using tc::NTHREADS;
using tc::UK;

constexpr int BN = 128;
#ifndef QRB_TCX_STAGES
#define QRB_TCX_STAGES 3
#endif
constexpr int RAW_STAGES = QRB_TCX_STAGES;  // raw tiles in flight (3 measured best of 3-5)
constexpr int RAW_A = BM * BK * 4;   // 16 KB
constexpr int RAW_B = BN * BK * 4;   // 16 KB
constexpr int PLANE = 16384;         // one hi or lo plane of a 128 x 32 operand tile
constexpr int PLANE_SETS = 2;      // split of stage t+1 overlaps the MMAs of stage t
// A_TMEM policies keep A in tensor memory: a plane set holds B hi / lo only.
template <bool A_TMEM>
constexpr int plane_set_bytes() { return (A_TMEM ? 2 : 4) * PLANE; }
// Pipeline shape of a launch: RS raw stages, PS plane / TMEM-operand sets, LONGK = drain the
// TMEM accumulator into float32 registers in long reductions, MINB = CTAs per SM it is built for.
template <int RS_, int PS_, bool LONGK_, int MINB_>
struct Cfg {
  static constexpr int RS = RS_, PS = PS_, MINB = MINB_;
  static constexpr bool LONGK = LONGK_;
};
// One CTA per SM, 3 raw stages and 2 plane sets (the split of stage t+1 overlaps the MMAs of
// stage t inside the CTA); the only shape that drains, so every K is allowed.
using CfgWide = Cfg<RAW_STAGES, PLANE_SETS, true, 1>;
// Two CTAs per SM for K <= 512: 2 raw stages, 1 plane set and no drain registers (<= 112
// registers, 97 KB of shared memory); one CTA's epilogue and split overlap the other's MMAs.
using CfgDual = Cfg<2, 1, false, 2>;
constexpr int kDualMaxK = 512;

template <class Pb, class C = CfgWide>
constexpr int smem_bytes() {
  return C::RS * (RAW_A + RAW_B) + C::PS * plane_set_bytes<Pb::A_TMEM>() + 1024 + 128;
}

struct Maps {
  CUtensorMap a;  // raw A source
  CUtensorMap b;  // raw B source
};

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(tc::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(tc::smem_u32(bar))
      : "memory");
}

// Raw tile of an operand whose rows (tile rows = M or N index) are contiguous in k:
// one box {32 k, 128 rows}, 128-byte swizzle.  Element (r, k) sits at sw128_off(r, k/4) + 4*(k%4).
// Raw tile of an operand stored k-major (X[k][r]): one unswizzled box {128 r, 32 k}; element
// (r, k) at 512 k + 4 r.  (Four swizzled {32, 32} boxes were measured slower: the copy engine
// spends most of its time per box, not per byte, on these small boxes.)  The row-per-thread
// A reads and the 4 x 4 micro-block B reads of such a tile are bank-conflict free as is.
template <bool KMAJOR>
__device__ __forceinline__ void issue_raw(char* dst, const CUtensorMap* map, int r0, int k0,
                                          int z, uint64_t* bar) {
  if (KMAJOR) tma_load_3d(dst, map, k0, r0, z, bar);
  else tma_load_3d(dst, map, r0, k0, z, bar);
}

// 4(row) x 4(k) micro-block (rows 4*rb.., k 4*kc..) out of a raw tile.
template <bool KMAJOR>
__device__ __forceinline__ void read_raw(const char* raw, int rb, int kc, float (&v)[4][4]) {
  if (KMAJOR) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 t = *reinterpret_cast<const float4*>(raw + tc::sw128_off(4 * rb + i, kc));
      v[i][0] = t.x; v[i][1] = t.y; v[i][2] = t.z; v[i][3] = t.w;
    }
  } else {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float4 t = *reinterpret_cast<const float4*>(raw + (4 * kc + kk) * 512 + 16 * rb);
      v[0][kk] = t.x; v[1][kk] = t.y; v[2][kk] = t.z; v[3][kk] = t.w;
    }
  }
}

// Policy additions over the tc_ops policies: A_KMAJOR / B_KMAJOR (raw layout of the sources
// described by the two tensor maps), TILE_SCALE (B transform with a per-column scale:
// col_scale, fixB_scaled; otherwise fixB).
#ifdef QRB_PANEL_TIMERS
// test-kit profiling build: cycle sums per phase over all CTAs, of split thread 0 (slots 0-3)
// and of the issuing thread (slots 4-5)
#define QRB_GT(who, i)                                                     \
  do {                                                                     \
    if (tid == (who)) {                                                    \
      const long long now_ = clock64();                                    \
      atomicAdd(reinterpret_cast<unsigned long long*>(&g_panel_timers[i]), \
                (unsigned long long)(now_ - gt_prev_));                    \
      gt_prev_ = now_;                                                     \
    }                                                                      \
  } while (0)
#else
#define QRB_GT(who, i) do { } while (0)
#endif

// Warp roles: warps 0-7 split raw tiles into hi/lo planes and run the epilogue; warp 8 (one
// elected lane) issues the TMA loads and the MMAs.  tcgen05.mma issue blocks while the tensor
// pipe works through the previous stage, so the issuing thread must not be one the split waits
// for: with a CTA-wide barrier per stage the split, the waits and the MMAs ran back to back.
// Hand-offs are mbarriers only:
//   full[s]     TMA -> split      raw tiles of stage t landed          (tx bytes)
//   pfull[ps]   split -> issuer   planes of stage t written            (256 arrivals)
//   mma_bar[ps] MMAs -> split     planes of stage t free / TMEM ready  (tcgen05.commit)
constexpr int XTHREADS = NTHREADS + 32;
#ifndef QRB_TCX_BALL
#define QRB_TCX_BALL 1
#endif
// A-in-TMEM tiles: every split warp also takes one B micro-block (else warps 4-7 take two each)
constexpr bool kBAll = QRB_TCX_BALL != 0;
constexpr int TM_A = BN;              // TMEM: accumulator in columns [0, BN), A sets after it
constexpr int TM_COLS = 256;          // BN + 2 sets x (hi, lo) x BK columns, power of two

template <class Pb, class C = CfgWide>
__global__ void __launch_bounds__(XTHREADS, C::MINB)
    tcx_gemm_kernel(const __grid_constant__ Maps maps, typename Pb::Args a) {
  constexpr int RAW_STAGES = C::RS, PLANE_SETS = C::PS;
  extern __shared__ __align__(1024) char smraw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  char* rawA = sm;                                  // [RAW_STAGES][RAW_A]
  char* rawB = sm + RAW_STAGES * RAW_A;             // [RAW_STAGES][RAW_B]
  // [PLANE_SETS] x {b_hi, b_lo} (A_TMEM) or {a_hi, a_lo, b_hi, b_lo}
  constexpr int PSET = plane_set_bytes<Pb::A_TMEM>(), PB = Pb::A_TMEM ? 0 : 2 * PLANE;
  char* pl0 = sm + RAW_STAGES * (RAW_A + RAW_B);
  uint64_t* full = reinterpret_cast<uint64_t*>(pl0 + PLANE_SETS * PSET);  // [RAW_STAGES]
  uint64_t* mma_bar = full + RAW_STAGES;                                          // [PLANE_SETS]
  uint64_t* pfull = mma_bar + PLANE_SETS;                                         // [PLANE_SETS]
  static_assert(smem_bytes<Pb, C>() + BN * 4 <= 227 * 1024 / C::MINB, "tcx shared memory");
  uint32_t* tslot = reinterpret_cast<uint32_t*>(pfull + PLANE_SETS);

  const int64_t b = blockIdx.z;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  if (!Pb::live(m0, n0, BM, BN)) return;
  int M, N, K;
  Pb::dims(a, M, N, K);
  if (m0 >= M || n0 >= N) return;
  int kb, ke;
  Pb::krange(a, m0, n0, kb, ke);
  const int nk = (ke > kb) ? (ke - kb + BK - 1) / BK : 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool issuer_warp = warp == NTHREADS / 32;
#ifdef QRB_PANEL_TIMERS
  long long gt_prev_ = clock64();
#endif

  // issuer-side progress (TMA stages issued, MMA stages committed) and whether a timeout's
  // drain completed; read after the CTA barrier that follows the role loops
  __shared__ int s_issued, s_committed, s_drained;
  if (warp == 0) {
    tc::tmem_alloc(tslot, TM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    s_issued = s_committed = 0;
    s_drained = 1;
    for (int s = 0; s < RAW_STAGES; ++s) tc::mbar_init(&full[s], 1);
    for (int p = 0; p < PLANE_SETS; ++p) {
      tc::mbar_init(&mma_bar[p], 1);
      tc::mbar_init(&pfull[p], NTHREADS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Start the tile's epilogue reads (read-modify-write policies) on their way to L2 so that
  // they overlap the main loop: 128 rows x 4 lines of 128 bytes.
  for (int idx = tid; idx < BM * 4; idx += XTHREADS) {
    const int row = idx >> 2, j = n0 + 32 * (idx & 3);
    if (m0 + row < M && j < N) {
      const void* p = Pb::c_addr(a, b, m0 + row, j);
      if (p) asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    }
  }
  // per-column scale of the B transform (QApplyX: d_j^{-1/2}), read once per tile
  __shared__ __align__(16) float tscale[BN];
  if constexpr (Pb::TILE_SCALE)
    for (int j = tid; j < BN; j += XTHREADS) tscale[j] = Pb::col_scale(a, b, n0 + j);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  // Long reductions drain the TMEM accumulator into float32 registers every DRAIN stages:
  // TMEM accumulation does not round to nearest on each add, and over K = 2048 the drift is
  // large enough to make a Gram indefinite.  Short reductions (nk <= 2 * DRAIN) never drain.
  constexpr int DRAIN = 8;
  const bool drains = C::LONGK && nk > 2 * DRAIN;
  float racc[C::LONGK ? BN / 2 : 1];
#pragma unroll
  for (int i = 0; i < (C::LONGK ? BN / 2 : 1); ++i) racc[i] = 0.f;
  const int lq = warp & 3;
  bool ok = true;

  if (issuer_warp) {
    if (lane == 0) {
      int o_ar, o_ak, o_br, o_bk;  // where the operands start inside the mapped buffers
      Pb::org(a, o_ar, o_ak, o_br, o_bk);
      auto issue = [&](int t) {  // raw tiles of k-step t into slot t % RAW_STAGES
        const int s = t % RAW_STAGES, k0 = kb + t * BK;
        mbar_expect_tx(&full[s], RAW_A + RAW_B);
        issue_raw<Pb::A_KMAJOR>(rawA + s * RAW_A, &maps.a, m0 + o_ar, k0 + o_ak, (int)b, &full[s]);
        issue_raw<Pb::B_KMAJOR>(rawB + s * RAW_B, &maps.b, n0 + o_br, k0 + o_bk, (int)b, &full[s]);
      };
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.b)) : "memory");
      for (int t = 0; t < nk && t < RAW_STAGES; ++t) { issue(t); s_issued = t + 1; }
      constexpr uint32_t IDESC = tc::idesc_tf32(BM, BN);
      for (int t = 0; t < nk; ++t) {
        const int ps = t % PLANE_SETS;
        char* pl = pl0 + ps * PSET;
        // on a timeout nothing more is issued; what is in flight is drained below
        if (!tc::mbar_wait(&pfull[ps], (t / PLANE_SETS) & 1)) { ok = false; break; }
        tc::tc_fence_after();
        QRB_GT(NTHREADS, 4);
        if (t + RAW_STAGES < nk) {  // slot t % RAW_STAGES has been split
          issue(t + RAW_STAGES);
          s_issued = t + RAW_STAGES + 1;
        }
        const uint32_t bh = tc::smem_u32(pl + PB), bl = tc::smem_u32(pl + PB + PLANE);
#pragma unroll
        for (int kk = 0; kk < BK / UK; ++kk) {
          const uint32_t koff = kk * UK * 4;
          const uint64_t dbh = tc::sdesc_sw128(bh + koff), dbl = tc::sdesc_sw128(bl + koff);
          const bool fresh = (drains ? (t % DRAIN == 0) : (t == 0)) && kk == 0;
          if constexpr (Pb::A_TMEM) {
            const uint32_t ah = tmem + TM_A + ps * 2 * BK + kk * UK, al = ah + BK;
            tc::mma_tf32_ta(tmem, al, dbh, IDESC, fresh ? 0u : 1u);
            tc::mma_tf32_ta(tmem, ah, dbl, IDESC, 1u);
            tc::mma_tf32_ta(tmem, ah, dbh, IDESC, 1u);
          } else {
            const uint64_t dah = tc::sdesc_sw128(tc::smem_u32(pl) + koff);
            const uint64_t dal = tc::sdesc_sw128(tc::smem_u32(pl + PLANE) + koff);
            tc::mma_tf32(tmem, dal, dbh, IDESC, fresh ? 0u : 1u);
            tc::mma_tf32(tmem, dah, dbl, IDESC, 1u);
            tc::mma_tf32(tmem, dah, dbh, IDESC, 1u);
          }
        }
        tc::mma_commit(&mma_bar[ps]);
        s_committed = t + 1;
        QRB_GT(NTHREADS, 5);
      }
    }
  } else {
    // Split roles.  Warps 0-3: thread = tile row r (its TMEM lane) of A; it reads the row's 32
    // k values from the raw tile and writes tf32 hi / lo into the A columns of this stage's
    // TMEM set (A never goes through shared-memory planes).  Warps 4-7: B, two 4 x 4
    // micro-blocks per thread into the shared-memory planes; the 8 threads of a quarter-warp
    // take column blocks 8g + q and k chunks (q + c) % 8, so their 16-byte accesses fall on 8
    // distinct bank groups for both raw layouts and for the swizzled plane writes.
    const bool a_role = warp < 4;
    const int r = 32 * warp + lane;
    QRB_GT(0, 0);
    for (int t = 0; t < nk; ++t) {
      const int s = t % RAW_STAGES, k0 = kb + t * BK;
      const int ps = t % PLANE_SETS;        // plane / TMEM set of this stage
      char* pl = pl0 + ps * PSET;
      if (ok && !tc::mbar_wait(&full[s], (t / RAW_STAGES) & 1)) ok = false;
      QRB_GT(0, 1);
      // set ps was last read by the MMAs of stage t - PLANE_SETS (its commit completed phase
      // t / PLANE_SETS - 1 of mma_bar[ps])
      if (t >= PLANE_SETS && ok && !tc::mbar_wait(&mma_bar[ps], ((t / PLANE_SETS) - 1) & 1))
        ok = false;
      QRB_GT(0, 2);
      if (!Pb::A_TMEM) {
        // all 256 threads: one A and one B micro-block each, both into shared-memory planes
        const int sq = tid & 7, sg = tid >> 3;
        const int mb = 8 * (sg & 3) + sq, kc = (sq + (sg >> 2)) & 7;
        float v[4][4];
        read_raw<Pb::A_KMAJOR>(rawA + s * RAW_A, mb, kc, v);
        tc::put4x4(pl, pl + PLANE, 4 * mb, kc, v);
        read_raw<Pb::B_KMAJOR>(rawB + s * RAW_B, mb, kc, v);
        if constexpr (Pb::TILE_SCALE)
          Pb::fixB_scaled(a, n0 + 4 * mb, k0 + 4 * kc, tscale + 4 * mb, v);
        else
          Pb::fixB(a, b, n0 + 4 * mb, k0 + 4 * kc, v);
        tc::put4x4(pl + PB, pl + PB + PLANE, 4 * mb, kc, v);
      } else if (a_role) {
        const char* raw = rawA + s * RAW_A;
        float hi[BK], lo[BK];
        if (Pb::A_KMAJOR) {
#pragma unroll
          for (int c = 0; c < BK / 4; ++c) {
            const float4 x = *reinterpret_cast<const float4*>(raw + tc::sw128_off(r, c));
            hi[4 * c] = x.x; hi[4 * c + 1] = x.y; hi[4 * c + 2] = x.z; hi[4 * c + 3] = x.w;
          }
        } else {
#pragma unroll
          for (int k = 0; k < BK; ++k) hi[k] = *reinterpret_cast<const float*>(raw + 512 * k + 4 * r);
        }
#pragma unroll
        for (int k = 0; k < BK; ++k) {
          const float x = hi[k];
          hi[k] = tc::tf32_rn_int(x);
          lo[k] = tc::tf32_rn_int(x - hi[k]);
        }
        const uint32_t ta = tmem + ((uint32_t)(32 * warp) << 16) + TM_A + ps * 2 * BK;
        tc::tmem_st32(ta, hi);
        tc::tmem_st32(ta + BK, lo);
      }
      if (Pb::A_TMEM && (kBAll || !a_role)) {
        // B micro-blocks: one per thread over all 8 warps (kBAll), or two per thread of warps 4-7
#pragma unroll
        for (int rep = 0; rep < (kBAll ? 1 : 2); ++rep) {
          const int idx = kBAll ? tid : (tid - 128) + 128 * rep, sq = idx & 7, sg = idx >> 3;
          const int jb = 8 * (sg & 3) + sq, kc = (sq + (sg >> 2)) & 7;
          float v[4][4];
          read_raw<Pb::B_KMAJOR>(rawB + s * RAW_B, jb, kc, v);
          if constexpr (Pb::TILE_SCALE)
            Pb::fixB_scaled(a, n0 + 4 * jb, k0 + 4 * kc, tscale + 4 * jb, v);
          else
            Pb::fixB(a, b, n0 + 4 * jb, k0 + 4 * kc, v);
          tc::put4x4(pl + PB, pl + PB + PLANE, 4 * jb, kc, v);
        }
      }
      tc::fence_async_smem();   // generic-proxy plane writes -> visible to the MMAs
      tc::tc_fence_before();    // orders the tcgen05.st of A and any earlier tcgen05.ld
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(&pfull[ps]))
                   : "memory");
      QRB_GT(0, 3);
      if (drains && (t + 1) % DRAIN == 0 && t + 1 < nk) {
        if (ok && !tc::mbar_wait(&mma_bar[ps], (t / PLANE_SETS) & 1)) ok = false;
        tc::tc_fence_after();
        if constexpr (C::LONGK) {
#pragma unroll
          for (int c = 0; c < BN / 2; c += 32) {
            float v2[32];
            tc::tmem_ld32(tmem + ((uint32_t)(32 * lq) << 16) + (warp >> 2) * (BN / 2) + c, v2);
#pragma unroll
            for (int i = 0; i < 32; ++i) racc[c + i] += v2[i];
          }
        }
      }
    }
    // the last commit covers every MMA issued before it
    if (nk >= 1 && ok) {
      const int t = nk - 1;
      if (!tc::mbar_wait(&mma_bar[t % PLANE_SETS], (t / PLANE_SETS) & 1)) ok = false;
    }
    tc::tc_fence_after();
  }

  const bool failed = __syncthreads_or(!ok);
  if (failed && issuer_warp && lane == 0) {
    // Drain before the TMEM is freed and the CTA exits: the last commit covers every MMA
    // issued (commit t completes phase t / PLANE_SETS of mma_bar[t % PLANE_SETS]), and each
    // of the last
    // RAW_STAGES TMA stages issued completes phase u / RAW_STAGES of full[u % RAW_STAGES]
    // (parity waits do not consume a phase, so waiting on one already seen is harmless).
    bool drained = true;
    const int nc = s_committed, ni = s_issued;
    if (nc > 0 && !tc::mbar_wait(&mma_bar[(nc - 1) % PLANE_SETS], ((nc - 1) / PLANE_SETS) & 1))
      drained = false;
    for (int u = (ni > RAW_STAGES ? ni - RAW_STAGES : 0); u < ni; ++u)
      if (!tc::mbar_wait(&full[u % RAW_STAGES], (u / RAW_STAGES) & 1)) drained = false;
    if (!drained) s_drained = 0;
  }
  if (failed) {
    if (tid == 0) atomicOr(Pb::info(a, b), INFO_DEVICE_TIMEOUT);
  } else if (!issuer_warp) {
    const int m = m0 + 32 * lq + lane;
    constexpr int CPW = BN / 2;
#pragma unroll
    for (int c = 0; c < CPW; c += 32) {
      const int col = (warp >> 2) * CPW + c;
      float v[32];
      if (nk > 0) tc::tmem_ld32(tmem + ((uint32_t)(32 * lq) << 16) + col, v);
      else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      if constexpr (C::LONGK) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += racc[c + i];
      }
      if (m < M && n0 + col < N) Pb::store(a, b, m, n0 + col, v, M, N);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  QRB_GT(0, 6);
  if (warp == 0 && s_drained) tc::tmem_dealloc(tmem, TM_COLS);
}

// ---- policies: the tc_ops ones plus the raw-layout flags ----
struct GramX : tc::GramTC {
  static constexpr bool A_KMAJOR = false, B_KMAJOR = false;  // X[k][m], X[k][j]
  static constexpr bool A_TMEM = true;
  __device__ static void org(const Args&, int& ar, int& ak, int& br, int& bk) { ar = ak = br = bk = 0; }
  static constexpr bool TILE_SCALE = false;
};
struct QApplyX : tc::QApplyTC {
  static constexpr bool A_KMAJOR = true, B_KMAJOR = true;    // X[m][k], RL[j][k]
  // A (X rows) in TMEM; the transformed B is split by all 8 warps (1.35 / 1.84 ms per pass-1 /
  // pass-2 launch of 768 matrices vs 1.41 / 1.96 with both operands in shared-memory planes)
  static constexpr bool A_TMEM = true;
  __device__ static void org(const Args&, int& ar, int& ak, int& br, int& bk) { ar = ak = br = bk = 0; }
  static constexpr bool TILE_SCALE = true;
  __device__ static float col_scale(const Args& a, int64_t b, int j) {
    return (j < a.n) ? 1.f / sqrtf(a.D[b * a.n + j]) : 0.f;
  }
  // QApplyTC::fixB with d_j^{-1/2} from the tile's shared copy (rs[i] for column j0 + i)
  __device__ static void fixB_scaled(const Args& a, int j0, int k0, const float* rs,
                                     float (&v)[4][4]) {
    const float4 r4 = *reinterpret_cast<const float4*>(rs);  // one 16-byte shared load
    const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = j0 + i;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int k = k0 + kk;
        float r;
        if (j >= a.n || k > j) r = 0.f;
        else if (k < j) r = a.pass2 ? -(v[i][kk] * rv[i]) : v[i][kk] * rv[i];
        else r = a.pass2 ? (1.f - rv[i]) : rv[i];
        v[i][kk] = r;
      }
    }
  }
};
// T = the output dtype; B (A of the factorization) is always read as float32 (a 16-bit input
// is widened into the workspace first, as the reference's .to(float32) does)
template <typename T>
struct ClosureXT : tc::ClosureTC<T> {
  using Args = typename tc::ClosureTC<T>::Args;
  static constexpr bool A_KMAJOR = false, B_KMAJOR = false;  // Q[k][m], A[k][j]
  static constexpr bool A_TMEM = true;
  __device__ static void org(const Args&, int& ar, int& ak, int& br, int& bk) { ar = ak = br = bk = 0; }
  static constexpr bool TILE_SCALE = false;
};
using ClosureX = ClosureXT<float>;

// K = block updates of the two-level Cholesky elimination (see SyrkTC / LinvBlkTC in
// qrb_tc_ops.cuh) on the TMA-fed tile.  org() places the operand tiles inside the mapped
// buffers: SyrkX reads R rows [kb, ke) at columns [ke, n) for both operands (m-major);
// LinvBlkX reads the W buffer (rows [ke, n), k-major, ldw columns) and the Bp buffer (ldw
// rows of n columns, m-major).
struct SyrkX : tc::SyrkTC {
  static constexpr bool A_KMAJOR = false, B_KMAJOR = false;  // R[kb + k][ke + m]
  static constexpr bool A_TMEM = true, TILE_SCALE = false;
  __device__ static void org(const Args& a, int& ar, int& ak, int& br, int& bk) {
    ar = br = a.k1;
    ak = bk = a.k0;
  }
  __device__ static float row_scale(const Args&, int64_t, int) { return 0.f; }
  __device__ static void fixA_row(const Args&, int, int, float, float (&)[BK]) {}
};
struct LinvBlkX : tc::LinvBlkTC {
  static constexpr bool A_KMAJOR = true, B_KMAJOR = false;   // W[ke + m][k], Bp[k][j]
  static constexpr bool A_TMEM = true, TILE_SCALE = false;
  __device__ static void org(const Args& a, int& ar, int& ak, int& br, int& bk) {
    ar = a.ke;
    ak = br = bk = 0;
  }
  __device__ static float row_scale(const Args&, int64_t, int) { return 0.f; }
  __device__ static void fixA_row(const Args&, int, int, float, float (&)[BK]) {}
};

}  // namespace tcx
}  // namespace qrb
