// Blackwell (sm_100a) GEMM on 5th-generation tensor cores:  C[M,N] = A[M,K] · W[N,K]^T with
// the same fused epilogue functors as the warp-level path (gemm_mma.cuh).
//
//   * TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast) stages 128×64 A tiles and
//     BN×64 W tiles into a STAGES-deep shared-memory ring guarded by mbarriers;
//   * one thread issues tcgen05.mma (kind::f16, M=128, N=BN, K=16 per instruction) with the
//     accumulator in tensor memory; tcgen05.commit releases ring slots and hands finished
//     accumulators to the epilogue;
//   * the accumulator is double buffered in TMEM (2·BN columns), so eight epilogue warps drain
//     tile i (tcgen05.ld → registers → functor) while the MMA warp accumulates tile i+1;
//   * persistent CTAs (one per SM) walk the tiles M-fastest, so the CTAs working at the same
//     time share W tiles through L2 and every weight byte comes from HBM about once;
//   * two cluster modes: a K split between two CTAs (KS = 2) for long-K GEMMs of few tiles, and
//     256-row tiles on a CTA pair with tcgen05 cta_group::2 (CG = 2) for GEMMs of many tiles.
// Every mbarrier wait is bounded (about one second of globaltimer); on timeout the kernel sets
// *err, leaves its loops, waits for its own tensor-core work and frees TMEM before returning.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace pi0 {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;                       // 64 × 16-bit = one 128-byte swizzle row
// epilogue warps: EPQ per TMEM lane quarter (a warp may only read its quarter's lanes), taking
// every EPQ-th 32-column chunk of the tile, so a tile drains EPQ times as fast as with one
constexpr int EPQ = 2;
constexpr int EPI_WARPS = 4 * EPQ;
constexpr int NT = 64 + 32 * EPI_WARPS;      // + the TMA producer warp and the MMA warp
constexpr unsigned long long kTimeoutNs = 1000000000ull;

enum ErrCode { ERR_NONE = 0, ERR_TIMEOUT_PRODUCER = 1, ERR_TIMEOUT_MMA = 2, ERR_TIMEOUT_EPI = 3 };

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of parity `parity` to complete; false (and *err = code) after ~1 s, or as
// soon as another role has reported an error (unless `bail` is false: drain waits). The hot
// loop only polls the barrier; the clock is read every 128 polls and the (global) error flag
// every 8192, so a completed phase is seen without a memory round trip in the way.
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int* err, int code,
                                            bool bail) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 127) == 0) {
      if (globaltimer() - t0 > kTimeoutNs) {
        atomicCAS(err, 0, code);
        return false;
      }
      if (bail && (it & 8191) == 0 && *(volatile int*)err != 0) return false;
    }
  }
}
// (the polling loop is out of line: it is rarely entered more than once per wait, and keeping it
// out of every call site keeps the kernels' code small)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          bool bail = true) {
  if (mbar_try(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, err, code, bail);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle layout written by TMA:
// rows of 128 B, 8-row (1024 B) swizzle atoms, so the stride between 8-row groups is 1024 B.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);     // start address
  d |= (uint64_t)1 << 16;                      // leading-dimension byte offset (unused here)
  d |= (uint64_t)(1024 >> 4) << 32;            // stride-dimension byte offset
  d |= (uint64_t)1 << 46;                      // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                      // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: fp32 accumulate, A and B of the same 16-bit
// type (fp16 or bf16), both K-major.
template <typename T>
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | ((Tr<T>::kBf16 ? 1u : 0u) << 7)          // A format
         | ((Tr<T>::kBf16 ? 1u : 0u) << 10)         // B format
         | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// ---- CTA-pair forms (tcgen05 cta_group::2): the even CTA of a cluster pair issues one MMA that
// reads A (128 rows each) and B (half the columns each) from both CTAs' shared memory at the
// same offsets and writes each CTA's 128 accumulator rows into that CTA's tensor memory ----
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t a, uint64_t b,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// arrive on the barrier at this offset in both CTAs of the pair once the pair's MMAs complete
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on `bar_cluster`, a
// shared::cluster address that may be the peer CTA's barrier (the pair's loads all complete on
// the even CTA's barrier, where its MMA issuer waits)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes × 32 consecutive 32-bit columns: thread i of the warp gets lane (quarter·32 + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- thread-block clusters: rank, barrier, distributed shared memory ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// the address of this CTA's shared-memory location `saddr` in the CTA of cluster rank `rank`
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int BN, int STAGES, int CG = 1>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN / CG * BK * 2;  // a CTA pair stages half of W each
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BYTES = STAGES * STAGE + 1024;  // + alignment slack
  // double-buffered accumulator, rounded up to the power of two tcgen05.alloc requires
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128
                                        : 2 * BN <= 256 ? 256 : 512;
};

// KS = 2: split-K over a cluster of two CTAs, one output tile per cluster (grid = 2·tiles, at
// most one wave). Rank r accumulates k-blocks [r·⌈nk/2⌉, (r+1)·⌈nk/2⌉) and finishes output
// columns [r·BN/2, (r+1)·BN/2): it parks the other half of its accumulator in its drained ring,
// and after a cluster barrier adds the peer's parked half to its own through distributed shared
// memory (p0 + p1, the same sum on both ranks) before the epilogue.
//
// CG = 2: one 256 × BN output tile per cluster pair on tcgen05 cta_group::2 (persistent pairs,
// grid = 2·pairs). Each CTA stages its own 128 rows of A and its own BN/2 rows of W per k-block,
// so a pair moves (256 + BN)·64 elements for a 256 × BN × 64 product where two single CTAs move
// 2·(128 + BN)·64: a third less shared-memory ingress per SM at BN = 256. The even CTA issues
// the MMAs; both CTAs' loads complete on its ring barriers (it arms them for the pair's bytes);
// its commits arrive on the same barrier in both CTAs (ring slots, finished accumulators); both
// CTAs' epilogue warps drain their own 128 rows from their own tensor memory and report the
// drained accumulator to the even CTA.
template <typename T, int BN, int STAGES, class Epi, int KS = 1, int CG = 1>
__global__ void __launch_bounds__(NT, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   int M, int N, int K, Epi epi, int* err) {
  using S = Smem<BN, STAGES, CG>;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(KS == 1 || (KS == 2 && BN % 64 == 0 && 128 * (BN / 2 + 4) * 4 <= STAGES * S::STAGE),
                "split-K pair: parked half must fit the ring");
  static_assert(CG == 1 || (CG == 2 && KS == 1 && BN % 32 == 0 && BN >= 64),
                "CTA-pair tiles: no K split, W half at least 32 rows");
  constexpr int TM = BM * CG;  // rows of one output tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2], drain, recv;
  __shared__ uint32_t s_tmem;
  bool epi_ok = false;  // KS > 1, epilogue warps: this CTA's accumulator is complete

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + TM - 1) / TM, n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const uint32_t rank = (KS > 1 || CG > 1) ? cluster_rank() : 0;
  const bool leader = CG == 1 || rank == 0;      // issues the MMAs (CG = 2: the even CTA)
  const int mrow = CG > 1 ? (int)rank * BM : 0;  // this CTA's rows inside a pair tile
  const int nk_all = (K + BK - 1) / BK, kper = (nk_all + KS - 1) / KS;
  const int kb0 = KS > 1 ? (int)rank * kper : 0, nk = max(0, min(nk_all, kb0 + kper) - kb0);
  const int t_first = blockIdx.x / (KS * CG), t_step = gridDim.x / (KS * CG);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS * CG);
    }
    mbar_init(&drain, 1);
    mbar_init(&recv, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {  // the same columns in both CTAs' tensor memory
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&s_tmem)),
                   "r"(S::TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&s_tmem)),
                   "r"(S::TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  // CG = 2: both CTAs' barriers are initialised and the pair's tensor memory allocated before
  // either CTA loads into, commits to or arrives on the other's barriers
  if constexpr (CG == 2) cluster_sync();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;  // bit s: stage s has a load in flight or landed (phase ph_of[s])
      uint32_t ph_of = 0;
      for (int t = t_first; t < tiles; t += t_step) {
        const int m0 = (t % m_tiles) * TM + mrow, n0 = (t / m_tiles) * BN + (int)rank * (BN / 2) * (CG - 1);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, err, ERR_TIMEOUT_PRODUCER)) goto producer_done;
          uint8_t* st = sbase + s * S::STAGE;
          if constexpr (CG == 2) {
            if (leader) mbar_expect_tx(&full[s], 2 * S::STAGE);  // both CTAs' bytes
            const uint32_t fb = map_rank(smem_u32(&full[s]), 0);
            tma_load_2d_pair(st, &tmA, fb, (kb0 + kb) * BK, m0);
            tma_load_2d_pair(st + S::A_BYTES, &tmB, fb, (kb0 + kb) * BK, n0);
          } else {
            mbar_expect_tx(&full[s], S::STAGE);
            tma_load_2d(st, &tmA, &full[s], (kb0 + kb) * BK, m0);
            tma_load_2d(st + S::A_BYTES, &tmB, &full[s], (kb0 + kb) * BK, n0);
          }
          issued |= 1u << s;
          ph_of = (ph_of & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    producer_done:
      // never leave with a TMA write into this CTA's shared memory still in flight (the odd CTA
      // of a pair: its loads complete on the even CTA's barrier, which the MMAs that read them
      // wait for; their commit on this CTA's slot barrier says they have landed)
      for (int st = 0; st < STAGES; ++st)
        if (issued & (1u << st)) {
          if (leader)
            mbar_wait(&full[st], (ph_of >> st) & 1u, err, ERR_TIMEOUT_PRODUCER, false);
          else
            mbar_wait(&empty[st], (ph_of >> st) & 1u, err, ERR_TIMEOUT_PRODUCER, false);
        }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // MMA issuer
      constexpr uint32_t idesc = idesc_f16<T>(TM, BN);
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      for (int t = t_first; t < tiles; t += t_step, ++i) {
        const int acc = i & 1;
        const uint32_t aph = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1, err, ERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[s], ph, err, ERR_TIMEOUT_MMA)) goto mma_done;
          tc_fence_after();
          const uint32_t sa = smem_u32(sbase + s * S::STAGE);
          const uint64_t da = desc_sw128(sa), db = desc_sw128(sa + S::A_BYTES);
          if constexpr (CG == 2) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16_pair(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
            umma_commit_pair_both(&empty[s]);
          } else {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)  // +32 B per K step inside the swizzle row
              umma_f16(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
            umma_commit(&empty[s]);
          }
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if constexpr (CG == 2)
          umma_commit_pair_both(&tfull[acc]);
        else
          umma_commit(&tfull[acc]);
      }
    mma_done:
      // every issued MMA completes before TMEM is released
      if constexpr (CG == 2)
        umma_commit_pair(&drain);
      else
        umma_commit(&drain);
      mbar_wait(&drain, 0, err, ERR_TIMEOUT_MMA, false);
    }
  } else if (KS > 1) {  // split-K pair: park the peer's half of the accumulator
    const int q = warp & 3, sub = (warp - 2) >> 2;
    if (t_first < tiles) {  // operands of the columns this rank finishes, requested early
      const int prow = (t_first % m_tiles) * BM + q * 32 + lane;
      const int pn0 = (t_first / m_tiles) * BN + (int)rank * (BN / 2);
      if (prow < M)
        for (int c = sub * 32; c < BN / 2 && pn0 + c < N; c += 32 * EPQ) epi.prefetch(prow, pn0 + c);
    }
    bool ok = t_first < tiles && nk > 0;
    if (ok && lane == 0) ok = mbar_wait(&tfull[0], 0, err, ERR_TIMEOUT_EPI);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    epi_ok = ok;
    if (ok) {
      tc_fence_after();
      constexpr int H = BN / 2, XLD = H + 4;
      float* park = reinterpret_cast<float*>(sbase) + (q * 32 + lane) * XLD;
      const int pc0 = (1 - (int)rank) * H;
#pragma unroll 1
      for (int c = sub * 32; c < H; c += 32 * EPQ) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + pc0 + c, v);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(park + c + 4 * u) =
              make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                          __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // park -> bulk copy engine
    }
  } else {  // epilogue warps: TMEM lane quarter = warp % 4, chunk residue = (warp - 2) / 4
    const int q = warp & 3, sub = (warp - 2) >> 2;
    int i = 0;
    for (int t = t_first; t < tiles; t += t_step, ++i) {
      const int acc = i & 1;
      const uint32_t aph = (i >> 1) & 1;
      const int m0 = (t % m_tiles) * TM + mrow, n0 = (t / m_tiles) * BN;
      // request every global operand of this warp's chunks into L1 while the accumulator is
      // still being computed (the epilogue warps are otherwise idle then)
      {
        const int prow = m0 + q * 32 + lane;
        if (prow < M)
          for (int c = sub * 32; c < BN && n0 + c < N; c += 32 * EPQ) epi.prefetch(prow, n0 + c);
      }
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&tfull[acc], aph, err, ERR_TIMEOUT_EPI);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      // one thread per accumulator row; each 32-column chunk goes through the functor's
      // vectorised chunk32 (operands loaded before results are stored)
#pragma unroll 1
      for (int c = sub * 32; c < BN; c += 32 * EPQ) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * BN + c, v);
        if (row < M) {
          const float* vf = reinterpret_cast<const float*>(v);
          if (!(n0 + c + 32 <= N && epi.chunk32(row, n0 + c, vf))) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = n0 + c + 2 * j;
              if (col < N) epi(row, col, vf[2 * j], vf[2 * j + 1]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&tempty[acc]);
        else  // the even CTA's MMA issuer reuses the pair's accumulator
          mbar_arrive_cluster(map_rank(smem_u32(&tempty[acc]), 0));
      }
    }
  }

  if constexpr (KS > 1) {
    // every rank's half is parked: each rank pushes its parked block into the peer's ring with
    // bulk shared::cluster copies (completing on the peer's recv barrier), then adds the block
    // it received (local shared memory) to its own half and finishes those columns
    constexpr int H = BN / 2, XLD = H + 4;
    constexpr uint32_t PARK = BM * XLD * 4, PART = PARK / 4;
    static_assert(2 * PARK <= STAGES * S::STAGE && PART % 16 == 0, "park + receive in the ring");
    if (threadIdx.x == 64) mbar_expect_tx(&recv, PARK);  // armed before the peer can send
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (threadIdx.x == 64 && epi_ok) {
      const uint32_t src = smem_u32(sbase), dst = map_rank(smem_u32(sbase) + PARK, 1u - rank);
      const uint32_t mb = map_rank(smem_u32(&recv), 1u - rank);
#pragma unroll
      for (uint32_t part = 0; part < 4; ++part)
        asm volatile(
            "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], "
            "%2, [%3];" ::"r"(dst + part * PART),
            "r"(src + part * PART), "r"(PART), "r"(mb)
            : "memory");
    }
    bool got = false;
    if (warp >= 2 && epi_ok) {
      if (lane == 0) got = mbar_wait(&recv, 0, err, ERR_TIMEOUT_EPI);
      got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
    }
    if (got) {
      tc_fence_after();
      const int q = warp & 3, sub = (warp - 2) >> 2, t = t_first;
      const int m0 = (t % m_tiles) * BM, n0 = (t / m_tiles) * BN + (int)rank * H;
      const int row = m0 + q * 32 + lane;
      const float* rcv = reinterpret_cast<const float*>(sbase + PARK) + (q * 32 + lane) * XLD;
#pragma unroll 1
      for (int c = sub * 32; c < H; c += 32 * EPQ) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (int)rank * H + c, v);
        float4 pv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pv[u] = *reinterpret_cast<const float4*>(rcv + c + 4 * u);
        float vf[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          vf[4 * u] = __uint_as_float(v[4 * u]) + pv[u].x;
          vf[4 * u + 1] = __uint_as_float(v[4 * u + 1]) + pv[u].y;
          vf[4 * u + 2] = __uint_as_float(v[4 * u + 2]) + pv[u].z;
          vf[4 * u + 3] = __uint_as_float(v[4 * u + 3]) + pv[u].w;
        }
        if (row < M) {
          if (!(n0 + c + 32 <= N && epi.chunk32(row, n0 + c, vf))) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = n0 + c + 2 * j;
              if (col < N) epi(row, col, vf[2 * j], vf[2 * j + 1]);
            }
          }
        }
      }
    }
    // the peer has received this CTA's block (or given up) before either CTA exits
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  // CG = 2: the even CTA's MMAs (which read this CTA's shared memory and write its tensor
  // memory) have completed and neither CTA arrives on the other's barriers any more
  if constexpr (CG == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(S::TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(S::TMEM_COLS));
  }
}

}  // namespace tc
}  // namespace pi0
