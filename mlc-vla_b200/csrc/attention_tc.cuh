// Multi-query attention on 5th-generation tensor cores (fp16 models, one kv head), for both
// halves of the M1 path (gemma_dual.py:97-122 `_sdpa`; prefill attn_prefill_e0 :236-253,
// denoise attn_decode_e1 :255-275).
//
// A CTA owns 128 query rows (row j of batch b = token j / H, head j % H) and a range of 64-key
// tiles; the key tiles of a row tile may be split over a cluster of CTAs, whose partials are
// merged through distributed shared memory in rank order.
//   * S = Q·Kᵀ: tcgen05.mma kind::f16, M=128, N=64, K=hd, fp32 accumulator in TMEM. q (post-RoPE,
//     pre-scaled by hd^-0.5) and k (post-RoPE, stored at half scale so that no finite fp16-range
//     value can overflow) are rounded to fp16 by the q/k/v epilogue: the same 10-bit mantissa as
//     the tf32 inputs tensor cores take for fp32 operands, with round-to-nearest; the product is
//     accumulated in fp32 and doubled exactly.
//   * softmax: one thread per row reads its 64 logits from TMEM, adds the fp32 pad mask (0 / -1e9
//     for prefix keys, 0 for suffix keys), and keeps a running max m and sum l in fp32. The
//     probabilities exp(s − m), from CUDA's fast exponential intrinsic (__expf, relative error
//     about 2^-21, far below their rounding to fp16), are rounded to fp16 (the V dtype) and
//     written to shared memory as the A operand of the next MMA. O is rescaled only when the row max grows by more than
//     e^8 (then O is read from TMEM, scaled and written back); until then probabilities are taken
//     against the older, smaller max, at most e^8 ≈ 2981, well inside fp16.
//   * O += P·V: tcgen05.mma kind::f16, M=128, N=hd, K=64, V read MN-major straight from its
//     cache layout ([keys, hd], hd contiguous), fp32 accumulator in TMEM (hd columns).
//   * final O / l (or, with key splits, the (m, l, O) partials merged across the cluster).
// Warp roles: warp 0 TMA producer (Q once; K and V tiles through separate 2-slot rings, a K slot
// refilled once its S MMA is done and a V slot once its P·V is done; cached prefix tiles are
// requested before griddepcontrol.wait), warp 1 MMA issuer, warps 2-5 softmax/epilogue.
// All waits are bounded (gemm_tc.cuh: mbar_wait).
//
// LO = true is the reference's default attn_logits_dtype "float32" (fp32 q·k operands,
// gemma_dual.py:115): q and the half-scale k are split into fp16 pairs x = hi + lo with
// hi = fp16(x) and lo = fp16(x − hi) (both written by the q/k/v epilogue, or by
// keys_half_scale_kernel for the caller's cache), and S accumulates lo_q·hi_k + hi_q·lo_k +
// hi_q·hi_k in fp32: 22 bits of operand precision, the dropped lo·lo term below 2^-21 of the
// product, and a lo part that falls into the fp16 subnormal range is off by at most 2^-25 in
// absolute terms. Q_hi stays resident; for every key tile and 64-wide head-dim block, one ring
// stage carries that block of Q_lo (re-read from L2 per key tile), K_hi and K_lo, so shared memory
// stays at the size of the single-product layout.
#pragma once

#include "gemm_skinny.cuh"

namespace pi0 {
namespace atc {

using namespace tc;
using sk::workers_sync;

constexpr int KB = 64;             // keys per tile
constexpr int NT = 192;
constexpr float kRescale = 8.0f;   // rescale O when the row max grows by more than this

template <int HD, bool LO = false>
struct AtcSmem {
  static constexpr int NKB = HD / 64;               // 64-wide head-dim blocks
  static constexpr int Q_BYTES = 128 * HD * 2;      // NKB boxes [64 hd × 128 rows]
  static constexpr int QBLK = 128 * 64 * 2;         // LO: one Q_lo box
  static constexpr int KBLK = KB * 64 * 2;          // one [64 hd × 64 keys] box
  // K ring slot: a whole K tile (NKB boxes), or (LO) one head-dim block of Q_lo, K_hi and K_lo
  static constexpr int K_BYTES = LO ? QBLK + 2 * KBLK : KB * HD * 2;
  static constexpr int V_BYTES = KB * HD * 2;
  static constexpr int STAGE = K_BYTES + V_BYTES;
  static constexpr int P_OFF = Q_BYTES + 2 * STAGE;
  static constexpr int P_BYTES = 128 * KB * 2;      // [128 rows × 64 keys] fp16
  static constexpr int LOAD = P_OFF + P_BYTES;
  // key-split merge (after the key loop, aliasing the loop buffers): this CTA's partial as
  // normalised fp16 rows O/l [128][HD] and fp32 (m, l) [128][2], then the received row blocks of
  // every split: [splits][rpr][HD] fp16 and [splits][rpr][2] fp32, rpr·splits ≤ 160 rows (≤ 16
  // splits, rpr = ⌈128 / splits⌉ rounded up to even)
  static constexpr int P16 = 128 * HD * 2;
  static constexpr int PML = P16;                   // + 128·8
  static constexpr int R16 = PML + 1024;            // + 160·HD·2
  static constexpr int RML = R16 + 160 * HD * 2;    // + 160·8
  static constexpr int MERGE = RML + 160 * 8;
  static constexpr int BYTES = (LOAD > MERGE ? LOAD : MERGE) + 1024;
};

struct AtcArgs {
  int rows;           // query rows per batch element: Tq·H
  int LA, LB;         // keys of segment A (prefix cache) and B (suffix; 0 in prefill)
  int ntA, nt;        // key tiles of A, all key tiles
  int tps;            // key tiles per split
  const float* maskA; // [B, LA] additive fp32, or null
  void* out;          // [B·rows, HD] fp16
  int* err;
  int a_ready;        // segment A was written before the previous kernel
  int ya0;            // row of segment A's first key in its tensor map (layer offset)
  // > 0: the suffix keys are folded into the last prefix tile, whose first `tail` rows are the
  // prefix's last keys (LA % 64, a multiple of 8) and whose next LB rows are the suffix keys
  // (tail + LB ≤ 64); the B tensor maps then have boxes of 64 − tail rows and the tail maps of
  // `tail` rows. 0: segment B has tiles of its own.
  int tail;
  uint32_t v_lbo, v_sbo;  // MN-major V descriptor: byte stride between 64-dim blocks / 8-key groups
};

// Shared-memory matrix descriptor, MN-major operand in the 128-byte swizzle layout that TMA
// writes for a [64 contiguous elements × rows] box.
__device__ __forceinline__ uint64_t desc_sw128_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Barriers and small buffers of one attention CTA (static shared memory of the calling kernel).
struct AtcShared {
  uint64_t q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full, s_free, p_full, pv_done,
      drain, recv;
  float mask[KB];
  float w[128][16];
  float inv[128];
};

// One thread: initialise the barriers (before the CTA-wide barrier that precedes attn_tile).
__device__ __forceinline__ void atc_init(AtcShared& sm) {
  mbar_init(&sm.q_full, 1);
  for (int s = 0; s < 2; ++s) {
    mbar_init(&sm.k_full[s], 1);
    mbar_init(&sm.k_empty[s], 1);
    mbar_init(&sm.v_full[s], 1);
    mbar_init(&sm.v_empty[s], 1);
  }
  mbar_init(&sm.s_full, 1);
  mbar_init(&sm.s_free, 4);
  mbar_init(&sm.p_full, 4);
  mbar_init(&sm.pv_done, 1);
  mbar_init(&sm.drain, 1);
  mbar_init(&sm.recv, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One thread: invalidate the barriers of a finished attn_tile (no copy or MMA is pending on them)
// before atc_init makes them fresh for the next one.
__device__ __forceinline__ void atc_inval(AtcShared& sm) {
  uint64_t* b[15] = {&sm.q_full, &sm.k_full[0], &sm.k_full[1], &sm.k_empty[0], &sm.k_empty[1],
                     &sm.v_full[0], &sm.v_full[1], &sm.v_empty[0], &sm.v_empty[1], &sm.s_full,
                     &sm.s_free, &sm.p_full, &sm.pv_done, &sm.drain, &sm.recv};
#pragma unroll
  for (int i = 0; i < 15; ++i)
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(b[i])) : "memory");
}

// The work of one CTA: query rows [row0, row0 + 128) of batch element b against key tiles
// [tbeg, tbeg + n), split `rank` of `nsplit` (the splits of a row tile are consecutive cluster
// ranks and are merged here when nsplit > 1; every rank of the cluster calls this). TMEM: S in
// columns [0, 64), O in [256, 256 + HD) of `tmem` (512 columns). pdl: called from a kernel
// launched with programmatic dependent launch (cached prefix tiles are requested before its
// griddepcontrol.wait). tmQL / tmKAL / tmKBL: the lo parts of q and k (LO only).
template <int HD, bool LO>
__device__ __forceinline__ void attn_tile(const CUtensorMap& tmQ, const CUtensorMap& tmKA,
                                          const CUtensorMap& tmVA, const CUtensorMap& tmKB,
                                          const CUtensorMap& tmVB, const CUtensorMap& tmQL,
                                          const CUtensorMap& tmKAL, const CUtensorMap& tmKBL,
                                          const CUtensorMap& tmKAT, const CUtensorMap& tmVAT,
                                          const CUtensorMap& tmKALT,
                                          const AtcArgs& a, int b, int row0, int tbeg, int n,
                                          int nsplit, uint32_t rank, uint8_t* base,
                                          AtcShared& sm, uint32_t tmem, bool pdl) {
  using S = AtcSmem<HD, LO>;
  constexpr int NKB = S::NKB;
  uint64_t& q_full = sm.q_full;
  uint64_t* k_full = sm.k_full;
  uint64_t* k_empty = sm.k_empty;
  uint64_t* v_full = sm.v_full;
  uint64_t* v_empty = sm.v_empty;
  uint64_t& s_full = sm.s_full;
  uint64_t& s_free = sm.s_free;
  uint64_t& p_full = sm.p_full;
  uint64_t& pv_done = sm.pv_done;
  uint64_t& drain = sm.drain;
  float* s_mask = sm.mask;
  float(*s_w)[16] = sm.w;
  float* s_inv = sm.inv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* sQ = base;
  uint8_t* sP = base + S::P_OFF;
  auto sK = [&](int s) { return base + S::Q_BYTES + s * S::STAGE; };
  auto sV = [&](int s) { return base + S::Q_BYTES + s * S::STAGE + S::K_BYTES; };

  // one K (is_v = false) or V tile of key tile i into ring slot i & 1
  // the folded tile (a.tail > 0): prefix rows [0, tail) and suffix rows [tail, 64) of one box
  // position come from two loads; tail is a multiple of 8, so the second box starts on a
  // 1024-byte swizzle atom and keeps the 128-byte swizzle pattern of the tile
  auto folded = [&](int tile) { return a.tail > 0 && tile == a.ntA - 1; };
  auto load_rows = [&](uint8_t* dst, const CUtensorMap* mA, const CUtensorMap* mAt,
                       const CUtensorMap* mB, uint64_t* bar, int col, int tile) {
    if (folded(tile)) {
      tma_load_2d(dst, mAt, bar, col, a.ya0 + b * a.LA + tile * KB);
      tma_load_2d(dst + a.tail * 128, mB, bar, col, b * a.LB);
    } else if (tile < a.ntA) {
      tma_load_2d(dst, mA, bar, col, a.ya0 + b * a.LA + tile * KB);
    } else {
      tma_load_2d(dst, mB, bar, col, b * a.LB + (tile - a.ntA) * KB);
    }
  };
  auto issue = [&](int i, bool is_v) {
    const int s = i & 1, tile = tbeg + i;
    uint64_t* bar = is_v ? &v_full[s] : &k_full[s];
    uint8_t* dst = is_v ? sV(s) : sK(s);
    mbar_expect_tx(bar, is_v ? S::V_BYTES : S::K_BYTES);
#pragma unroll
    for (int kb = 0; kb < NKB; ++kb)
      load_rows(dst + kb * (KB * 128), is_v ? &tmVA : &tmKA, is_v ? &tmVAT : &tmKAT,
                is_v ? &tmVB : &tmKB, bar, kb * 64, tile);
  };

  // LO: ring stage j = (key tile j / NKB, head-dim block j % NKB) into K slot j & 1: that block
  // of Q_lo, K_hi and K_lo. issue_lo_k requests the K parts (arming the stage for all three),
  // issue_lo_q the Q_lo part.
  auto issue_lo_k = [&](int j) {
    const int s = j & 1, tile = tbeg + j / NKB, kb = j % NKB;
    uint8_t* dst = sK(s);
    mbar_expect_tx(&k_full[s], S::K_BYTES);
    load_rows(dst + S::QBLK, &tmKA, &tmKAT, &tmKB, &k_full[s], kb * 64, tile);
    load_rows(dst + S::QBLK + S::KBLK, &tmKAL, &tmKALT, &tmKBL, &k_full[s], kb * 64, tile);
  };
  auto issue_lo_q = [&](int j) {
    const int s = j & 1, kb = j % NKB;
    tma_load_2d(sK(s), &tmQL, &k_full[s], kb * 64, b * a.rows + row0);
  };

  // tiles of the cached prefix do not depend on the previous kernel: request them before its
  // completion (LO: the K parts of the first two ring stages and V of the first two tiles; the
  // stages' Q_lo, which does depend on it, follows the wait)
  int issued = 0;     // V (and, !LO, K) of tiles [0, issued) requested
  int pre_k = 0;      // LO: K parts of ring stages [0, pre_k) requested
  if (pdl && tid == 0 && a.a_ready) {
    const int nready = a.tail > 0 ? a.ntA - 1 : a.ntA;  // the folded tile holds suffix keys
    if constexpr (LO) {
      for (; pre_k < min(n * NKB, 2) && tbeg + pre_k / NKB < nready; ++pre_k) issue_lo_k(pre_k);
      for (; issued < min(n, 2) && tbeg + issued < nready; ++issued) issue(issued, true);
    } else {
      for (; issued < min(n, 2) && tbeg + issued < nready; ++issued) {
        issue(issued, false);
        issue(issued, true);
      }
    }
  }
  if (pdl) {
    pdl_trigger();
    pdl_wait();
  }

  if (warp == 0) {
    if (lane == 0) {  // producer
      mbar_expect_tx(&q_full, S::Q_BYTES);
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb)
        tma_load_2d(sQ + kb * (128 * 128), &tmQ, &q_full, kb * 64, b * a.rows + row0);
      if constexpr (LO) {
        int jk = 0;  // ring stages [0, jk) requested; V of tiles [0, issued)
        for (int j = 0; j < pre_k; ++j) issue_lo_q(j);  // complete the early stages
        jk = pre_k;
        for (int i = 0; i < n; ++i) {
          bool ok = true;
          for (int kb = 0; kb < NKB && ok; ++kb) {
            const int j = i * NKB + kb;
            if (j < pre_k) continue;
            if (j >= 2 && !mbar_wait(&k_empty[j & 1], ((j >> 1) - 1) & 1, a.err,
                                     ERR_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            issue_lo_k(j);
            issue_lo_q(j);
            jk = j + 1;
          }
          if (!ok) break;
          if (i < issued) continue;  // V requested before the dependency wait
          if (i >= 2 && !mbar_wait(&v_empty[i & 1], ((i >> 1) - 1) & 1, a.err, ERR_TIMEOUT_PRODUCER))
            break;
          issue(i, true);
          issued = i + 1;
        }
        mbar_wait(&q_full, 0, a.err, ERR_TIMEOUT_PRODUCER, false);
        for (int j = max(0, jk - 2); j < jk; ++j)
          mbar_wait(&k_full[j & 1], (j >> 1) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
        for (int i = max(0, issued - 2); i < issued; ++i)
          mbar_wait(&v_full[i & 1], (i >> 1) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
      } else {
      int issued_k = issued;  // K of tiles [0, issued_k) requested; V of [0, issued)
      for (int i = issued; i < n; ++i) {
        const uint32_t ph = ((i >> 1) - 1) & 1;
        if (i >= 2 && !mbar_wait(&k_empty[i & 1], ph, a.err, ERR_TIMEOUT_PRODUCER)) break;
        issue(i, false);
        issued_k = i + 1;
        if (i >= 2 && !mbar_wait(&v_empty[i & 1], ph, a.err, ERR_TIMEOUT_PRODUCER)) break;
        issue(i, true);
        issued = i + 1;
      }
      // no copy into this CTA's shared memory may still be in flight when it exits
      mbar_wait(&q_full, 0, a.err, ERR_TIMEOUT_PRODUCER, false);
      for (int i = max(0, issued_k - 2); i < issued_k; ++i)
        mbar_wait(&k_full[i & 1], (i >> 1) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
      for (int i = max(0, issued - 2); i < issued; ++i)
        mbar_wait(&v_full[i & 1], (i >> 1) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {  // MMA issuer
      constexpr uint32_t id_s = idesc_f16<__half>(128, KB);
      constexpr uint32_t id_o = idesc_f16<__half>(128, HD) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(&q_full, 0, a.err, ERR_TIMEOUT_MMA);
      auto qk = [&](int i) -> bool {
        if constexpr (LO) {
          for (int kb = 0; kb < NKB; ++kb) {
            const int j = i * NKB + kb, s = j & 1;
            if (!mbar_wait(&k_full[s], (j >> 1) & 1, a.err, ERR_TIMEOUT_MMA)) return false;
            tc_fence_after();
            const uint64_t dqh = desc_sw128(smem_u32(sQ + kb * (128 * 128)));
            const uint64_t dql = desc_sw128(smem_u32(sK(s)));
            const uint64_t dkh = desc_sw128(smem_u32(sK(s) + S::QBLK));
            const uint64_t dkl = desc_sw128(smem_u32(sK(s) + S::QBLK + S::KBLK));
#pragma unroll
            for (int k = 0; k < 4; ++k)  // the small cross terms first
              umma_f16(tmem, dql + 2 * k, dkh + 2 * k, id_s, (kb | k) != 0);
#pragma unroll
            for (int k = 0; k < 4; ++k) umma_f16(tmem, dqh + 2 * k, dkl + 2 * k, id_s, 1u);
#pragma unroll
            for (int k = 0; k < 4; ++k) umma_f16(tmem, dqh + 2 * k, dkh + 2 * k, id_s, 1u);
            umma_commit(&k_empty[s]);
          }
          umma_commit(&s_full);
          return true;
        } else {
        const int s = i & 1;
        if (!mbar_wait(&k_full[s], (i >> 1) & 1, a.err, ERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb) {
          const uint64_t da = desc_sw128(smem_u32(sQ + kb * (128 * 128)));
          const uint64_t db = desc_sw128(smem_u32(sK(s) + kb * (KB * 128)));
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16(tmem, da + 2 * k, db + 2 * k, id_s, (kb | k) != 0);
        }
        umma_commit(&s_full);
        umma_commit(&k_empty[s]);
        return true;
        }
      };
      auto pv = [&](int i) -> bool {
        const int s = i & 1;
        if (!mbar_wait(&p_full, i & 1, a.err, ERR_TIMEOUT_MMA) ||
            !mbar_wait(&v_full[s], (i >> 1) & 1, a.err, ERR_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint64_t da = desc_sw128(smem_u32(sP));
        const uint64_t db = desc_sw128_mn(smem_u32(sV(s)), a.v_lbo, a.v_sbo);
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 16 keys (2048 bytes of V rows) per step
          umma_f16(tmem + 256, da + 2 * k, db + (uint64_t)(128 * k), id_o, (i | k) != 0);
        umma_commit(&v_empty[s]);
        umma_commit(&pv_done);
        return true;
      };
      ok = ok && qk(0);
      for (int i = 0; i < n && ok; ++i) {
        if (i + 1 < n) ok = mbar_wait(&s_free, i & 1, a.err, ERR_TIMEOUT_MMA) && qk(i + 1);
        ok = ok && pv(i);
      }
      // every issued MMA completes before TMEM is released
      umma_commit(&drain);
      mbar_wait(&drain, 0, a.err, ERR_TIMEOUT_MMA, false);
    }
  } else {  // warps 2-5: softmax, one thread per query row
    const int q4 = warp & 3, r = q4 * 32 + lane, wt = tid - 64;
    const uint32_t tS = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t tO = tS + 256;
    float m_ref = -1e30f, l = 0.f;
    auto mask_of = [&](int tile) -> float {
      if (folded(tile)) {
        if (wt < a.tail) {
          const int key = tile * KB + wt;
          return a.maskA ? a.maskA[(size_t)b * a.LA + key] : 0.f;
        }
        return wt - a.tail < a.LB ? 0.f : -1e30f;
      }
      if (tile < a.ntA) {
        const int key = tile * KB + wt;
        return key < a.LA ? (a.maskA ? a.maskA[(size_t)b * a.LA + key] : 0.f) : -1e30f;
      }
      const int key = (tile - a.ntA) * KB + wt;
      return key < a.LB ? 0.f : -1e30f;
    };
    float mnext = (wt < KB && n > 0) ? mask_of(tbeg) : 0.f;
    // after a failed (timed-out) wait the loop keeps running without work, so the four warps
    // always meet at the same named barriers
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      workers_sync();  // everyone is done with the previous tile's mask
      if (wt < KB) s_mask[wt] = mnext;
      workers_sync();
      if (wt < KB && i + 1 < n) mnext = mask_of(tbeg + i + 1);
      if (ok) ok = mbar_wait(&s_full, i & 1, a.err, ERR_TIMEOUT_EPI);
      ok = !__any_sync(0xffffffffu, !ok);
      uint32_t s0[32], s1[32];
      if (ok) {
        tc_fence_after();
        tmem_ld32(tS, s0);
        tmem_ld32(tS + 32, s1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free);
      }
      if (!ok) continue;
      float sv[KB];
      float mt = -1e30f;
#pragma unroll
      for (int j = 0; j < KB; ++j) {
        const float raw = __uint_as_float(j < 32 ? s0[j] : s1[j - 32]);
        sv[j] = __fadd_rn(2.f * raw, s_mask[j]);
        mt = fmaxf(mt, sv[j]);
      }
      if (i == 0) {
        m_ref = mt;
      } else {
        // O and the P buffer are free once the previous P·V has finished
        ok = mbar_wait(&pv_done, (i - 1) & 1, a.err, ERR_TIMEOUT_EPI);
        ok = !__any_sync(0xffffffffu, !ok);
        if (!ok) continue;
        tc_fence_after();
        const bool need = mt > m_ref + kRescale;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? expf(m_ref - mt) : 1.f;
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t ov[32];
            tmem_ld32(tO + c, ov);
#pragma unroll
            for (int j = 0; j < 32; ++j) ov[j] = __float_as_uint(__uint_as_float(ov[j]) * alpha);
            tmem_st32(tO + c, ov);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          if (need) {
            l *= alpha;
            m_ref = mt;
          }
        }
      }
      // probabilities against m_ref, rounded to fp16, into the swizzled A operand
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < KB / 8; ++c) {
        uint32_t w4[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float p0 = __expf(sv[8 * c + 2 * h] - m_ref);
          const float p1 = __expf(sv[8 * c + 2 * h + 1] - m_ref);
          rs += p0 + p1;
          w4[h] = Tr<__half>::pack(p0, p1);
        }
        *reinterpret_cast<uint4*>(sP + r * 128 + ((c ^ (r & 7)) << 4)) =
            make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      l += rs;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
    }
    if (ok && n > 0) {
      ok = mbar_wait(&pv_done, (n - 1) & 1, a.err, ERR_TIMEOUT_EPI, false);
      tc_fence_after();
    }
    const bool have = __all_sync(0xffffffffu, ok) && n > 0;
    if (nsplit == 1) {
      const int j = row0 + r;
      __half* out = reinterpret_cast<__half*>(a.out) + ((size_t)b * a.rows + j) * HD;
      const float inv = have && l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t ov[32];
        if (have) tmem_ld32(tO + c, ov);
        uint4 pk[4];
        uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
        for (int h = 0; h < 16; ++h)
          pw[h] = have ? Tr<__half>::pack(__uint_as_float(ov[2 * h]) * inv,
                                          __uint_as_float(ov[2 * h + 1]) * inv)
                       : 0u;
        if (j < a.rows)
#pragma unroll
          for (int u = 0; u < 4; ++u) reinterpret_cast<uint4*>(out + c)[u] = pk[u];
      }
    } else {
      // partial of this split for the merge: the row normalised by its own sum, O / l, in fp16
      // (bounded by max |v|, so no overflow), and (m, l) in fp32
      __half* sO = reinterpret_cast<__half*>(base);
      float* sML = reinterpret_cast<float*>(base + S::PML);
      const float inv = have && l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t ov[32];
        if (have) tmem_ld32(tO + c, ov);
        uint4 pk[4];
        uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
        for (int h = 0; h < 16; ++h)
          pw[h] = have ? Tr<__half>::pack(__uint_as_float(ov[2 * h]) * inv,
                                          __uint_as_float(ov[2 * h + 1]) * inv)
                       : 0u;
#pragma unroll
        for (int u = 0; u < 4; ++u) reinterpret_cast<uint4*>(sO + r * HD + c)[u] = pk[u];
      }
      sML[2 * r] = have && l > 0.f ? m_ref : -1e30f;
      sML[2 * r + 1] = have ? l : 0.f;
    }
  }

  if (nsplit > 1) {
    // ---- merge the key splits of this row tile: rank r finishes rows [r·rpr, (r+1)·rpr) ----
    // Every split pushes its normalised partial rows of rank r's block (one bulk copy for O, one
    // for (m, l)) into rank r's receive buffer, completing on rank r's `recv` barrier; rank r then
    // merges from its own shared memory: out = Σ_s c_s·o_s with c_s = e^(m_s − M)·l_s / Σ e^(m − M)·l,
    // summed in split order.
    const int rpr = ((128 + nsplit - 1) / nsplit + 1) & ~1;  // even: 16-byte (m, l) blocks
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // every split's partial is written and its loop buffers are free
    const __half* sO = reinterpret_cast<const __half*>(base);
    const float* sML = reinterpret_cast<const float*>(base + S::PML);
    __half* rO = reinterpret_cast<__half*>(base + S::R16);
    float* rML = reinterpret_cast<float*>(base + S::RML);
    if ((int)rank < nsplit && tid < nsplit) {  // split `rank`, thread t: rank t's row block
      const int r0 = tid * rpr, nr = max(0, min(128, r0 + rpr) - r0);
      if (nr > 0) {
        const uint32_t mb = map_rank(smem_u32(&sm.recv), (uint32_t)tid);
        const uint32_t dO = map_rank(smem_u32(rO + (size_t)rank * rpr * HD), (uint32_t)tid);
        const uint32_t dM = map_rank(smem_u32(rML + (size_t)rank * rpr * 2), (uint32_t)tid);
        asm volatile(
            "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dO),
            "r"(smem_u32(sO + (size_t)r0 * HD)), "r"((uint32_t)(nr * HD * 2)), "r"(mb)
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dM),
            "r"(smem_u32(sML + (size_t)r0 * 2)), "r"((uint32_t)(nr * 8)), "r"(mb)
            : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    const int rbeg = (int)rank * rpr, rend = min(128, rbeg + rpr), nme = max(0, rend - rbeg);
    if ((int)rank < nsplit && nme > 0) {
      if (tid == 0) {
        mbar_expect_tx(&sm.recv, (uint32_t)(nsplit * nme * (HD * 2 + 8)));
        mbar_wait(&sm.recv, 0, a.err, ERR_TIMEOUT_EPI, false);
      }
      __syncthreads();
      for (int rr = tid; rr < nme; rr += NT) {  // merge coefficients of row rbeg + rr
        float mm[16], ll[16];
        float M = -1e30f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          mm[c] = c < nsplit ? rML[((size_t)c * rpr + rr) * 2] : -1e30f;
          ll[c] = c < nsplit ? rML[((size_t)c * rpr + rr) * 2 + 1] : 0.f;
          M = fmaxf(M, mm[c]);
        }
        float L = 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float w = c < nsplit ? expf(mm[c] - M) * ll[c] : 0.f;
          s_w[rr][c] = w;
          L += w;
        }
        s_inv[rr] = L > 0.f ? 1.f / L : 0.f;
      }
      __syncthreads();
      const int items = nme * (HD / 8);
      for (int it = tid; it < items; it += NT) {  // (row, 8 dims)
        const int rr = it / (HD / 8), d = (it % (HD / 8)) * 8;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int c = 0; c < nsplit; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(rO + ((size_t)c * rpr + rr) * HD + d);
          const __half* e = reinterpret_cast<const __half*>(&v);
          const float wc = s_w[rr][c] * s_inv[rr];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += wc * __half2float(e[j]);
        }
        const int row = row0 + rbeg + rr;
        if (row < a.rows) {
          uint4 o;
          uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int j = 0; j < 4; ++j) ow[j] = Tr<__half>::pack(acc[2 * j], acc[2 * j + 1]);
          *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.out) + ((size_t)b * a.rows + row) * HD + d) = o;
        }
      }
    }
    if ((int)rank < nsplit && tid < nsplit) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncthreads();
  }
}

// tmQL / tmKAL / tmKBL: the lo parts of q and k (LO only; the hi maps otherwise, unused).
template <int HD, bool LO>
__global__ void __launch_bounds__(NT, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKA,
                   const __grid_constant__ CUtensorMap tmVA, const __grid_constant__ CUtensorMap tmKB,
                   const __grid_constant__ CUtensorMap tmVB, const __grid_constant__ CUtensorMap tmQL,
                   const __grid_constant__ CUtensorMap tmKAL,
                   const __grid_constant__ CUtensorMap tmKBL,
                   const __grid_constant__ CUtensorMap tmKAT,
                   const __grid_constant__ CUtensorMap tmVAT,
                   const __grid_constant__ CUtensorMap tmKALT, AtcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  __shared__ AtcShared sm;
  __shared__ uint32_t s_tmem;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    atc_init(sm);
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKA);
    tma_prefetch_desc(&tmVA);
    if (LO) {
      tma_prefetch_desc(&tmQL);
      tma_prefetch_desc(&tmKAL);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"(512u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int tbeg = blockIdx.y * a.tps;
  const int n = max(0, min(a.nt, tbeg + a.tps) - tbeg);
  attn_tile<HD, LO>(tmQ, tmKA, tmVA, tmKB, tmVB, tmQL, tmKAL, tmKBL, tmKAT, tmVAT, tmKALT, a,
                    blockIdx.z,
                    blockIdx.x * 128, tbeg, n, gridDim.y, cluster_rank(), base, sm, tmem, true);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u));
  }
}

}  // namespace atc
}  // namespace pi0
