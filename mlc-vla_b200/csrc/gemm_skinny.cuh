// Weight-streaming GEMM for the denoise step (M = B·S activation rows ≤ 128, e.g. 50):
//   Y[M, N] = X[M, K] · W[N, K]^T  with the fused epilogue functors of gemm_mma.cuh.
//
// The M=50 projections are HBM-bound (every weight byte is used M times), so the kernel is
// built around streaming W once at full bandwidth while staying small enough that the CTAs of
// two consecutive kernels fit on one SM together:
//   * the weights are pre-packed (at pi0_set_params) into 16 KB blocks, one per (128-row tile,
//     64-wide k-block), each already the 128-byte-swizzled K-major shared-memory image, and a
//     tile's k-blocks are contiguous: a CTA streams its weight slice with one-dimensional
//     cp.async.bulk copies — sequential DRAM, no tensor map;
//   * swap-AB on tcgen05: the weight tile is the MMA's A operand (M = 128 weight rows) and the
//     activations are B (N = NA = 64 or 128 rows, zero past M), accumulator [128 × NA] fp32 in
//     TMEM;
//   * a RING-deep shared-memory pipeline (weight block + activation block per stage) with
//     warp-specialised roles: warp 0 streams blocks (weights by bulk copy, activations by TMA),
//     warp 1 issues the MMAs and frees stages with tcgen05.commit, warps 2-5 normalise the
//     activation blocks in place (NORM) and run the epilogue. Shared memory does not grow with
//     K: ~100 KB per CTA, two CTAs per SM;
//   * the epilogue's global operands are prefetched into L1 right after the dependency wait;
//   * split-K over a thread-block cluster of C ≤ 8 CTAs: rank r owns k-blocks
//     [r·kbpc, (r+1)·kbpc) of one tile; partial accumulators are summed through distributed
//     shared memory in rank order (deterministic), each rank finishing 128/C weight rows;
//   * programmatic dependent launch: the first RING weight blocks are requested before
//     griddepcontrol.wait, so a kernel's weight stream overlaps the kernel producing its
//     activations;
//   * optional fusions: NORM builds B = adaRMSNorm(x) in shared memory from the residual stream
//     and per-row Σx² partials; SSQ makes the residual epilogue emit those partials (one per
//     (tile, rank), deterministic) for the next norm-fused GEMM.
// Every mbarrier wait is bounded (gemm_tc.cuh: mbar_wait); on timeout the kernel sets *err,
// waits for the copies it issued, and frees TMEM before returning.
#pragma once

#include "gemm_tc.cuh"

namespace pi0 {
namespace sk {

using namespace tc;

// one-dimensional bulk copy global -> this CTA's shared memory, completing on an mbarrier
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// barrier among the 128 threads of warps 2-5 (activation producers / epilogue)
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

constexpr int RING = 4;               // pipeline stages
constexpr int W_BLOCK = BM * BK * 2;  // 16 KB: one packed (tile, k-block) weight block
constexpr int PLD = BM + 4;           // partial row stride (floats): activation-row major
constexpr int MAX_C = 8;              // cluster size limit (portable clusters)
constexpr int SSQ_MAX_PARTS = 256;    // row Σx² partials per row (multiple of 16)
constexpr int NT = 192;               // threads per CTA

template <int NA>
struct SkSmem {
  static constexpr int X_BLOCK = NA * BK * 2;
  static constexpr int STAGE = W_BLOCK + X_BLOCK;  // multiple of 1024 (swizzle atoms)
  static constexpr int LOAD = RING * STAGE;
  static constexpr int PART = NA * PLD * 4;        // after the MMAs: partial accumulator
  static constexpr int ITEM = NA * 32 * 4;         // after the MMAs: SSQ per-item squares
  static constexpr int BYTES = (LOAD > PART + ITEM ? LOAD : PART + ITEM) + 1024;
};

struct SkArgs {
  int M, N, K;
  int kbpc;              // k-blocks per CTA
  int C;                 // cluster size = number of K splits (power of two ≤ MAX_C)
  int* err;
  const void* wpack;     // pre-packed weights, or null to load W through the tensor map
  // NORM: B = x / sqrt(Σx²/K + eps) · (1 + scale) + shift, (scale, shift) = mod[0:K], mod[K:2K]
  const void* x;         // [M, K] residual stream, model dtype
  const void* mod;       // modulation row of this step
  float eps;
  const float* ssq_in;   // [M][ssq_parts] partial Σx² of the rows of x
  // SSQ: ssq_out[m][tile·C + rank] = Σ over the rank's output columns of x_new² (the values
  // the epilogue returns); CTA (0, 0) zeroes the slots [tiles·C, ssq_parts)
  float* ssq_out;
  int ssq_parts;
};

// Packs a row-major [N, K] 16-bit matrix into (tile, k-block) blocks of 128 × 64 elements in the
// 128-byte-swizzle K-major layout: chunk c (8 elements) of block row r sits at r·128 +
// ((c ^ (r & 7))·16). Rows ≥ N and columns ≥ K are zero. One thread per 16-byte chunk.
__global__ void pack_sw128_kernel(uint16_t* __restrict__ dst, const uint16_t* __restrict__ src,
                                  int N, int K, int nkb, size_t total_chunks) {
  size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= total_chunks) return;
  const int cs = (int)(id & 7);
  size_t rest = id >> 3;
  const int r = (int)(rest % BM);
  rest /= BM;
  const int kb = (int)(rest % nkb);
  const size_t t = rest / nkb;
  const size_t row = t * BM + r;
  const int col = kb * BK + ((cs ^ (r & 7)) << 3);
  uint4 v = make_uint4(0, 0, 0, 0);
  if (row < (size_t)N && col < K) v = *reinterpret_cast<const uint4*>(src + row * K + col);
  *reinterpret_cast<uint4*>(dst + ((t * nkb + kb) * BM + r) * BK + cs * 8) = v;
}

// Group-quantised weight blocks, in the same (tile, k-block) order as the 16-bit packed blocks,
// qw_block(QB) bytes per 128×64 block. Chunk c of a row = columns 8c..8c+7 of the block; pair h
// of a chunk = columns 8c+2h, 8c+2h+1. The codes are re-ordered at bind time so that one shift
// and one mask put a pair's two codes at bits 0 and 16 of a register:
//   q4 (q4f16_1 / q4bf16_1: G = 32, w = (code − 7)·s): [128 rows × 8 words], word c of a row
//      holds chunk c with the code of column 2h at bits 4h and of column 2h+1 at bits 16 + 4h;
//      then [128 rows × 2 scales] (columns 0-31, 32-63). 4608 bytes.
//   q3 (q3f16_1: G = 40, w = (code − 3)·s): low two bits of every code in [128 rows × 4 words]
//      (chunk c, pair h at bits 8·(c&1) + 2h and +16 of word c>>1), the third bit in
//      [128 rows × 2 words] (pair p = 4c + h at bit p&15 and +16 of word p>>4), then
//      [128 rows × 4 scales]: the three groups a 64-wide block can touch (groups start at
//      multiples of 40, always on a chunk boundary) and a zero pad. 4096 bytes.
// The kernel loads a block into the tail of the stage's weight slot and dequantises it in place
// into the 16 KB swizzled image the MMA reads.
__host__ __device__ constexpr int qw_block(int qb) { return qb == 4 ? BM * 36 : BM * 32; }
__host__ __device__ constexpr int qw_off(int qb) { return W_BLOCK - qw_block(qb); }

// Packs rows [row0, row0 + n) of a fused matrix from one quantised Linear (reference layout:
// q_weight [.., ceil(K/G)·G/epw] uint32 with code k at word k/epw, bits bits·(k%epw); q_scale
// [.., ceil(K/G)] 16-bit): destination row row0 + r takes source row idx ? idx[r] : r.
// K % 64 == 0. One thread per (row, k-block), scalar loads (the caller's buffers need only their
// natural alignment); rows past the matrix stay as the caller zeroed them.
template <int QB>
__global__ void pack_q_kernel(uint8_t* __restrict__ dst, const uint32_t* __restrict__ qw,
                              const uint16_t* __restrict__ qs, const int* __restrict__ idx, int n,
                              int K, int row0, int nkb) {
  const int id = blockIdx.x * blockDim.x + threadIdx.x;
  const int rl = id / nkb, kb = id - rl * nkb;
  if (rl >= n) return;
  const int src = idx ? idx[rl] : rl;
  const int r = row0 + rl, rr = r % BM;
  uint8_t* blk = dst + ((size_t)(r / BM) * nkb + kb) * qw_block(QB);
  if constexpr (QB == 4) {
    const uint32_t* w = qw + (size_t)src * (K / 8) + kb * 8;
    uint32_t* oc = reinterpret_cast<uint32_t*>(blk + rr * 32);
    for (int c = 0; c < 8; ++c) {
      const uint32_t v = w[c];  // column 8c + j at bits 4j
      uint32_t o = 0;
      for (int h = 0; h < 4; ++h)
        o |= ((v >> (8 * h)) & 15u) << (4 * h) | ((v >> (8 * h + 4)) & 15u) << (16 + 4 * h);
      oc[c] = o;
    }
    const uint16_t* sc = qs + (size_t)src * (K / 32) + kb * 2;
    uint16_t* os = reinterpret_cast<uint16_t*>(blk + BM * 32 + rr * 4);
    os[0] = sc[0];
    os[1] = sc[1];
  } else {
    const int ng = (K + 39) / 40;
    const uint32_t* w = qw + (size_t)src * ng * 4;
    uint32_t lo[4] = {0, 0, 0, 0}, hi[2] = {0, 0};
    for (int c = 0; c < 8; ++c)
      for (int h = 0; h < 4; ++h)
        for (int e = 0; e < 2; ++e) {
          const int k = kb * 64 + 8 * c + 2 * h + e;
          const uint32_t code = (w[k / 10] >> (3 * (k % 10))) & 7u;
          lo[c >> 1] |= (code & 3u) << (8 * (c & 1) + 2 * h + 16 * e);
          const int p = 4 * c + h;
          hi[p >> 4] |= (code >> 2) << ((p & 15) + 16 * e);
        }
    uint32_t* ol = reinterpret_cast<uint32_t*>(blk + rr * 16);
    uint32_t* oh = reinterpret_cast<uint32_t*>(blk + BM * 16 + rr * 8);
    for (int j = 0; j < 4; ++j) ol[j] = lo[j];
    oh[0] = hi[0];
    oh[1] = hi[1];
    uint16_t* os = reinterpret_cast<uint16_t*>(blk + BM * 24 + rr * 8);
    const int g0 = kb * 64 / 40;
    for (int t = 0; t < 3; ++t) os[t] = g0 + t < ng ? qs[(size_t)src * ng + g0 + t] : (uint16_t)0;
    os[3] = 0;
  }
}

// Two codes (bits 0-3 and 16-19 of x, higher bits clear) -> the model-dtype pair
// RN((code − off)·g) = dequantize_kernel's arithmetic. fp16: x | 0x6400 is the half 1024 + code,
// so the subtraction is exact and the one rounding is the half multiply's (the exact product
// rounded to nearest, as the fp32 product rounded to half is). bf16: the same in fp32 through
// 2^23 + code, then one rounding to bf16.
template <typename T, int OFF>
__device__ __forceinline__ uint32_t dequant_pair(uint32_t x, uint32_t g2, float g) {
  if constexpr (Tr<T>::kBf16) {
    const float a = __uint_as_float(0x4B000000u | (x & 0xFFFFu)) - (8388608.f + OFF);
    const float b = __uint_as_float(0x4B000000u | (x >> 16)) - (8388608.f + OFF);
    return Tr<T>::pack(a * g, b * g);
  } else {
    const uint32_t v = x | 0x64006400u;
    const __half2 c = __hsub2(*reinterpret_cast<const __half2*>(&v),
                              __halves2half2(__ushort_as_half((unsigned short)(0x6400 + OFF)),
                                             __ushort_as_half((unsigned short)(0x6400 + OFF))));
    const __half2 r = __hmul2(c, *reinterpret_cast<const __half2*>(&g2));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
}

// Dequantises the block at `slot + qw_off(QB)` (k-block kb of the matrix) into the swizzled
// K-major image at `slot` (row r, 16-byte chunk c at r·128 + ((c ^ (r & 7))·16)). Worker thread
// wt owns row wt; every thread reads its inputs before any writes (the output overlaps the
// input), hence the barrier in the middle.
template <typename T, int QB>
__device__ __forceinline__ void dequant_inplace(uint8_t* slot, int wt, int kb) {
  const uint8_t* blk = slot + qw_off(QB);
  uint32_t cw[8];        // q4: one word per chunk; q3: low planes 0-3, high planes 4-5
  uint16_t sraw[3];      // the block's scales, raw
  if constexpr (QB == 4) {
    const uint4 c0 = reinterpret_cast<const uint4*>(blk + wt * 32)[0];
    const uint4 c1 = reinterpret_cast<const uint4*>(blk + wt * 32)[1];
    cw[0] = c0.x; cw[1] = c0.y; cw[2] = c0.z; cw[3] = c0.w;
    cw[4] = c1.x; cw[5] = c1.y; cw[6] = c1.z; cw[7] = c1.w;
    const uint32_t sc = *reinterpret_cast<const uint32_t*>(blk + BM * 32 + wt * 4);
    sraw[0] = (uint16_t)sc;
    sraw[1] = (uint16_t)(sc >> 16);
    sraw[2] = 0;
  } else {
    const uint4 l = *reinterpret_cast<const uint4*>(blk + wt * 16);
    const uint2 h = *reinterpret_cast<const uint2*>(blk + BM * 16 + wt * 8);
    const uint2 sc = *reinterpret_cast<const uint2*>(blk + BM * 24 + wt * 8);
    cw[0] = l.x; cw[1] = l.y; cw[2] = l.z; cw[3] = l.w;
    cw[4] = h.x; cw[5] = h.y; cw[6] = 0u; cw[7] = 0u;
    sraw[0] = (uint16_t)sc.x;
    sraw[1] = (uint16_t)(sc.x >> 16);
    sraw[2] = (uint16_t)sc.y;
  }
  workers_sync();
  const int r0 = (kb * 64) % 40;  // q3: column of the block's first element inside its group
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    int gi;
    if constexpr (QB == 4) gi = c >> 2;
    else gi = (r0 + 8 * c) / 40;
    const uint16_t sb = gi == 0 ? sraw[0] : (gi == 1 ? sraw[1] : sraw[2]);
    const uint32_t g2 = (uint32_t)sb * 0x10001u;  // the scale in both halves
    const float g = Tr<T>::f(*reinterpret_cast<const T*>(&sb));
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      if constexpr (QB == 4) {
        o[h] = dequant_pair<T, 7>((cw[c] >> (4 * h)) & 0x000F000Fu, g2, g);
      } else {
        const uint32_t lo2 = (cw[c >> 1] >> (8 * (c & 1) + 2 * h)) & 0x00030003u;
        const int p = 4 * c + h;
        const uint32_t hi1 = ((cw[4 + (p >> 4)] >> (p & 15)) & 0x00010001u) << 2;
        o[h] = dequant_pair<T, 3>(lo2 | hi1, g2, g);
      }
    }
    *reinterpret_cast<uint4*>(slot + wt * 128 + ((c ^ (wt & 7)) << 4)) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// NORM: normalises one raw x block in place. The block holds x[0:NA, 64 columns] as written by
// TMA in the 128-byte swizzle layout (element (r, k) at r·128 + ((k/8) ^ (r & 7))·16 + (k%8)·2,
// rows ≥ M and columns ≥ K zero-filled). Worker thread wt (0..127) owns 16-byte column chunk
// q = wt & 7 of rows (wt >> 3) + 16·u; (sc, sh) are that chunk's 8 scale / shift values.
//   B = RN16( RN(RN(x / den) · RN(1 + scale)) + shift ),  den = sqrt(Σx²/K + eps)
// (gemma_dual.py:76-88, fp32 arithmetic, one rounding per operation).
template <typename T, int NA>
__device__ __forceinline__ void norm_inplace(const SkArgs& a, uint8_t* xb, uint4 sc, uint4 sh,
                                             const float* s_den, const float* s_rcp, int wt) {
  const int q = wt & 7;
  const T* es = reinterpret_cast<const T*>(&sc);
  const T* eh = reinterpret_cast<const T*>(&sh);
  float s1[8], shf[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    s1[e] = __fadd_rn(1.f, Tr<T>::f(es[e]));
    shf[e] = Tr<T>::f(eh[e]);
  }
#pragma unroll 1
  for (int u = 0; u < NA / 16; ++u) {
    const int r = (wt >> 3) + 16 * u;
    if (r >= a.M) break;  // zero rows stay zero
    uint4* p = reinterpret_cast<uint4*>(xb + r * 128 + ((q ^ (r & 7)) << 4));
    const uint4 v = *p;
    const T* e = reinterpret_cast<const T*>(&v);
    const float den = s_den[r], rcp = s_rcp[r];
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float n0 = div_by_rcp(Tr<T>::f(e[2 * j]), den, rcp);
      const float n1 = div_by_rcp(Tr<T>::f(e[2 * j + 1]), den, rcp);
      o[j] = Tr<T>::pack(__fadd_rn(__fmul_rn(n0, s1[2 * j]), shf[2 * j]),
                         __fadd_rn(__fmul_rn(n1, s1[2 * j + 1]), shf[2 * j + 1]));
    }
    *p = make_uint4(o[0], o[1], o[2], o[3]);
  }
  // generic-proxy smem writes -> visible to the tensor core (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// QB: 0 = 16-bit weights (packed blocks or a tensor map), 4 / 3 = group-quantised blocks
// (pack_q_kernel) dequantised in shared memory by the worker warps.
template <typename T, int NA, bool NORM, bool SSQ, class Epi, int QB = 0>
__global__ void __launch_bounds__(NT, 2) skinny_kernel(const __grid_constant__ CUtensorMap tmW,
                                                       const __grid_constant__ CUtensorMap tmX,
                                                       SkArgs a, Epi epi) {
  using S = SkSmem<NA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  // full_w / full_x: copy landed; ready_x (NORM or QB): the stage's blocks are normalised /
  // dequantised; empty: MMAs done with a stage
  __shared__ __align__(8) uint64_t full_w[RING], full_x[RING], ready_x[RING], empty[RING], bar_mma;
  __shared__ uint32_t s_tmem;
  __shared__ int s_ok, s_stop;
  __shared__ float s_den[NORM ? NA : 1], s_rcp[NORM ? NA : 1];  // NORM: row sqrt(ms + eps), 1/it

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = a.C;
  const uint32_t rank = cluster_rank();  // 0 for a cluster of one
  const int tile = blockIdx.x / C;
  const int n0 = tile * BM;
  const int nkb = (a.K + BK - 1) / BK;
  const int kb0 = rank * a.kbpc;
  const int nk = max(0, min(nkb, kb0 + a.kbpc) - kb0);
  auto stage_w = [&](int s) { return base + s * S::STAGE; };
  auto stage_x = [&](int s) { return base + s * S::STAGE + W_BLOCK; };

  if (tid == 0) {
    for (int s = 0; s < RING; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&full_x[s], 1);
      mbar_init(&ready_x[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&bar_mma, 1);
    s_stop = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (!a.wpack) tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"((uint32_t)NA));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  constexpr int WB = QB ? qw_block(QB) : W_BLOCK;  // bytes of one weight block in global memory
  const uint8_t* wsrc =
      a.wpack ? reinterpret_cast<const uint8_t*>(a.wpack) + ((size_t)tile * nkb + kb0) * WB
              : nullptr;
  auto issue_w = [&](int i) {
    const int s = i % RING;
    mbar_expect_tx(&full_w[s], WB);
    if (QB) bulk_load(stage_w(s) + qw_off(QB), wsrc + (size_t)i * WB, WB, &full_w[s]);
    else if (wsrc) bulk_load(stage_w(s), wsrc + (size_t)i * WB, WB, &full_w[s]);
    else tma_load_2d(stage_w(s), &tmW, &full_w[s], (kb0 + i) * BK, n0);
  };

  // weights never depend on the previous kernel: fill the ring before waiting on it
  int issued = 0, issued_x = 0;  // thread 0: weight / activation blocks issued
  if (tid == 0)
    for (; issued < min(nk, RING); ++issued) issue_w(issued);
  pdl_trigger();
  // QB: the worker warps dequantise those first blocks while the previous kernel finishes (the
  // weights do not depend on it); without NORM such a stage is then ready but for its x block
  int pre = 0;
  if constexpr (QB != 0) {
    if (warp >= 2) {
      const int wt = tid - 64;
      for (; pre < min(nk, RING); ++pre) {
        if (!mbar_wait(&full_w[pre], 0, a.err, ERR_TIMEOUT_EPI)) s_stop = 1;
        workers_sync();
        if (s_stop) break;
        dequant_inplace<T, QB>(stage_w(pre), wt, kb0 + pre);
        if constexpr (!NORM) {
          workers_sync();
          if (wt == 0) mbar_arrive(&ready_x[pre]);
        }
      }
    }
  }
  pdl_wait();

  // the epilogue's global operands (residual rows, gates, RoPE tables) do not depend on the
  // accumulator: request them into L1 early, so the epilogue does not wait on L2 round trips
  auto prefetch_epi = [&]() {
    const int R = BM / C, quads = R / 4, total = quads * a.M;
    for (int it = tid; it < total; it += NT) {
      const int g = it % quads, m = it / quads;
      const int n = n0 + rank * R + 4 * g;
      if (n < a.N) epi.prefetch(m, n);
    }
  };

  if (warp == 0) {
    if (lane == 0) {  // producer: weight blocks past the first RING, all activation blocks
      for (int i = 0; i < nk; ++i) {
        const int s = i % RING;
        if (i >= RING) {
          if (!mbar_wait(&empty[s], ((i / RING) - 1) & 1, a.err, ERR_TIMEOUT_PRODUCER)) break;
          issue_w(i);
          issued = i + 1;
        }
        mbar_expect_tx(&full_x[s], S::X_BLOCK);
        tma_load_2d(stage_x(s), &tmX, &full_x[s], (kb0 + i) * BK, 0);
        issued_x = i + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = idesc_f16<T>(BM, NA);
      for (int i = 0; i < nk; ++i) {
        const int s = i % RING;
        const uint32_t ph = (i / RING) & 1;
        if ((!QB && !mbar_wait(&full_w[s], ph, a.err, ERR_TIMEOUT_MMA)) ||
            ((NORM || QB) && !mbar_wait(&ready_x[s], ph, a.err, ERR_TIMEOUT_MMA)) ||
            (!NORM && !mbar_wait(&full_x[s], ph, a.err, ERR_TIMEOUT_MMA)))
          break;
        tc_fence_after();
        const uint64_t da = desc_sw128(smem_u32(stage_w(s)));
        const uint64_t db = desc_sw128(smem_u32(stage_x(s)));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(&bar_mma);  // arrives once every issued MMA is done (at once if none)
    }
  } else {
    if (NORM || QB) {  // warps 2-5: per stage, dequantise the weight block (QB) and normalise
                       // the raw x block (NORM) in place once their copies have landed
      const int wt = tid - 64;
      const T* mod = reinterpret_cast<const T*>(a.mod);
      const uint4 z = make_uint4(0, 0, 0, 0);
      auto load_mod = [&](int i, uint4& c1, uint4& c2) {
        const int col = (kb0 + i) * BK + (wt & 7) * 8;
        const bool in = col < a.K;
        c1 = in ? *reinterpret_cast<const uint4*>(mod + col) : z;
        c2 = in ? *reinterpret_cast<const uint4*>(mod + a.K + col) : z;
      };
      uint4 sc = z, sh = z;
      if constexpr (NORM) {
        if (nk > 0) load_mod(0, sc, sh);
        if (wt < a.M) {  // M ≤ NA ≤ 128: one row per thread; partials summed in slot order
          const float4* p = reinterpret_cast<const float4*>(a.ssq_in + (size_t)wt * a.ssq_parts);
          float ss = 0.f;
          for (int i = 0; i < a.ssq_parts / 4; i += 4) {
            float4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = p[i + j];
#pragma unroll
            for (int j = 0; j < 4; ++j) ss = ((ss + v[j].x) + v[j].y + v[j].z) + v[j].w;
          }
          const float den = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps));
          s_den[wt] = den;
          s_rcp[wt] = __frcp_rn(den);
        }
        workers_sync();
      }
      for (int i = 0; i < nk; ++i) {
        const int s = i % RING;
        const uint32_t ph = (i / RING) & 1;
        if (s_stop) break;  // a wait before the previous kernel's end gave up
        if constexpr (QB != 0) {
          if (i >= pre) {
            if (!mbar_wait(&full_w[s], ph, a.err, ERR_TIMEOUT_EPI)) s_stop = 1;
            workers_sync();
            if (s_stop) break;
            dequant_inplace<T, QB>(stage_w(s), wt, kb0 + i);
          } else if (!NORM) {
            continue;  // dequantised and marked ready before the wait
          }
        }
        if constexpr (NORM) {
          uint4 nsc = z, nsh = z;
          if (i + 1 < nk) load_mod(i + 1, nsc, nsh);
          if (!mbar_wait(&full_x[s], ph, a.err, ERR_TIMEOUT_EPI)) s_stop = 1;
          workers_sync();
          if (s_stop) break;
          norm_inplace<T, NA>(a, stage_x(s), sc, sh, s_den, s_rcp, wt);
          sc = nsc;
          sh = nsh;
        }
        workers_sync();
        if (wt == 0) mbar_arrive(&ready_x[s]);
      }
    }
  }
  // one call site for every thread: idle lanes and, in NORM launches, the workers once their
  // blocks are done (the epilogue is still about a microsecond away)
  prefetch_epi();

  // ---- accumulator -> shared memory partial ----
  if (tid == 64) s_ok = mbar_wait(&bar_mma, 0, a.err, ERR_TIMEOUT_EPI, false) ? 1 : 0;
  if (tid == 0) {
    // drain: every copy this thread issued has landed before the ring memory is reused (the
    // normal path consumed them all; this matters after a timeout)
    for (int i = max(0, issued - RING); i < issued; ++i)
      mbar_wait(&full_w[i % RING], (i / RING) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
    for (int i = max(0, issued_x - RING); i < issued_x; ++i)
        mbar_wait(&full_x[i % RING], (i / RING) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
  }
  __syncthreads();
  const bool ok = s_ok != 0 && nk > 0;
  tc_fence_after();
  float* part = reinterpret_cast<float*>(base);  // [NA][PLD], aliases the drained ring
  if (warp >= 2) {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int wrow = q * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < NA; c += 32) {
      uint32_t v[32];
      if (ok) {
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) part[(c + j) * PLD + wrow] = __uint_as_float(v[j]);
    }
  }
  tc_fence_before();
  cluster_sync();

  // ---- split-K reduction + epilogue: rank r finishes weight rows [r·R, (r+1)·R) ----
  // One (activation row, 4 weight rows) item per iteration, the C partials of an item loaded
  // together, and a single call site of the epilogue: every CTA runs this code once, so it is
  // kept short (instruction fetch, not arithmetic, bounds a cold one-pass epilogue).
  const int R = BM / C, quads = R / 4;
  const uint32_t pbase = smem_u32(part);
  const int total = quads * a.M;
  float* s_item = reinterpret_cast<float*>(base + S::PART);
#pragma unroll 1
  for (int it = tid; it < total; it += NT) {
    const int g = it % quads, m = it / quads;
    const uint32_t off = pbase + (uint32_t)(m * PLD + rank * R + 4 * g) * 4u;
    float4 v[MAX_C];
#pragma unroll
    for (int c = 0; c < MAX_C; ++c)
      if (c < C) v[c] = ld_cluster4(map_rank(off, c));
    float4 sum = v[0];
#pragma unroll
    for (int c = 1; c < MAX_C; ++c)
      if (c < C) {
        sum.x += v[c].x;
        sum.y += v[c].y;
        sum.z += v[c].z;
        sum.w += v[c].w;
      }
    float sq = 0.f;
    const int nb = n0 + rank * R + 4 * g;
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      const int n = nb + 2 * h;
      if (n >= a.N) break;
      const float v0 = h ? sum.z : sum.x, v1 = h ? sum.w : sum.y;
      if constexpr (SSQ) {
        const float2 p = epi(m, n, v0, v1);
        sq += p.x * p.x + p.y * p.y;
      } else {
        epi(m, n, v0, v1);
      }
    }
    if constexpr (SSQ) s_item[it] = sq;
  }
  if constexpr (SSQ) {
    __syncthreads();
    const int parts_used = (int)gridDim.x;  // tiles · C
    for (int m = tid; m < a.M; m += NT) {
      float q = 0.f;
      for (int g = 0; g < quads; ++g) q += s_item[m * quads + g];
      a.ssq_out[(size_t)m * a.ssq_parts + tile * C + rank] = q;
      if (blockIdx.x == 0)
        for (int p = parts_used; p < a.ssq_parts; ++p) a.ssq_out[(size_t)m * a.ssq_parts + p] = 0.f;
    }
  }
  cluster_sync();  // keep this CTA's shared memory alive until every rank has read it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)NA));
  }
}

}  // namespace sk
}  // namespace pi0
