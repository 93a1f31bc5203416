// Weight-streaming GEMM for the denoise step (M = B·S activation rows ≤ 128, e.g. 50):
//   Y[M, N] = X[M, K] · W[N, K]^T  with the fused epilogue functors of gemm_mma.cuh.
//
// The M=50 projections are HBM-bound (every weight byte is used 50 times), so the kernel is
// built around streaming W once at full bandwidth:
//   * the weights are pre-packed (at pi0_set_params) into 16 KB blocks, one per (128-row tile,
//     64-wide k-block), each already the 128-byte-swizzled K-major shared-memory image, and a
//     tile's k-blocks are contiguous: a CTA pulls its whole weight slice with one-dimensional
//     cp.async.bulk copies — sequential DRAM streams, no tensor map;
//   * swap-AB on tcgen05: the weight tile is the MMA's A operand (M = 128 weight rows) and the
//     activations are B (N = NA = 64 or 128 rows, zero past M), accumulator [128 × NA] fp32 in
//     TMEM;
//   * split-K over a thread-block cluster of C CTAs (C ≤ 16): rank r owns k-blocks
//     [r·kbpc, (r+1)·kbpc) of one tile; partial accumulators are summed through distributed
//     shared memory in rank order (deterministic), each rank finishing 128/C weight rows;
//   * programmatic dependent launch: the weight copies are issued before griddepcontrol.wait,
//     so a kernel's weight stream overlaps the tail of the kernel producing its activations;
//   * optional fusions: NORM builds B = adaRMSNorm(x) in shared memory from the residual stream
//     and per-row Σx² partials; SSQ makes the residual epilogue emit those partials (one per
//     128-row tile, deterministic) for the next norm-fused GEMM.
#pragma once

#include "gemm_tc.cuh"

namespace pi0 {
namespace sk {

using namespace tc;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
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
__device__ __forceinline__ float ld_cluster1(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
// one-dimensional bulk copy global -> this CTA's shared memory, completing on an mbarrier
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

constexpr int KBPC_MAX = 4;           // k-blocks (of 64) per CTA
constexpr int W_BLOCK = BM * BK * 2;  // 16 KB: one packed (tile, k-block) weight block
constexpr int PLD = BM + 4;           // partial row stride (floats): activation-row major
constexpr int NORM_ITEMS = 4;         // 16-byte chunks a thread normalises per batch

template <int NA>
struct SkSmem {
  static constexpr int X_BLOCK = NA * BK * 2;
  static constexpr int LOAD = KBPC_MAX * (W_BLOCK + X_BLOCK);
  static constexpr int PART = NA * PLD * 4;
  static constexpr int BYTES = (LOAD > PART ? LOAD : PART) + 1024;
};

struct SkArgs {
  int M, N, K;
  int kbpc;              // k-blocks per CTA (≤ KBPC_MAX)
  int C;                 // cluster size = number of K splits
  int* err;
  const void* wpack;     // pre-packed weights, or null to load W through the tensor map
  // NORM: B = x / sqrt(Σx²/K + eps) · (1 + scale) + shift, (scale, shift) = mod[0:K], mod[K:2K]
  const void* x;         // [M, K] residual stream, model dtype
  const void* mod;       // modulation row of this step
  float eps;
  const float* ssq_in;   // [M][ssq_parts] partial Σx² of the rows of x
  // SSQ: ssq_out[m][tile] = Σ over the tile's 128 features of x_new² (epilogue return values)
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

// NORM prologue: writes this CTA's k-blocks of B = adaRMSNorm(x) into the swizzled smem operand.
template <typename T, int NA>
__device__ __forceinline__ void norm_to_smem(const SkArgs& a, uint8_t* sX, int kb0, int nk,
                                             float* s_den) {
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int m = tid; m < a.M; m += nt) {
    const float* p = a.ssq_in + (size_t)m * a.ssq_parts;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = i < a.ssq_parts ? p[i] : 0.f;  // loads issued together
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) ss += v[i];
    s_den[m] = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps));
  }
  __syncthreads();
  const T* x = reinterpret_cast<const T*>(a.x);
  const T* mod = reinterpret_cast<const T*>(a.mod);
  const int cpr = nk * 8;  // 16-byte chunks per row in this CTA
  const int total = NA * cpr;
  const int c0 = kb0 * 8;
  for (int base = tid; base < total; base += nt * NORM_ITEMS) {
    uint4 xv[NORM_ITEMS], sc[NORM_ITEMS], sh[NORM_ITEMS];
#pragma unroll
    for (int u = 0; u < NORM_ITEMS; ++u) {
      const int it = base + u * nt;
      if (it >= total) continue;
      const int r = it / cpr, c = c0 + it % cpr;
      if (r < a.M) {
        xv[u] = *reinterpret_cast<const uint4*>(x + (size_t)r * a.K + c * 8);
        sc[u] = *reinterpret_cast<const uint4*>(mod + c * 8);
        sh[u] = *reinterpret_cast<const uint4*>(mod + a.K + c * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < NORM_ITEMS; ++u) {
      const int it = base + u * nt;
      if (it >= total) continue;
      const int r = it / cpr, cl = it % cpr;
      uint4 outv = make_uint4(0, 0, 0, 0);
      if (r < a.M) {
        const float den = s_den[r];
        const T* e = reinterpret_cast<const T*>(&xv[u]);
        const T* es = reinterpret_cast<const T*>(&sc[u]);
        const T* eh = reinterpret_cast<const T*>(&sh[u]);
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float v2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int q = 2 * j + h;
            const float n = __fdiv_rn(Tr<T>::f(e[q]), den);
            v2[h] = __fadd_rn(__fmul_rn(n, __fadd_rn(1.f, Tr<T>::f(es[q]))), Tr<T>::f(eh[q]));
          }
          o[j] = Tr<T>::pack(v2[0], v2[1]);
        }
        outv = make_uint4(o[0], o[1], o[2], o[3]);
      }
      const int kb = cl >> 3, q = cl & 7;
      *reinterpret_cast<uint4*>(sX + kb * (NA * BK * 2) + r * 128 + ((q ^ (r & 7)) << 4)) = outv;
    }
  }
  // generic-proxy smem writes -> visible to the tensor core (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T, int NA, bool NORM, bool SSQ, class Epi>
__global__ void __launch_bounds__(128) skinny_kernel(const __grid_constant__ CUtensorMap tmW,
                                                     const __grid_constant__ CUtensorMap tmX,
                                                     SkArgs a, Epi epi) {
  using S = SkSmem<NA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t bar_w, bar_x, bar_mma;
  __shared__ uint32_t s_tmem;
  __shared__ int s_ok;
  __shared__ float s_small[NA];                // NORM: row denominators; SSQ: rank partials
  __shared__ float s_item[SSQ ? NA * 32 : 1];  // SSQ: per-item squares

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = a.C;
  const uint32_t rank = C > 1 ? cluster_rank() : 0;
  const int tile = blockIdx.x / C;
  const int n0 = tile * BM;
  const int nkb = (a.K + BK - 1) / BK;
  const int kb0 = rank * a.kbpc;
  const int nk = max(0, min(nkb, kb0 + a.kbpc) - kb0);
  uint8_t* sW = base;
  uint8_t* sX = base + KBPC_MAX * W_BLOCK;
  float* part = reinterpret_cast<float*>(base);  // reused after the MMAs: [NA][PLD]

  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_x, 1);
    mbar_init(&bar_mma, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (!a.wpack) tma_prefetch_desc(&tmW);
    if (!NORM) tma_prefetch_desc(&tmX);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem)),
                 "r"((uint32_t)NA));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  // weights never depend on the previous kernel: start streaming them before waiting on it
  if (tid == 0 && nk > 0) {
    mbar_expect_tx(&bar_w, nk * W_BLOCK);
    if (a.wpack) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.wpack) +
                           ((size_t)tile * nkb + kb0) * W_BLOCK;
      for (int i = 0; i < nk; ++i) bulk_load(sW + i * W_BLOCK, src + i * W_BLOCK, W_BLOCK, &bar_w);
    } else {
      for (int i = 0; i < nk; ++i) tma_load_2d(sW + i * W_BLOCK, &tmW, &bar_w, (kb0 + i) * BK, n0);
    }
  }
  pdl_trigger();
  pdl_wait();
  if (NORM) {
    if (nk > 0) norm_to_smem<T, NA>(a, sX, kb0, nk, s_small);
    __syncthreads();
  }
  if (tid == 0) {
    if (nk > 0) {
      if (!NORM) {
        mbar_expect_tx(&bar_x, nk * S::X_BLOCK);
        for (int i = 0; i < nk; ++i)
          tma_load_2d(sX + i * S::X_BLOCK, &tmX, &bar_x, (kb0 + i) * BK, 0);
      }
      bool ok = mbar_wait(&bar_w, 0, a.err, ERR_TIMEOUT_MMA, false) &&
                (NORM || mbar_wait(&bar_x, 0, a.err, ERR_TIMEOUT_MMA, false));
      if (ok) {
        tc_fence_after();
        constexpr uint32_t idesc = idesc_f16<T>(BM, NA);
        for (int i = 0; i < nk; ++i) {
          const uint64_t da = desc_sw128(smem_u32(sW + i * W_BLOCK));
          const uint64_t db = desc_sw128(smem_u32(sX + i * S::X_BLOCK));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
        }
      }
    }
    umma_commit(&bar_mma);  // arrives once every issued MMA is done (at once if none)
    s_ok = mbar_wait(&bar_mma, 0, a.err, ERR_TIMEOUT_EPI, false) ? 1 : 0;
  }
  __syncthreads();
  const bool ok = s_ok != 0;
  tc_fence_after();
  // accumulator -> shared partial part[act row][weight row] (weight row = TMEM lane)
  const int wrow = warp * 32 + lane;
  if (nk > 0 && ok) {
#pragma unroll 1
    for (int c = 0; c < NA; c += 32) {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) part[(c + j) * PLD + wrow] = __uint_as_float(v[j]);
    }
  } else {
    for (int j = 0; j < NA; ++j) part[j * PLD + wrow] = 0.f;
  }
  tc_fence_before();
  if (C > 1) cluster_sync();
  else __syncthreads();

  // rank r finishes weight rows [r·R, (r+1)·R) of the tile: each item is 4 consecutive weight
  // rows of one activation row, read from all C ranks with 16-byte loads issued together and
  // summed in rank order (deterministic)
  const int R = BM / C, quads = R / 4;
  const uint32_t pbase = smem_u32(part);
  const int total = quads * a.M;
  const int lc = 31 - __clz(C);      // C is a power of two ≤ 16
  const int ipb = 16 >> lc;          // items per batch: 16 loads in flight per thread
  for (int base = tid; base < total; base += blockDim.x * ipb) {
    float4 v[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int u = q >> lc, c = q & (C - 1);
      const int it = base + u * blockDim.x;
      v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (u < ipb && it < total) {
        const int g = it % quads, m = it / quads;
        const uint32_t off = pbase + (uint32_t)(m * PLD + rank * R + 4 * g) * 4u;
        v[q] = ld_cluster4(C > 1 ? map_rank(off, c) : off);
      }
    }
    // per item: sum its C partials in rank order (static register indices only)
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      sum.x += v[q].x;
      sum.y += v[q].y;
      sum.z += v[q].z;
      sum.w += v[q].w;
      if ((q & (C - 1)) == C - 1) {
        const int u = q >> lc;
        const int it = base + u * blockDim.x;
        if (u < ipb && it < total) {
          const int g = it % quads, m = it / quads;
          const int n = n0 + rank * R + 4 * g;
          if constexpr (SSQ) {
            float sq = 0.f;
            if (n < a.N) {
              const float2 p = epi(m, n, sum.x, sum.y);
              sq += p.x * p.x + p.y * p.y;
            }
            if (n + 2 < a.N) {
              const float2 p = epi(m, n + 2, sum.z, sum.w);
              sq += p.x * p.x + p.y * p.y;
            }
            s_item[it] = sq;
          } else {
            if (n < a.N) epi(m, n, sum.x, sum.y);
            if (n + 2 < a.N) epi(m, n + 2, sum.z, sum.w);
          }
        }
        sum = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  if constexpr (SSQ) {
    __syncthreads();
    for (int m = tid; m < a.M; m += blockDim.x) {
      float q = 0.f;
      for (int g = 0; g < quads; ++g) q += s_item[m * quads + g];
      s_small[m] = q;
    }
    if (C > 1) cluster_sync();
    else __syncthreads();
    if (rank == 0) {
      const uint32_t sb = smem_u32(s_small);
      for (int m = tid; m < a.M; m += blockDim.x) {
        float q = 0.f;
        for (int c = 0; c < C; ++c) q += ld_cluster1(C > 1 ? map_rank(sb + m * 4, c) : sb + m * 4);
        a.ssq_out[(size_t)m * a.ssq_parts + tile] = q;
      }
    }
  }
  if (C > 1) cluster_sync();  // keep this CTA's shared memory alive until every rank has read it
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)NA));
  }
}

}  // namespace sk
}  // namespace pi0
