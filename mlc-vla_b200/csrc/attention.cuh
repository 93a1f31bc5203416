// Multi-query attention for both halves of the M1 path (gemma_dual.py:97-122 `_sdpa`):
//   * prefill: P prefix queries per head against the P prefix keys just written to the cache
//     (attn_prefill_e0, gemma_dual.py:236-253);
//   * denoise: S suffix queries per head against [P cached prefix keys ; S suffix keys]
//     (attn_decode_e1, gemma_dual.py:255-275).
// Numerics follow the reference: q and k are fp32 (post-RoPE, q pre-scaled by hd^-0.5), logits
// are accumulated in fp32 and the additive fp32 pad mask (0 / -1e9, prefix keys only) is added
// before a fp32 softmax; probabilities are rounded to the model dtype and multiplied by the
// model-dtype V with fp32 accumulation. The q·k operands follow the reference's
// attn_logits_dtype (gemma_dual.py:115: q and k cast to it, product accumulated in fp32):
//   * "float32" (its default): fp32 operands, on tf32 tensor cores as three products of the
//     split x = big + small (big = tf32(x), small = tf32(x − big)): big·big + big·small +
//     small·big, which carries the 22-bit operand precision of fp32 accumulation (the dropped
//     small·small term is below 2^-21 of the product);
//   * the model dtype: q and k rounded to fp16 / bf16 first, then one tf32 product, which is
//     exact for 16-bit operands.
// The softmax is online (flash style), so probabilities are rounded before the final 1/l
// normalisation rather than after it.
//
// Rows of one CTA tile are (t, g) pairs of one kv head: row j -> t = j / G, head = kvh·G + j % G
// with G = H / KV, so every row of a tile shares the tile's K/V (MQA: all heads of a token).
// gridDim = (row tiles, key splits, B·KV). K/V tiles of 32 keys are double buffered with
// cp.async; tiles of cached prefix keys do not depend on the previous kernel and are requested
// before griddepcontrol.wait. With several key splits the CTAs of one row tile form a cluster
// and merge their (m, l, O) partials through distributed shared memory in rank order, so no
// separate combine kernel runs.
#pragma once

#include "common.cuh"

namespace pi0 {

template <typename T>
struct AttnArgs {
  const float* q;      // [B, Tq, H, hd]
  const float* kA;     // segment A keys   [B, KV, LA, hd] fp32 (the prefix cache of one layer)
  const T* vA;         //           values [B, KV, LA, hd]
  const float* maskA;  // [B, LA] additive fp32, or null
  int LA;
  const float* kB;     // segment B (suffix keys/values) [B, KV, LB, hd], LB may be 0
  const T* vB;
  int LB;
  int Tq, H, KV;
  int keys_per_split;  // multiple of the key tile width
  T* out;              // [B, Tq, H·hd]
  int a_is_ready;      // segment A was written before the previous kernel (the prefix cache
                       // during denoise): its tiles may be requested before griddepcontrol.wait
  int logits_f32;      // 1: fp32 q·k operands (attn_logits_dtype "float32"); 0: model dtype
};

// tf32 operand pair (big, small) of an fp32 value: big = tf32(x), small = tf32(x − big)
__device__ __forceinline__ void tf32_split(float x, uint32_t& big, uint32_t& small) {
  big = to_tf32(x);
  small = to_tf32(x - __uint_as_float(big));
}

constexpr int ATT_BQ = 64;   // query rows per CTA (4 warps × 16)
constexpr int ATT_BK = 32;   // keys per tile

template <int HD, int BK = ATT_BK>
struct AttnSmem {
  static constexpr int QLD = HD + 4;   // fp32 row stride (conflict-free tf32 fragment loads)
  static constexpr int KLD = HD + 4;
  static constexpr int VLD = HD + 8;   // 16-bit row stride (conflict-free ldmatrix.trans)
  static constexpr int Q_BYTES = ATT_BQ * QLD * 4;
  static constexpr int K_BYTES = BK * KLD * 4;
  static constexpr int V_BYTES = BK * VLD * 2;
  static constexpr int STAGE = K_BYTES + V_BYTES + BK * 4;
  static constexpr int BYTES = Q_BYTES + 2 * STAGE;
  // after the key loop: partial O [64][HD + 4] fp32 and (m, l) [64][2] reuse the same space
  static constexpr int OLD = HD + 4;
  static_assert(ATT_BQ * OLD * 4 + ATT_BQ * 8 <= BYTES, "combine buffer");
};

__device__ __forceinline__ uint32_t attn_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void attn_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t attn_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float2 attn_ld2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}

template <typename T, int HD, int BK>
__global__ void __launch_bounds__(128) attn_kernel(AttnArgs<T> a) {
  using SM = AttnSmem<HD, BK>;
  constexpr int NT8 = BK / 8, NK16 = BK / 16;  // score n-tiles, PV k-steps per key tile
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sQ = reinterpret_cast<float*>(smem_raw);
  auto sK = [&](int s) { return reinterpret_cast<float*>(smem_raw + SM::Q_BYTES + s * SM::STAGE); };
  auto sV = [&](int s) {
    return reinterpret_cast<T*>(smem_raw + SM::Q_BYTES + s * SM::STAGE + SM::K_BYTES);
  };
  auto sMask = [&](int s) {
    return reinterpret_cast<float*>(smem_raw + SM::Q_BYTES + s * SM::STAGE + SM::K_BYTES + SM::V_BYTES);
  };

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.H / a.KV;
  const int rows = a.Tq * G;
  const int bk = blockIdx.z, b = bk / a.KV, kvh = bk % a.KV;
  const int row0 = blockIdx.x * ATT_BQ;
  const int nsplit = gridDim.y;
  const int split = blockIdx.y;
  const int Ltot = a.LA + a.LB;
  const int kbeg = split * a.keys_per_split;
  const int kend = min(Ltot, kbeg + a.keys_per_split);
  const int ntiles = max(0, (kend - kbeg + BK - 1) / BK);

  const float* kA = a.kA + ((size_t)b * a.KV + kvh) * a.LA * HD;
  const T* vA = a.vA + ((size_t)b * a.KV + kvh) * a.LA * HD;
  const float* kB = a.kB ? a.kB + ((size_t)b * a.KV + kvh) * a.LB * HD : nullptr;
  const T* vB = a.vB ? a.vB + ((size_t)b * a.KV + kvh) * a.LB * HD : nullptr;
  const float* mA = a.maskA ? a.maskA + (size_t)b * a.LA : nullptr;

  // K/V tile of keys [k0, k0 + BK) into stage s (zero-filled past kend)
  auto load_tile = [&](int s, int k0) {
    float* dk = sK(s);
    T* dv = sV(s);
    for (int i = tid; i < BK * (HD / 4); i += 128) {
      const int r = i / (HD / 4), ch = i % (HD / 4);
      const int key = k0 + r;
      const bool ok = key < kend;
      const float* src = ok ? (key < a.LA ? kA + (size_t)key * HD : kB + (size_t)(key - a.LA) * HD) : kA;
      cp_async16(dk + r * SM::KLD + ch * 4, src + (ok ? ch * 4 : 0), ok ? 16 : 0);
    }
    for (int i = tid; i < BK * (HD / 8); i += 128) {
      const int r = i / (HD / 8), ch = i % (HD / 8);
      const int key = k0 + r;
      const bool ok = key < kend;
      const T* src = ok ? (key < a.LA ? vA + (size_t)key * HD : vB + (size_t)(key - a.LA) * HD) : vA;
      cp_async16(dv + r * SM::VLD + ch * 8, src + (ok ? ch * 8 : 0), ok ? 16 : 0);
    }
    if (tid < BK) {
      const int key = k0 + tid;
      float mv;
      if (key >= kend) mv = -1e30f;                   // outside this split: contributes 0
      else if (key < a.LA) mv = mA ? mA[key] : 0.f;    // prefix pad mask
      else mv = 0.f;                                   // suffix keys are always visible
      sMask(s)[tid] = mv;
    }
  };

  // tiles made only of cached prefix keys (and their mask) are independent of the previous
  // kernel: start the first one before waiting on it
  const bool t0_independent = a.a_is_ready && ntiles > 0 && kbeg + BK <= a.LA;
  if (t0_independent) load_tile(0, kbeg);
  cp_async_commit();
  pdl_trigger();
  pdl_wait();
  if (ntiles > 0 && !t0_independent) load_tile(0, kbeg);
  // Q tile (written by the q/k/v projection)
  for (int i = tid; i < ATT_BQ * (HD / 4); i += 128) {
    const int r = i / (HD / 4), ch = i % (HD / 4);
    const int j = row0 + r;
    float* dst = sQ + r * SM::QLD + ch * 4;
    if (j < rows) {
      const int t = j / G, h = kvh * G + (j - t * G);
      cp_async16(dst, a.q + (((size_t)b * a.Tq + t) * a.H + h) * HD + ch * 4, 16);
    } else {
      *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  cp_async_commit();

  const int gq = lane >> 2, tq = lane & 3;
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-1e30f, -1e30f}, l_r[2] = {0.f, 0.f};

  for (int t = 0; t < ntiles; ++t) {
    const int s = t & 1;
    if (t + 1 < ntiles) load_tile(s ^ 1, kbeg + (t + 1) * BK);  // prefetch the next tile
    cp_async_commit();
    cp_async_wait<1>();  // everything but the just-issued prefetch has landed
    __syncthreads();
    const float* kt = sK(s);
    const T* vt = sV(s);
    const float* mt = sMask(s);

    // S = Q K^T for this warp's 16 rows × BK keys
    float sc[NT8][4];
#pragma unroll
    for (int n = 0; n < NT8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
    const float* qw = sQ + (warp * 16) * SM::QLD;
    if (a.logits_f32) {
#pragma unroll 2
      for (int kk = 0; kk < HD; kk += 8) {
        uint32_t ab[4], as[4];
        tf32_split(qw[gq * SM::QLD + kk + tq], ab[0], as[0]);
        tf32_split(qw[(gq + 8) * SM::QLD + kk + tq], ab[1], as[1]);
        tf32_split(qw[gq * SM::QLD + kk + tq + 4], ab[2], as[2]);
        tf32_split(qw[(gq + 8) * SM::QLD + kk + tq + 4], ab[3], as[3]);
#pragma unroll
        for (int n = 0; n < NT8; ++n) {
          uint32_t bb[2], bs[2];
          tf32_split(kt[(n * 8 + gq) * SM::KLD + kk + tq], bb[0], bs[0]);
          tf32_split(kt[(n * 8 + gq) * SM::KLD + kk + tq + 4], bb[1], bs[1]);
          mma1688_tf32(sc[n], as, bb);  // small terms first
          mma1688_tf32(sc[n], ab, bs);
          mma1688_tf32(sc[n], ab, bb);
        }
      }
    } else {
#pragma unroll 4
      for (int kk = 0; kk < HD; kk += 8) {
        uint32_t af[4];  // 16-bit values are exact in tf32
        af[0] = to_tf32(Tr<T>::r(qw[gq * SM::QLD + kk + tq]));
        af[1] = to_tf32(Tr<T>::r(qw[(gq + 8) * SM::QLD + kk + tq]));
        af[2] = to_tf32(Tr<T>::r(qw[gq * SM::QLD + kk + tq + 4]));
        af[3] = to_tf32(Tr<T>::r(qw[(gq + 8) * SM::QLD + kk + tq + 4]));
#pragma unroll
        for (int n = 0; n < NT8; ++n) {
          uint32_t bf[2];
          bf[0] = to_tf32(Tr<T>::r(kt[(n * 8 + gq) * SM::KLD + kk + tq]));
          bf[1] = to_tf32(Tr<T>::r(kt[(n * 8 + gq) * SM::KLD + kk + tq + 4]));
          mma1688_tf32(sc[n], af, bf);
        }
      }
    }
    // mask, online softmax
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < NT8; ++n) {
      const float mk0 = mt[n * 8 + tq * 2], mk1 = mt[n * 8 + tq * 2 + 1];
      sc[n][0] += mk0;
      sc[n][1] += mk1;
      sc[n][2] += mk0;
      sc[n][3] += mk1;
      mx[0] = fmaxf(mx[0], fmaxf(sc[n][0], sc[n][1]));
      mx[1] = fmaxf(mx[1], fmaxf(sc[n][2], sc[n][3]));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) corr[h] = expf(m_r[h] - mx[h]);
    uint32_t pf[NK16][4];  // P as m16n8k16 A fragments (16 keys each)
#pragma unroll
    for (int n = 0; n < NT8; ++n) {
      // CUDA's fast exponential (relative error about 2^-21; the probabilities are then rounded
      // to the V dtype)
      const float p0 = __expf(sc[n][0] - mx[0]), p1 = __expf(sc[n][1] - mx[0]);
      const float p2 = __expf(sc[n][2] - mx[1]), p3 = __expf(sc[n][3] - mx[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int kt2 = n >> 1, hi = n & 1;
      pf[kt2][hi * 2 + 0] = Tr<T>::pack(p0, p1);
      pf[kt2][hi * 2 + 1] = Tr<T>::pack(p2, p3);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_r[h] = l_r[h] * corr[h] + rs[h];
      m_r[h] = mx[h];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kt2 = 0; kt2 < NK16; ++kt2) {
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t b0, b1, b2, b3;
        const T* p = vt + (kt2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * SM::VLD + i * 8 +
                     (lane >> 4) * 8;
        ldsm_x4_t(b0, b1, b2, b3, p);
        uint32_t bb0[2] = {b0, b1}, bb1[2] = {b2, b3};
        mma16816<T>(o[i], pf[kt2], bb0);
        mma16816<T>(o[i + 1], pf[kt2], bb1);
      }
    }
    __syncthreads();  // this stage is refilled two tiles later
  }
  cp_async_wait<0>();

  if (nsplit == 1) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = row0 + warp * 16 + gq + h * 8;
      if (j >= rows) continue;
      const int t = j / G, head = kvh * G + (j - t * G);
      const float inv = 1.f / l_r[h];
      T* dst = a.out + ((size_t)b * a.Tq + t) * a.H * HD + (size_t)head * HD;
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) {
        const int d = i * 8 + tq * 2;
        *reinterpret_cast<uint32_t*>(dst + d) = Tr<T>::pack(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
      }
    }
    return;
  }

  // ---- merge the key splits of this row tile (cluster along grid.y) ----
  __syncthreads();
  float* sO = reinterpret_cast<float*>(smem_raw);            // [64][OLD] unnormalised O
  float* sML = sO + ATT_BQ * SM::OLD;                          // [64][2] (m, l)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = warp * 16 + gq + h * 8;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
      *reinterpret_cast<float2*>(sO + r * SM::OLD + i * 8 + tq * 2) = make_float2(o[i][2 * h], o[i][2 * h + 1]);
    if (tq == 0) {
      sML[r * 2 + 0] = m_r[h];
      sML[r * 2 + 1] = l_r[h];
    }
  }
  attn_cluster_sync();
  // rank r finishes rows [r·RPR, (r+1)·RPR) of the tile from every rank's partial, in rank order
  const uint32_t rank = attn_cluster_rank();
  const int rpr = ATT_BQ / nsplit;
  const uint32_t oaddr = smem_u32(sO), maddr = smem_u32(sML);
  __shared__ float s_w[ATT_BQ][16];
  __shared__ float s_inv[ATT_BQ];
  if (tid < rpr) {
    const int r = rank * rpr + tid;
    float mm[16], ll[16];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      if (c < nsplit) {
        const float2 ml = attn_ld2(attn_map(maddr + r * 8, c));
        mm[c] = ml.x;
        ll[c] = ml.y;
      }
    float M = -1e30f;
#pragma unroll
    for (int c = 0; c < 16; ++c)
      if (c < nsplit) M = fmaxf(M, mm[c]);
    float L = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c)
      if (c < nsplit) {
        const float w = expf(mm[c] - M);
        s_w[tid][c] = w;
        L += w * ll[c];
      }
    s_inv[tid] = 1.f / L;
  }
  __syncthreads();
  for (int it = tid; it < rpr * (HD / 2); it += 128) {
    const int rr = it / (HD / 2), d = (it % (HD / 2)) * 2;
    const int r = rank * rpr + rr;
    const int j = row0 + r;
    float2 pv[16];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      if (c < nsplit) pv[c] = attn_ld2(attn_map(oaddr + (r * SM::OLD + d) * 4, c));
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c)
      if (c < nsplit) {
        s0 += s_w[rr][c] * pv[c].x;
        s1 += s_w[rr][c] * pv[c].y;
      }
    if (j < rows) {
      const int t = j / G, head = kvh * G + (j - t * G);
      T* dst = a.out + ((size_t)b * a.Tq + t) * a.H * HD + (size_t)head * HD;
      *reinterpret_cast<uint32_t*>(dst + d) = Tr<T>::pack(s0 * s_inv[rr], s1 * s_inv[rr]);
    }
  }
  attn_cluster_sync();  // peers may still read this CTA's partial
}

}  // namespace pi0
