// Multi-query attention for both halves of the M1 path (gemma_dual.py:97-122 `_sdpa`):
//   * prefill: P prefix queries per head against the P prefix keys just written to the cache
//     (attn_prefill_e0, gemma_dual.py:236-253);
//   * denoise: S suffix queries per head against [P cached prefix keys ; S suffix keys]
//     (attn_decode_e1, gemma_dual.py:255-275).
// Numerics follow the reference: q and k are fp32 (post-RoPE, q pre-scaled by hd^-0.5), logits
// are accumulated in fp32 and the additive fp32 pad mask (0 / -1e9, prefix keys only) is added
// before a fp32 softmax; probabilities are rounded to the model dtype and multiplied by the
// model-dtype V with fp32 accumulation. q·k runs on tf32 tensor cores (cvt.rna, 10-bit
// mantissa); the softmax is online (flash style), so probabilities are rounded before the final
// 1/l normalisation rather than after it.
//
// Rows of one CTA tile are (t, g) pairs of one kv head: row j -> t = j / G, head = kvh·G + j % G
// with G = H / KV, so every row of a tile shares the tile's K/V (MQA: all heads of a token).
// gridDim = (row tiles, key splits, B·KV). With one split the kernel writes the normalised
// output; with several it writes (m, l, unnormalised O) partials that attn_combine merges.
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
  int keys_per_split;  // multiple of ATT_BK
  T* out;              // [B, Tq, H·hd]
  float* part_o;       // [B·KV, rows, splits, hd]
  float* part_ml;      // [B·KV, rows, splits, 2]
};

constexpr int ATT_BQ = 64;   // query rows per CTA (4 warps × 16)
constexpr int ATT_BK = 32;   // keys per iteration

template <int HD>
struct AttnSmem {
  static constexpr int QLD = HD + 4;   // fp32 row stride (conflict-free tf32 fragment loads)
  static constexpr int KLD = HD + 4;
  static constexpr int VLD = HD + 8;   // 16-bit row stride (conflict-free ldmatrix.trans)
  static constexpr int BYTES = (ATT_BQ * QLD + ATT_BK * KLD) * 4 + ATT_BK * VLD * 2 + ATT_BK * 4;
};

template <typename T, int HD>
__global__ void __launch_bounds__(128) attn_kernel(AttnArgs<T> a) {
  using SM = AttnSmem<HD>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sQ = reinterpret_cast<float*>(smem_raw);
  float* sK = sQ + ATT_BQ * SM::QLD;
  T* sV = reinterpret_cast<T*>(sK + ATT_BK * SM::KLD);
  float* sMask = reinterpret_cast<float*>(sV + ATT_BK * SM::VLD);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.H / a.KV;
  const int rows = a.Tq * G;
  const int bk = blockIdx.z, b = bk / a.KV, kvh = bk % a.KV;
  const int row0 = blockIdx.x * ATT_BQ;
  const int split = blockIdx.y, nsplit = gridDim.y;
  const int Ltot = a.LA + a.LB;
  const int kbeg = split * a.keys_per_split;
  const int kend = min(Ltot, kbeg + a.keys_per_split);

  // Q tile
  for (int i = tid; i < ATT_BQ * (HD / 4); i += 128) {
    int r = i / (HD / 4), ch = i % (HD / 4);
    int j = row0 + r;
    float* dst = sQ + r * SM::QLD + ch * 4;
    if (j < rows) {
      int t = j / G, h = kvh * G + (j - t * G);
      const float* src = a.q + (((size_t)b * a.Tq + t) * a.H + h) * HD + ch * 4;
      cp_async16(dst, src, 16);
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

  const float* kA = a.kA + ((size_t)b * a.KV + kvh) * a.LA * HD;
  const T* vA = a.vA + ((size_t)b * a.KV + kvh) * a.LA * HD;
  const float* kB = a.kB ? a.kB + ((size_t)b * a.KV + kvh) * a.LB * HD : nullptr;
  const T* vB = a.vB ? a.vB + ((size_t)b * a.KV + kvh) * a.LB * HD : nullptr;
  const float* mA = a.maskA ? a.maskA + (size_t)b * a.LA : nullptr;

  for (int k0 = kbeg; k0 < kend; k0 += ATT_BK) {
    __syncthreads();  // previous tile fully consumed
    for (int i = tid; i < ATT_BK * (HD / 4); i += 128) {
      int r = i / (HD / 4), ch = i % (HD / 4);
      int key = k0 + r;
      const float* src = key < a.LA ? kA + (size_t)key * HD : kB + (size_t)(key - a.LA) * HD;
      bool ok = key < kend;
      cp_async16(sK + r * SM::KLD + ch * 4, ok ? src + ch * 4 : a.q, ok ? 16 : 0);
    }
    for (int i = tid; i < ATT_BK * (HD / 8); i += 128) {
      int r = i / (HD / 8), ch = i % (HD / 8);
      int key = k0 + r;
      const T* src = key < a.LA ? vA + (size_t)key * HD : vB + (size_t)(key - a.LA) * HD;
      bool ok = key < kend;
      cp_async16(sV + r * SM::VLD + ch * 8, ok ? src + ch * 8 : (const T*)a.q, ok ? 16 : 0);
    }
    if (tid < ATT_BK) {
      int key = k0 + tid;
      float mv;
      if (key >= kend) mv = -1e30f;                 // outside this split: contributes 0
      else if (key < a.LA) mv = mA ? mA[key] : 0.f;  // prefix pad mask
      else mv = 0.f;                                 // suffix keys are always visible
      sMask[tid] = mv;
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();

    // S = Q K^T for this warp's 16 rows × 32 keys
    float s[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    const float* qw = sQ + (warp * 16) * SM::QLD;
#pragma unroll 4
    for (int kk = 0; kk < HD; kk += 8) {
      uint32_t af[4];
      af[0] = to_tf32(qw[gq * SM::QLD + kk + tq]);
      af[1] = to_tf32(qw[(gq + 8) * SM::QLD + kk + tq]);
      af[2] = to_tf32(qw[gq * SM::QLD + kk + tq + 4]);
      af[3] = to_tf32(qw[(gq + 8) * SM::QLD + kk + tq + 4]);
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        uint32_t bf[2];
        bf[0] = to_tf32(sK[(n * 8 + gq) * SM::KLD + kk + tq]);
        bf[1] = to_tf32(sK[(n * 8 + gq) * SM::KLD + kk + tq + 4]);
        mma1688_tf32(s[n], af, bf);
      }
    }
    // mask, online softmax
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      float mk0 = sMask[n * 8 + tq * 2], mk1 = sMask[n * 8 + tq * 2 + 1];
      s[n][0] += mk0;
      s[n][1] += mk1;
      s[n][2] += mk0;
      s[n][3] += mk1;
      mx[0] = fmaxf(mx[0], fmaxf(s[n][0], s[n][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[n][2], s[n][3]));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) corr[h] = expf(m_r[h] - mx[h]);
    uint32_t pf[2][4];  // P as two m16n8k16 A fragments (keys 0-15, 16-31)
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      float p0 = expf(s[n][0] - mx[0]), p1 = expf(s[n][1] - mx[0]);
      float p2 = expf(s[n][2] - mx[1]), p3 = expf(s[n][3] - mx[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      int kt = n >> 1, hi = n & 1;
      pf[kt][hi * 2 + 0] = Tr<T>::pack(p0, p1);
      pf[kt][hi * 2 + 1] = Tr<T>::pack(p2, p3);
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
    for (int kt = 0; kt < 2; ++kt) {
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t b0, b1, b2, b3;
        const T* p = sV + (kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * SM::VLD + i * 8 +
                     (lane >> 4) * 8;
        ldsm_x4_t(b0, b1, b2, b3, p);
        uint32_t bb0[2] = {b0, b1}, bb1[2] = {b2, b3};
        mma16816<T>(o[i], pf[kt], bb0);
        mma16816<T>(o[i + 1], pf[kt], bb1);
      }
    }
  }

  // write out
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    int j = row0 + warp * 16 + gq + h * 8;
    if (j >= rows) continue;
    int t = j / G, head = kvh * G + (j - t * G);
    if (nsplit == 1) {
      float inv = 1.f / l_r[h];
      T* dst = a.out + ((size_t)b * a.Tq + t) * a.H * HD + (size_t)head * HD;
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) {
        int d = i * 8 + tq * 2;
        *reinterpret_cast<uint32_t*>(dst + d) =
            Tr<T>::pack(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
      }
    } else {
      size_t base = ((size_t)bk * rows + j) * nsplit + split;
      float* dst = a.part_o + base * HD;
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) {
        int d = i * 8 + tq * 2;
        *reinterpret_cast<float2*>(dst + d) = make_float2(o[i][2 * h], o[i][2 * h + 1]);
      }
      if (tq == 0) {
        a.part_ml[base * 2 + 0] = m_r[h];
        a.part_ml[base * 2 + 1] = l_r[h];
      }
    }
  }
}

// Merge split partials: O = Σ_s e^{m_s - M} O_s / Σ_s e^{m_s - M} l_s, rounded to the model dtype.
// grid (rows, B·KV), block hd/2 threads (2 dims each).
template <typename T>
__global__ void attn_combine_kernel(AttnArgs<T> a, int hd, int nsplit) {
  const int G = a.H / a.KV, rows = a.Tq * G;
  const int j = blockIdx.x, bk = blockIdx.y, b = bk / a.KV, kvh = bk % a.KV;
  const size_t base = ((size_t)bk * rows + j) * nsplit;
  float M = -1e30f;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, a.part_ml[(base + s) * 2]);
  float L = 0.f;
  for (int s = 0; s < nsplit; ++s) L += expf(a.part_ml[(base + s) * 2] - M) * a.part_ml[(base + s) * 2 + 1];
  const float inv = 1.f / L;
  const int t = j / G, head = kvh * G + (j - t * G);
  T* dst = a.out + ((size_t)b * a.Tq + t) * a.H * hd + (size_t)head * hd;
  for (int d = threadIdx.x * 2; d < hd; d += blockDim.x * 2) {
    float o0 = 0.f, o1 = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      float w = expf(a.part_ml[(base + s) * 2] - M);
      float2 v = *reinterpret_cast<const float2*>(a.part_o + (base + s) * hd + d);
      o0 += w * v.x;
      o1 += w * v.y;
    }
    *reinterpret_cast<uint32_t*>(dst + d) = Tr<T>::pack(o0 * inv, o1 * inv);
  }
}

}  // namespace pi0
