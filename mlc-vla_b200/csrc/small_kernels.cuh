// Row-wise kernels of the M1 path: RMSNorm (plain and adaRMS), the action in/out projections
// (K or N equal to action_dim) with the Euler update fused, weight repacking and group
// quantisation.
#pragma once

#include "common.cuh"

namespace pi0 {

// ---- RMSNorm (gemma_dual.py:75-89) -------------------------------------------------------
// normed = x / sqrt(Σx²/W + eps) in fp32; plain: ·(1 + w); ada: ·(1 + scale) + shift, where
// (scale, shift) = mod[0:W], mod[W:2W] of the modulation row of the request's group
// (mod + (row / rows_per_mod) · mod_stride). One warp per row; every lane issues all of its
// 16-byte loads before using any (W ≤ 32·8·RMS_CHUNKS). Output in the model dtype.
constexpr int RMS_CHUNKS = 16;

template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, T* __restrict__ out, int rows, int W,
                               float eps, const T* __restrict__ w, const T* __restrict__ mod,
                               int rows_per_mod, int mod_stride) {
  pdl_wait();
  pdl_trigger();
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nch = W / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * W);
  uint4 xv[RMS_CHUNKS];
#pragma unroll
  for (int c = 0; c < RMS_CHUNKS; ++c)
    if (c * 32 + lane < nch) xv[c] = __ldg(xr + c * 32 + lane);
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < RMS_CHUNKS; ++c)
    if (c * 32 + lane < nch) {
      const T* e = reinterpret_cast<const T*>(&xv[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float f = Tr<T>::f(e[j]);
        ss += f * f;
      }
    }
  ss = warp_sum(ss);
  const float denom = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)W), eps));
  const float rden = __frcp_rn(denom);  // x / denom below: div_by_rcp, bit-equal to IEEE division
  const T* m = mod ? mod + (size_t)(row / rows_per_mod) * mod_stride : nullptr;
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)row * W);
#pragma unroll
  for (int c = 0; c < RMS_CHUNKS; ++c) {
    const int ch = c * 32 + lane;
    if (ch >= nch) continue;
    const T* e = reinterpret_cast<const T*>(&xv[c]);
    uint4 a, b;
    if (m) {
      a = __ldg(reinterpret_cast<const uint4*>(m) + ch);          // scale
      b = __ldg(reinterpret_cast<const uint4*>(m + W) + ch);      // shift
    } else {
      a = __ldg(reinterpret_cast<const uint4*>(w) + ch);
    }
    const T* sa = reinterpret_cast<const T*>(&a);
    const T* sb = reinterpret_cast<const T*>(&b);
    uint32_t res[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float r2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int q = 2 * j + h;
        float n = div_by_rcp(Tr<T>::f(e[q]), denom, rden);
        r2[h] = m ? __fadd_rn(__fmul_rn(n, __fadd_rn(1.f, Tr<T>::f(sa[q]))), Tr<T>::f(sb[q]))
                  : __fmul_rn(n, __fadd_rn(1.f, Tr<T>::f(sa[q])));
      }
      res[j] = Tr<T>::pack(r2[0], r2[1]);
    }
    o[ch] = make_uint4(res[0], res[1], res[2], res[3]);
  }
}

// ---- action_in_proj (pi0_model.py:154,187): emb = round(round(x·Wᵀ) + b), K = action_dim ----
// x is the model-dtype x_t (XF32 = false) or the fp32 Euler state cast to the model dtype.
// One block per activation row: the row is staged in shared memory, each thread produces
// Wd / blockDim outputs.
// Also emits the row's Σ emb² into ssq[r·ssq_parts] (other parts zero) for the first norm-fused
// GEMM when ssq is not null.
template <typename T, bool XF32>
__global__ void action_in_kernel(const void* __restrict__ xin, int rows, int D,
                                 const T* __restrict__ W, const T* __restrict__ b, int Wd,
                                 T* __restrict__ out, float* __restrict__ ssq, int ssq_parts) {
  extern __shared__ float sxr[];
  __shared__ float s_red[32];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  for (int k = threadIdx.x; k < D; k += blockDim.x)
    sxr[k] = XF32 ? Tr<T>::r(reinterpret_cast<const float*>(xin)[(size_t)r * D + k])
                  : Tr<T>::f(reinterpret_cast<const T*>(xin)[(size_t)r * D + k]);
  __syncthreads();
  float sq = 0.f;
  for (int n = threadIdx.x; n < Wd; n += blockDim.x) {
    const T* wr = W + (size_t)n * D;
    float acc = 0.f;
#pragma unroll 8
    for (int k = 0; k < D; ++k) acc = fmaf(sxr[k], Tr<T>::f(wr[k]), acc);
    const float y = Tr<T>::r(Tr<T>::r(acc) + Tr<T>::f(b[n]));
    out[(size_t)r * Wd + n] = Tr<T>::t(y);
    sq += y * y;
  }
  if (ssq) {
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < ssq_parts) {
      float t = 0.f;
      if (threadIdx.x == 0)
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_red[w];
      ssq[(size_t)r * ssq_parts + threadIdx.x] = t;
    }
  }
}

// ---- final adaRMSNorm + action_out_proj (gemma_dual.py:432; pi0_model.py:162-163,192-193) --
// h = round(norm(x; mod)) with the final norm's modulation (scale, shift); v = float(round(
// round(h·Wᵀ) + b)); euler = 0: v_out = v; euler = 1: x = x + dt·v (fp32, no fused
// multiply-add, as numpy and the reference's separate multiply and add). One warp per (row, d).
// One warp: output d of activation row r (the body of action_out_kernel).
template <typename T>
__device__ __forceinline__ void action_out_warp(const T* __restrict__ h, int r, int d, int Wd,
                                                const T* __restrict__ mod, float eps,
                                                const T* __restrict__ W, const T* __restrict__ b,
                                                int D, float* __restrict__ out, int euler,
                                                float dt, int lane) {
  const uint4* hr = reinterpret_cast<const uint4*>(h + (size_t)r * Wd);
  const uint4* wr = reinterpret_cast<const uint4*>(W + (size_t)d * Wd);
  const int nch = Wd / 8;
  uint4 hv[RMS_CHUNKS], wv[RMS_CHUNKS];
#pragma unroll
  for (int c = 0; c < RMS_CHUNKS; ++c)
    if (c * 32 + lane < nch) {
      hv[c] = hr[c * 32 + lane];
      wv[c] = __ldg(wr + c * 32 + lane);
    }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < RMS_CHUNKS; ++c)
    if (c * 32 + lane < nch) {
      const T* a = reinterpret_cast<const T*>(&hv[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float f = Tr<T>::f(a[j]);
        ss += f * f;
      }
    }
  ss = warp_sum(ss);
  const float denom = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)Wd), eps));
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < RMS_CHUNKS; ++c)
    if (c * 32 + lane < nch) {
      const int ch = c * 32 + lane;
      const uint4 sc = reinterpret_cast<const uint4*>(mod)[ch];
      const uint4 sh = reinterpret_cast<const uint4*>(mod + Wd)[ch];
      const T* a = reinterpret_cast<const T*>(&hv[c]);
      const T* es = reinterpret_cast<const T*>(&sc);
      const T* eh = reinterpret_cast<const T*>(&sh);
      const T* bb = reinterpret_cast<const T*>(&wv[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float n = __fdiv_rn(Tr<T>::f(a[j]), denom);
        const float hn = Tr<T>::r(__fadd_rn(__fmul_rn(n, __fadd_rn(1.f, Tr<T>::f(es[j]))), Tr<T>::f(eh[j])));
        acc = fmaf(hn, Tr<T>::f(bb[j]), acc);
      }
    }
  acc = warp_sum(acc);
  if (lane == 0) {
    float v = Tr<T>::r(Tr<T>::r(acc) + Tr<T>::f(b[d]));
    float* o = out + (size_t)r * D + d;
    if (euler) *o = __fadd_rn(*o, __fmul_rn(dt, v));
    else *o = v;
  }
}

template <typename T>
__global__ void action_out_kernel(const T* __restrict__ h, int rows, int Wd,
                                  const T* __restrict__ mod, float eps,
                                  const T* __restrict__ W, const T* __restrict__ b, int D,
                                  float* __restrict__ out, int euler, float dt) {
  pdl_wait();
  pdl_trigger();
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows * D) return;
  int r = warp / D, d = warp - r * D;
  action_out_warp<T>(h, r, d, Wd, mod, eps, W, b, D, out, euler, dt, lane);
}

// ---- weight repack: dst row i = src row idx[i] (rows of K elements of 16-bit type) -------
__global__ void gather_rows_kernel(uint16_t* __restrict__ dst, const uint16_t* __restrict__ src,
                                   const int* __restrict__ idx, int rows, int K) {
  int r = blockIdx.x;
  if (r >= rows) return;
  const uint16_t* s = src + (size_t)idx[r] * K;
  uint16_t* d = dst + (size_t)r * K;
  if ((K & 7) == 0) {
    for (int i = threadIdx.x * 8; i < K; i += blockDim.x * 8)
      *reinterpret_cast<uint4*>(d + i) = *reinterpret_cast<const uint4*>(s + i);
  } else {
    for (int i = threadIdx.x; i < K; i += blockDim.x) d[i] = s[i];
  }
}

// ---- group quantisation (quant.py:176-266), one thread per (row, group) -------------------
// Every arithmetic step rounds to the model dtype as the reference's TE compute does: scale =
// round(max|w| / max_int); t = round(round(w / scale) + max_int); code = clamp(round-half-away
// (t), 0, 2·max_int) with max(NaN, 0) = 0.
template <typename T>
__global__ void quantize_kernel(const T* __restrict__ w, int64_t n_out, int64_t K, int G,
                                int bits, int epw, int maxint, uint32_t* __restrict__ qw,
                                T* __restrict__ qs) {
  int64_t ng = (K + G - 1) / G;
  int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= n_out * ng) return;
  int64_t n = id / ng, gi = id - n * ng;
  const T* wr = w + n * K;
  int64_t k0 = gi * G;
  float mx = -INFINITY;
  for (int i = 0; i < G; ++i)
    if (k0 + i < K) mx = fmaxf(mx, fabsf(Tr<T>::f(wr[k0 + i])));
  float s = Tr<T>::r(__fdiv_rn(mx, (float)maxint));
  qs[n * ng + gi] = Tr<T>::t(s);
  const int words = G / epw;
  uint32_t* out = qw + n * (ng * words) + gi * words;
  for (int wd = 0; wd < words; ++wd) {
    uint32_t acc = 0;
    for (int r = 0; r < epw; ++r) {
      int64_t k = k0 + wd * epw + r;
      uint32_t code = 0;
      if (k < K) {
        float t = Tr<T>::r(__fdiv_rn(Tr<T>::f(wr[k]), s));
        t = Tr<T>::r(__fadd_rn(t, (float)maxint));
        t = copysignf(floorf(fabsf(t) + 0.5f), t);
        t = t > 0.f ? t : 0.f;
        t = t < (float)(2 * maxint) ? t : (float)(2 * maxint);
        code = (uint32_t)t;
      }
      acc |= code << (r * bits);
    }
    out[wd] = acc;
  }
}

template <typename T>
__global__ void dequantize_kernel(const uint32_t* __restrict__ qw, const T* __restrict__ qs,
                                  int64_t n_out, int64_t K, int G, int bits, int epw, int maxint,
                                  T* __restrict__ w) {
  int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= n_out * K) return;
  int64_t n = id / K, k = id - n * K;
  int64_t ng = (K + G - 1) / G;
  int64_t words_per_row = ng * (G / epw);
  uint32_t word = qw[n * words_per_row + k / epw];
  uint32_t code = (word >> ((k % epw) * bits)) & ((1u << bits) - 1u);
  float s = Tr<T>::f(qs[n * ng + k / G]);
  w[id] = Tr<T>::t(((float)code - (float)maxint) * s);
}

// Language embedding (pi0_model.py:101-104, embed_language): out[t, :] = RN(table[id_t, :] · c)
// with c = sqrt(width) rounded to the model dtype (the Python constant takes the tensor's dtype),
// the product exact in fp32 and rounded once. One block per token, 16-byte chunks; an id outside
// [0, vocab) gives a zero row and sets *err to 1 (err may be null).
template <typename T>
__global__ void embed_language_kernel(const T* __restrict__ table, int64_t vocab, int width,
                                      const int* __restrict__ ids, T* __restrict__ out, float c,
                                      int* err) {
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool in = id >= 0 && (int64_t)id < vocab;
  if (!in && threadIdx.x == 0 && err) atomicExch(err, 1);
  const uint4* src = reinterpret_cast<const uint4*>(table + (in ? (size_t)id : 0) * width);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * width);
  for (int i = threadIdx.x; i < width / 8; i += blockDim.x) {
    uint4 v = in ? src[i] : make_uint4(0, 0, 0, 0);
    const T* e = reinterpret_cast<const T*>(&v);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = Tr<T>::pack(Tr<T>::f(e[2 * j]) * c, Tr<T>::f(e[2 * j + 1]) * c);
    dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// a / b through div_by_rcp (common.cuh), for the bit-for-bit comparison with IEEE division
__global__ void div_check_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                 float* __restrict__ out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = div_by_rcp(a[i], b[i], __frcp_rn(b[i]));
}

// Model-dtype copy of an fp32 K cache at half scale, the operand of the tensor-core attention
// (attention_tc.cuh): k16[i] = RN(0.5·k[i]); for fp32 logits also the lo part
// k16lo[i] = RN(0.5·k[i] − k16[i]) (k16lo may be null). n4 = elements / 4.
template <typename T>
__global__ void keys_half_scale_kernel(const float4* __restrict__ k, T* __restrict__ k16,
                                       T* __restrict__ k16lo, size_t n4) {
  // launched with programmatic dependent launch: the cache may still be being written by the
  // kernel before (a prefill on the same stream)
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 v = k[i];
  const float h[4] = {0.5f * v.x, 0.5f * v.y, 0.5f * v.z, 0.5f * v.w};
  uint2 o;
  o.x = Tr<T>::pack(h[0], h[1]);
  o.y = Tr<T>::pack(h[2], h[3]);
  reinterpret_cast<uint2*>(k16)[i] = o;
  if (k16lo) {
    o.x = Tr<T>::pack(h[0] - Tr<T>::r(h[0]), h[1] - Tr<T>::r(h[1]));
    o.y = Tr<T>::pack(h[2] - Tr<T>::r(h[2]), h[3] - Tr<T>::r(h[3]));
    reinterpret_cast<uint2*>(k16lo)[i] = o;
  }
}

}  // namespace pi0
