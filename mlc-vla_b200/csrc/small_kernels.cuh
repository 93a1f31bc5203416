// Row-wise and skinny kernels of the M1 path: RMSNorm (plain and adaRMS), the GEMV that
// streams the time-MLP and adaRMS-modulation weights, the action in/out projections (K or N
// equal to action_dim) with the Euler update fused, weight repacking and group quantisation.
#pragma once

#include "common.cuh"

namespace pi0 {

// ---- RMSNorm (gemma_dual.py:75-89) -------------------------------------------------------
// normed = x / sqrt(Σx²/W + eps) in fp32; plain: ·(1 + w); ada: ·(1 + scale) + shift, where
// (scale, shift) = mod[0:W], mod[W:2W] of the modulation row of the request's group
// (mod + (row / rows_per_mod) · mod_stride). One warp per row; output in the model dtype.
template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, T* __restrict__ out, int rows, int W,
                               float eps, const T* __restrict__ w, const T* __restrict__ mod,
                               int rows_per_mod, int mod_stride) {
  int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + (size_t)row * W;
  float ss = 0.f;
  for (int i = lane * 2; i < W; i += 64) {
    float a = Tr<T>::f(xr[i]), b = Tr<T>::f(xr[i + 1]);
    ss += a * a + b * b;
  }
  ss = warp_sum(ss);
  const float denom = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)W), eps));
  const T* m = mod ? mod + (size_t)(row / rows_per_mod) * mod_stride : nullptr;
  T* o = out + (size_t)row * W;
  for (int i = lane * 2; i < W; i += 64) {
    float r[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float n = __fdiv_rn(Tr<T>::f(xr[i + e]), denom);
      if (m) {
        r[e] = __fadd_rn(__fmul_rn(n, __fadd_rn(1.f, Tr<T>::f(m[i + e]))), Tr<T>::f(m[W + i + e]));
      } else {
        r[e] = __fmul_rn(n, __fadd_rn(1.f, Tr<T>::f(w[i + e])));
      }
    }
    *reinterpret_cast<uint32_t*>(o + i) = Tr<T>::pack(r[0], r[1]);
  }
}

// ---- GEMV for M ≤ GEMV_MMAX rows (time MLP, adaRMS modulations) --------------------------
// y[m, n] = act(round(round(Σ_k x[m,k]·W[n,k]) + b[n])), act ∈ {identity, silu→round}.
// One warp per weight row; 16-byte coalesced weight loads, four in flight per lane; x staged
// in shared memory as fp32. Each output's reduction order depends only on K, not on M, so the
// hoisted all-steps modulation (M = N steps) equals N single-step launches bit for bit.
constexpr int GEMV_MMAX = 16;

template <typename T>
__global__ void __launch_bounds__(256) gemv_kernel(const T* __restrict__ x, int M, int K,
                                                   const T* __restrict__ W,
                                                   const T* __restrict__ bias, int N,
                                                   T* __restrict__ y, int ldy, int act_silu) {
  extern __shared__ float sx[];  // [M][K]
  for (int i = threadIdx.x; i < M * K; i += blockDim.x) sx[i] = Tr<T>::f(x[i]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  for (int n = blockIdx.x * warps + threadIdx.x / 32; n < N; n += gridDim.x * warps) {
    const T* wr = W + (size_t)n * K;
    float acc[GEMV_MMAX];
#pragma unroll
    for (int m = 0; m < GEMV_MMAX; ++m) acc[m] = 0.f;
    for (int k0 = lane * 8; k0 < K; k0 += 32 * 8 * 4) {
      uint4 wv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int k = k0 + u * 256;
        wv[u] = k < K ? __ldg(reinterpret_cast<const uint4*>(wr + k)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int k = k0 + u * 256;
        if (k >= K) break;
        const T* wh = reinterpret_cast<const T*>(&wv[u]);
        float wf[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) wf[e] = Tr<T>::f(wh[e]);
#pragma unroll
        for (int m = 0; m < GEMV_MMAX; ++m) {
          if (m < M) {
            const float* xs = sx + m * K + k;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[m] = fmaf(wf[e], xs[e], acc[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < GEMV_MMAX; ++m) {
      if (m < M) {
        float v = warp_sum(acc[m]);
        if (lane == 0) {
          float r = Tr<T>::r(v);
          if (bias) r = Tr<T>::r(r + Tr<T>::f(bias[n]));
          if (act_silu) r = Tr<T>::r(silu_f(r));
          y[(size_t)m * ldy + n] = Tr<T>::t(r);
        }
      }
    }
  }
}

// ---- action_in_proj (pi0_model.py:154,187): emb = round(round(x·Wᵀ) + b), K = action_dim ----
// x is the model-dtype x_t (XF32 = false) or the fp32 Euler state cast to the model dtype.
template <typename T, bool XF32>
__global__ void action_in_kernel(const void* __restrict__ xin, int rows, int D,
                                 const T* __restrict__ W, const T* __restrict__ b, int Wd,
                                 T* __restrict__ out) {
  int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * Wd) return;
  int r = idx / Wd, n = idx - r * Wd;
  float acc = 0.f;
  for (int k = 0; k < D; ++k) {
    float xv = XF32 ? Tr<T>::r(reinterpret_cast<const float*>(xin)[(size_t)r * D + k])
                    : Tr<T>::f(reinterpret_cast<const T*>(xin)[(size_t)r * D + k]);
    acc = fmaf(xv, Tr<T>::f(W[(size_t)n * D + k]), acc);
  }
  float y = Tr<T>::r(Tr<T>::r(acc) + Tr<T>::f(b[n]));
  out[idx] = Tr<T>::t(y);
}

// ---- action_out_proj (pi0_model.py:162-163,192-193) ---------------------------------------
// v = float(round(round(h·Wᵀ) + b)); euler = 0: v_out = v; euler = 1: x = x + dt·v (fp32,
// no fused multiply-add, as numpy and the reference's separate multiply and add).
template <typename T>
__global__ void action_out_kernel(const T* __restrict__ h, int rows, int Wd,
                                  const T* __restrict__ W, const T* __restrict__ b, int D,
                                  float* __restrict__ out, int euler, float dt) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows * D) return;
  int r = warp / D, d = warp - r * D;
  const T* hr = h + (size_t)r * Wd;
  const T* wr = W + (size_t)d * Wd;
  float acc = 0.f;
  for (int k = lane * 2; k < Wd; k += 64)
    acc += Tr<T>::f(hr[k]) * Tr<T>::f(wr[k]) + Tr<T>::f(hr[k + 1]) * Tr<T>::f(wr[k + 1]);
  acc = warp_sum(acc);
  if (lane == 0) {
    float v = Tr<T>::r(Tr<T>::r(acc) + Tr<T>::f(b[d]));
    float* o = out + (size_t)r * D + d;
    if (euler) *o = __fadd_rn(*o, __fmul_rn(dt, v));
    else *o = v;
  }
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

}  // namespace pi0
