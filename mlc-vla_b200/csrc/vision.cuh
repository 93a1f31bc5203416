// embed_image (SigLIP So400m/14 + PaliGemma projector; reference python/mlc_vla/model/pi0/
// siglip.py:92-120, pi0_model.py:97-99) on the GPU: the patchify and LayerNorm kernels and the
// epilogue functors of its projections. The projections themselves run on the tile GEMM engines
// (gemm_tc.cuh for ≥ 128 rows) and the attention on attention.cuh (fp32 logits), with the head
// dimension padded to a multiple of 16 (72 -> 80, zero pad columns) so the attention's shapes
// are supported; the out-projection weight gets matching zero input columns at bind time.
#pragma once

#include "common.cuh"
#include "gemm_mma.cuh"

namespace pi0 {

// siglip.py:104-114 (channels-last image [B, H, W, C]): out[b·np + py·side + px][(i·p + j)·C + c] =
// image[b][py·p + i][px·p + j][c], columns [p·p·C, kpad) zero. One thread per output element.
template <typename T>
__global__ void patchify_kernel(const T* __restrict__ image, T* __restrict__ out, int nb, int img,
                                int patch, int C, int kpad) {
  pdl_wait();
  pdl_trigger();
  const int side = img / patch, np = side * side;
  const int64_t total = (int64_t)nb * np * kpad;
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= total) return;
  const int k = (int)(id % kpad);
  const int64_t row = id / kpad;
  const int b = (int)(row / np), pidx = (int)(row % np);
  const int py = pidx / side, px = pidx % side;
  T v = Tr<T>::t(0.f);
  if (k < patch * patch * C) {
    const int c = k % C, ij = k / C, i = ij / patch, j = ij % patch;
    v = image[(((int64_t)b * img + py * patch + i) * img + px * patch + j) * C + c];
  }
  out[id] = v;
}

// LayerNorm in fp32 (siglip.py:23-37): mean, biased variance, (x − mean) / sqrt(var + eps) · w + b,
// rounded once to the model dtype. One warp per row (W a multiple of 8, W ≤ 32·8·LN_CHUNKS).
constexpr int LN_CHUNKS = 8;
template <typename T>
__global__ void layernorm_kernel(const T* __restrict__ x, T* __restrict__ out, int rows, int W,
                                 float eps, const T* __restrict__ w, const T* __restrict__ b) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nch = W / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * W);
  float v[LN_CHUNKS][8];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < LN_CHUNKS; ++c) {
    const int ch = c * 32 + lane;
    if (ch < nch) {
      const uint4 u = xr[ch];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[c][j] = Tr<T>::f(e[j]);
        s += v[c][j];
      }
    }
  }
  const float mean = __fdiv_rn(warp_sum(s), (float)W);
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < LN_CHUNKS; ++c)
    if (c * 32 + lane < nch)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = __fsub_rn(v[c][j], mean);
        q = fmaf(d, d, q);
      }
  const float var = __fdiv_rn(warp_sum(q), (float)W);
  const float den = sqrtf(__fadd_rn(var, eps));
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)row * W);
#pragma unroll
  for (int c = 0; c < LN_CHUNKS; ++c) {
    const int ch = c * 32 + lane;
    if (ch >= nch) continue;
    const uint4 wu = reinterpret_cast<const uint4*>(w)[ch];
    const uint4 bu = reinterpret_cast<const uint4*>(b)[ch];
    const T* we = reinterpret_cast<const T*>(&wu);
    const T* be = reinterpret_cast<const T*>(&bu);
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float y[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int k = 2 * j + h;
        const float n = __fdiv_rn(__fsub_rn(v[c][k], mean), den);
        y[h] = __fadd_rn(__fmul_rn(n, Tr<T>::f(we[k])), Tr<T>::f(be[k]));
      }
      r[j] = Tr<T>::pack(y[0], y[1]);
    }
    o[ch] = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

// Zero-filled column re-layout at bind time: dst row r, column group g (of `groups`), element d <
// src_group = src row r, column g·src_group + d; the dst group stride is dst_group (≥ src_group).
// Pads the patch-embedding K (588 -> 640) and the out-projection's per-head input columns.
__global__ void regroup_cols_kernel(uint16_t* __restrict__ dst, int dst_ld,
                                    const uint16_t* __restrict__ src, int src_ld, int rows,
                                    int groups, int src_group, int dst_group) {
  const int64_t total = (int64_t)rows * groups * src_group;
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= total) return;
  const int d = (int)(id % src_group);
  const int64_t rg = id / src_group;
  const int g = (int)(rg % groups), r = (int)(rg / groups);
  dst[(size_t)r * dst_ld + (size_t)g * dst_group + d] = src[(size_t)r * src_ld + (size_t)g * src_group + d];
}

// ---- epilogues (operator() on a column pair, chunk32 declined: the per-pair path runs) ----

// patch embedding + position embedding: x = RN(RN(RN(acc) + b) + pos[row mod np]) (siglip.py:116-117)
template <typename T>
struct EpiBiasPos {
  T* x;
  int ld;
  const T* bias;
  const T* pos;
  int np;
  __device__ void prefetch(int, int) const {}
  __device__ void operator()(int r, int c, float v0, float v1) const {
    const T* pr = pos + (size_t)(r % np) * ld + c;
    const float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    const float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    *reinterpret_cast<uint32_t*>(x + (size_t)r * ld + c) =
        Tr<T>::pack(a + Tr<T>::f(pr[0]), b + Tr<T>::f(pr[1]));
  }
  __device__ bool chunk32(int, int, const float*) const { return false; }
};

// residual with a biased Linear: x = RN(x + RN(RN(acc) + b)) (siglip.py:86-87)
template <typename T>
struct EpiResidBias {
  T* x;
  int ld;
  const T* bias;
  __device__ void prefetch(int r, int c) const { pf_l1(x + (size_t)r * ld + c); }
  __device__ void operator()(int r, int c, float v0, float v1) const {
    T* p = x + (size_t)r * ld + c;
    const float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    const float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    *reinterpret_cast<uint32_t*>(p) = Tr<T>::pack(Tr<T>::f(p[0]) + a, Tr<T>::f(p[1]) + b);
  }
  __device__ bool chunk32(int, int, const float*) const { return false; }
};

// fc1 + GELU-tanh: h = RN(gelu(RN(RN(acc) + b))) (siglip.py:46-47; GELU evaluated in fp32)
template <typename T>
struct EpiBiasGelu {
  T* h;
  int ld;
  const T* bias;
  __device__ void prefetch(int, int) const {}
  __device__ void operator()(int r, int c, float v0, float v1) const {
    const float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    const float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    *reinterpret_cast<uint32_t*>(h + (size_t)r * ld + c) = Tr<T>::pack(gelu_tanh_f(a), gelu_tanh_f(b));
  }
  __device__ bool chunk32(int, int, const float*) const { return false; }
};

// fused q/k/v with biases (siglip.py:58-66): column c of [q | k | v] (each `hid` wide, heads of
// hd) of token row r = image·T + t. q = RN(RN(RN(acc) + b) · RN(hd^-0.5)) -> fp32 [img, T, H, hdp];
// k = RN(RN(acc) + b) -> fp32 [img, H, T, hdp]; v (the same) -> model dtype [img, H, T, hdp].
// Columns [hd, hdp) of every head stay as the caller zeroed them.
template <typename T>
struct EpiVisionQkv {
  float* q;
  float* k;
  T* v;
  const T* bias;
  int T_len, H, hd, hdp;
  float qscale;  // hd^-0.5 rounded to the model dtype (the constant takes the tensor's dtype)
  __device__ void prefetch(int, int) const {}
  __device__ void operator()(int r, int c, float v0, float v1) const {
    const int hid = H * hd;
    const int which = c / hid, cc = c - which * hid;
    const int head = cc / hd, d = cc - head * hd;
    const int img = r / T_len, t = r - img * T_len;
    const float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    const float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    if (which == 0) {
      float* p = q + (((size_t)img * T_len + t) * H + head) * hdp + d;
      p[0] = Tr<T>::r(a * qscale);
      p[1] = Tr<T>::r(b * qscale);
    } else {
      const size_t o = (((size_t)img * H + head) * T_len + t) * hdp + d;
      if (which == 1) {
        k[o] = a;
        k[o + 1] = b;
      } else {
        *reinterpret_cast<uint32_t*>(v + o) = Tr<T>::pack(a, b);
      }
    }
  }
  __device__ bool chunk32(int, int, const float*) const { return false; }
};

}  // namespace pi0
