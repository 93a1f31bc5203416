// embed_image (SigLIP So400m/14 + PaliGemma projector; reference python/mlc_vla/model/pi0/
// siglip.py:92-120, pi0_model.py:97-99) on the GPU: the patchify, LayerNorm and attention
// kernels and the epilogue functors of its projections. The projections run on the tcgen05 tile
// GEMM (gemm_tc.cuh); the attention (vattn_kernel below) works on heads padded to a multiple of
// 16 (72 -> 80, zero pad columns) so its MMA shapes apply; the out-projection weight gets the
// matching zero input columns at bind time.
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
  const float rden = __frcp_rn(den);  // (x − mean) / den below: div_by_rcp, bit-equal to IEEE
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
        const float n = div_by_rcp(__fsub_rn(v[c][k], mean), den, rden);
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

// ---- attention (siglip.py:58-72) ----------------------------------------------------------
// Bidirectional multi-head attention over the T patches of each image, with q (pre-scaled), k
// and v in the model dtype: the reference forms the logits from fp32 copies of the model-dtype
// q·scale and k, i.e. exact products of 16-bit values accumulated in fp32, which is what the
// 16-bit m16n8k16 tensor-core MMA with fp32 accumulation computes. fp32 online softmax (CUDA's
// fast exponential), probabilities rounded to the model dtype for P·V (fp32 accumulation), output
// normalised by 1/Σ and rounded once.
//   q [n, T, H, HD], k / v [n, H, T, HD] (HD = the padded head width, zero pad columns),
//   out [n, T, H·HD]. grid = (ceil(T / 64), 1, n·H), 128 threads: warp w owns query rows
//   16w .. 16w+15 of the tile; K/V tiles of 64 keys in a VA_ST-deep cp.async ring, all of them
//   requested up front when T ≤ 256 (one load latency per CTA instead of one per tile).
constexpr int VA_BQ = 64, VA_BK = 64, VA_ST = 4;
template <int HD>
struct VattnSmem {
  static constexpr int LD = HD + 8;  // 16-bit row stride: conflict-free ldmatrix rows
  static constexpr int Q_BYTES = VA_BQ * LD * 2;
  static constexpr int KV_BYTES = VA_BK * LD * 2;
  static constexpr int STAGE = 2 * KV_BYTES;
  static constexpr int BYTES = Q_BYTES + VA_ST * STAGE;
};

template <typename T, int HD>
__global__ void __launch_bounds__(128) vattn_kernel(const T* __restrict__ q,
                                                    const T* __restrict__ k,
                                                    const T* __restrict__ v, T* __restrict__ out,
                                                    int T_len, int H) {
  static_assert(HD % 16 == 0, "head width");
  using SM = VattnSmem<HD>;
  constexpr int LD = SM::LD, NT8 = VA_BK / 8, NK16 = VA_BK / 16, CH = HD / 8;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sQ = reinterpret_cast<T*>(smem_raw);
  auto sK = [&](int s) { return reinterpret_cast<T*>(smem_raw + SM::Q_BYTES + s * SM::STAGE); };
  auto sV = [&](int s) {
    return reinterpret_cast<T*>(smem_raw + SM::Q_BYTES + s * SM::STAGE + SM::KV_BYTES);
  };
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.z, img = bh / H, head = bh - img * H;
  const int row0 = blockIdx.x * VA_BQ;
  const T* kb = k + (size_t)bh * T_len * HD;
  const T* vb = v + (size_t)bh * T_len * HD;
  auto load_kv = [&](int s, int k0) {
    for (int i = tid; i < VA_BK * CH; i += 128) {
      const int r = i / CH, ch = i - r * CH, key = k0 + r;
      const bool ok = key < T_len;
      const size_t off = (size_t)(ok ? key : 0) * HD + ch * 8;
      cp_async16(sK(s) + r * LD + ch * 8, kb + off, ok ? 16 : 0);
      cp_async16(sV(s) + r * LD + ch * 8, vb + off, ok ? 16 : 0);
    }
  };
  pdl_trigger();
  pdl_wait();
  for (int i = tid; i < VA_BQ * CH; i += 128) {
    const int r = i / CH, ch = i - r * CH, t = row0 + r;
    const bool ok = t < T_len;
    cp_async16(sQ + r * LD + ch * 8, q + (((size_t)img * T_len + (ok ? t : 0)) * H + head) * HD + ch * 8,
               ok ? 16 : 0);
  }
  const int ntiles = (T_len + VA_BK - 1) / VA_BK;
  // VA_ST groups in flight (Q travels with tile 0; empty groups keep the count uniform)
#pragma unroll
  for (int t = 0; t < VA_ST; ++t) {
    if (t < ntiles) load_kv(t, t * VA_BK);
    cp_async_commit();
  }

  const int gq = lane >> 2, tq = lane & 3;
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-1e30f, -1e30f}, l_r[2] = {0.f, 0.f};
  uint32_t qf[HD / 16][4];

  for (int t = 0; t < ntiles; ++t) {
    const int s = t % VA_ST;
    cp_async_wait<VA_ST - 1>();  // tile t has landed (VA_ST + t groups committed so far)
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk)
        ldsm_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3],
                sQ + (warp * 16 + (lane & 15)) * LD + kk * 16 + (lane >> 4) * 8);
    }
    const T* kt = sK(s);
    const T* vt = sV(s);
    float sc[NT8][4];
#pragma unroll
    for (int n = 0; n < NT8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int j = 0; j < NT8; j += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3,
                kt + (j * 8 + (lane & 7) + ((lane >> 4) << 3)) * LD + kk * 16 + ((lane >> 3) & 1) * 8);
        const uint32_t bb0[2] = {b0, b1}, bb1[2] = {b2, b3};
        mma16816<T>(sc[j], qf[kk], bb0);
        mma16816<T>(sc[j + 1], qf[kk], bb1);
      }
    }
    if ((t + 1) * VA_BK > T_len) {  // keys past T contribute nothing
#pragma unroll
      for (int n = 0; n < NT8; ++n) {
        const int key = t * VA_BK + n * 8 + tq * 2;
        if (key >= T_len) sc[n][0] = sc[n][2] = -1e30f;
        if (key + 1 >= T_len) sc[n][1] = sc[n][3] = -1e30f;
      }
    }
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < NT8; ++n) {
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
    for (int h = 0; h < 2; ++h) corr[h] = __expf(m_r[h] - mx[h]);
    uint32_t pf[NK16][4];
#pragma unroll
    for (int n = 0; n < NT8; ++n) {
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
#pragma unroll
    for (int kt2 = 0; kt2 < NK16; ++kt2) {
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3,
                  vt + (kt2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + i * 8 + (lane >> 4) * 8);
        const uint32_t bb0[2] = {b0, b1}, bb1[2] = {b2, b3};
        mma16816<T>(o[i], pf[kt2], bb0);
        mma16816<T>(o[i + 1], pf[kt2], bb1);
      }
    }
    __syncthreads();  // every warp is done with slot s: refill it with tile t + VA_ST
    if (t + VA_ST < ntiles) load_kv(s, (t + VA_ST) * VA_BK);
    cp_async_commit();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int tok = row0 + warp * 16 + gq + h * 8;
    if (tok >= T_len) continue;
    const float inv = 1.f / l_r[h];
    T* dst = out + ((size_t)img * T_len + tok) * H * HD + (size_t)head * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
      *reinterpret_cast<uint32_t*>(dst + i * 8 + tq * 2) = Tr<T>::pack(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
  }
}

// ---- epilogues (operator() on a column pair; chunk32 on 32 columns with 16-byte accesses) ----

// patch embedding + position embedding: x = RN(RN(RN(acc) + b) + pos[row mod np]) (siglip.py:116-117)
template <typename T>
struct EpiBiasPos {
  T* x;
  int ld;
  const T* bias;
  const T* pos;
  int np;
  __device__ void prefetch(int r, int c) const {
    pf_l1(bias + c);
    pf_l1(pos + (size_t)(r % np) * ld + c);
  }
  __device__ void operator()(int r, int c, float v0, float v1) const {
    const T* pr = pos + (size_t)(r % np) * ld + c;
    const float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    const float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    *reinterpret_cast<uint32_t*>(x + (size_t)r * ld + c) =
        Tr<T>::pack(a + Tr<T>::f(pr[0]), b + Tr<T>::f(pr[1]));
  }
  __device__ bool chunk32(int r, int c0, const float* v) const {
    T* o = x + (size_t)r * ld + c0;
    const T* pr = pos + (size_t)(r % np) * ld + c0;
    if (!al16(o) || !al16(pr) || !al16(bias + c0)) return false;
    uint4 bv[4], pv[4], ov[4];
    ld16x4(bias + c0, bv);
    ld16x4(pr, pv);
    const T* be = reinterpret_cast<const T*>(bv);
    const T* pe = reinterpret_cast<const T*>(pv);
    uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float a = Tr<T>::r(Tr<T>::r(v[2 * j]) + Tr<T>::f(be[2 * j]));
      const float b = Tr<T>::r(Tr<T>::r(v[2 * j + 1]) + Tr<T>::f(be[2 * j + 1]));
      ow[j] = Tr<T>::pack(a + Tr<T>::f(pe[2 * j]), b + Tr<T>::f(pe[2 * j + 1]));
    }
    st16x4(o, ov);
    return true;
  }
};

// residual with a biased Linear: x = RN(x + RN(RN(acc) + b)) (siglip.py:86-87)
template <typename T>
struct EpiResidBias {
  T* x;
  int ld;
  const T* bias;
  __device__ void prefetch(int r, int c) const {
    pf_l1(x + (size_t)r * ld + c);
    pf_l1(bias + c);
  }
  __device__ void operator()(int r, int c, float v0, float v1) const {
    T* p = x + (size_t)r * ld + c;
    const float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    const float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    *reinterpret_cast<uint32_t*>(p) = Tr<T>::pack(Tr<T>::f(p[0]) + a, Tr<T>::f(p[1]) + b);
  }
  __device__ bool chunk32(int r, int c0, const float* v) const {
    T* p = x + (size_t)r * ld + c0;
    if (!al16(p) || !al16(bias + c0)) return false;
    uint4 xv[4], bv[4], ov[4];
    ld16x4(p, xv);
    ld16x4(bias + c0, bv);
    const T* xe = reinterpret_cast<const T*>(xv);
    const T* be = reinterpret_cast<const T*>(bv);
    uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float a = Tr<T>::r(Tr<T>::r(v[2 * j]) + Tr<T>::f(be[2 * j]));
      const float b = Tr<T>::r(Tr<T>::r(v[2 * j + 1]) + Tr<T>::f(be[2 * j + 1]));
      ow[j] = Tr<T>::pack(Tr<T>::f(xe[2 * j]) + a, Tr<T>::f(xe[2 * j + 1]) + b);
    }
    st16x4(p, ov);
    return true;
  }
};

// fc1 + GELU-tanh: h = RN(gelu(RN(RN(acc) + b))) (siglip.py:46-47; GELU evaluated in fp32)
template <typename T>
struct EpiBiasGelu {
  T* h;
  int ld;
  const T* bias;
  __device__ void prefetch(int, int c) const { pf_l1(bias + c); }
  __device__ void operator()(int r, int c, float v0, float v1) const {
    const float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    const float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    *reinterpret_cast<uint32_t*>(h + (size_t)r * ld + c) = Tr<T>::pack(gelu_tanh_f(a), gelu_tanh_f(b));
  }
  __device__ bool chunk32(int r, int c0, const float* v) const {
    T* o = h + (size_t)r * ld + c0;
    if (!al16(o) || !al16(bias + c0)) return false;
    uint4 bv[4], ov[4];
    ld16x4(bias + c0, bv);
    const T* be = reinterpret_cast<const T*>(bv);
    uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float a = Tr<T>::r(Tr<T>::r(v[2 * j]) + Tr<T>::f(be[2 * j]));
      const float b = Tr<T>::r(Tr<T>::r(v[2 * j + 1]) + Tr<T>::f(be[2 * j + 1]));
      ow[j] = Tr<T>::pack(gelu_tanh_f(a), gelu_tanh_f(b));
    }
    st16x4(o, ov);
    return true;
  }
};

// fused q/k/v with biases (siglip.py:58-66): column c of [q | k | v] (each `hid` wide, heads of
// hd) of token row r = image·T + t. q = RN(RN(RN(acc) + b) · RN(hd^-0.5)) -> [img, T, H, hdp];
// k and v = RN(RN(acc) + b) -> [img, H, T, hdp]; all in the model dtype. Columns [hd, hdp) of
// every head stay as the caller zeroed them.
template <typename T>
struct EpiVisionQkv {
  T* q;
  T* k;
  T* v;
  const T* bias;
  int T_len, H, hd, hdp;
  float qscale;  // hd^-0.5 rounded to the model dtype (the constant takes the tensor's dtype)
  __device__ void prefetch(int, int c) const { pf_l1(bias + c); }
  __device__ T* dst(int which, int img, int t, int head, int d) const {
    if (which == 0) return q + (((size_t)img * T_len + t) * H + head) * hdp + d;
    return (which == 1 ? k : v) + (((size_t)img * H + head) * T_len + t) * hdp + d;
  }
  __device__ void operator()(int r, int c, float v0, float v1) const {
    const int hid = H * hd;
    const int which = c / hid, cc = c - which * hid;
    const int head = cc / hd, d = cc - head * hd;
    const int img = r / T_len, t = r - img * T_len;
    float a = Tr<T>::r(Tr<T>::r(v0) + Tr<T>::f(bias[c]));
    float b = Tr<T>::r(Tr<T>::r(v1) + Tr<T>::f(bias[c + 1]));
    if (which == 0) {  // the product of two 16-bit values is exact in fp32: one rounding
      a *= qscale;
      b *= qscale;
    }
    *reinterpret_cast<uint32_t*>(dst(which, img, t, head, d)) = Tr<T>::pack(a, b);
  }
  // 32 columns of one of q / k / v (hid a multiple of 32); heads of hd a multiple of 8, so every
  // aligned group of 8 columns lies in one head and one 16-byte segment
  __device__ bool chunk32(int r, int c0, const float* acc) const {
    const int hid = H * hd;
    if (hid % 32 || hd % 8 || !al16(bias + c0)) return false;
    uint4 bv[4];
    ld16x4(bias + c0, bv);
    const T* be = reinterpret_cast<const T*>(bv);
    const int which = c0 / hid, cc0 = c0 - which * hid;
    const float sc = which == 0 ? qscale : 1.f;
    float y[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = Tr<T>::r(Tr<T>::r(acc[j]) + Tr<T>::f(be[j])) * sc;
    const int img = r / T_len, t = r - img * T_len;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int cc = cc0 + 8 * g, head = cc / hd, d = cc - head * hd;
      uint4 u;
      u.x = Tr<T>::pack(y[8 * g], y[8 * g + 1]);
      u.y = Tr<T>::pack(y[8 * g + 2], y[8 * g + 3]);
      u.z = Tr<T>::pack(y[8 * g + 4], y[8 * g + 5]);
      u.w = Tr<T>::pack(y[8 * g + 6], y[8 * g + 7]);
      *reinterpret_cast<uint4*>(dst(which, img, t, head, d)) = u;
    }
    return true;
  }
};

}  // namespace pi0
