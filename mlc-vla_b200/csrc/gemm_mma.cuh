// Tiled GEMM  C[M,N] = A[M,K] · W[N,K]^T  (A and W row-major, K contiguous — the reference's
// nn.Linear layout [out, in]) on warp-level mma.sync tensor cores, fp32 accumulation, with the
// epilogue fused: every Linear of the π0.5 backbone ends in one of the epilogue functors below
// (RoPE + K/V-cache write for q/k/v, residual add, gated residual add, GeGLU).
//
// Split-K: gridDim.z > 1 splits K; every split writes its fp32 partial tile to a workspace and
// the last split to arrive (atomic ticket per output tile) sums the partials in split order and
// runs the epilogue, so results do not depend on arrival order. The ticket is reset by that
// last split, so the same workspace is reusable (and CUDA-graph replayable) without clearing.
#pragma once

#include "common.cuh"

namespace pi0 {

template <typename T>
struct GemmArgs {
  const T* A;
  int lda;
  const T* W;
  int ldw;
  int M, N, K;
  int k_split_len;   // K range of one split (multiple of 32)
  float* ws;         // split-K partials [splits][M][N]
  int* tickets;      // one int per output tile, zero between launches
};

// ---- epilogues: operator()(row, col, v(col), v(col+1)); col is even ----
// chunk32(row, col0, v[32]) is the same epilogue for 32 consecutive columns (col0 a multiple of
// 32, all columns valid): every global operand of the chunk is loaded with 16-byte vectors before
// any result is stored, so a read-modify-write epilogue costs one memory round trip per chunk
// instead of one per column pair (a store to the array an operand is read from orders the next
// load after it). It returns false, having done nothing, when a pointer is not 16-byte aligned;
// the caller then runs operator() per pair.

__device__ __forceinline__ bool al16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}
template <typename T>
__device__ __forceinline__ void ld16x4(const T* p, uint4 (&v)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = reinterpret_cast<const uint4*>(p)[i];
}
template <typename T>
__device__ __forceinline__ void st16x4(T* p, const uint4 (&v)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(p)[i] = v[i];
}


// y = round(round(acc) + bias) (nn.Linear: matmul, then bias add; bias optional), then
// optionally round(silu(y)) (the time MLP, pi0_model.py:106-109), stored in the model dtype.
template <typename T>
struct EpiStore {
  T* out;
  int ldo;
  const T* bias;
  int silu = 0;
  __device__ void prefetch(int, int c) const {
    if (bias) pf_l1(bias + c);
  }
  __device__ void operator()(int r, int c, float v0, float v1) const {
    float a = Tr<T>::r(v0), b = Tr<T>::r(v1);
    if (bias) {
      a = Tr<T>::r(a + Tr<T>::f(bias[c]));
      b = Tr<T>::r(b + Tr<T>::f(bias[c + 1]));
    }
    if (silu) {
      a = silu_f(a);
      b = silu_f(b);
    }
    *reinterpret_cast<uint32_t*>(out + (size_t)r * ldo + c) = Tr<T>::pack(a, b);
  }
  __device__ bool chunk32(int r, int c0, const float* v) const {
    T* o = out + (size_t)r * ldo + c0;
    if (!al16(o) || (bias && !al16(bias + c0))) return false;
    uint4 bv[4];
    if (bias) ld16x4(bias + c0, bv);
    const T* be = reinterpret_cast<const T*>(bv);
    uint4 ov[4];
    uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float a = Tr<T>::r(v[2 * j]), b = Tr<T>::r(v[2 * j + 1]);
      if (bias) {
        a = Tr<T>::r(a + Tr<T>::f(be[2 * j]));
        b = Tr<T>::r(b + Tr<T>::f(be[2 * j + 1]));
      }
      if (silu) {
        a = silu_f(a);
        b = silu_f(b);
      }
      ow[j] = Tr<T>::pack(a, b);
    }
    st16x4(o, ov);
    return true;
  }
};

template <typename T>
struct EpiResid {  // prefix residual (gemma_dual.py:338,340): x = round(x + round(acc))
  T* x;
  int ldx;
  __device__ void prefetch(int r, int c) const { pf_l1(x + (size_t)r * ldx + c); }
  __device__ void operator()(int r, int c, float v0, float v1) const {
    T* p = x + (size_t)r * ldx + c;
    float a = Tr<T>::f(p[0]) + Tr<T>::r(v0);
    float b = Tr<T>::f(p[1]) + Tr<T>::r(v1);
    *reinterpret_cast<uint32_t*>(p) = Tr<T>::pack(a, b);
  }
  __device__ bool chunk32(int r, int c0, const float* v) const {
    T* p = x + (size_t)r * ldx + c0;
    if (!al16(p)) return false;
    uint4 xv[4];
    ld16x4(p, xv);
    const T* xe = reinterpret_cast<const T*>(xv);
    uint4 ov[4];
    uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      ow[j] = Tr<T>::pack(Tr<T>::f(xe[2 * j]) + Tr<T>::r(v[2 * j]),
                          Tr<T>::f(xe[2 * j + 1]) + Tr<T>::r(v[2 * j + 1]));
    st16x4(p, ov);
    return true;
  }
};

template <typename T>
struct EpiGatedResid {  // suffix residual (gemma_dual.py:91-94): x = round(x + round(round(acc)·gate))
  T* x;
  int ldx;
  const T* gate;      // [rows_per_gate_group ...]: gate[(r / rows_per_gate) * gate_stride + c]
  int rows_per_gate;  // rows that share one gate vector (S·B when the time is shared)
  int gate_stride;
  __device__ void prefetch(int r, int c) const {
    pf_l1(x + (size_t)r * ldx + c);
    pf_l1(gate + (size_t)(r / rows_per_gate) * gate_stride + c);
  }
  // returns the new (rounded) x values, from which the next norm's Σx² partials are formed
  __device__ float2 operator()(int r, int c, float v0, float v1) const {
    const T* g = gate + (size_t)(r / rows_per_gate) * gate_stride + c;
    T* p = x + (size_t)r * ldx + c;
    float a = Tr<T>::r(Tr<T>::f(p[0]) + Tr<T>::r(Tr<T>::r(v0) * Tr<T>::f(g[0])));
    float b = Tr<T>::r(Tr<T>::f(p[1]) + Tr<T>::r(Tr<T>::r(v1) * Tr<T>::f(g[1])));
    *reinterpret_cast<uint32_t*>(p) = Tr<T>::pack(a, b);
    return make_float2(a, b);
  }
  __device__ bool chunk32(int r, int c0, const float* v) const {
    const T* g = gate + (size_t)(r / rows_per_gate) * gate_stride + c0;
    T* p = x + (size_t)r * ldx + c0;
    if (!al16(p) || !al16(g)) return false;
    uint4 xv[4], gv[4];
    ld16x4(p, xv);
    ld16x4(g, gv);
    const T* xe = reinterpret_cast<const T*>(xv);
    const T* ge = reinterpret_cast<const T*>(gv);
    uint4 ov[4];
    uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float a = Tr<T>::r(Tr<T>::f(xe[2 * j]) + Tr<T>::r(Tr<T>::r(v[2 * j]) * Tr<T>::f(ge[2 * j])));
      const float b = Tr<T>::r(Tr<T>::f(xe[2 * j + 1]) +
                               Tr<T>::r(Tr<T>::r(v[2 * j + 1]) * Tr<T>::f(ge[2 * j + 1])));
      ow[j] = Tr<T>::pack(a, b);
    }
    st16x4(p, ov);
    return true;
  }
};

// GeGLU (gemma_dual.py:132-135) on interleaved gate/up weights: packed weight row 2j is gate
// row j and row 2j+1 is up row j, so (col, col+1) = (gate_j, up_j).
// h[r, j] = round(round(gelu_tanh(round(gate))) · round(up)).
template <typename T>
struct EpiGeglu {
  T* h;
  int ldh;
  __device__ void prefetch(int, int) const {}
  __device__ void operator()(int r, int c, float v0, float v1) const {
    float g = Tr<T>::r(gelu_tanh_f(Tr<T>::r(v0)));
    h[(size_t)r * ldh + (c >> 1)] = Tr<T>::t(g * Tr<T>::r(v1));
  }
  __device__ bool chunk32(int r, int c0, const float* v) const {
    T* o = h + (size_t)r * ldh + (c0 >> 1);
    if (!al16(o)) return false;
    uint4 ov[2];
    uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g0 = Tr<T>::r(gelu_tanh_f(Tr<T>::r(v[4 * j])));
      const float g1 = Tr<T>::r(gelu_tanh_f(Tr<T>::r(v[4 * j + 2])));
      ow[j] = Tr<T>::pack(g0 * Tr<T>::r(v[4 * j + 1]), g1 * Tr<T>::r(v[4 * j + 3]));
    }
    reinterpret_cast<uint4*>(o)[0] = ov[0];
    reinterpret_cast<uint4*>(o)[1] = ov[1];
    return true;
  }
};

// q/k/v projection with RoPE and the K/V-cache write fused (gemma_dual.py:236-275).
// Packed weight rows of the q and k blocks are permuted per head so that columns (2i, 2i+1)
// hold original dims (i, i + hd/2); v rows keep their order.
//   q  -> fp32 [rows, H, hd], rotated and scaled by hd^-0.5
//   k  -> fp32 cache [B, KV, T, hd] at (b, kvh, pos), rotated
//   v  -> model-dtype cache, same layout
// Rows are r = b·T + pos. RoPE tables: cos/sin[(b·cs_bstride) + pos·(hd/2) + i] fp32.
template <typename T>
struct EpiQkvRope {
  float* q;
  float* k;
  T* v;
  const float* cos;
  const float* sin;
  int cs_bstride;
  int T_len;     // positions per request
  int H, KV, hd;
  int col0;      // global column offset of this launch (skip q rows for the last prefill layer)
  float qscale;
  // tensor-core attention operands (optional): q in the model dtype instead of fp32 q, and a
  // model-dtype copy of k at half scale next to the fp32 cache entry; for fp32 logits also their
  // lo parts x − fp16(x) (q16lo / k16lo, set together with q16 / k16)
  T* q16 = nullptr;
  T* k16 = nullptr;
  T* q16lo = nullptr;
  T* k16lo = nullptr;
  __device__ void prefetch(int r, int c_local) const {
    const int c = c_local + col0;
    if (c < (H + KV) * hd) {
      const int cc = c < H * hd ? c : c - H * hd;
      const int b = r / T_len, pos = r - b * T_len;
      const size_t t = (size_t)b * cs_bstride + (size_t)pos * (hd >> 1) + ((cc % hd) >> 1);
      pf_l1(cos + t);
      pf_l1(sin + t);
    }
  }
  __device__ void operator()(int r, int c_local, float v0, float v1) const {
    int c = c_local + col0;
    int hq = H * hd, hkv = KV * hd;
    int b = r / T_len, pos = r - b * T_len;
    if (c < hq + hkv) {
      bool isq = c < hq;
      int cc = isq ? c : c - hq;
      int head = cc / hd, i = (cc - head * hd) >> 1, half = hd >> 1;
      size_t t = (size_t)b * cs_bstride + (size_t)pos * half + i;
      float cs = cos[t], sn = sin[t];
      float x1 = Tr<T>::r(v0), x2 = Tr<T>::r(v1);
      float o1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      float o2 = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
      if (isq) {
        const size_t qo = ((size_t)r * H + head) * hd;
        if (q16) {
          const float a1 = __fmul_rn(o1, qscale), a2 = __fmul_rn(o2, qscale);
          q16[qo + i] = Tr<T>::t(a1);
          q16[qo + i + half] = Tr<T>::t(a2);
          if (q16lo) {
            q16lo[qo + i] = Tr<T>::t(a1 - Tr<T>::r(a1));
            q16lo[qo + i + half] = Tr<T>::t(a2 - Tr<T>::r(a2));
          }
        } else {
          q[qo + i] = __fmul_rn(o1, qscale);
          q[qo + i + half] = __fmul_rn(o2, qscale);
        }
      } else {
        const size_t ko = (((size_t)b * KV + head) * T_len + pos) * hd;
        k[ko + i] = o1;
        k[ko + i + half] = o2;
        if (k16) {
          k16[ko + i] = Tr<T>::t(0.5f * o1);
          k16[ko + i + half] = Tr<T>::t(0.5f * o2);
          if (k16lo) {
            k16lo[ko + i] = Tr<T>::t(0.5f * o1 - Tr<T>::r(0.5f * o1));
            k16lo[ko + i + half] = Tr<T>::t(0.5f * o2 - Tr<T>::r(0.5f * o2));
          }
        }
      }
    } else {
      int cc = c - hq - hkv;
      int head = cc / hd, d = cc - head * hd;
      T* p = v + (((size_t)b * KV + head) * T_len + pos) * hd + d;
      *reinterpret_cast<uint32_t*>(p) = Tr<T>::pack(v0, v1);
    }
  }
  // 32 columns = 16 RoPE pairs (i0 .. i0+15) of one head, or 32 v dims of one head
  __device__ bool chunk32(int r, int c_local0, const float* val) const {
    if (hd < 32) return false;
    const int c0 = c_local0 + col0;
    const int hq = H * hd, hkv = KV * hd;
    const int b = r / T_len, pos = r - b * T_len;
    if (c0 < hq + hkv) {
      const bool isq = c0 < hq;
      const int cc = isq ? c0 : c0 - hq;
      const int head = cc / hd, i0 = (cc - head * hd) >> 1, half = hd >> 1;
      const size_t t = (size_t)b * cs_bstride + (size_t)pos * half + i0;
      const size_t off = isq ? ((size_t)r * H + head) * hd
                             : (((size_t)b * KV + head) * T_len + pos) * hd;
      float* base = isq ? q + off : k + off;
      T* base16 = isq ? q16 : k16;
      T* lo16 = isq ? q16lo : k16lo;
      if (!al16(cos + t) || !al16(sin + t)) return false;
      if (base16) {
        if (!al16(base16 + off + i0) || !al16(base16 + off + i0 + half)) return false;
      }
      if (lo16) {
        if (!al16(lo16 + off + i0) || !al16(lo16 + off + i0 + half)) return false;
      }
      if ((!isq || !q16) && (!al16(base + i0) || !al16(base + i0 + half))) return false;
      float cs[16], sn[16];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        *reinterpret_cast<float4*>(cs + 4 * u) = reinterpret_cast<const float4*>(cos + t)[u];
        *reinterpret_cast<float4*>(sn + 4 * u) = reinterpret_cast<const float4*>(sin + t)[u];
      }
      float o1[16], o2[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float x1 = Tr<T>::r(val[2 * j]), x2 = Tr<T>::r(val[2 * j + 1]);
        o1[j] = __fsub_rn(__fmul_rn(x1, cs[j]), __fmul_rn(x2, sn[j]));
        o2[j] = __fadd_rn(__fmul_rn(x2, cs[j]), __fmul_rn(x1, sn[j]));
        if (isq) {
          o1[j] = __fmul_rn(o1[j], qscale);
          o2[j] = __fmul_rn(o2[j], qscale);
        }
      }
      if (!isq || !q16) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          reinterpret_cast<float4*>(base + i0)[u] = *reinterpret_cast<const float4*>(o1 + 4 * u);
          reinterpret_cast<float4*>(base + i0 + half)[u] = *reinterpret_cast<const float4*>(o2 + 4 * u);
        }
      }
      if (base16) {
        const float sc = isq ? 1.f : 0.5f;  // k at half scale
        uint4 h1[2], h2[2];
        uint32_t* w1 = reinterpret_cast<uint32_t*>(h1);
        uint32_t* w2 = reinterpret_cast<uint32_t*>(h2);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          w1[j] = Tr<T>::pack(sc * o1[2 * j], sc * o1[2 * j + 1]);
          w2[j] = Tr<T>::pack(sc * o2[2 * j], sc * o2[2 * j + 1]);
        }
        reinterpret_cast<uint4*>(base16 + off + i0)[0] = h1[0];
        reinterpret_cast<uint4*>(base16 + off + i0)[1] = h1[1];
        reinterpret_cast<uint4*>(base16 + off + i0 + half)[0] = h2[0];
        reinterpret_cast<uint4*>(base16 + off + i0 + half)[1] = h2[1];
        if (lo16) {  // the residuals x − fp16(x), exact in fp32, rounded to fp16
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float a0 = sc * o1[2 * j], a1 = sc * o1[2 * j + 1];
            const float b0 = sc * o2[2 * j], b1 = sc * o2[2 * j + 1];
            w1[j] = Tr<T>::pack(a0 - Tr<T>::r(a0), a1 - Tr<T>::r(a1));
            w2[j] = Tr<T>::pack(b0 - Tr<T>::r(b0), b1 - Tr<T>::r(b1));
          }
          reinterpret_cast<uint4*>(lo16 + off + i0)[0] = h1[0];
          reinterpret_cast<uint4*>(lo16 + off + i0)[1] = h1[1];
          reinterpret_cast<uint4*>(lo16 + off + i0 + half)[0] = h2[0];
          reinterpret_cast<uint4*>(lo16 + off + i0 + half)[1] = h2[1];
        }
      }
    } else {
      const int cc = c0 - hq - hkv;
      const int head = cc / hd, d = cc - head * hd;
      T* p = v + (((size_t)b * KV + head) * T_len + pos) * hd + d;
      if (!al16(p)) return false;
      uint4 ov[4];
      uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
      for (int j = 0; j < 16; ++j) ow[j] = Tr<T>::pack(val[2 * j], val[2 * j + 1]);
      st16x4(p, ov);
    }
    return true;
  }
};

// ---- kernel ----
template <typename T, int BM, int BN, int WM, int WN, int STAGES>
struct GemmCfg {
  static constexpr int BK = 32;
  static constexpr int LDS = BK + 8;  // halves per smem row (80 B: conflict-free ldmatrix)
  static constexpr int WARPS_M = BM / WM, WARPS_N = BN / WN;
  static constexpr int NT = WARPS_M * WARPS_N * 32;
  static constexpr int MI = WM / 16, NI = WN / 8;
  static constexpr int SMEM = STAGES * (BM + BN) * LDS * 2;
};

template <typename T, int BM, int BN, int WM, int WN, int STAGES, class Epi>
__global__ void __launch_bounds__(GemmCfg<T, BM, BN, WM, WN, STAGES>::NT)
    gemm_mma_kernel(GemmArgs<T> g, Epi epi) {
  using C = GemmCfg<T, BM, BN, WM, WN, STAGES>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sA = reinterpret_cast<T*>(smem_raw);
  T* sB = sA + STAGES * BM * C::LDS;
  __shared__ int s_last;
  pdl_wait();
  pdl_trigger();

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp / C::WARPS_N, wn = warp % C::WARPS_N;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int kbeg = blockIdx.z * g.k_split_len;
  const int kend = min(g.K, kbeg + g.k_split_len);
  const int nk = (kend - kbeg) / C::BK;

  auto load_stage = [&](int stage, int kt) {
    const int k0 = kbeg + kt * C::BK;
    T* a = sA + stage * BM * C::LDS;
    T* b = sB + stage * BN * C::LDS;
    for (int i = tid; i < BM * 4; i += C::NT) {
      int row = i >> 2, ch = i & 3;
      int gr = m0 + row;
      const T* src = g.A + (size_t)min(gr, g.M - 1) * g.lda + k0 + ch * 8;
      cp_async16(a + row * C::LDS + ch * 8, src, gr < g.M ? 16 : 0);
    }
    for (int i = tid; i < BN * 4; i += C::NT) {
      int row = i >> 2, ch = i & 3;
      int gr = n0 + row;
      const T* src = g.W + (size_t)min(gr, g.N - 1) * g.ldw + k0 + ch * 8;
      cp_async16(b + row * C::LDS + ch * 8, src, gr < g.N ? 16 : 0);
    }
  };

  float acc[C::MI][C::NI][4];
#pragma unroll
  for (int i = 0; i < C::MI; ++i)
#pragma unroll
    for (int j = 0; j < C::NI; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < nk) load_stage(s, s);
    cp_async_commit();
  }

  for (int kt = 0; kt < nk; ++kt) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    {
      int nxt = kt + STAGES - 1;
      if (nxt < nk) load_stage(nxt % STAGES, nxt);
      cp_async_commit();
    }
    const T* a = sA + (kt % STAGES) * BM * C::LDS;
    const T* b = sB + (kt % STAGES) * BN * C::LDS;
#pragma unroll
    for (int ks = 0; ks < C::BK; ks += 16) {
      uint32_t af[C::MI][4], bf[C::NI][2];
#pragma unroll
      for (int i = 0; i < C::MI; ++i) {
        const T* p = a + (wm * WM + i * 16 + (lane & 15)) * C::LDS + ks + (lane >> 4) * 8;
        ldsm_x4(af[i][0], af[i][1], af[i][2], af[i][3], p);
      }
#pragma unroll
      for (int j = 0; j < C::NI; j += 2) {
        const T* p = b + (wn * WN + j * 8 + (lane & 7) + ((lane >> 4) << 3)) * C::LDS + ks +
                     ((lane >> 3) & 1) * 8;
        ldsm_x4(bf[j][0], bf[j][1], bf[j + 1][0], bf[j + 1][1], p);
      }
#pragma unroll
      for (int i = 0; i < C::MI; ++i)
#pragma unroll
        for (int j = 0; j < C::NI; ++j) mma16816<T>(acc[i][j], af[i], bf[j]);
    }
  }
  cp_async_wait<0>();

  const int gq = lane >> 2, tq = lane & 3;
  if (gridDim.z > 1) {
    // deterministic split-K fix-up
    float* part = g.ws + (size_t)blockIdx.z * g.M * g.N;
#pragma unroll
    for (int i = 0; i < C::MI; ++i)
#pragma unroll
      for (int j = 0; j < C::NI; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int r = m0 + wm * WM + i * 16 + gq + h * 8;
          int c = n0 + wn * WN + j * 8 + tq * 2;
          if (r < g.M && c < g.N)
            *reinterpret_cast<float2*>(part + (size_t)r * g.N + c) =
                make_float2(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
        }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      int* t = g.tickets + blockIdx.y * gridDim.x + blockIdx.x;
      int prev = atomicAdd(t, 1);
      s_last = (prev == (int)gridDim.z - 1);
      if (s_last) *t = 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
#pragma unroll
    for (int i = 0; i < C::MI; ++i)
#pragma unroll
      for (int j = 0; j < C::NI; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int r = m0 + wm * WM + i * 16 + gq + h * 8;
          int c = n0 + wn * WN + j * 8 + tq * 2;
          if (r < g.M && c < g.N) {
            float s0 = 0.f, s1 = 0.f;
            for (int z = 0; z < (int)gridDim.z; ++z) {
              float2 v = __ldcg(reinterpret_cast<const float2*>(g.ws + (size_t)z * g.M * g.N +
                                                               (size_t)r * g.N + c));
              s0 += v.x;
              s1 += v.y;
            }
            epi(r, c, s0, s1);
          }
        }
    return;
  }
#pragma unroll
  for (int i = 0; i < C::MI; ++i)
#pragma unroll
    for (int j = 0; j < C::NI; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int r = m0 + wm * WM + i * 16 + gq + h * 8;
        int c = n0 + wn * WN + j * 8 + tq * 2;
        if (r < g.M && c < g.N) epi(r, c, acc[i][j][2 * h], acc[i][j][2 * h + 1]);
      }
}

}  // namespace pi0
