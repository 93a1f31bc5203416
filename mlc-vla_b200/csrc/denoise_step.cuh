// One persistent kernel for a whole denoise step (decode_suffix + action in/out, the reference's
// denoise_step_kv body: pi0_model.py:142-163, gemma_dual.py:343-351,417-433) at batch 1, fp16,
// one kv head: action_in, then per layer q/k/v (adaRMSNorm fused) → attention → o_proj + gated
// residual → gate_up (adaRMSNorm fused) + GeGLU → down + gated residual, then the final
// adaRMSNorm + action_out (+ the Euler update). The step's ~92 dependent launches become phases of
// one launch separated by grid barriers, and every CTA loads the weights of its next phase while
// the barrier is still open, so a phase starts with its weights already in shared memory.
//
// Grid: every co-resident cluster of 8 CTAs (one CTA per SM; 15 clusters on a B200). Phases:
//   * GEMM phases (weight-streaming, swap-AB tcgen05 MMA as in gemm_skinny.cuh): a host-built
//     plan gives every CTA a (tile, split group, k-range). A split group is s ∈ {1, 2, 4, 8}
//     consecutive ranks of a cluster that share one 128-row weight tile over K; their partial
//     accumulators are summed through distributed shared memory in rank order (deterministic)
//     and each rank finishes 128/s weight rows with the fused epilogue. Weight blocks go through a
//     RING-slot shared-memory ring that persists across phases; block q of the CTA's whole
//     sequence uses slot q % RING, so all roles agree on slots and mbarrier parities without
//     re-initialising anything.
//   * attention phase: clusters 0 .. row_tiles-1 each own a 128-row tile of the 400 query rows
//     and split its key tiles over their 8 ranks (attention_tc.cuh's algorithm, including the
//     fp32-logits hi/lo variant); the split partials are merged in the cluster.
//   * action_in / action_out: SIMT phases (small_kernels.cuh's arithmetic).
// Grid barrier: the CTAs of a cluster meet at a cluster barrier, rank 0 arrives on a global
// counter and waits for the generation to change (bounded: about a second), and its verdict is
// handed to the cluster's ranks through distributed shared memory, so every CTA of a cluster
// leaves a failed barrier together and the cluster barriers stay matched. On any timeout the
// kernel records the error code and every cluster stops at the next grid barrier.
// While a phase runs, each CTA also asks L2 for the weight blocks of its next-but-one GEMM phase
// (cp.async.bulk.prefetch.L2), so the ring loads issued at the barrier read L2, not HBM.
#pragma once

#include "attention_tc.cuh"
#include "small_kernels.cuh"

namespace pi0 {
namespace ds {

using namespace tc;
using sk::W_BLOCK;
using sk::workers_sync;

constexpr int CL = 8;          // cluster size
constexpr int RING = 7;        // weight ring slots
constexpr int NA = 64;         // activation rows (B·S ≤ 64)
constexpr int NT = 192;        // threads: warp 0 copies, warp 1 MMAs, warps 2-5 workers
constexpr int X_BLOCK = NA * BK * 2;     // 8 KB activation block
constexpr int STAGE = W_BLOCK + X_BLOCK; // 24 KB
constexpr int RECV_OFF = RING * STAGE;   // split-K receive buffer, outside the ring
constexpr int RECV_BYTES = BM * NA * 4;  // s slices of [M][128/s] fp32 = 128·M floats
constexpr int SSQ_PARTS = 64;            // row Σx² partials per row (8 tiles × 8 ranks)
constexpr int ERR_TIMEOUT_GRID = 5;      // error code: a grid barrier gave up

enum GemmKind { G_QKV = 0, G_O = 1, G_GU = 2, G_D = 3, G_NUM = 4 };

// One CTA's share of a GEMM phase: weight tile `tile` (-1: idle), split group of `s` ranks
// starting at cluster rank `g0`, k-blocks [kb0, kb0 + nk).
struct Work {
  int16_t tile, s, g0, kb0, nk, pad[3];
};

struct Layer {                 // packed weight blocks of one action-expert layer
  const uint8_t* w[G_NUM];
};

struct StepArgs {
  int M;                       // activation rows (S)
  int W1, F1, H, hd, S, P, L, D;
  const Layer* layers;         // [L]
  const Work* plan;            // [G_NUM][grid]
  int tiles[G_NUM], nkb[G_NUM], N[G_NUM], K[G_NUM];
  const void* mods;            // this step's modulation rows [(2L+1)·3·W1]
  void* x;                     // residual stream [M, W1]
  void* attn;                  // attention output [M, H·hd]
  void* h;                     // MLP hidden [M, F1]
  float* ssq;                  // [M][SSQ_PARTS]
  // q/k/v epilogue
  float* qs;
  float* ksuf;
  void* vsuf;
  void* q16;
  void* q16lo;
  void* k16;
  void* k16lo;
  const float* scos;
  const float* ssin;
  float qscale;
  // attention: prefix cache rows of layer l start at l·P (batch 1, one kv head)
  const float* maskA;          // [P]
  int att_row_tiles, att_tps, att_splits, att_ntA, att_nt;
  const void* kA16;            // half-scale prefix keys (hi, lo) and values, for L2 prefetches
  const void* kA16lo;
  const void* vA;
  // action in / out
  const void* x_in;
  int x_is_f32;
  const void* ain_w;
  const void* ain_b;
  const void* aout_w;
  const void* aout_b;
  float* out;
  int euler;
  float dt;
  float eps;
  int* err;
  unsigned long long* bar;     // grid barrier word (arrivals | generation << 32), zero at creation
};

// L2 prefetch of `bytes` at `p` (16-byte aligned, a multiple of 16 bytes)
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long atom_add_acqrel64(unsigned long long* p,
                                                                unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.add.acq_rel.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_add_release64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.add.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Grid barrier over `nclusters` clusters. `bar` is one 64-bit word: arrivals of the current
// generation in the low half, the generation in the high half. Rank 0 of each cluster arrives with
// an acq_rel add, which returns the generation it arrived in; the last arrival adds
// 2^32 − nclusters (count back to zero, generation + 1) with release semantics, and the others
// poll until the generation changes (bounded: about a second). No reset is needed between
// launches. Returns false, the same in every CTA of a cluster, when the barrier timed out or a
// kernel reported an error; `s_ok` is a shared word of every CTA, and rank 0 writes its verdict
// into each rank's copy.
__device__ __noinline__ bool grid_sync(unsigned long long* bar, unsigned nclusters, int* err,
                                       uint32_t* s_ok) {
  // this thread's generic-proxy writes -> visible to the TMA loads of other CTAs
  asm volatile("fence.proxy.async.global;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (cluster_rank() == 0 && threadIdx.x == 0) {
    uint32_t ok = 1;
    // the acq_rel arrival releases the cluster's writes (ordered before it by the cluster
    // barrier; release is cumulative) and the generation poll below acquires everyone's
    const unsigned long long old = atom_add_acqrel64(bar, 1ull);
    const unsigned gen = (unsigned)(old >> 32);
    if ((unsigned)old == nclusters - 1) {
      red_add_release64(bar, (1ull << 32) - (unsigned long long)nclusters);
    } else {
      const unsigned long long t0 = globaltimer();
      for (uint32_t it = 1;; ++it) {
        if ((unsigned)(ld_acquire64(bar) >> 32) != gen) break;
        if ((it & 63) == 0) {
          if (globaltimer() - t0 > kTimeoutNs) {
            atomicCAS(err, 0, ERR_TIMEOUT_GRID);
            ok = 0;
            break;
          }
          if (*(volatile int*)err != 0) {
            ok = 0;
            break;
          }
        }
      }
    }
    if (ok && *(volatile int*)err != 0) ok = 0;
    for (uint32_t r = 0; r < CL; ++r) st_cluster_u32(map_rank(smem_u32(s_ok), r), ok);
  }
  cluster_sync();
  tc_fence_after();
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return *(volatile uint32_t*)s_ok != 0;
}

// Shared state of one CTA that outlives the phases (static shared memory of the kernel).
struct Sh {
  uint64_t full_w[RING], full_x[RING], ready_x[RING], empty[RING], bar_mma, recv_bar;
  uint32_t rx_par;         // bit s: parity of slot s's next ready_x completion (norm phases)
  uint32_t recv_uses;      // completed receives on recv_bar
  atc::AtcShared att;      // attention phase (its barriers are re-initialised every layer)
  uint32_t tmem;
  uint32_t ok;             // grid barrier verdict (written by rank 0 of the cluster)
  uint32_t mma_ok;         // GEMM phase: the accumulator is complete
  int stop;
  uint32_t w_end, x_end;   // thread 0: sequence number after the last issued weight / x block
  float den[NA], rcp[NA];  // NORM: per-row sqrt(mean x² + eps) and its reciprocal
  uint4 mod[16][2][8];     // NORM: the (scale, shift) chunks of this CTA's k-blocks
};

__device__ __forceinline__ uint8_t* stage_w(uint8_t* base, int s) { return base + s * STAGE; }
__device__ __forceinline__ uint8_t* stage_x(uint8_t* base, int s) { return base + s * STAGE + W_BLOCK; }

// Thread 0: the weight blocks [from, to) of a GEMM phase whose first block has sequence number
// seq; a slot is refilled once the MMAs of its previous block are done.
__device__ __forceinline__ bool issue_weights(Sh& sh, uint8_t* base, const uint8_t* wsrc,
                                              uint32_t seq, int from, int to, int* err) {
  for (int i = from; i < to; ++i) {
    const uint32_t q = seq + i, s = q % RING, use = q / RING;
    if (use > 0 && !mbar_wait(&sh.empty[s], (use - 1) & 1, err, ERR_TIMEOUT_PRODUCER)) return false;
    mbar_expect_tx(&sh.full_w[s], W_BLOCK);
    sk::bulk_load(stage_w(base, s), wsrc + (size_t)i * W_BLOCK, W_BLOCK, &sh.full_w[s]);
    sh.w_end = q + 1;
  }
  return true;
}

// The source of this CTA's weight blocks in a GEMM phase (null when idle).
__device__ __forceinline__ const uint8_t* work_src(const StepArgs& a, const Layer& ly, int g,
                                                   const Work& w) {
  if (w.tile < 0 || w.nk <= 0) return nullptr;
  return ly.w[g] + ((size_t)w.tile * a.nkb[g] + w.kb0) * W_BLOCK;
}

// One GEMM phase: Y[M, N] = X[M, K] · W[N, K]^T for this CTA's work item, fused epilogue `epi`.
// wpre: weight blocks already issued for this phase (issue_weights before the barrier); seq: the
// CTA's k-block sequence number (advanced by w.nk); gph: GEMM phases so far (bar_mma parity).
// Every CTA of a cluster calls this (idle ones too: the two cluster barriers must match).
template <typename T, bool NORM, bool SSQ, class Epi>
__device__ __noinline__ void gemm_phase(const StepArgs& a, Sh& sh, uint8_t* base, const Work& w,
                           const uint8_t* wsrc, const CUtensorMap* tmX, const T* mod, int N, int K,
                           const Epi& epi, uint32_t& seq, int wpre, uint32_t gph, bool& ok) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = (w.tile >= 0 && ok) ? w.nk : 0;
  const int M = a.M;
  if (nk > 0) {
    {  // the epilogue's global operands (residual rows, gates, RoPE tables) into L1 now
      const int R = BM / w.s, quads = R / 4, total = quads * M;
      const int rr = (int)cluster_rank() - w.g0;
      for (int it = tid; it < total; it += NT) {
        const int g = it % quads, m = it / quads;
        const int n = w.tile * BM + rr * R + 4 * g;
        if (n < N) epi.prefetch(m, n);
      }
    }
    if (warp == 0) {
      if (lane == 0) {  // producer: the rest of the weights, every activation block
        bool good = true;
        for (int i = 0; i < nk && good; ++i) {
          const uint32_t q = seq + i, s = q % RING;
          if (i >= wpre) good = issue_weights(sh, base, wsrc, seq, i, i + 1, a.err);
          if (!good) break;
          mbar_expect_tx(&sh.full_x[s], X_BLOCK);
          tma_load_2d(stage_x(base, s), tmX, &sh.full_x[s], (w.kb0 + i) * BK, 0);
          sh.x_end = q + 1;
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {  // MMA issuer
        constexpr uint32_t idesc = idesc_f16<T>(BM, NA);
        const uint32_t rx = sh.rx_par;
        for (int i = 0; i < nk; ++i) {
          const uint32_t q = seq + i, s = q % RING, ph = (q / RING) & 1;
          const uint32_t rph = ((rx >> s) ^ (uint32_t)(i / RING)) & 1;
          if (!mbar_wait(&sh.full_w[s], ph, a.err, ERR_TIMEOUT_MMA) ||
              !(NORM ? mbar_wait(&sh.ready_x[s], rph, a.err, ERR_TIMEOUT_MMA)
                     : mbar_wait(&sh.full_x[s], ph, a.err, ERR_TIMEOUT_MMA)))
            break;
          tc_fence_after();
          const uint64_t da = desc_sw128(smem_u32(stage_w(base, s)));
          const uint64_t db = desc_sw128(smem_u32(stage_x(base, s)));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(sh.tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
          umma_commit(&sh.empty[s]);
        }
        umma_commit(&sh.bar_mma);
      }
    } else if (NORM) {  // workers: normalise every activation block in place for the MMA
      const int wt = tid - 64;
      if constexpr (NORM) {
        // the (scale, shift) chunks of every k-block of this CTA, requested together
        const uint4 z4 = make_uint4(0, 0, 0, 0);
        for (int it = wt; it < nk * 16; it += 128) {
          const int i = it >> 4, half = (it >> 3) & 1, c = it & 7;
          const int col = (w.kb0 + i) * BK + c * 8;
          sh.mod[i & 15][half][c] = col < K ? *reinterpret_cast<const uint4*>(mod + half * K + col) : z4;
        }
        if (wt < M) {  // row wt: its Σx² partials, all loads issued before the sum (slot order)
          const float4* p = reinterpret_cast<const float4*>(a.ssq + (size_t)wt * SSQ_PARTS);
          float4 v[SSQ_PARTS / 4];
#pragma unroll
          for (int j = 0; j < SSQ_PARTS / 4; ++j) v[j] = p[j];
          float ss = 0.f;
#pragma unroll
          for (int j = 0; j < SSQ_PARTS / 4; ++j) ss = ((ss + v[j].x) + v[j].y + v[j].z) + v[j].w;
          const float den = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps));
          sh.den[wt] = den;
          sh.rcp[wt] = __frcp_rn(den);
        }
        workers_sync();
      }
      sk::SkArgs na{};
      na.M = M;
      for (int i = 0; i < nk; ++i) {
        const uint32_t q = seq + i, s = q % RING, ph = (q / RING) & 1;
        uint4 sc, sh2;
        if constexpr (NORM) {
          sc = sh.mod[i & 15][0][wt & 7];
          sh2 = sh.mod[i & 15][1][wt & 7];
        }
        if (!mbar_wait(&sh.full_x[s], ph, a.err, ERR_TIMEOUT_EPI)) sh.stop = 1;
        workers_sync();
        if (sh.stop) break;
        if constexpr (NORM) sk::norm_inplace<T, NA>(na, stage_x(base, s), sc, sh2, sh.den, sh.rcp, wt);
        workers_sync();
        if (wt == 0) mbar_arrive(&sh.ready_x[s]);
      }
    }
    seq += (uint32_t)nk;
    // ---- accumulator -> this CTA's partial, one contiguous slice per destination rank ----
    // part[(d·M + m)·R + r] = row d·R + r of the weight tile, activation row m (aliases ring
    // slots 0-1, all consumed); destination d finishes weight rows [d·R, (d+1)·R)
    if (tid == 64) sh.mma_ok = mbar_wait(&sh.bar_mma, gph & 1, a.err, ERR_TIMEOUT_EPI, false) ? 1 : 0;
    __syncthreads();
    const bool acc_ok = sh.mma_ok != 0 && sh.stop == 0;
    if (!acc_ok) ok = false;
    tc_fence_after();
    const int S_ = w.s, R = BM / S_, rr = (int)cluster_rank() - w.g0;
    float* part = reinterpret_cast<float*>(base);
    if (warp >= 2) {
      const int qd = warp & 3, wrow = qd * 32 + lane;
      const int d = wrow / R, r = wrow - d * R;
#pragma unroll 1
      for (int c = 0; c < M; c += 32) {
        uint32_t v[32];
        if (acc_ok) {
          tmem_ld32(sh.tmem + ((uint32_t)(qd * 32) << 16) + c, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0u;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c + j < M) part[((d * M) + c + j) * R + r] = __uint_as_float(v[j]);
      }
    }
    tc_fence_before();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // part -> bulk copy engine
    __syncthreads();
    // ---- split group: push slice d to rank g0 + d (its receive buffer, row block of our rank),
    // completing on that rank's recv_bar; then wait for the s slices of our own rows ----
    const float* src = part;  // s = 1: the own partial is the whole tile
    const uint32_t slice = (uint32_t)(M * R * 4);
    if (S_ > 1) {
      if (tid < S_) {
        const uint32_t peer = (uint32_t)(w.g0 + tid);
        const uint32_t dst = map_rank(smem_u32(base + RECV_OFF + (size_t)rr * slice), peer);
        const uint32_t mb = map_rank(smem_u32(&sh.recv_bar), peer);
        asm volatile(
            "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
            "r"(smem_u32(part + (size_t)tid * M * R)), "r"(slice), "r"(mb)
            : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        if (tid == 0) mbar_expect_tx(&sh.recv_bar, (uint32_t)S_ * slice);
      }
      if (tid == 64 && !mbar_wait(&sh.recv_bar, sh.recv_uses & 1, a.err, ERR_TIMEOUT_EPI, false))
        sh.mma_ok = 0;
      __syncthreads();
      if (sh.mma_ok == 0) ok = false;
      src = reinterpret_cast<const float*>(base + RECV_OFF);
    }
    // ---- reduction in rank order + epilogue: item = (activation row m, 4 weight rows) ----
    const int quads = R / 4, total = quads * M;
    const int n0 = w.tile * BM;
    float* s_item = reinterpret_cast<float*>(base + (size_t)S_ * slice + 1024);  // after part
#pragma unroll 1
    for (int it = tid; it < total; it += NT) {
      const int g = it % quads, m = it / quads;
      const float4* p = reinterpret_cast<const float4*>(src + (size_t)m * R + 4 * g);
      float4 sum = p[0];
#pragma unroll
      for (int c = 1; c < CL; ++c)
        if (c < S_) {
          const float4 v = p[(size_t)c * M * R / 4];
          sum.x += v.x;
          sum.y += v.y;
          sum.z += v.z;
          sum.w += v.w;
        }
      float sq = 0.f;
      const int nb = n0 + rr * R + 4 * g;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        const int n = nb + 2 * hh;
        if (n >= N) break;
        const float v0 = hh ? sum.z : sum.x, v1 = hh ? sum.w : sum.y;
        if constexpr (SSQ) {
          const float2 pr = epi(m, n, v0, v1);
          sq += pr.x * pr.x + pr.y * pr.y;
        } else {
          epi(m, n, v0, v1);
        }
      }
      if constexpr (SSQ) s_item[it] = sq;
    }
    if constexpr (SSQ) {
      __syncthreads();
      for (int m = tid; m < M; m += NT) {
        float qq = 0.f;
        for (int g = 0; g < quads; ++g) qq += s_item[m * quads + g];
        a.ssq[(size_t)m * SSQ_PARTS + w.tile * S_ + rr] = qq;
      }
    }
    // the ring may be refilled once the pushes have read `part` and every thread is done
    if (S_ > 1 && tid < S_) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      if (S_ > 1) ++sh.recv_uses;
      if (NORM) {  // ready_x completions of this phase: slot (seq0 + i) % RING for i < nk
        uint32_t flip = 0;
        for (int i = 0; i < nk; ++i) flip ^= 1u << ((seq - (uint32_t)nk + (uint32_t)i) % RING);
        sh.rx_par ^= flip;
      }
    }
    __syncthreads();
  } else {
    seq += (uint32_t)(w.tile >= 0 ? w.nk : 0);
  }
}

// action_in_proj (pi0_model.py:154,187): emb = RN(RN(x·Wᵀ) + b) for all M rows, K = D. CTA u < 64
// computes output columns [u·W1/64, (u+1)·W1/64) of every row (the fp32 fma chain in k order of
// action_in_kernel) and the row Σx² partial of those columns into slot u of a.ssq.
template <typename T>
__device__ __noinline__ void action_in_phase(const StepArgs& a, uint8_t* base, bool work) {
  const int u = blockIdx.x, tid = threadIdx.x;
  const int M = a.M, D = a.D, W1 = a.W1, cols = W1 / SSQ_PARTS;
  if (!work || u >= SSQ_PARTS) return;
  float* sx = reinterpret_cast<float*>(base);                 // [M][D]
  float* sy = sx + M * D;                                     // [M][cols]
  for (int i = tid; i < M * D; i += NT)
    sx[i] = a.x_is_f32 ? Tr<T>::r(reinterpret_cast<const float*>(a.x_in)[i])
                       : Tr<T>::f(reinterpret_cast<const T*>(a.x_in)[i]);
  __syncthreads();
  const T* W = reinterpret_cast<const T*>(a.ain_w);
  const T* bias = reinterpret_cast<const T*>(a.ain_b);
  T* x = reinterpret_cast<T*>(a.x);
  for (int i = tid; i < M * cols; i += NT) {
    const int m = i / cols, n = u * cols + (i - (i / cols) * cols);
    const T* wr = W + (size_t)n * D;
    float acc = 0.f;
    for (int k = 0; k < D; ++k) acc = fmaf(sx[m * D + k], Tr<T>::f(wr[k]), acc);
    const float y = Tr<T>::r(Tr<T>::r(acc) + Tr<T>::f(bias[n]));
    x[(size_t)m * W1 + n] = Tr<T>::t(y);
    sy[i] = y;
  }
  __syncthreads();
  for (int m = tid; m < M; m += NT) {
    float q = 0.f;
    for (int c = 0; c < cols; ++c) q += sy[m * cols + c] * sy[m * cols + c];
    a.ssq[(size_t)m * SSQ_PARTS + u] = q;
  }
  __syncthreads();
}

// final adaRMSNorm + action_out_proj (+ Euler): one warp per (row, output), over the grid
template <typename T>
__device__ __noinline__ void action_out_phase(const StepArgs& a, bool work) {
  if (!work) return;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (NT / 32) + (threadIdx.x >> 5), nw = gridDim.x * (NT / 32);
  const T* mod = reinterpret_cast<const T*>(a.mods) + (size_t)(2 * a.L) * 3 * a.W1;
  for (int it = gw; it < a.M * a.D; it += nw) {
    const int r = it / a.D, d = it - r * a.D;
    action_out_warp<T>(reinterpret_cast<const T*>(a.x), r, d, a.W1, mod, a.eps,
                       reinterpret_cast<const T*>(a.aout_w), reinterpret_cast<const T*>(a.aout_b),
                       a.D, a.out, a.euler, a.dt, lane);
  }
}

// The attention phase of one CTA of an attention cluster (separately register-allocated).
template <bool LO>
__device__ __forceinline__ void attn_phase(const CUtensorMap& tmQ, const CUtensorMap& tmKA,
                                        const CUtensorMap& tmVA, const CUtensorMap& tmKB,
                                        const CUtensorMap& tmVB, const CUtensorMap& tmQL,
                                        const CUtensorMap& tmKAL, const CUtensorMap& tmKBL,
                                        const atc::AtcArgs& aa, int row0, int tbeg, int n,
                                        int nsplit, uint32_t rank, uint8_t* base, Sh& sh) {
  atc::attn_tile<256, LO>(tmQ, tmKA, tmVA, tmKB, tmVB, tmQL, tmKAL, tmKBL, tmKA, tmVA, tmKAL, aa,
                                0, row0, tbeg,
                                n, nsplit, rank, base, sh.att, sh.tmem, false);
}

// Thread 0: ask L2 for this CTA's weight blocks of GEMM phase g of layer l.
__device__ __forceinline__ void l2_weights(const StepArgs& a, int g, int l, const Work& w) {
  if (l >= a.L || w.tile < 0 || w.nk <= 0) return;
  prefetch_l2(work_src(a, a.layers[l], g, w), (uint32_t)w.nk * W_BLOCK);
}

// Thread 0 (the others only compute the count): the first RING weight blocks of this CTA's GEMM
// phase g of layer l into the ring (the next phase's weights, issued before the barrier).
__device__ __noinline__ int prefetch_next(const StepArgs& a, Sh& sh, uint8_t* base, int g, int l,
                                          uint32_t seq, bool& ok) {
  const Work w = a.plan[g * gridDim.x + blockIdx.x];
  const int n = (l < a.L && w.tile >= 0) ? min((int)w.nk, RING) : 0;
  if (threadIdx.x == 0 && n > 0 && ok)
    if (!issue_weights(sh, base, work_src(a, a.layers[l], g, w), seq, 0, n, a.err)) ok = false;
  return n;
}

// GEMM phase g of layer l with its epilogue (see gemm_phase). Returns the CTA's work item.
template <int G>
__device__ __noinline__ void layer_gemm(const StepArgs& a, const CUtensorMap* tm, Sh& sh,
                                        uint8_t* base, int l, uint32_t& seq, int wpre,
                                        uint32_t& gph, bool& ok) {
  using T = __half;
  const Work w = a.plan[G * gridDim.x + blockIdx.x];
  const Layer& ly = a.layers[l];
  const T* mods = reinterpret_cast<const T*>(a.mods);
  const T* m_in = mods + (size_t)(2 * l) * 3 * a.W1;
  const T* m_post = mods + (size_t)(2 * l + 1) * 3 * a.W1;
  const uint8_t* src = work_src(a, ly, G, w);
  if constexpr (G == G_QKV) {
    EpiQkvRope<T> eq{a.qs, a.ksuf, reinterpret_cast<T*>(a.vsuf), a.scos, a.ssin,
                     a.S * (a.hd / 2), a.S, a.H, 1, a.hd, 0, a.qscale};
    eq.q16 = reinterpret_cast<T*>(a.q16);
    eq.k16 = reinterpret_cast<T*>(a.k16);
    eq.q16lo = reinterpret_cast<T*>(a.q16lo);
    eq.k16lo = reinterpret_cast<T*>(a.k16lo);
    gemm_phase<T, true, false>(a, sh, base, w, src, tm, m_in, a.N[G], a.K[G], eq, seq, wpre, gph, ok);
  } else if constexpr (G == G_O) {
    gemm_phase<T, false, true>(a, sh, base, w, src, tm, nullptr, a.N[G], a.K[G],
                               EpiGatedResid<T>{reinterpret_cast<T*>(a.x), a.W1, m_in + 2 * a.W1, a.M, 0},
                               seq, wpre, gph, ok);
  } else if constexpr (G == G_GU) {
    gemm_phase<T, true, false>(a, sh, base, w, src, tm, m_post, a.N[G], a.K[G],
                               EpiGeglu<T>{reinterpret_cast<T*>(a.h), a.F1}, seq, wpre, gph, ok);
  } else {
    gemm_phase<T, false, true>(a, sh, base, w, src, tm, nullptr, a.N[G], a.K[G],
                               EpiGatedResid<T>{reinterpret_cast<T*>(a.x), a.W1, m_post + 2 * a.W1, a.M, 0},
                               seq, wpre, gph, ok);
  }
  if (w.tile >= 0 && w.nk > 0) ++gph;
}

// Thread 0 at the start of a phase: L2 requests for this CTA's weights of GEMM phase g of layer
// l and (att) its prefix K/V tiles of layer l's attention.
__device__ __noinline__ void l2_ahead(const StepArgs& a, int g, int l, bool att, uint32_t rank) {
  if (threadIdx.x != 0) return;
  if (l < a.L) l2_weights(a, g, l, a.plan[g * gridDim.x + blockIdx.x]);
  if (att && l < a.L) {
    const int tbeg = (int)rank * a.att_tps;
    const int t1 = min(a.att_ntA, tbeg + a.att_tps);
    if (t1 > tbeg) {
      const size_t row = (size_t)l * a.P + (size_t)tbeg * atc::KB;
      const size_t rows = min((size_t)(t1 - tbeg) * atc::KB, (size_t)a.P - (size_t)tbeg * atc::KB);
      const uint32_t bytes = (uint32_t)(rows * a.hd * 2);
      prefetch_l2(reinterpret_cast<const uint8_t*>(a.kA16) + row * a.hd * 2, bytes);
      prefetch_l2(reinterpret_cast<const uint8_t*>(a.vA) + row * a.hd * 2, bytes);
      if (a.kA16lo != a.kA16)
        prefetch_l2(reinterpret_cast<const uint8_t*>(a.kA16lo) + row * a.hd * 2, bytes);
    }
  }
}

// Tensor maps: tmX / tmA / tmH the activations x [M, W1], attention output [M, H·hd], MLP hidden
// [M, F1] (NA-row boxes); tmQ / tmQL q16 and its lo part [S·H, hd] (128-row boxes); tmKA / tmKAL /
// tmVA the half-scale prefix keys (hi, lo) and the values of all layers [L·P, hd]; tmKB / tmKBL /
// tmVB the suffix keys and values [S, hd] (64-row boxes).
template <bool LO>
__global__ void __launch_bounds__(NT, 1)
    denoise_step_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmQL, const __grid_constant__ CUtensorMap tmKA,
                        const __grid_constant__ CUtensorMap tmKAL, const __grid_constant__ CUtensorMap tmVA,
                        const __grid_constant__ CUtensorMap tmKB, const __grid_constant__ CUtensorMap tmKBL,
                        const __grid_constant__ CUtensorMap tmVB, const __grid_constant__ StepArgs a) {
  using T = __half;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  __shared__ Sh sh;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int cl = blockIdx.x / CL;
  const unsigned ncl = (unsigned)(gridDim.x / CL);
  const uint32_t rank = cluster_rank();

  if (tid == 0) {
    for (int s = 0; s < RING; ++s) {
      mbar_init(&sh.full_w[s], 1);
      mbar_init(&sh.full_x[s], 1);
      mbar_init(&sh.ready_x[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    mbar_init(&sh.bar_mma, 1);
    mbar_init(&sh.recv_bar, 1);
    sh.rx_par = 0;
    sh.recv_uses = 0;
    atc::atc_init(sh.att);
    sh.stop = 0;
    sh.w_end = 0;
    sh.x_end = 0;
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmH);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sh.tmem)),
                 "r"(512u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every rank's barriers are initialised before any DSMEM traffic
  tc_fence_after();

  const bool att_cta = cl < a.att_row_tiles;
  uint32_t seq = 0, gph = 0;
  bool ok = true;   // this CTA's work so far is sound (a failed wait clears it)
  bool run = true;  // the grid is still in step (cluster-uniform: grid barrier verdicts)

  action_in_phase<T>(a, base, true);
  int wpre = prefetch_next(a, sh, base, G_QKV, 0, seq, ok);
  run = grid_sync(a.bar, ncl, a.err, &sh.ok);

  for (int l = 0; l < a.L && run; ++l) {
    // ---- q/k/v: adaRMSNorm(x) · Wqkvᵀ, RoPE, q and the suffix K/V (fp16 hi / lo copies) ----
    l2_ahead(a, G_O, l, att_cta, rank);
    layer_gemm<G_QKV>(a, &tmX, sh, base, l, seq, wpre, gph, ok);
    wpre = att_cta ? 0 : prefetch_next(a, sh, base, G_O, l, seq, ok);
    if (tid == 0) tma_prefetch_desc(&tmA);
    run = grid_sync(a.bar, ncl, a.err, &sh.ok);
    if (!run) break;
    // ---- attention over [prefix cache of layer l ; suffix K/V] ----
    l2_ahead(a, G_GU, l, false, rank);
    if (att_cta) {
      if (tid == 0) {  // fresh barriers for this layer's attention (the last one is drained)
        atc::atc_inval(sh.att);
        atc::atc_init(sh.att);
      }
      __syncthreads();
      atc::AtcArgs aa{};
      aa.rows = a.S * a.H;
      aa.LA = a.P;
      aa.LB = a.S;
      aa.ntA = a.att_ntA;
      aa.nt = a.att_nt;
      aa.tps = a.att_tps;
      aa.maskA = a.maskA;
      aa.out = a.attn;
      aa.err = a.err;
      aa.ya0 = l * a.P;
      aa.v_lbo = atc::KB * 128;
      aa.v_sbo = 1024;
      const int tbeg = (int)rank * a.att_tps;
      const int n = (ok && (int)rank < a.att_splits) ? max(0, min(a.att_nt, tbeg + a.att_tps) - tbeg) : 0;
      attn_phase<LO>(tmQ, tmKA, tmVA, tmKB, tmVB, tmQL, tmKAL, tmKBL, aa, cl * 128, tbeg, n,
                     a.att_splits, rank, base, sh);
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      wpre = prefetch_next(a, sh, base, G_O, l, seq, ok);
    }
    run = grid_sync(a.bar, ncl, a.err, &sh.ok);
    if (!run) break;
    // ---- o_proj + gated residual (+ row Σx² partials) ----
    l2_ahead(a, G_D, l, false, rank);
    layer_gemm<G_O>(a, &tmA, sh, base, l, seq, wpre, gph, ok);
    wpre = prefetch_next(a, sh, base, G_GU, l, seq, ok);
    if (tid == 0) tma_prefetch_desc(&tmX);
    run = grid_sync(a.bar, ncl, a.err, &sh.ok);
    if (!run) break;
    // ---- gate_up (adaRMSNorm fused) + GeGLU ----
    l2_ahead(a, G_QKV, l + 1, false, rank);
    layer_gemm<G_GU>(a, &tmX, sh, base, l, seq, wpre, gph, ok);
    wpre = prefetch_next(a, sh, base, G_D, l, seq, ok);
    if (tid == 0) tma_prefetch_desc(&tmH);
    run = grid_sync(a.bar, ncl, a.err, &sh.ok);
    if (!run) break;
    // ---- down + gated residual (+ row Σx² partials) ----
    l2_ahead(a, G_O, l + 1, false, rank);
    layer_gemm<G_D>(a, &tmH, sh, base, l, seq, wpre, gph, ok);
    wpre = prefetch_next(a, sh, base, G_QKV, l + 1, seq, ok);
    if (tid == 0) tma_prefetch_desc(&tmX);
    run = grid_sync(a.bar, ncl, a.err, &sh.ok);
  }
  if (run) action_out_phase<T>(a, ok);

  // ---- exit: no copy may still be writing this CTA's shared memory ----
  if (tid == 0) {  // the last fill of every slot (weights, x) has landed
    for (uint32_t q = sh.w_end > RING ? sh.w_end - RING : 0; q < sh.w_end; ++q)
      mbar_wait(&sh.full_w[q % RING], (q / RING) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
    for (uint32_t q = sh.x_end > RING ? sh.x_end - RING : 0; q < sh.x_end; ++q)
      mbar_wait(&sh.full_x[q % RING], (q / RING) & 1, a.err, ERR_TIMEOUT_PRODUCER, false);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sh.tmem), "r"(512u));
  }
}

}  // namespace ds
}  // namespace pi0
