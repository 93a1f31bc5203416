// libpi0b200.so — context, parameter table, weight arena and the three exported functions of
// the π0.5 M1 hot path (prefill, denoise_step_kv, denoise_loop_kv) behind the C ABI declared in
// include/pi0b200.h.
//
// One context owns, on one GPU:
//   * the parameter table in the reference's export order (names, shapes, dtypes);
//   * a weight arena holding a repacked copy of the caller's parameters: per layer the q/k/v
//     rows of each expert are concatenated (q and k rows permuted per head for the RoPE
//     epilogue), gate/up rows are interleaved for the GeGLU epilogue, and the 2·L+1 adaRMS
//     modulation matrices of the action expert are concatenated into one matrix so a single
//     weight-streaming launch produces every modulation of a step (or of all N steps);
//   * workspaces sized for cfg.max_batch requests, the prefix RoPE table, split-K and
//     attention partial buffers, and the CUDA graphs of denoise_loop_kv.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "pi0b200.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "common.cuh"
#include "gemm_mma.cuh"
#include "gemm_tc.cuh"
#include "gemm_skinny.cuh"
#include "small_kernels.cuh"
#include "denoise_step.cuh"

using namespace pi0;

namespace {

enum Role {
  R_Q, R_K, R_V, R_O, R_GU, R_D,   // attention / MLP linears (expert e, layer l)
  R_LN_IN, R_LN_POST,              // expert-0 plain norm weights
  R_MOD_W, R_MOD_B,                // expert-1 modulation (block index in `layer`)
  R_FINAL0,                        // expert-0 final norm weight (unused on the M1 path)
  R_AIN_W, R_AIN_B, R_AOUT_W, R_AOUT_B, R_TIN_W, R_TIN_B, R_TOUT_W, R_TOUT_B
};

struct Entry {
  std::string name;
  int ndim;
  int64_t shape[2];
  int dtype;
  Role role;
  int expert;
  int layer;  // layer index, or modulation block for R_MOD_*
  int in_dim = 0;  // quantised Linear entries: the unpadded input width K
};

struct LayerW {
  void* qkv;   // [Hq + 2·Hkv, W]
  void* o;     // [W, Hq]
  void* gu;    // [2F, W] interleaved
  void* d;     // [W, F]
  void* ln_in;
  void* ln_post;
  // action expert only: the same matrices packed for the weight-streaming GEMM
  void *qkv_p = nullptr, *o_p = nullptr, *gu_p = nullptr, *d_p = nullptr;
  // quantised models: the same matrices as group-quantised blocks (pack_q_kernel layout), which
  // the weight-streaming kernel dequantises in shared memory; null when not in use
  void *qkv_q = nullptr, *o_q = nullptr, *gu_q = nullptr, *d_q = nullptr;
};

struct GraphKey {
  int batch;
  const void* p[9];
  bool operator<(const GraphKey& o) const {
    if (batch != o.batch) return batch < o.batch;
    return std::memcmp(p, o.p, sizeof(p)) < 0;
  }
};

}  // namespace

struct pi0_ctx {
  pi0_config cfg{};
  int device = 0;
  std::string err;
  std::vector<Entry> table;
  bool have_params = false;
  size_t esz = 2;

  // weights
  void* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<LayerW> pre, suf;
  void *mod_w = nullptr, *mod_b = nullptr;
  void *ain_w = nullptr, *ain_b = nullptr, *aout_w = nullptr, *aout_b = nullptr;
  void *tin_w = nullptr, *tin_b = nullptr, *tout_w = nullptr, *tout_b = nullptr;
  void *mod_w_p = nullptr, *tin_p = nullptr, *tout_p = nullptr;  // packed copies
  void *mod_w_q = nullptr, *tin_q = nullptr, *tout_q = nullptr;  // quantised blocks (qb != 0)
  int qb = 0;  // 4 / 3: the weight-streaming GEMMs read q4 / q3 blocks; 0: 16-bit blocks
  float* ssq = nullptr;  // [max_batch·S][ssq_parts] row Σx² partials of the suffix stream
  int ssq_parts = 1;
  int* perm_q = nullptr;   // RoPE row permutation of a q block (H·hd rows)
  int* perm_k = nullptr;   // ... of a k block (KV·hd rows)
  int* perm_gu0 = nullptr; // gate/up interleave for F0
  int* perm_gu1 = nullptr; // ... for F1
  float* rope_cos = nullptr;  // prefix RoPE table [P, hd/2]
  float* rope_sin = nullptr;
  // the M0 joint denoise_step: its own prefix K/V cache, an all-valid prefix mask and the suffix
  // RoPE tables at positions P .. P+S-1, for every request of a batch
  float *m0_keys = nullptr, *m0_mask = nullptr, *m0_cos = nullptr, *m0_sin = nullptr;
  void* m0_values = nullptr;

  // workspaces
  void *xp = nullptr, *xpn = nullptr, *attn_p = nullptr, *hp = nullptr;
  float* qp = nullptr;
  void *xs = nullptr, *xsn = nullptr, *attn_s = nullptr, *hs = nullptr, *vsuf = nullptr;
  float *qs = nullptr, *ksuf = nullptr;
  // tensor-core attention (fp16 models, one kv head): model-dtype q, and k copies at half scale
  bool attn_tc = false;
  void *q16p = nullptr, *q16s = nullptr, *kpre16 = nullptr, *ksuf16 = nullptr;
  // fp32 attention logits (the reference's default): q·k from fp32 operands. With the tensor-core
  // attention, the fp16 lo parts x − fp16(x) of the same q and half-scale k
  bool logits_f32 = true;
  void *q16p_lo = nullptr, *q16s_lo = nullptr, *kpre16_lo = nullptr, *ksuf16_lo = nullptr;
  bool pdl_barrier = false;  // the next launch waits for full completion of the previous one
  // persistent denoise step (denoise_step.cuh): batch-1 fp16 π0.5-width models
  bool step_kernel = false;
  int step_grid = 0;
  ds::Work* step_plan = nullptr;    // [G_NUM][step_grid]
  ds::Layer* step_layers = nullptr; // [depth]
  unsigned long long* step_bar = nullptr;  // grid barrier word
  int step_tiles[ds::G_NUM] = {}, step_nkb[ds::G_NUM] = {}, step_N[ds::G_NUM] = {},
      step_K[ds::G_NUM] = {};
  int att_row_tiles = 0, att_tps = 0, att_splits = 0, att_ntA = 0, att_nt = 0;
  std::string step_why;             // why the persistent step is not used (empty: it is)
  void* qscratch = nullptr;  // quantised parameters: one dequantised Linear at a time
  size_t qscratch_elems = 0;
  void *t1 = nullptr, *cond = nullptr, *mods = nullptr;
  float* splitk_ws = nullptr;
  size_t splitk_floats = 0;
  int* tickets = nullptr;
  int* dev_err = nullptr;  // device error flag written by bounded waits
  int num_sms = 148;
  bool use_tc = true;      // tensor-core (tcgen05) GEMMs for M >= 128
  bool pdl = true;         // programmatic dependent launch between the kernels of a chain
  bool cta_pair = true;    // CTA-pair tiles for GEMMs of two or more waves (PI0_CTA_PAIR=0: off)

  cudaStream_t cap_stream = nullptr;
  std::map<GraphKey, std::pair<cudaGraphExec_t, int64_t>> graphs;  // exec, kernel nodes

  // measurement
  int64_t launches = 0;
  bool prof_on = false;
  struct ProfRec {
    int fam;
    cudaEvent_t a, b;
  };
  std::vector<ProfRec> prof;
  std::vector<cudaEvent_t> ev_pool;

  std::vector<void*> allocs;
};

namespace {

// kernel families reported by pi0_profile_read
enum Fam {
  F_PRE_NORM, F_PRE_QKV, F_PRE_ATTN, F_PRE_O, F_PRE_GU, F_PRE_DOWN,
  F_DEN_TIME_MODS, F_DEN_ACT_IN, F_DEN_NORM, F_DEN_QKV, F_DEN_ATTN, F_DEN_O, F_DEN_GU,
  F_DEN_DOWN, F_DEN_ACT_OUT, F_DEN_KEYS16, F_DEN_STEP,
  F_VIS_PATCH, F_VIS_NORM, F_VIS_QKV, F_VIS_ATTN, F_VIS_O, F_VIS_FC1, F_VIS_FC2, F_VIS_PROJ, F_NUM
};
const char* kFamName[F_NUM] = {
  "prefill.rmsnorm", "prefill.qkv_rope_gemm", "prefill.attention", "prefill.o_gemm",
  "prefill.gate_up_geglu_gemm", "prefill.down_gemm",
  "denoise.time_mlp_modulation_gemm", "denoise.action_in", "denoise.ada_rmsnorm",
  "denoise.qkv_rope_gemm", "denoise.attention", "denoise.o_gemm", "denoise.gate_up_geglu_gemm",
  "denoise.down_gemm", "denoise.action_out_euler", "denoise.prefix_keys_fp16",
  "denoise.step_persistent",
  "vision.patchify_embed_gemm", "vision.layernorm", "vision.qkv_gemm", "vision.attention",
  "vision.out_gemm", "vision.fc1_gelu_gemm", "vision.fc2_gemm", "vision.projector_gemm"};

int fail(pi0_ctx* c, int code, const std::string& msg) {
  if (c) c->err = msg;
  return code;
}

#define CK(call)                                                                      \
  do {                                                                                \
    cudaError_t e_ = (call);                                                          \
    if (e_ != cudaSuccess)                                                            \
      return fail(ctx, PI0_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define CKL()                                                                         \
  do {                                                                                \
    cudaError_t e_ = cudaGetLastError();                                              \
    if (e_ != cudaSuccess)                                                            \
      return fail(ctx, PI0_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e_) + \
                                         " at " + __FILE__ + ":" + std::to_string(__LINE__)); \
  } while (0)

#define TRY(...)          \
  do {                    \
    int r_ = (__VA_ARGS__); \
    if (r_) return r_;    \
  } while (0)

int dev_alloc(pi0_ctx* ctx, void** p, size_t bytes) {
  if (bytes == 0) bytes = 16;
  CK(cudaMalloc(p, bytes));
  ctx->allocs.push_back(*p);
  return 0;
}

// Brackets the launches of one kernel family with events while profiling is on.
struct Prof {
  pi0_ctx* c;
  cudaStream_t st;
  int idx = -1;
  Prof(pi0_ctx* ctx, int fam, cudaStream_t s) : c(ctx), st(s) {
    if (!c->prof_on) return;
    cudaEvent_t a, b;
    if (c->ev_pool.size() >= 2) {
      a = c->ev_pool.back(); c->ev_pool.pop_back();
      b = c->ev_pool.back(); c->ev_pool.pop_back();
    } else {
      cudaEventCreate(&a);
      cudaEventCreate(&b);
    }
    cudaEventRecordWithFlags(a, st, cudaEventRecordExternal);  // a graph node under capture
    c->prof.push_back({fam, a, b});
    idx = (int)c->prof.size() - 1;
  }
  ~Prof() {
    if (idx >= 0) cudaEventRecordWithFlags(c->prof[idx].b, st, cudaEventRecordExternal);
  }
};

// Launch through cudaLaunchKernelEx: programmatic dependent launch (kernels start their
// independent prologue while the previous kernel drains) and an optional cluster.
template <typename... KArgs, typename... Args>
int launch(pi0_ctx* ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t st, dim3 cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int n = 0;
  const bool pdl = ctx->pdl && !ctx->pdl_barrier;
  ctx->pdl_barrier = false;
  if (pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = cluster.x;
    at[n].val.clusterDim.y = cluster.y;
    at[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess)
    return fail(ctx, PI0_ERR_CUDA, std::string("cudaLaunchKernelEx: ") + cudaGetErrorString(e));
  ctx->launches += 1;
  return 0;
}

// ---- parameter table (reference export order; see mlc_vla/model/pi0/pi0_model.py) ----------
void build_table(pi0_ctx* c) {
  const pi0_config& g = c->cfg;
  const int hq = g.num_heads * g.head_dim, hkv = g.num_kv_heads * g.head_dim;
  const int W[2] = {g.vlm_width, g.ae_width}, F[2] = {g.vlm_mlp_dim, g.ae_mlp_dim};
  const int dt = g.dtype;
  const bool q = g.quant != PI0_QUANT_NONE;
  const int G = g.quant == PI0_QUANT_Q3 ? 40 : 32, epw = g.quant == PI0_QUANT_Q3 ? 10 : 8;
  auto lin = [&](const std::string& name, int out, int in, bool bias, Role rw, Role rb, int e,
                 int l) {
    if (!q) {
      c->table.push_back({name + ".weight", 2, {out, in}, dt, rw, e, l});
    } else {
      int64_t ng = (in + G - 1) / G;
      c->table.push_back({name + ".q_weight", 2, {out, ng * (G / epw)}, PI0_U32, rw, e, l, in});
      c->table.push_back({name + ".q_scale", 2, {out, ng}, dt, rw, e, l, in});
    }
    if (bias) c->table.push_back({name + ".bias", 1, {out, 0}, dt, rb, e, l});
  };
  for (int l = 0; l < g.depth; ++l) {
    std::string p = "backbone.layers." + std::to_string(l) + ".";
    for (int e = 0; e < 2; ++e) {
      std::string a = p + "self_attn.experts." + std::to_string(e) + ".";
      lin(a + "q_proj", hq, W[e], false, R_Q, R_Q, e, l);
      lin(a + "k_proj", hkv, W[e], false, R_K, R_K, e, l);
      lin(a + "v_proj", hkv, W[e], false, R_V, R_V, e, l);
      lin(a + "o_proj", W[e], hq, false, R_O, R_O, e, l);
    }
    for (int e = 0; e < 2; ++e) {
      std::string m = p + "mlp." + std::to_string(e) + ".";
      lin(m + "gate_up_proj", 2 * F[e], W[e], false, R_GU, R_GU, e, l);
      lin(m + "down_proj", W[e], F[e], false, R_D, R_D, e, l);
    }
    const char* lns[2] = {"input_layernorm", "post_attention_layernorm"};
    for (int k = 0; k < 2; ++k) {
      c->table.push_back({p + lns[k] + ".0.weight", 1, {W[0], 0}, dt, k ? R_LN_POST : R_LN_IN, 0, l});
      lin(p + lns[k] + ".1.modulation", 3 * W[1], W[1], true, R_MOD_W, R_MOD_B, 1, 2 * l + k);
    }
  }
  c->table.push_back({"backbone.final_norm.0.weight", 1, {W[0], 0}, dt, R_FINAL0, 0, 0});
  lin("backbone.final_norm.1.modulation", 3 * W[1], W[1], true, R_MOD_W, R_MOD_B, 1, 2 * g.depth);
  lin("action_in_proj", W[1], g.action_dim, true, R_AIN_W, R_AIN_B, 1, 0);
  lin("action_out_proj", g.action_dim, W[1], true, R_AOUT_W, R_AOUT_B, 1, 0);
  lin("time_mlp_in", W[1], W[1], true, R_TIN_W, R_TIN_B, 1, 0);
  lin("time_mlp_out", W[1], W[1], true, R_TOUT_W, R_TOUT_B, 1, 0);
}

int validate(const pi0_config& g, std::string& why) {
  auto bad = [&](const char* m) { why = m; return PI0_ERR_INVALID; };
  if (g.dtype != PI0_F16 && g.dtype != PI0_BF16) {
    why = "model dtype must be float16 or bfloat16 on the GPU path";
    return PI0_ERR_UNSUPPORTED;
  }
  if (g.quant != PI0_QUANT_NONE && g.quant != PI0_QUANT_Q4 && g.quant != PI0_QUANT_Q3)
    return bad("unknown quant format");
  int hd = g.head_dim;
  if (!(hd == 16 || hd == 32 || hd == 64 || hd == 128 || hd == 256)) {
    why = "head_dim must be one of 16, 32, 64, 128, 256";
    return PI0_ERR_UNSUPPORTED;
  }
  if (g.depth < 1 || g.num_heads < 1 || g.num_kv_heads < 1 || g.num_heads % g.num_kv_heads)
    return bad("depth/num_heads/num_kv_heads invalid (num_heads must be a multiple of num_kv_heads)");
  if (g.vlm_width % 32 || g.ae_width % 32 || g.vlm_mlp_dim % 32 || g.ae_mlp_dim % 32 ||
      (g.num_heads * hd) % 32)
    return bad("widths, mlp dims and num_heads*head_dim must be multiples of 32");
  if (g.vlm_width <= 0 || g.ae_width <= 0 || g.vlm_mlp_dim <= 0 || g.ae_mlp_dim <= 0)
    return bad("widths and mlp dims must be positive");
  if (g.prefix_len < 1 || g.action_horizon < 1 || g.action_dim < 1 || g.num_denoise_steps < 1)
    return bad("prefix_len, action_horizon, action_dim and num_denoise_steps must be >= 1");
  if (g.max_batch < 1) return bad("max_batch must be >= 1");
  if (g.ae_width > 4096 || g.vlm_width > 4096)
    return bad("expert widths above 4096 are not supported");
  if (g.action_dim > 4096) return bad("action_dim above 4096 is not supported");
  if (g.attn_logits != PI0_LOGITS_F32 && g.attn_logits != PI0_LOGITS_MODEL_DTYPE)
    return bad("attn_logits must be PI0_LOGITS_F32 or PI0_LOGITS_MODEL_DTYPE");
  return 0;
}


// ---- TMA tensor maps (driver entry point fetched through the runtime, no libcuda link) ------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

int get_encode(pi0_ctx* ctx) {
  if (g_encode) return 0;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess || !fn)
    return fail(ctx, PI0_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
  g_encode = (EncodeTiledFn)fn;
  return 0;
}

// 2-D K-major tile map of a [rows, cols] 16-bit matrix with row stride ld (elements):
// box = 64 columns (128 B, one swizzle row) × box_rows rows, zero fill out of bounds.
int make_tmap(pi0_ctx* ctx, CUtensorMap* m, const void* base, int rows, int cols, int ld,
              int box_rows, bool bf16) {
  TRY(get_encode(ctx));
  if (((uintptr_t)base & 15) || ((size_t)ld * 2) % 16)
    return fail(ctx, PI0_ERR_INVALID, "TMA operand must be 16-byte aligned with 16-byte row stride");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ctx, PI0_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return 0;
}

template <typename T, int BN, int ST, class Epi>
int gemm_tc_launch(pi0_ctx* ctx, const T* A, int lda, const T* W, int ldw, int M, int N, int K,
                   const Epi& epi, cudaStream_t st, int fam) {
  CUtensorMap ta, tb;
  const bool bf = Tr<T>::kBf16;
  TRY(make_tmap(ctx, &ta, A, M, K, lda, tc::BM, bf));
  TRY(make_tmap(ctx, &tb, W, N, K, ldw, BN, bf));
  const int tiles = ((M + tc::BM - 1) / tc::BM) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, ctx->num_sms);
  Prof pr(ctx, fam, st);
  return launch(ctx, tc::gemm_tc_kernel<T, BN, ST, Epi>, dim3(grid), dim3(tc::NT),
                tc::Smem<BN, ST>::BYTES, st, dim3(1, 1, 1), ta, tb, M, N, K, epi, ctx->dev_err);
}

// Split-K pair (gemm_tc_kernel KS = 2) with 128×256 tiles: for a GEMM whose 256-wide tiles fill
// under half the SMs but whose K is long (the prefill down projection: 64 tiles, K = 16384), two
// CTAs per tile keep every SM's tensor pipe fed from a 4-stage ring of 256-wide stages, which a
// 128-wide tile's ring of the same size cannot (its stages drain faster than L2 refills them).
bool use_splitk_pair(int M, int N, int K, int sms) {
  const int tiles = ((M + tc::BM - 1) / tc::BM) * ((N + 255) / 256);
  return K >= 64 * tc::BK && 2 * tiles <= sms && 4 * tiles > sms;
}
template <typename T, class Epi, int BN = 256, int ST = 4>
int gemm_tc_pair_launch(pi0_ctx* ctx, const T* A, int lda, const T* W, int ldw, int M, int N,
                        int K, const Epi& epi, cudaStream_t st, int fam) {
  CUtensorMap ta, tb;
  const bool bf = Tr<T>::kBf16;
  TRY(make_tmap(ctx, &ta, A, M, K, lda, tc::BM, bf));
  TRY(make_tmap(ctx, &tb, W, N, K, ldw, BN, bf));
  const int tiles = ((M + tc::BM - 1) / tc::BM) * ((N + BN - 1) / BN);
  if ((K + tc::BK - 1) / tc::BK < 2)
    return fail(ctx, PI0_ERR_UNSUPPORTED, "split-K pair: K must span at least two k-blocks");
  Prof pr(ctx, fam, st);
  return launch(ctx, tc::gemm_tc_kernel<T, BN, ST, Epi, 2>, dim3(2 * tiles), dim3(tc::NT),
                tc::Smem<BN, ST>::BYTES, st, dim3(2, 1, 1), ta, tb, M, N, K, epi, ctx->dev_err);
}

// CTA-pair tiles (gemm_tc_kernel CG = 2): 256 × 256 output tiles on tcgen05 cta_group::2,
// persistent pairs; each CTA of a pair loads 128 rows of A and 128 rows of W per k-block
// instead of 128 + 256. Used where the pair tiles fill the SMs at least twice over (the prefill
// gate/up projection: 512 pair tiles at batch 1; every prefill projection at batch 8), so each
// pair streams several tiles through a full ring. On GEMMs of one wave (the batch-1 q/k/v and
// o projections, the vision projections) they measured 5-20 % slower than single-CTA tiles.
template <int BN> constexpr int pair_stages() { return BN == 256 ? 6 : 8; }
bool use_cta_pair(int M, int N, int sms) {
  const int pairs = ((M + 255) / 256) * ((N + 255) / 256);
  return M > 256 && N % 256 == 0 && pairs >= 2 * (sms / 2);
}
template <typename T, int BN, class Epi>
int gemm_tc_cg2_launch(pi0_ctx* ctx, const T* A, int lda, const T* W, int ldw, int M, int N,
                       int K, const Epi& epi, cudaStream_t st, int fam) {
  constexpr int ST = pair_stages<BN>();
  CUtensorMap ta, tb;
  const bool bf = Tr<T>::kBf16;
  TRY(make_tmap(ctx, &ta, A, M, K, lda, tc::BM, bf));
  TRY(make_tmap(ctx, &tb, W, N, K, ldw, BN / 2, bf));
  const int pairs = ((M + 2 * tc::BM - 1) / (2 * tc::BM)) * ((N + BN - 1) / BN);
  const int grid = 2 * std::min(pairs, ctx->num_sms / 2);
  Prof pr(ctx, fam, st);
  return launch(ctx, tc::gemm_tc_kernel<T, BN, ST, Epi, 1, 2>, dim3(grid), dim3(tc::NT),
                tc::Smem<BN, ST, 2>::BYTES, st, dim3(2, 1, 1), ta, tb, M, N, K, epi,
                ctx->dev_err);
}

template <typename T>
int rmsnorm(pi0_ctx* ctx, const T* x, T* out, int rows, int W, const T* w, const T* mod,
            int rows_per_mod, int mod_stride, cudaStream_t st, int fam);
template <typename T, class Epi>
int gemm(pi0_ctx* ctx, const T* A, int lda, const T* W, int ldw, int M, int N, int K,
         const Epi& epi, cudaStream_t st, int fam, int engine = 0);

// Weight-streaming path for M ≤ 128 activation rows (see gemm_skinny.cuh). Cluster size C (the
// K split) is the smallest power of two ≤ 8 that gives at least 128 CTAs, as long as every CTA
// keeps at least two k-blocks to stream; norm-fused launches also split until a CTA's blocks
// fit the ring, so all of its raw activation blocks are requested at once.
int skinny_split(int N, int K, bool norm) {
  const int nkb = (K + 63) / 64, tiles = (N + 127) / 128;
  int C = 1;
  while (C < sk::MAX_C && nkb >= 4 * C &&
         (tiles * C < 128 || (norm && (nkb + C - 1) / C > sk::RING)))
    C *= 2;
  return C;
}

// Row Σx² partial slots of the suffix residual stream: one per (tile, rank) of the widest
// residual-producing projection (o_proj, down_proj), rounded up to a multiple of 16.
int ssq_slots(const pi0_config& c) {
  const int W1 = c.ae_width;
  const int tiles = (W1 + 127) / 128;
  const int p = tiles * std::max(skinny_split(W1, c.num_heads * c.head_dim, false),
                                 skinny_split(W1, c.ae_mlp_dim, false));
  return (p + 15) / 16 * 16;
}

struct SkOpt {
  const void* wpack = nullptr;  // packed weights (pack_sw128 layout), or null: tensor map on W
  const void* mod = nullptr;    // NORM: modulation row (scale | shift)
};

template <typename T, int NA, bool NORM, bool SSQ, int QB = 0, class Epi>
int skinny_launch(pi0_ctx* ctx, const T* X, int ldx, const T* W, int ldw, int M, int N, int K,
                  const Epi& epi, cudaStream_t st, int fam, SkOpt o) {
  const int nkb = (K + 63) / 64, tiles = (N + 127) / 128;
  const int C = skinny_split(N, K, NORM);
  const int kbpc = (nkb + C - 1) / C;
  if (NORM && (K % 8 || ldx != K))
    return fail(ctx, PI0_ERR_UNSUPPORTED, "norm-fused GEMM needs K % 8 == 0 and dense rows");
  if (SSQ && tiles * C > ctx->ssq_parts)
    return fail(ctx, PI0_ERR_INVALID, "row-sum partials: more (tile, rank) pairs than slots");
  CUtensorMap tw, tx;
  const bool bf = Tr<T>::kBf16;
  TRY(make_tmap(ctx, &tw, W, N, K, ldw, tc::BM, bf));
  TRY(make_tmap(ctx, &tx, X, M, K, ldx, NA, bf));
  sk::SkArgs a{M, N, K, kbpc, C, ctx->dev_err, o.wpack, X, o.mod, ctx->cfg.rms_norm_eps,
               ctx->ssq, ctx->ssq, ctx->ssq_parts};
  Prof pr(ctx, fam, st);
  return launch(ctx, sk::skinny_kernel<T, NA, NORM, SSQ, Epi, QB>, dim3(tiles * C), dim3(sk::NT),
                sk::SkSmem<NA>::BYTES, st, dim3(C, 1, 1), tw, tx, a, epi);
}

// Denoise-path projection: the weight-streaming kernel for M ≤ 128 (group-quantised blocks `Wq`
// when the context has them, else packed 16-bit weights `Wp`), the tensor-core tile kernel
// otherwise (row-major `W`). NORM: the input is adaRMSNorm(A; mod) (fused for M ≤ 128, a
// separate norm kernel into `scratch` otherwise). SSQ: the epilogue also emits the row Σx²
// partials of its output stream.
template <typename T, bool NORM, bool SSQ, class Epi>
int gemm_w(pi0_ctx* ctx, const T* A, int lda, const T* W, const T* Wp, const void* Wq, int M,
           int N, int K, const Epi& epi, cudaStream_t st, int fam, const T* mod = nullptr,
           T* scratch = nullptr) {
  SkOpt o;
  o.wpack = Wp;
  o.mod = mod;
  if (M <= 128 && Wq && ctx->qb) {
    o.wpack = Wq;
    if (ctx->qb == 4)
      return M <= 64 ? skinny_launch<T, 64, NORM, SSQ, 4>(ctx, A, lda, W, K, M, N, K, epi, st, fam, o)
                     : skinny_launch<T, 128, NORM, SSQ, 4>(ctx, A, lda, W, K, M, N, K, epi, st, fam, o);
    return M <= 64 ? skinny_launch<T, 64, NORM, SSQ, 3>(ctx, A, lda, W, K, M, N, K, epi, st, fam, o)
                   : skinny_launch<T, 128, NORM, SSQ, 3>(ctx, A, lda, W, K, M, N, K, epi, st, fam, o);
  }
  if (M <= 64) return skinny_launch<T, 64, NORM, SSQ>(ctx, A, lda, W, K, M, N, K, epi, st, fam, o);
  if (M <= 128) return skinny_launch<T, 128, NORM, SSQ>(ctx, A, lda, W, K, M, N, K, epi, st, fam, o);
  if (NORM) {
    TRY(rmsnorm<T>(ctx, A, scratch, M, K, nullptr, mod, M, 0, st, F_DEN_NORM));
    return gemm<T>(ctx, scratch, K, W, K, M, N, K, epi, st, fam);
  }
  return gemm<T>(ctx, A, lda, W, K, M, N, K, epi, st, fam);
}

// Waves-aware tile width for the tensor-core GEMM: the widest of 256 / 160 / 128 whose last
// wave is fullest.
int pick_bn(int M, int N, int sms) {
  const int cands[3] = {256, 160, 128};
  int best = 128;
  double best_eff = -1.0;
  for (int bn : cands) {
    int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
    int waves = (tiles + sms - 1) / sms;
    double eff = (double)tiles / (waves * sms) * ((double)N / (((N + bn - 1) / bn) * bn));
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = bn;
    }
  }
  return best;
}

// ---- GEMM launch --------------------------------------------------------------------------
template <typename T, int BM, int BN, int WM, int WN, int ST, class Epi>
int gemm_launch_cfg(pi0_ctx* ctx, const T* A, int lda, const T* W, int ldw, int M, int N, int K,
                    const Epi& epi, int splits, cudaStream_t st, int fam) {
  using C = GemmCfg<T, BM, BN, WM, WN, ST>;
  auto kern = gemm_mma_kernel<T, BM, BN, WM, WN, ST, Epi>;
  GemmArgs<T> g{A, lda, W, ldw, M, N, K, 0, ctx->splitk_ws, ctx->tickets};
  int ksteps = K / 32;
  splits = std::max(1, std::min(splits, ksteps));
  int per = (ksteps + splits - 1) / splits;
  splits = (ksteps + per - 1) / per;
  g.k_split_len = per * 32;
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, splits);
  if (splits > 1) {
    if ((size_t)splits * M * N > ctx->splitk_floats)
      return fail(ctx, PI0_ERR_INVALID, "split-K workspace too small");
    if ((size_t)grid.x * grid.y > (1u << 16)) return fail(ctx, PI0_ERR_INVALID, "too many tiles");
  }
  Prof pr(ctx, fam, st);
  return launch(ctx, kern, grid, dim3(C::NT), C::SMEM, st, dim3(1, 1, 1), g, epi);
}

template <typename T, class Epi>
int gemm(pi0_ctx* ctx, const T* A, int lda, const T* W, int ldw, int M, int N, int K,
         const Epi& epi, cudaStream_t st, int fam, int engine) {
  if ((engine == 0 && M <= 128 && ctx->use_tc) || engine == 3) {
    if (M <= 64) return skinny_launch<T, 64, false, false>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam, SkOpt{});
    return skinny_launch<T, 128, false, false>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam, SkOpt{});
  }
  if (engine == 5) return gemm_tc_cg2_launch<T, 256>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam);
  if ((engine == 0 && M >= 128 && ctx->use_tc) || engine == 1 || engine == 4) {
    if (engine == 4 || (engine == 0 && use_splitk_pair(M, N, K, ctx->num_sms)))
      return gemm_tc_pair_launch<T>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam);
    if (engine == 0 && ctx->cta_pair && use_cta_pair(M, N, ctx->num_sms))
      return gemm_tc_cg2_launch<T, 256>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam);
    switch (pick_bn(M, N, ctx->num_sms)) {
      case 256: return gemm_tc_launch<T, 256, 4>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam);
      case 160: return gemm_tc_launch<T, 160, 5>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam);
      default: return gemm_tc_launch<T, 128, 6>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam);
    }
  }
  if (M >= 256) {
    return gemm_launch_cfg<T, 128, 128, 64, 32, 4>(ctx, A, lda, W, ldw, M, N, K, epi, 1, st, fam);
  }
  int tiles = ((M + 63) / 64) * ((N + 63) / 64);
  int splits = std::max(1, (2 * ctx->num_sms + tiles - 1) / tiles);
  splits = std::min(splits, std::max(1, K / 128));
  return gemm_launch_cfg<T, 64, 64, 32, 32, 4>(ctx, A, lda, W, ldw, M, N, K, epi, splits, st, fam);
}

// ---- attention launch ----------------------------------------------------------------------
// Key splits (a power of two ≤ max_splits, so the splits of a row tile form one cluster): grow
// while the grid stays within two waves over the SMs and every split keeps at least one key tile.
int attn_splits(int rows, int batch, int KV, int ltot, int num_sms, int max_splits) {
  const int row_tiles = (rows + ATT_BQ - 1) / ATT_BQ;
  const int ctas = row_tiles * batch * KV;
  int splits = 1;
  while (splits < max_splits && ctas * splits * 2 <= 2 * num_sms &&
         splits * 2 * ATT_BK <= ltot + ATT_BK)
    splits *= 2;
  return splits;
}
int attn_kps(int ltot, int splits) {
  int kps = (ltot + splits - 1) / splits;
  return (kps + ATT_BK - 1) / ATT_BK * ATT_BK;
}

// The denoise step (segment A = the prefix cache, ready before the previous kernel) splits the
// keys over up to 16 CTAs of one cluster; prefill has enough row tiles without splitting.
template <typename T, int HD>
int attn_launch_hd(pi0_ctx* ctx, AttnArgs<T> a, int batch, bool allow_split, cudaStream_t st,
                   int fam) {
  Prof pr(ctx, fam, st);
  const int G = a.H / a.KV, rows = a.Tq * G;
  const int row_tiles = (rows + ATT_BQ - 1) / ATT_BQ;
  const int ltot = a.LA + a.LB;
  const int splits = attn_splits(rows, batch, a.KV, ltot, ctx->num_sms, allow_split ? 16 : 1);
  a.keys_per_split = attn_kps(ltot, splits);
  dim3 grid(row_tiles, splits, batch * a.KV);
  return launch(ctx, attn_kernel<T, HD, ATT_BK>, grid, dim3(128), AttnSmem<HD, ATT_BK>::BYTES, st,
                dim3(1, splits, 1), a);
}

template <typename T>
int attn_launch(pi0_ctx* ctx, AttnArgs<T> a, int batch, bool allow_split, cudaStream_t st,
                int fam) {
  switch (ctx->cfg.head_dim) {
    case 16: return attn_launch_hd<T, 16>(ctx, a, batch, allow_split, st, fam);
    case 32: return attn_launch_hd<T, 32>(ctx, a, batch, allow_split, st, fam);
    case 64: return attn_launch_hd<T, 64>(ctx, a, batch, allow_split, st, fam);
    case 128: return attn_launch_hd<T, 128>(ctx, a, batch, allow_split, st, fam);
    case 256: return attn_launch_hd<T, 256>(ctx, a, batch, allow_split, st, fam);
  }
  return fail(ctx, PI0_ERR_UNSUPPORTED, "head_dim");
}


template <typename T>
int rmsnorm(pi0_ctx* ctx, const T* x, T* out, int rows, int W, const T* w, const T* mod,
            int rows_per_mod, int mod_stride, cudaStream_t st, int fam) {
  Prof pr(ctx, fam, st);
  int blocks = (rows + 7) / 8;
  return launch(ctx, rmsnorm_kernel<T>, dim3(blocks), dim3(256), 0, st, dim3(1, 1, 1), x, out, rows, W,
                ctx->cfg.rms_norm_eps, w, mod, rows_per_mod, mod_stride);
}

// time conditions and all 2·L+1 modulations for `nsteps` time embeddings [nsteps, W1]
template <typename T>
int time_and_mods(pi0_ctx* ctx, const T* te, int nsteps, cudaStream_t st) {
  const pi0_config& g = ctx->cfg;
  const int W1 = g.ae_width;
  const int nmod = (2 * g.depth + 1) * 3 * W1;
  T* t1 = (T*)ctx->t1;
  T* cond = (T*)ctx->cond;
  // three weight-streaming GEMMs with M = nsteps: time_mlp_in + SiLU, time_mlp_out + SiLU, and
  // every adaRMS modulation of the step(s) at once
  for (int m0 = 0; m0 < nsteps; m0 += 64) {
    const int mm = std::min(64, nsteps - m0);
    TRY((gemm_w<T, false, false>(ctx, te + (size_t)m0 * W1, W1, (const T*)ctx->tin_w,
                                 (const T*)ctx->tin_p, ctx->tin_q, mm, W1, W1,
                                 EpiStore<T>{t1 + (size_t)m0 * W1, W1, (const T*)ctx->tin_b, 1}, st,
                                 F_DEN_TIME_MODS)));
    TRY((gemm_w<T, false, false>(ctx, t1 + (size_t)m0 * W1, W1, (const T*)ctx->tout_w,
                                 (const T*)ctx->tout_p, ctx->tout_q, mm, W1, W1,
                                 EpiStore<T>{cond + (size_t)m0 * W1, W1, (const T*)ctx->tout_b, 1},
                                 st, F_DEN_TIME_MODS)));
    TRY((gemm_w<T, false, false>(ctx, cond + (size_t)m0 * W1, W1, (const T*)ctx->mod_w,
                                 (const T*)ctx->mod_w_p, ctx->mod_w_q, mm, nmod, W1,
                                 EpiStore<T>{(T*)ctx->mods + (size_t)m0 * nmod, nmod,
                                             (const T*)ctx->mod_b, 0},
                                 st, F_DEN_TIME_MODS)));
  }
  return 0;
}

// Tensor-core attention (attention_tc.cuh) of `rows` = Tq·H query rows per request over key
// segment A (kA16 / vA, LA keys) and segment B (kB16 / vB, LB keys, may be 0). Key splits: as
// many as keep the grid within one wave (at most 16, one cluster), with every split at least
// one 64-key tile.
template <int HD>
int attn_tc_launch_hd(pi0_ctx* ctx, int B, const __half* q16, const __half* q16lo, int rows,
                      const __half* kA16, const __half* kA16lo, const __half* vA, int LA,
                      const __half* kB16, const __half* kB16lo, const __half* vB, int LB,
                      const float* mask, __half* out, int a_ready, cudaStream_t st, int fam) {
  const bool lo = q16lo != nullptr;
  // Fold the suffix keys into the prefix's last, partial tile when they fit in it (decode: 968
  // prefix keys leave 8 in the last tile, the 50 suffix keys fill it to 58): one tile fewer, so
  // every key split can hold a single tile. The tile's rows come from two loads whose boxes are
  // `tail` and 64 − tail rows high.
  const int tail = LA % atc::KB;
  const bool fold = a_ready && LB > 0 && tail > 0 && tail % 8 == 0 && tail + LB <= atc::KB;
  const int brows = fold ? atc::KB - tail : atc::KB;
  CUtensorMap tq, tka, tva, tkb, tvb, tql, tkal, tkbl, tkat, tvat, tkalt;
  TRY(make_tmap(ctx, &tq, q16, B * rows, HD, HD, 128, false));
  TRY(make_tmap(ctx, &tka, kA16, B * LA, HD, HD, atc::KB, false));
  TRY(make_tmap(ctx, &tva, vA, B * LA, HD, HD, atc::KB, false));
  if (LB > 0) {
    TRY(make_tmap(ctx, &tkb, kB16, B * LB, HD, HD, brows, false));
    TRY(make_tmap(ctx, &tvb, vB, B * LB, HD, HD, brows, false));
  } else {
    tkb = tka;
    tvb = tva;
  }
  if (lo) {
    TRY(make_tmap(ctx, &tql, q16lo, B * rows, HD, HD, 128, false));
    TRY(make_tmap(ctx, &tkal, kA16lo, B * LA, HD, HD, atc::KB, false));
    if (LB > 0) TRY(make_tmap(ctx, &tkbl, kB16lo, B * LB, HD, HD, brows, false));
    else tkbl = tkal;
  } else {
    tql = tq;
    tkal = tka;
    tkbl = tkb;
  }
  if (fold) {
    TRY(make_tmap(ctx, &tkat, kA16, B * LA, HD, HD, tail, false));
    TRY(make_tmap(ctx, &tvat, vA, B * LA, HD, HD, tail, false));
    if (lo) TRY(make_tmap(ctx, &tkalt, kA16lo, B * LA, HD, HD, tail, false));
    else tkalt = tkat;
  } else {
    tkat = tka;
    tvat = tva;
    tkalt = tkal;
  }
  atc::AtcArgs a{};
  a.rows = rows;
  a.LA = LA;
  a.LB = LB;
  a.ntA = (LA + atc::KB - 1) / atc::KB;
  a.nt = fold ? a.ntA : a.ntA + (LB + atc::KB - 1) / atc::KB;
  a.tail = fold ? tail : 0;
  const int row_tiles = (rows + 127) / 128;
  int splits = std::max(1, std::min(16, ctx->num_sms / std::max(1, row_tiles * B)));
  splits = std::min(splits, a.nt);
  a.tps = (a.nt + splits - 1) / splits;
  splits = (a.nt + a.tps - 1) / a.tps;
  a.maskA = mask;
  a.out = out;
  a.err = ctx->dev_err;
  a.a_ready = a_ready;
  a.v_lbo = atc::KB * 128;  // next 64-dim block of a V tile
  a.v_sbo = 1024;           // next 8 keys
  Prof pr(ctx, fam, st);
  if (lo)
    return launch(ctx, atc::attn_tc_kernel<HD, true>, dim3(row_tiles, splits, B), dim3(atc::NT),
                  atc::AtcSmem<HD, true>::BYTES, st, dim3(1, splits, 1), tq, tka, tva, tkb, tvb,
                  tql, tkal, tkbl, tkat, tvat, tkalt, a);
  return launch(ctx, atc::attn_tc_kernel<HD, false>, dim3(row_tiles, splits, B), dim3(atc::NT),
                atc::AtcSmem<HD, false>::BYTES, st, dim3(1, splits, 1), tq, tka, tva, tkb, tvb,
                tql, tkal, tkbl, tkat, tvat, tkalt, a);
}

// q16lo / kA16lo / kB16lo: the fp16 lo parts for fp32 logits (null: model-dtype logits)
int attn_tc_launch(pi0_ctx* ctx, int B, const __half* q16, const __half* q16lo, int rows,
                   const __half* kA16, const __half* kA16lo, const __half* vA, int LA,
                   const __half* kB16, const __half* kB16lo, const __half* vB, int LB,
                   const float* mask, __half* out, int a_ready, cudaStream_t st, int fam) {
  switch (ctx->cfg.head_dim) {
    case 64: return attn_tc_launch_hd<64>(ctx, B, q16, q16lo, rows, kA16, kA16lo, vA, LA, kB16, kB16lo, vB, LB, mask, out, a_ready, st, fam);
    case 128: return attn_tc_launch_hd<128>(ctx, B, q16, q16lo, rows, kA16, kA16lo, vA, LA, kB16, kB16lo, vB, LB, mask, out, a_ready, st, fam);
    case 256: return attn_tc_launch_hd<256>(ctx, B, q16, q16lo, rows, kA16, kA16lo, vA, LA, kB16, kB16lo, vB, LB, mask, out, a_ready, st, fam);
  }
  return fail(ctx, PI0_ERR_UNSUPPORTED, "tensor-core attention: head_dim must be 64, 128 or 256");
}

// K cache (fp32, caller's layout) -> model-dtype copy at half scale for the tensor-core
// attention; the next launch waits for it to complete (no programmatic overlap), so the cached
// tiles the attention requests before its own dependency wait are already converted.
int convert_prefix_keys(pi0_ctx* ctx, int B, const float* keys, cudaStream_t st) {
  const pi0_config& g = ctx->cfg;
  const size_t n = (size_t)g.depth * B * g.num_kv_heads * g.prefix_len * g.head_dim;
  const size_t n4 = n / 4;
  Prof pr(ctx, F_DEN_KEYS16, st);
  TRY(launch(ctx, keys_half_scale_kernel<__half>, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0,
             st, dim3(1, 1, 1), reinterpret_cast<const float4*>(keys), (__half*)ctx->kpre16,
             (__half*)ctx->kpre16_lo, n4));
  ctx->pdl_barrier = true;
  return 0;
}

// ---- persistent denoise step ---------------------------------------------------------------
// Work plan of one GEMM phase over `grid` CTAs in clusters of ds::CL (denoise_step.cuh): every
// 128-row weight tile gets a split group of s ranks, s the largest power of two ≤ 8 with
// tiles·s ≤ grid, and (unless `uniform`) tiles are promoted to 2s while CTAs are left; groups are
// packed into clusters largest first (power-of-two sizes, so a group never straddles a cluster
// and its first rank is a multiple of its size). Rank j of a group takes k-blocks
// [j·⌈nkb/s⌉, (j+1)·⌈nkb/s⌉). Returns false when no plan exists.
bool step_gemm_plan(int grid, int tiles, int nkb, bool uniform, ds::Work* out, int* s_out) {
  int smax = 0;
  for (int sz = ds::CL; sz >= 1; sz >>= 1)
    if (tiles * sz <= grid) {
      smax = sz;
      break;
    }
  if (!smax) return false;
  std::vector<int> sz(tiles, smax);
  if (!uniform && smax < ds::CL) {
    int left = grid - tiles * smax;
    for (int t = 0; t < tiles && left >= smax; ++t) {
      sz[t] = 2 * smax;
      left -= smax;
    }
  }
  for (int i = 0; i < grid; ++i) out[i] = ds::Work{-1, 0, 0, 0, 0, {0, 0, 0}};
  const int ncl = grid / ds::CL;
  std::vector<int> used(ncl, 0);
  std::vector<int> order(tiles);
  for (int t = 0; t < tiles; ++t) order[t] = t;
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return sz[x] > sz[y]; });
  for (int t : order) {
    const int g = sz[t], kbpc = (nkb + g - 1) / g;
    int c = 0;
    while (c < ncl && used[c] + g > ds::CL) ++c;
    if (c == ncl) return false;
    const int g0 = used[c];
    used[c] += g;
    for (int j = 0; j < g; ++j) {
      const int kb0 = j * kbpc, nk = std::min(nkb, kb0 + kbpc) - kb0;
      if (nk <= 0) return false;
      out[c * ds::CL + g0 + j] = ds::Work{(int16_t)t, (int16_t)g, (int16_t)g0, (int16_t)kb0,
                                          (int16_t)nk, {0, 0, 0}};
    }
  }
  if (s_out) *s_out = uniform ? smax : 0;
  return true;
}

// Decides at context creation whether denoise steps run as one persistent launch, and builds its
// plans. Opt-in: PI0_STEP_KERNEL=1 in the environment (measured slower than the per-kernel chain
// on a B200: 1.9 against 1.3 ms per π0.5 step, so the chain is the default). Requirements: fp16
// weights (not quantised), the tensor-core attention with head_dim 256, an action expert of width
// 1024 (8 tiles × 8-rank splits = the 64 row Σx² partial slots), S ≤ 64 suffix rows, enough
// co-resident clusters of 8.
int setup_step_kernel(pi0_ctx* ctx) {
  const pi0_config& g = ctx->cfg;
  ctx->step_kernel = false;
  const char* env = std::getenv("PI0_STEP_KERNEL");
  if (!env || env[0] != '1') return ctx->step_why = "not enabled (PI0_STEP_KERNEL=1)", 0;
  if (g.dtype != PI0_F16 || ctx->qb || !ctx->attn_tc || g.head_dim != 256 || g.num_kv_heads != 1)
    return ctx->step_why = "needs unquantised fp16 weights and one kv head of dim 256", 0;
  if (g.ae_width != 1024 || g.action_horizon > ds::NA || g.ae_mlp_dim % 64 ||
      (g.num_heads * g.head_dim) % 64)
    return ctx->step_why = "needs an action expert of width 1024 and at most 64 suffix rows", 0;
  const bool lo = ctx->logits_f32;
  auto kern = lo ? ds::denoise_step_kernel<true> : ds::denoise_step_kernel<false>;
  const int smem = std::max(lo ? atc::AtcSmem<256, true>::BYTES : atc::AtcSmem<256, false>::BYTES,
                            ds::RECV_OFF + ds::RECV_BYTES + 1024);
  CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ds::CL * 16);
  cfg.blockDim = dim3(ds::NT);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = ds::CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int ncl = 0;
  CK(cudaOccupancyMaxActiveClusters(&ncl, kern, &cfg));
  const int S = g.action_horizon, H = g.num_heads, hd = g.head_dim;
  const int hq = H * hd, W1 = g.ae_width, F1 = g.ae_mlp_dim, P = g.prefix_len;
  ctx->att_row_tiles = (S * H + 127) / 128;
  if (ncl < ctx->att_row_tiles || ncl < 2)
    return ctx->step_why = "too few co-resident clusters of 8", 0;
  const int grid = ncl * ds::CL;
  const int N[ds::G_NUM] = {hq + 2 * g.num_kv_heads * hd, W1, 2 * F1, W1};
  const int K[ds::G_NUM] = {W1, hq, W1, F1};
  std::vector<ds::Work> plan((size_t)ds::G_NUM * grid);
  for (int k = 0; k < ds::G_NUM; ++k) {
    ctx->step_N[k] = N[k];
    ctx->step_K[k] = K[k];
    ctx->step_tiles[k] = (N[k] + 127) / 128;
    ctx->step_nkb[k] = (K[k] + 63) / 64;
    const bool ssq = k == ds::G_O || k == ds::G_D;  // residual phases: uniform 8-rank groups
    int su = 0;
    if (!step_gemm_plan(grid, ctx->step_tiles[k], ctx->step_nkb[k], ssq, &plan[(size_t)k * grid],
                        &su))
      return ctx->step_why = "no work plan for a projection", 0;
    if (ssq && ctx->step_tiles[k] * su != ds::SSQ_PARTS)
      return ctx->step_why = "residual projections do not give 64 row partials", 0;
  }
  ctx->att_ntA = (P + atc::KB - 1) / atc::KB;
  ctx->att_nt = ctx->att_ntA + (S + atc::KB - 1) / atc::KB;
  ctx->att_tps = (ctx->att_nt + ds::CL - 1) / ds::CL;
  ctx->att_splits = (ctx->att_nt + ctx->att_tps - 1) / ctx->att_tps;
  TRY(dev_alloc(ctx, (void**)&ctx->step_plan, plan.size() * sizeof(ds::Work)));
  CK(cudaMemcpy(ctx->step_plan, plan.data(), plan.size() * sizeof(ds::Work), cudaMemcpyHostToDevice));
  std::vector<ds::Layer> layers(g.depth);
  for (int l = 0; l < g.depth; ++l) {
    const LayerW& w = ctx->suf[l];
    layers[l].w[ds::G_QKV] = (const uint8_t*)w.qkv_p;
    layers[l].w[ds::G_O] = (const uint8_t*)w.o_p;
    layers[l].w[ds::G_GU] = (const uint8_t*)w.gu_p;
    layers[l].w[ds::G_D] = (const uint8_t*)w.d_p;
  }
  TRY(dev_alloc(ctx, (void**)&ctx->step_layers, layers.size() * sizeof(ds::Layer)));
  CK(cudaMemcpy(ctx->step_layers, layers.data(), layers.size() * sizeof(ds::Layer),
                cudaMemcpyHostToDevice));
  TRY(dev_alloc(ctx, (void**)&ctx->step_bar, sizeof(unsigned long long)));
  CK(cudaMemset(ctx->step_bar, 0, sizeof(unsigned long long)));
  ctx->step_grid = grid;
  ctx->step_kernel = true;
  ctx->step_why.clear();
  return 0;
}

// One denoise step (batch 1) as one persistent launch: x_in the model-dtype x_t (x_is_f32 false)
// or the fp32 Euler state; out v (euler 0) or the state updated by x += dt·v. The prefix keys'
// half-scale fp16 copies (and lo parts) must be current (convert_prefix_keys).
int step_launch(pi0_ctx* ctx, const __half* values, const void* x_in, bool x_is_f32,
                const __half* mods, const float* scos, const float* ssin, const float* mask,
                float* out, int euler, float dt, cudaStream_t st) {
  const pi0_config& g = ctx->cfg;
  const int S = g.action_horizon, H = g.num_heads, hd = g.head_dim, P = g.prefix_len;
  const int hq = H * hd, W1 = g.ae_width, F1 = g.ae_mlp_dim, L = g.depth;
  const bool lo = ctx->logits_f32;
  CUtensorMap tx, ta, th, tq, tql, tka, tkal, tva, tkb, tkbl, tvb;
  TRY(make_tmap(ctx, &tx, ctx->xs, S, W1, W1, ds::NA, false));
  TRY(make_tmap(ctx, &ta, ctx->attn_s, S, hq, hq, ds::NA, false));
  TRY(make_tmap(ctx, &th, ctx->hs, S, F1, F1, ds::NA, false));
  TRY(make_tmap(ctx, &tq, ctx->q16s, S * H, hd, hd, 128, false));
  TRY(make_tmap(ctx, &tql, lo ? ctx->q16s_lo : ctx->q16s, S * H, hd, hd, 128, false));
  TRY(make_tmap(ctx, &tka, ctx->kpre16, L * P, hd, hd, atc::KB, false));
  TRY(make_tmap(ctx, &tkal, lo ? ctx->kpre16_lo : ctx->kpre16, L * P, hd, hd, atc::KB, false));
  TRY(make_tmap(ctx, &tva, values, L * P, hd, hd, atc::KB, false));
  TRY(make_tmap(ctx, &tkb, ctx->ksuf16, S, hd, hd, atc::KB, false));
  TRY(make_tmap(ctx, &tkbl, lo ? ctx->ksuf16_lo : ctx->ksuf16, S, hd, hd, atc::KB, false));
  TRY(make_tmap(ctx, &tvb, ctx->vsuf, S, hd, hd, atc::KB, false));
  ds::StepArgs a{};
  a.M = S;
  a.W1 = W1;
  a.F1 = F1;
  a.H = H;
  a.hd = hd;
  a.S = S;
  a.P = P;
  a.L = L;
  a.D = g.action_dim;
  a.layers = ctx->step_layers;
  a.plan = ctx->step_plan;
  for (int k = 0; k < ds::G_NUM; ++k) {
    a.tiles[k] = ctx->step_tiles[k];
    a.nkb[k] = ctx->step_nkb[k];
    a.N[k] = ctx->step_N[k];
    a.K[k] = ctx->step_K[k];
  }
  a.mods = mods;
  a.x = ctx->xs;
  a.attn = ctx->attn_s;
  a.h = ctx->hs;
  a.ssq = ctx->ssq;
  a.qs = ctx->qs;
  a.ksuf = ctx->ksuf;
  a.vsuf = ctx->vsuf;
  a.q16 = ctx->q16s;
  a.q16lo = ctx->q16s_lo;
  a.k16 = ctx->ksuf16;
  a.k16lo = ctx->ksuf16_lo;
  a.scos = scos;
  a.ssin = ssin;
  a.qscale = (float)std::pow((double)hd, -0.5);
  a.maskA = mask;
  a.att_row_tiles = ctx->att_row_tiles;
  a.att_tps = ctx->att_tps;
  a.att_splits = ctx->att_splits;
  a.att_ntA = ctx->att_ntA;
  a.att_nt = ctx->att_nt;
  a.kA16 = ctx->kpre16;
  a.kA16lo = ctx->kpre16_lo;
  a.vA = values;
  a.x_in = x_in;
  a.x_is_f32 = x_is_f32 ? 1 : 0;
  a.ain_w = ctx->ain_w;
  a.ain_b = ctx->ain_b;
  a.aout_w = ctx->aout_w;
  a.aout_b = ctx->aout_b;
  a.out = out;
  a.euler = euler;
  a.dt = dt;
  a.eps = g.rms_norm_eps;
  a.err = ctx->dev_err;
  a.bar = ctx->step_bar;
  const int smem = std::max(lo ? atc::AtcSmem<256, true>::BYTES : atc::AtcSmem<256, false>::BYTES,
                            ds::RECV_OFF + ds::RECV_BYTES + 1024);
  Prof pr(ctx, F_DEN_STEP, st);
  ctx->pdl_barrier = true;  // every CTA must be resident together: no overlap with the previous kernel
  auto kern = lo ? ds::denoise_step_kernel<true> : ds::denoise_step_kernel<false>;
  TRY(launch(ctx, kern, dim3(ctx->step_grid), dim3(ds::NT), smem, st, dim3(ds::CL, 1, 1), tx, ta,
             th, tq, tql, tka, tkal, tva, tkb, tkbl, tvb, a));
  ctx->pdl_barrier = true;
  return 0;
}

// ---- prefill ---------------------------------------------------------------------------------
template <typename T>
int run_prefill(pi0_ctx* ctx, int B, const T* prefix, const float* mask, float* keys, T* values,
                cudaStream_t st) {
  const pi0_config& g = ctx->cfg;
  const int P = g.prefix_len, W0 = g.vlm_width, F0 = g.vlm_mlp_dim, hd = g.head_dim;
  const int H = g.num_heads, KV = g.num_kv_heads, hq = H * hd, hkv = KV * hd;
  const int M = B * P;
  T* x = (T*)ctx->xp;
  T* xn = (T*)ctx->xpn;
  T* attn = (T*)ctx->attn_p;
  T* h = (T*)ctx->hp;
  CK(cudaMemcpyAsync(x, prefix, (size_t)M * W0 * sizeof(T), cudaMemcpyDeviceToDevice, st));
  const size_t kv_layer = (size_t)B * KV * P * hd;
  for (int l = 0; l < g.depth; ++l) {
    const LayerW& w = ctx->pre[l];
    float* kl = keys + l * kv_layer;
    T* vl = values + l * kv_layer;
    TRY(rmsnorm<T>(ctx, x, xn, M, W0, (const T*)w.ln_in, nullptr, 1, 0, st, F_PRE_NORM));
    EpiQkvRope<T> eq{ctx->qp, kl, vl, ctx->rope_cos, ctx->rope_sin, 0, P, H, KV, hd, 0,
                     (float)std::pow((double)hd, -0.5)};
    T* k16 = ctx->attn_tc ? (T*)ctx->kpre16 + l * kv_layer : nullptr;
    T* k16lo = ctx->kpre16_lo ? (T*)ctx->kpre16_lo + l * kv_layer : nullptr;
    if (ctx->attn_tc) {
      eq.q16 = (T*)ctx->q16p;
      eq.k16 = k16;
      eq.q16lo = (T*)ctx->q16p_lo;
      eq.k16lo = k16lo;
    }
    const bool last = l == g.depth - 1;
    if (last) {  // only k and v of the last layer are ever read
      eq.col0 = hq;
      TRY(gemm<T>(ctx, xn, W0, (const T*)w.qkv + (size_t)hq * W0, W0, M, 2 * hkv, W0, eq, st,
                  F_PRE_QKV));
      break;
    }
    TRY(gemm<T>(ctx, xn, W0, (const T*)w.qkv, W0, M, hq + 2 * hkv, W0, eq, st, F_PRE_QKV));
    if constexpr (!Tr<T>::kBf16) {
      if (ctx->attn_tc) {
        TRY(attn_tc_launch(ctx, B, (const __half*)ctx->q16p, (const __half*)ctx->q16p_lo, P * H,
                           (const __half*)k16, (const __half*)k16lo, (const __half*)vl, P, nullptr,
                           nullptr, nullptr, 0, mask, (__half*)attn, 0, st, F_PRE_ATTN));
        TRY(gemm<T>(ctx, attn, hq, (const T*)w.o, hq, M, W0, hq, EpiResid<T>{x, W0}, st, F_PRE_O));
        TRY(rmsnorm<T>(ctx, x, xn, M, W0, (const T*)w.ln_post, nullptr, 1, 0, st, F_PRE_NORM));
        TRY(gemm<T>(ctx, xn, W0, (const T*)w.gu, W0, M, 2 * F0, W0, EpiGeglu<T>{h, F0}, st,
                    F_PRE_GU));
        TRY(gemm<T>(ctx, h, F0, (const T*)w.d, F0, M, W0, F0, EpiResid<T>{x, W0}, st, F_PRE_DOWN));
        continue;
      }
    }
    AttnArgs<T> a{};
    a.q = ctx->qp;
    a.kA = kl;
    a.vA = vl;
    a.maskA = mask;
    a.LA = P;
    a.kB = nullptr;
    a.vB = nullptr;
    a.LB = 0;
    a.Tq = P;
    a.H = H;
    a.KV = KV;
    a.out = attn;
    a.logits_f32 = ctx->logits_f32 ? 1 : 0;
    TRY(attn_launch<T>(ctx, a, B, false, st, F_PRE_ATTN));
    TRY(gemm<T>(ctx, attn, hq, (const T*)w.o, hq, M, W0, hq, EpiResid<T>{x, W0}, st, F_PRE_O));
    TRY(rmsnorm<T>(ctx, x, xn, M, W0, (const T*)w.ln_post, nullptr, 1, 0, st, F_PRE_NORM));
    TRY(gemm<T>(ctx, xn, W0, (const T*)w.gu, W0, M, 2 * F0, W0, EpiGeglu<T>{h, F0}, st,
                F_PRE_GU));
    TRY(gemm<T>(ctx, h, F0, (const T*)w.d, F0, M, W0, F0, EpiResid<T>{x, W0}, st, F_PRE_DOWN));
  }
  return 0;
}

// ---- one suffix pass (decode_suffix + action_out) with modulations `mods` -------------------
// x_in: model-dtype x_t (x_is_f32 = false) or the fp32 Euler state (x_is_f32 = true).
// out: v (euler = 0) or the fp32 state updated in place by x += dt·v (euler = 1).
template <typename T>
int run_suffix(pi0_ctx* ctx, int B, const float* keys, const T* values, const void* x_in,
               bool x_is_f32, const T* mods, const float* scos, const float* ssin,
               const float* mask, float* out, int euler, float dt, cudaStream_t st) {
  const pi0_config& g = ctx->cfg;
  const int P = g.prefix_len, S = g.action_horizon, D = g.action_dim, W1 = g.ae_width;
  const int F1 = g.ae_mlp_dim, hd = g.head_dim, H = g.num_heads, KV = g.num_kv_heads;
  const int hq = H * hd, hkv = KV * hd, M = B * S;
  const int mstride = 3 * W1;
  T* x = (T*)ctx->xs;
  T* xn = (T*)ctx->xsn;
  T* attn = (T*)ctx->attn_s;
  T* h = (T*)ctx->hs;
  if constexpr (!Tr<T>::kBf16) {
    if (ctx->step_kernel && B == 1)  // the whole step as one persistent launch
      return step_launch(ctx, (const __half*)values, x_in, x_is_f32, (const __half*)mods, scos,
                         ssin, mask, out, euler, dt, st);
  }
  {
    Prof pr(ctx, F_DEN_ACT_IN, st);
    const size_t sm = (size_t)D * sizeof(float);
    float* ssq = M <= 128 ? ctx->ssq : nullptr;
    if (x_is_f32)
      TRY(launch(ctx, action_in_kernel<T, true>, dim3(M), dim3(256), sm, st, dim3(1, 1, 1), x_in, M, D,
                 (const T*)ctx->ain_w, (const T*)ctx->ain_b, W1, x, ssq, ctx->ssq_parts));
    else
      TRY(launch(ctx, action_in_kernel<T, false>, dim3(M), dim3(256), sm, st, dim3(1, 1, 1), x_in, M, D,
                 (const T*)ctx->ain_w, (const T*)ctx->ain_b, W1, x, ssq, ctx->ssq_parts));
  }
  const size_t kv_layer = (size_t)B * KV * P * hd;
  for (int l = 0; l < g.depth; ++l) {
    const LayerW& w = ctx->suf[l];
    const T* m_in = mods + (size_t)(2 * l) * mstride;
    const T* m_post = mods + (size_t)(2 * l + 1) * mstride;
    EpiQkvRope<T> eq{ctx->qs, ctx->ksuf, (T*)ctx->vsuf, scos, ssin, S * (hd / 2), S, H, KV, hd, 0,
                     (float)std::pow((double)hd, -0.5)};
    if (ctx->attn_tc) {
      eq.q16 = (T*)ctx->q16s;
      eq.k16 = (T*)ctx->ksuf16;
      eq.q16lo = (T*)ctx->q16s_lo;
      eq.k16lo = (T*)ctx->ksuf16_lo;
    }
    TRY((gemm_w<T, true, false>(ctx, x, W1, (const T*)w.qkv, (const T*)w.qkv_p, w.qkv_q, M, hq + 2 * hkv,
                                W1, eq, st, F_DEN_QKV, m_in, xn)));
    bool done_attn = false;
    if constexpr (!Tr<T>::kBf16) {
      if (ctx->attn_tc) {
        const __half* kA16lo =
            ctx->kpre16_lo ? (const __half*)ctx->kpre16_lo + l * kv_layer : nullptr;
        TRY(attn_tc_launch(ctx, B, (const __half*)ctx->q16s, (const __half*)ctx->q16s_lo, S * H,
                           (const __half*)ctx->kpre16 + l * kv_layer, kA16lo,
                           (const __half*)values + l * kv_layer, P, (const __half*)ctx->ksuf16,
                           (const __half*)ctx->ksuf16_lo, (const __half*)ctx->vsuf, S, mask,
                           (__half*)attn, 1, st, F_DEN_ATTN));
        done_attn = true;
      }
    }
    if (!done_attn) {
    AttnArgs<T> a{};
    a.q = ctx->qs;
    a.kA = keys + l * kv_layer;
    a.vA = values + l * kv_layer;
    a.maskA = mask;
    a.LA = P;
    a.kB = ctx->ksuf;
    a.vB = (const T*)ctx->vsuf;
    a.LB = S;
    a.Tq = S;
    a.H = H;
    a.KV = KV;
    a.out = attn;
    a.a_is_ready = 1;  // the prefix K/V cache comes from prefill, not from this step
    a.logits_f32 = ctx->logits_f32 ? 1 : 0;
    TRY(attn_launch<T>(ctx, a, B, true, st, F_DEN_ATTN));
    }
    TRY((gemm_w<T, false, true>(ctx, attn, hq, (const T*)w.o, (const T*)w.o_p, w.o_q, M, W1, hq,
                                EpiGatedResid<T>{x, W1, m_in + 2 * W1, M, 0}, st, F_DEN_O)));
    TRY((gemm_w<T, true, false>(ctx, x, W1, (const T*)w.gu, (const T*)w.gu_p, w.gu_q, M, 2 * F1, W1,
                                EpiGeglu<T>{h, F1}, st, F_DEN_GU, m_post, xn)));
    TRY((gemm_w<T, false, true>(ctx, h, F1, (const T*)w.d, (const T*)w.d_p, w.d_q, M, W1, F1,
                                EpiGatedResid<T>{x, W1, m_post + 2 * W1, M, 0}, st, F_DEN_DOWN)));
  }
  {
    Prof pr(ctx, F_DEN_ACT_OUT, st);
    int warps = M * D;
    TRY(launch(ctx, action_out_kernel<T>, dim3((warps * 32 + 255) / 256), dim3(256), 0, st,
               dim3(1, 1, 1),
               (const T*)x, M, W1, mods + (size_t)(2 * g.depth) * mstride, ctx->cfg.rms_norm_eps,
               (const T*)ctx->aout_w, (const T*)ctx->aout_b, D, out, euler, dt));
  }
  return 0;
}

template <typename T>
int run_step(pi0_ctx* ctx, int B, const float* keys, const T* values, const T* x_t, const T* te,
             const float* scos, const float* ssin, const float* mask, float* v_out,
             cudaStream_t st) {
  if (ctx->attn_tc) TRY(convert_prefix_keys(ctx, B, keys, st));
  if (ctx->step_kernel && B == 1)  // a launch cut short can leave arrivals behind: start clean
    CK(cudaMemsetAsync(ctx->step_bar, 0, sizeof(unsigned long long), st));
  TRY(time_and_mods<T>(ctx, te, 1, st));
  return run_suffix<T>(ctx, B, keys, values, x_t, false, (const T*)ctx->mods, scos, ssin, mask,
                       v_out, 0, 0.f, st);
}

template <typename T>
int run_loop_body(pi0_ctx* ctx, int B, const float* keys, const T* values, const float* x0,
                  const T* tes, const float* scos, const float* ssin, const float* mask,
                  float* x_out, cudaStream_t st) {
  const pi0_config& g = ctx->cfg;
  const int N = g.num_denoise_steps;
  const size_t nmod = (size_t)(2 * g.depth + 1) * 3 * g.ae_width;
  if (x_out != x0)
    CK(cudaMemcpyAsync(x_out, x0, (size_t)B * g.action_horizon * g.action_dim * sizeof(float),
                       cudaMemcpyDeviceToDevice, st));
  if (ctx->attn_tc) TRY(convert_prefix_keys(ctx, B, keys, st));
  if (ctx->step_kernel && B == 1)  // a launch cut short can leave arrivals behind: start clean
    CK(cudaMemsetAsync(ctx->step_bar, 0, sizeof(unsigned long long), st));
  TRY(time_and_mods<T>(ctx, tes, N, st));
  const float dt = (float)(-1.0 / N);
  for (int i = 0; i < N; ++i)
    TRY(run_suffix<T>(ctx, B, keys, values, x_out, true, (const T*)ctx->mods + i * nmod, scos,
                      ssin, mask, x_out, 1, dt, st));
  return 0;
}

// ---- kernel attributes (set once at context creation: never inside a graph capture) --------
template <typename T, int BM, int BN, int WM, int WN, int ST, class Epi>
int attr_gemm(pi0_ctx* ctx) {
  CK(cudaFuncSetAttribute(gemm_mma_kernel<T, BM, BN, WM, WN, ST, Epi>,
                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                          GemmCfg<T, BM, BN, WM, WN, ST>::SMEM));
  return 0;
}
template <typename T, int BN, int ST, class Epi, int KS = 1, int CG = 1>
int attr_tc(pi0_ctx* ctx) {
  CK(cudaFuncSetAttribute(tc::gemm_tc_kernel<T, BN, ST, Epi, KS, CG>,
                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                          tc::Smem<BN, ST, CG>::BYTES));
  return 0;
}
template <typename T, int NA, class Epi, bool SSQ = false>
int attr_sk(pi0_ctx* ctx) {
  for (auto k : {sk::skinny_kernel<T, NA, false, SSQ, Epi>, sk::skinny_kernel<T, NA, !SSQ, SSQ, Epi>,
                 sk::skinny_kernel<T, NA, false, SSQ, Epi, 4>, sk::skinny_kernel<T, NA, !SSQ, SSQ, Epi, 4>,
                 sk::skinny_kernel<T, NA, false, SSQ, Epi, 3>, sk::skinny_kernel<T, NA, !SSQ, SSQ, Epi, 3>}) {
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, sk::SkSmem<NA>::BYTES));
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  }
  return 0;
}
template <typename T, class Epi>
int attr_gemm_both(pi0_ctx* ctx) {
  TRY((attr_sk<T, 64, Epi>(ctx)));
  TRY((attr_sk<T, 128, Epi>(ctx)));
  TRY((attr_gemm<T, 128, 128, 64, 32, 4, Epi>(ctx)));
  TRY((attr_gemm<T, 64, 64, 32, 32, 4, Epi>(ctx)));
  TRY((attr_tc<T, 256, 4, Epi>(ctx)));
  TRY((attr_tc<T, 256, 4, Epi, 2>(ctx)));
  TRY((attr_tc<T, 160, 5, Epi>(ctx)));
  TRY((attr_tc<T, 128, 6, Epi>(ctx)));
  TRY((attr_tc<T, 256, pair_stages<256>(), Epi, 1, 2>(ctx)));
  return 0;
}
template <typename T, int HD>
int attr_attn(pi0_ctx* ctx) {
  CK(cudaFuncSetAttribute(attn_kernel<T, HD, ATT_BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          AttnSmem<HD, ATT_BK>::BYTES));
  CK(cudaFuncSetAttribute(attn_kernel<T, HD, ATT_BK>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                          1));
  return 0;
}
template <int HD, bool LO>
int attr_attn_tc(pi0_ctx* ctx) {
  CK(cudaFuncSetAttribute(atc::attn_tc_kernel<HD, LO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          atc::AtcSmem<HD, LO>::BYTES));
  CK(cudaFuncSetAttribute(atc::attn_tc_kernel<HD, LO>,
                          cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  return 0;
}
template <typename T>
int setup_attrs(pi0_ctx* ctx) {
  if (ctx->attn_tc) {
    const bool lo = ctx->logits_f32;
    switch (ctx->cfg.head_dim) {
      case 64: TRY(lo ? attr_attn_tc<64, true>(ctx) : attr_attn_tc<64, false>(ctx)); break;
      case 128: TRY(lo ? attr_attn_tc<128, true>(ctx) : attr_attn_tc<128, false>(ctx)); break;
      case 256: TRY(lo ? attr_attn_tc<256, true>(ctx) : attr_attn_tc<256, false>(ctx)); break;
    }
  }
  TRY(attr_gemm_both<T, EpiQkvRope<T>>(ctx));
  TRY(attr_gemm_both<T, EpiResid<T>>(ctx));
  TRY(attr_gemm_both<T, EpiGatedResid<T>>(ctx));
  TRY((attr_sk<T, 64, EpiGatedResid<T>, true>(ctx)));
  TRY((attr_sk<T, 128, EpiGatedResid<T>, true>(ctx)));
  TRY(attr_gemm_both<T, EpiGeglu<T>>(ctx));
  TRY(attr_gemm_both<T, EpiStore<T>>(ctx));
  switch (ctx->cfg.head_dim) {
    case 16: TRY((attr_attn<T, 16>(ctx))); break;
    case 32: TRY((attr_attn<T, 32>(ctx))); break;
    case 64: TRY((attr_attn<T, 64>(ctx))); break;
    case 128: TRY((attr_attn<T, 128>(ctx))); break;
    case 256: TRY((attr_attn<T, 256>(ctx))); break;
  }
  return 0;
}

// ---- set params ---------------------------------------------------------------------------
int upload_ints(pi0_ctx* ctx, int** dst, const std::vector<int>& v) {
  TRY(dev_alloc(ctx, (void**)dst, v.size() * sizeof(int)));
  CK(cudaMemcpy(*dst, v.data(), v.size() * sizeof(int), cudaMemcpyHostToDevice));
  return 0;
}

std::vector<int> rope_perm(int heads, int hd) {
  // packed row h·hd + 2i + c  <-  original row h·hd + i + c·hd/2
  std::vector<int> p(heads * hd);
  for (int h = 0; h < heads; ++h)
    for (int i = 0; i < hd / 2; ++i)
      for (int c = 0; c < 2; ++c) p[h * hd + 2 * i + c] = h * hd + i + c * (hd / 2);
  return p;
}
std::vector<int> gu_perm(int F) {
  // packed row 2j = gate row j, 2j + 1 = up row j (= original row F + j)
  std::vector<int> p(2 * F);
  for (int j = 0; j < F; ++j) {
    p[2 * j] = j;
    p[2 * j + 1] = F + j;
  }
  return p;
}

int gather(pi0_ctx* ctx, void* dst, const void* src, const int* idx, int rows, int K,
           cudaStream_t st) {
  gather_rows_kernel<<<rows, 128, 0, st>>>((uint16_t*)dst, (const uint16_t*)src, idx, rows, K);
  CKL();
  return 0;
}

int copy(pi0_ctx* ctx, void* dst, const void* src, size_t bytes, cudaStream_t st) {
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st));
  return 0;
}

int alloc_all(pi0_ctx* ctx) {
  const pi0_config& g = ctx->cfg;
  const size_t e = ctx->esz;
  const int L = g.depth, hd = g.head_dim, H = g.num_heads, KV = g.num_kv_heads;
  const size_t hq = (size_t)H * hd, hkv = (size_t)KV * hd;
  const size_t W0 = g.vlm_width, W1 = g.ae_width, F0 = g.vlm_mlp_dim, F1 = g.ae_mlp_dim;
  const size_t B = g.max_batch, P = g.prefix_len, S = g.action_horizon, D = g.action_dim;
  const int N = g.num_denoise_steps;

  // weight arena: every block starts on a 256-byte boundary
  const size_t nmodw = (size_t)(2 * L + 1) * 3 * W1;
  auto pad = [&](size_t elems) { return ((elems * e + 255) / 256) * 256; };
  size_t arena = 0;
  for (int l = 0; l < L; ++l)
    arena += pad((hq + 2 * hkv) * W0) + pad(W0 * hq) + pad(2 * F0 * W0) + pad(W0 * F0) +
             2 * pad(W0) + pad((hq + 2 * hkv) * W1) + pad(W1 * hq) + pad(2 * F1 * W1) +
             pad(W1 * F1);
  arena += pad(nmodw * W1) + pad(nmodw) + pad(W1 * D) + pad(W1) + pad(D * W1) + pad(D) +
           2 * (pad(W1 * W1) + pad(W1));
  // packed copies of the weight-streaming matrices (action expert, modulations, time MLP)
  auto packed = [&](size_t n, size_t k) {
    return ((n + 127) / 128) * ((k + 63) / 64) * (size_t)sk::W_BLOCK;
  };
  arena += L * (packed(hq + 2 * hkv, W1) + packed(W1, hq) + packed(2 * F1, W1) + packed(W1, F1)) +
           packed(nmodw, W1) + 2 * packed(W1, W1);
  // quantised models whose action-expert dimensions are whole 64-wide k-blocks: the same
  // matrices as group-quantised blocks, dequantised inside the weight-streaming kernel
  ctx->qb = 0;
  if (e == 2 && W1 % 64 == 0 && hq % 64 == 0 && F1 % 64 == 0)
    ctx->qb = g.quant == PI0_QUANT_Q4 ? 4 : g.quant == PI0_QUANT_Q3 ? 3 : 0;
  auto qpacked = [&](size_t n, size_t k) {
    return ((n + 127) / 128) * ((k + 63) / 64) * (size_t)sk::qw_block(ctx->qb);
  };
  const size_t qbytes =
      ctx->qb ? L * (qpacked(hq + 2 * hkv, W1) + qpacked(W1, hq) + qpacked(2 * F1, W1) +
                     qpacked(W1, F1)) +
                    qpacked(nmodw, W1) + 2 * qpacked(W1, W1)
              : 0;
  arena += qbytes;
  ctx->arena_bytes = arena;
  TRY(dev_alloc(ctx, &ctx->arena, ctx->arena_bytes));
  char* p = (char*)ctx->arena;
  auto take = [&](size_t elems) {
    void* r = p;
    p += pad(elems);
    return r;
  };
  ctx->pre.resize(L);
  ctx->suf.resize(L);
  for (int l = 0; l < L; ++l) {
    LayerW& a = ctx->pre[l];
    a.qkv = take((hq + 2 * hkv) * W0);
    a.o = take(W0 * hq);
    a.gu = take(2 * F0 * W0);
    a.d = take(W0 * F0);
    a.ln_in = take(W0);
    a.ln_post = take(W0);
    LayerW& s = ctx->suf[l];
    s.qkv = take((hq + 2 * hkv) * W1);
    s.o = take(W1 * hq);
    s.gu = take(2 * F1 * W1);
    s.d = take(W1 * F1);
    s.ln_in = s.ln_post = nullptr;
  }
  ctx->mod_w = take(nmodw * W1);
  ctx->mod_b = take(nmodw);
  ctx->ain_w = take(W1 * D);
  ctx->ain_b = take(W1);
  ctx->aout_w = take(D * W1);
  ctx->aout_b = take(D);
  ctx->tin_w = take(W1 * W1);
  ctx->tin_b = take(W1);
  ctx->tout_w = take(W1 * W1);
  ctx->tout_b = take(W1);
  auto take_bytes = [&](size_t bytes) {
    void* r = p;
    p += bytes;
    return r;
  };
  for (int l = 0; l < L; ++l) {
    LayerW& w = ctx->suf[l];
    w.qkv_p = take_bytes(packed(hq + 2 * hkv, W1));
    w.o_p = take_bytes(packed(W1, hq));
    w.gu_p = take_bytes(packed(2 * F1, W1));
    w.d_p = take_bytes(packed(W1, F1));
  }
  ctx->mod_w_p = take_bytes(packed(nmodw, W1));
  ctx->tin_p = take_bytes(packed(W1, W1));
  ctx->tout_p = take_bytes(packed(W1, W1));
  if (ctx->qb) {
    char* q0 = p;
    for (int l = 0; l < L; ++l) {
      LayerW& w = ctx->suf[l];
      w.qkv_q = take_bytes(qpacked(hq + 2 * hkv, W1));
      w.o_q = take_bytes(qpacked(W1, hq));
      w.gu_q = take_bytes(qpacked(2 * F1, W1));
      w.d_q = take_bytes(qpacked(W1, F1));
    }
    ctx->mod_w_q = take_bytes(qpacked(nmodw, W1));
    ctx->tin_q = take_bytes(qpacked(W1, W1));
    ctx->tout_q = take_bytes(qpacked(W1, W1));
    CK(cudaMemset(q0, 0, (size_t)(p - q0)));  // rows past a matrix: zero codes and scales
  }
  if ((size_t)(p - (char*)ctx->arena) > ctx->arena_bytes)
    return fail(ctx, PI0_ERR_INVALID, "internal: weight arena overflow");

  // permutations and the prefix RoPE table (float64 -> fp32, gemma_dual.py:24-44)
  TRY(upload_ints(ctx, &ctx->perm_q, rope_perm(H, hd)));
  TRY(upload_ints(ctx, &ctx->perm_k, rope_perm(KV, hd)));
  TRY(upload_ints(ctx, &ctx->perm_gu0, gu_perm((int)F0)));
  TRY(upload_ints(ctx, &ctx->perm_gu1, gu_perm((int)F1)));
  {
    std::vector<float> c(P * (hd / 2)), s(P * (hd / 2));
    for (size_t t = 0; t < P; ++t)
      for (int i = 0; i < hd / 2; ++i) {
        double ts = std::pow((double)g.rope_theta, (2.0 / hd) * i);
        double r = (double)t / ts;
        c[t * (hd / 2) + i] = (float)std::cos(r);
        s[t * (hd / 2) + i] = (float)std::sin(r);
      }
    TRY(dev_alloc(ctx, (void**)&ctx->rope_cos, c.size() * 4));
    TRY(dev_alloc(ctx, (void**)&ctx->rope_sin, s.size() * 4));
    CK(cudaMemcpy(ctx->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ctx->rope_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
  }

  // workspaces
  const size_t MP = B * P, MS = B * S;
  TRY(dev_alloc(ctx, &ctx->xp, MP * W0 * e));
  TRY(dev_alloc(ctx, &ctx->xpn, MP * W0 * e));
  TRY(dev_alloc(ctx, &ctx->attn_p, MP * hq * e));
  TRY(dev_alloc(ctx, &ctx->hp, MP * F0 * e));
  TRY(dev_alloc(ctx, (void**)&ctx->qp, MP * hq * 4));
  TRY(dev_alloc(ctx, &ctx->xs, MS * W1 * e));
  TRY(dev_alloc(ctx, &ctx->xsn, MS * W1 * e));
  TRY(dev_alloc(ctx, &ctx->attn_s, MS * hq * e));
  TRY(dev_alloc(ctx, &ctx->hs, MS * F1 * e));
  TRY(dev_alloc(ctx, (void**)&ctx->qs, MS * hq * 4));
  TRY(dev_alloc(ctx, (void**)&ctx->ksuf, B * hkv * S * 4));
  TRY(dev_alloc(ctx, &ctx->vsuf, B * hkv * S * e));
  ctx->attn_tc = e == 2 && g.dtype == PI0_F16 && KV == 1 && hd % 64 == 0 && hd <= 256;
  ctx->logits_f32 = g.attn_logits == PI0_LOGITS_F32;
  if (ctx->attn_tc) {
    TRY(dev_alloc(ctx, &ctx->q16p, MP * hq * e));
    TRY(dev_alloc(ctx, &ctx->q16s, MS * hq * e));
    TRY(dev_alloc(ctx, &ctx->kpre16, (size_t)g.depth * B * hkv * P * e));
    TRY(dev_alloc(ctx, &ctx->ksuf16, B * hkv * S * e));
    if (ctx->logits_f32) {
      TRY(dev_alloc(ctx, &ctx->q16p_lo, MP * hq * e));
      TRY(dev_alloc(ctx, &ctx->q16s_lo, MS * hq * e));
      TRY(dev_alloc(ctx, &ctx->kpre16_lo, (size_t)g.depth * B * hkv * P * e));
      TRY(dev_alloc(ctx, &ctx->ksuf16_lo, B * hkv * S * e));
    }
  }
  {
    const size_t kvn = (size_t)g.depth * B * KV * P * hd;
    TRY(dev_alloc(ctx, (void**)&ctx->m0_keys, kvn * 4));
    TRY(dev_alloc(ctx, &ctx->m0_values, kvn * e));
    TRY(dev_alloc(ctx, (void**)&ctx->m0_mask, B * P * 4));
    CK(cudaMemset(ctx->m0_mask, 0, B * P * 4));
    std::vector<float> c(B * S * (hd / 2)), sn(B * S * (hd / 2));
    for (size_t bb = 0; bb < B; ++bb)
      for (size_t t = 0; t < S; ++t)
        for (int i = 0; i < hd / 2; ++i) {  // float64 -> fp32, as the prefix table above
          const double r = (double)(P + t) / std::pow((double)g.rope_theta, (2.0 / hd) * i);
          c[(bb * S + t) * (hd / 2) + i] = (float)std::cos(r);
          sn[(bb * S + t) * (hd / 2) + i] = (float)std::sin(r);
        }
    TRY(dev_alloc(ctx, (void**)&ctx->m0_cos, c.size() * 4));
    TRY(dev_alloc(ctx, (void**)&ctx->m0_sin, sn.size() * 4));
    CK(cudaMemcpy(ctx->m0_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ctx->m0_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }
  TRY(dev_alloc(ctx, &ctx->t1, (size_t)N * W1 * e));
  TRY(dev_alloc(ctx, &ctx->cond, (size_t)N * W1 * e));
  TRY(dev_alloc(ctx, &ctx->mods, (size_t)N * nmodw * e));
  // split-K partials (GEMMs with M < 256 only): splits·M·N ≤ (2·SMs/tiles + 1)·M·N
  //   ≤ 2·SMs·64·64 + 256·maxN
  size_t maxN = std::max(std::max(hq + 2 * hkv, 2 * F1), std::max(std::max(W1, W0), 2 * F0));
  ctx->splitk_floats = (size_t)2 * ctx->num_sms * 64 * 64 + 256 * maxN;
  TRY(dev_alloc(ctx, (void**)&ctx->splitk_ws, ctx->splitk_floats * 4));
  TRY(dev_alloc(ctx, (void**)&ctx->tickets, (1 << 16) * 4));
  CK(cudaMemset(ctx->tickets, 0, (1 << 16) * 4));
  TRY(dev_alloc(ctx, (void**)&ctx->dev_err, 16));
  if (g.quant != PI0_QUANT_NONE) {
    // the widest Linear: gate_up of either expert, the modulations, or the projections
    size_t mx = std::max(2 * F0 * W0, 2 * F1 * W1);
    mx = std::max(mx, std::max((hq + 2 * hkv) * std::max(W0, W1), 3 * W1 * W1));
    mx = std::max(mx, std::max(W0 * F0, W1 * F1));
    ctx->qscratch_elems = mx;
    TRY(dev_alloc(ctx, &ctx->qscratch, mx * e));
  }
  ctx->ssq_parts = ssq_slots(ctx->cfg);
  if (ctx->ssq_parts > sk::SSQ_MAX_PARTS)
    return fail(ctx, PI0_ERR_UNSUPPORTED, "action-expert width too large for the row-sum partials");
  TRY(dev_alloc(ctx, (void**)&ctx->ssq, MS * ctx->ssq_parts * 4));
  CK(cudaMemset(ctx->dev_err, 0, 16));
  return 0;
}

template <typename T>
int dequant_into(pi0_ctx* ctx, int quant, const uint32_t* qw, const T* scale, int64_t n_out,
                 int64_t k, T* out, cudaStream_t st) {
  if (!qw) return fail(ctx, PI0_ERR_INVALID, "q_scale without its q_weight");
  if ((size_t)(n_out * k) > ctx->qscratch_elems)
    return fail(ctx, PI0_ERR_INVALID, "dequantisation scratch too small");
  const int G = quant == PI0_QUANT_Q3 ? 40 : 32, bits = quant == PI0_QUANT_Q3 ? 3 : 4;
  const int epw = quant == PI0_QUANT_Q3 ? 10 : 8, maxint = quant == PI0_QUANT_Q3 ? 3 : 7;
  const int64_t n = n_out * k;
  dequantize_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(qw, scale, n_out, k, G, bits, epw,
                                                                    maxint, out);
  CKL();
  return 0;
}

// Quantised Linear -> the group-quantised blocks of the weight-streaming GEMMs (action expert,
// modulations, time MLP), with the same row re-layout (RoPE / gate-up permutations, fused row
// offsets) as the 16-bit copies. Other Linears are left to the dequantised path.
int pack_quantised(pi0_ctx* ctx, const Entry& en, const uint32_t* qw, const void* scale,
                   cudaStream_t st) {
  if (!qw) return fail(ctx, PI0_ERR_INVALID, "q_scale without its q_weight");
  const pi0_config& g = ctx->cfg;
  const int hq = g.num_heads * g.head_dim, hkv = g.num_kv_heads * g.head_dim;
  const int W1 = g.ae_width, F1 = g.ae_mlp_dim;
  void* dst = nullptr;
  const int* idx = nullptr;
  int row0 = 0;
  if (en.role <= R_D && en.expert == 1) {
    const LayerW& w = ctx->suf[en.layer];
    switch (en.role) {
      case R_Q: dst = w.qkv_q; idx = ctx->perm_q; break;
      case R_K: dst = w.qkv_q; idx = ctx->perm_k; row0 = hq; break;
      case R_V: dst = w.qkv_q; row0 = hq + hkv; break;
      case R_O: dst = w.o_q; break;
      case R_GU: dst = w.gu_q; idx = ctx->perm_gu1; break;
      case R_D: dst = w.d_q; break;
      default: break;
    }
  } else if (en.role == R_MOD_W) {
    dst = ctx->mod_w_q;
    row0 = en.layer * 3 * W1;
  } else if (en.role == R_TIN_W) {
    dst = ctx->tin_q;
  } else if (en.role == R_TOUT_W) {
    dst = ctx->tout_q;
  }
  if (!dst) return 0;
  const int n = (int)en.shape[0], K = (int)en.in_dim, nkb = K / 64;
  if (K % 64 || (K != W1 && K != hq && K != F1))
    return fail(ctx, PI0_ERR_INVALID, "internal: quantised block layout for " + en.name);
  const int threads = n * nkb;
  if (ctx->qb == 4)
    sk::pack_q_kernel<4><<<(threads + 255) / 256, 256, 0, st>>>(
        (uint8_t*)dst, qw, (const uint16_t*)scale, idx, n, K, row0, nkb);
  else
    sk::pack_q_kernel<3><<<(threads + 255) / 256, 256, 0, st>>>(
        (uint8_t*)dst, qw, (const uint16_t*)scale, idx, n, K, row0, nkb);
  CKL();
  return 0;
}

template <typename T>
int set_params_impl(pi0_ctx* ctx, const void* const* params, cudaStream_t st) {
  const pi0_config& g = ctx->cfg;
  const int hd = g.head_dim, H = g.num_heads, KV = g.num_kv_heads;
  const size_t hq = (size_t)H * hd, hkv = (size_t)KV * hd;
  const size_t W[2] = {(size_t)g.vlm_width, (size_t)g.ae_width};
  const size_t F[2] = {(size_t)g.vlm_mlp_dim, (size_t)g.ae_mlp_dim};
  const size_t e = sizeof(T);
  const size_t W1 = g.ae_width;
  const uint32_t* qw = nullptr;  // q_weight of the quantised Linear whose q_scale comes next
  for (size_t i = 0; i < ctx->table.size(); ++i) {
    const Entry& en = ctx->table[i];
    const void* src = params[i];
    if (!src) return fail(ctx, PI0_ERR_INVALID, "null pointer for parameter " + en.name);
    if (en.dtype == PI0_U32) {
      qw = static_cast<const uint32_t*>(src);
      continue;
    }
    if (en.in_dim > 0 && ctx->qb) TRY(pack_quantised(ctx, en, qw, src, st));
    if (en.in_dim > 0) {
      // quantised Linear: w = (code − max_int)·scale in the model dtype, then the same re-layout
      // as an unquantised weight
      const int quant = g.quant;
      TRY(dequant_into<T>(ctx, quant, qw, static_cast<const T*>(src), en.shape[0], en.in_dim,
                          (T*)ctx->qscratch, st));
      src = ctx->qscratch;
      qw = nullptr;
    }
    const int l = en.layer, ex = en.expert;
    LayerW* lw = nullptr;
    if (en.role <= R_D) lw = ex == 0 ? &ctx->pre[l] : &ctx->suf[l];
    const size_t Wd = W[ex];
    switch (en.role) {
      case R_Q: TRY(gather(ctx, lw->qkv, src, ctx->perm_q, (int)hq, (int)Wd, st)); break;
      case R_K:
        TRY(gather(ctx, (char*)lw->qkv + hq * Wd * e, src, ctx->perm_k, (int)hkv, (int)Wd, st));
        break;
      case R_V: TRY(copy(ctx, (char*)lw->qkv + (hq + hkv) * Wd * e, src, hkv * Wd * e, st)); break;
      case R_O: TRY(copy(ctx, lw->o, src, Wd * hq * e, st)); break;
      case R_GU:
        TRY(gather(ctx, lw->gu, src, ex == 0 ? ctx->perm_gu0 : ctx->perm_gu1, (int)(2 * F[ex]),
                   (int)Wd, st));
        break;
      case R_D: TRY(copy(ctx, lw->d, src, Wd * F[ex] * e, st)); break;
      case R_LN_IN: TRY(copy(ctx, ctx->pre[l].ln_in, src, W[0] * e, st)); break;
      case R_LN_POST: TRY(copy(ctx, ctx->pre[l].ln_post, src, W[0] * e, st)); break;
      case R_MOD_W:
        TRY(copy(ctx, (char*)ctx->mod_w + (size_t)l * 3 * W1 * W1 * e, src, 3 * W1 * W1 * e, st));
        break;
      case R_MOD_B:
        TRY(copy(ctx, (char*)ctx->mod_b + (size_t)l * 3 * W1 * e, src, 3 * W1 * e, st));
        break;
      case R_FINAL0: break;  // the prefix expert's final norm feeds nothing on the M1 path
      case R_AIN_W: TRY(copy(ctx, ctx->ain_w, src, W1 * g.action_dim * e, st)); break;
      case R_AIN_B: TRY(copy(ctx, ctx->ain_b, src, W1 * e, st)); break;
      case R_AOUT_W: TRY(copy(ctx, ctx->aout_w, src, W1 * g.action_dim * e, st)); break;
      case R_AOUT_B: TRY(copy(ctx, ctx->aout_b, src, g.action_dim * e, st)); break;
      case R_TIN_W: TRY(copy(ctx, ctx->tin_w, src, W1 * W1 * e, st)); break;
      case R_TIN_B: TRY(copy(ctx, ctx->tin_b, src, W1 * e, st)); break;
      case R_TOUT_W: TRY(copy(ctx, ctx->tout_w, src, W1 * W1 * e, st)); break;
      case R_TOUT_B: TRY(copy(ctx, ctx->tout_b, src, W1 * e, st)); break;
    }
  }
  // pack the weight-streaming matrices (from the repacked row-major copies above)
  auto pack = [&](void* dst, const void* src, size_t n, size_t k) -> int {
    const int nkb = (int)((k + 63) / 64);
    const size_t chunks = ((n + 127) / 128) * nkb * 128 * 8;
    sk::pack_sw128_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
        (uint16_t*)dst, (const uint16_t*)src, (int)n, (int)k, nkb, chunks);
    CKL();
    return 0;
  };
  for (int l = 0; l < g.depth; ++l) {
    const LayerW& w = ctx->suf[l];
    TRY(pack(w.qkv_p, w.qkv, hq + 2 * hkv, W[1]));
    TRY(pack(w.o_p, w.o, W[1], hq));
    TRY(pack(w.gu_p, w.gu, 2 * F[1], W[1]));
    TRY(pack(w.d_p, w.d, W[1], F[1]));
  }
  TRY(pack(ctx->mod_w_p, ctx->mod_w, (size_t)(2 * g.depth + 1) * 3 * W1, W1));
  TRY(pack(ctx->tin_p, ctx->tin_w, W1, W1));
  TRY(pack(ctx->tout_p, ctx->tout_w, W1, W1));
  return 0;
}

bool is_bf16(const pi0_ctx* c) { return c->cfg.dtype == PI0_BF16; }

// Profiling mode: capture `body` (kernel launches and the event records that bracket them) into
// a one-shot graph and replay it on `stream`, so the recorded intervals are device time without
// host launch gaps.
template <class F>
int run_profiled(pi0_ctx* ctx, cudaStream_t stream, F body) {
  cudaStream_t cs = ctx->cap_stream;
  CK(cudaStreamSynchronize(stream));
  CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  int r = body(cs);
  cudaGraph_t graph = nullptr;
  cudaError_t ce = cudaStreamEndCapture(cs, &graph);
  if (r) {
    if (graph) cudaGraphDestroy(graph);
    return r;
  }
  if (ce != cudaSuccess) return fail(ctx, PI0_ERR_CUDA, std::string("capture: ") + cudaGetErrorString(ce));
  cudaGraphExec_t exec = nullptr;
  ce = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ce != cudaSuccess) return fail(ctx, PI0_ERR_CUDA, std::string("instantiate: ") + cudaGetErrorString(ce));
  ce = cudaGraphLaunch(exec, stream);
  cudaError_t ce2 = cudaStreamSynchronize(stream);
  cudaGraphExecDestroy(exec);
  if (ce != cudaSuccess || ce2 != cudaSuccess)
    return fail(ctx, PI0_ERR_CUDA, std::string("profiled replay: ") + cudaGetErrorString(ce != cudaSuccess ? ce : ce2));
  return 0;
}

// Captures `body` (the launches of one call) on the context's capture stream into an executable
// graph; *nodes = the kernels it launched (a replay adds them to the launch counter).
template <class F>
int capture_graph(pi0_ctx* ctx, F body, cudaGraphExec_t* exec, int64_t* nodes) {
  cudaStream_t cs = ctx->cap_stream;
  const int64_t before = ctx->launches;
  CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  int r = body(cs);
  cudaGraph_t graph = nullptr;
  cudaError_t ce = cudaStreamEndCapture(cs, &graph);
  *nodes = ctx->launches - before;
  ctx->launches = before;
  if (r) {
    if (graph) cudaGraphDestroy(graph);
    return r;
  }
  if (ce != cudaSuccess)
    return fail(ctx, PI0_ERR_CUDA, std::string("capture: ") + cudaGetErrorString(ce));
  ce = cudaGraphInstantiate(exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ce != cudaSuccess)
    return fail(ctx, PI0_ERR_CUDA, std::string("instantiate: ") + cudaGetErrorString(ce));
  return 0;
}

int check_ready(pi0_ctx* ctx, int batch) {
  if (!ctx) return PI0_ERR_INVALID;
  if (!ctx->have_params) return fail(ctx, PI0_ERR_NO_PARAMS, "pi0_set_params has not been called");
  if (batch < 1 || batch > ctx->cfg.max_batch)
    return fail(ctx, PI0_ERR_INVALID, "batch must be in [1, max_batch]");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return fail(ctx, PI0_ERR_CUDA, cudaGetErrorString(e));
  return 0;
}

}  // namespace

// =============================================================================================
// C ABI
// =============================================================================================
extern "C" {

int pi0_create(const pi0_config* cfg, int device, pi0_ctx** out) {
  if (!cfg || !out) return PI0_ERR_INVALID;
  *out = nullptr;
  pi0_ctx* ctx = new pi0_ctx();
  ctx->cfg = *cfg;
  ctx->device = device;
  std::string why;
  int r = validate(*cfg, why);
  if (r) {
    *out = ctx;
    return fail(ctx, r, why);
  }
  ctx->esz = 2;
  build_table(ctx);
  *out = ctx;
  CK(cudaSetDevice(device));
  int sms = 0;
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  ctx->num_sms = sms;
  if (const char* env = std::getenv("PI0_CTA_PAIR")) ctx->cta_pair = env[0] != '0';
  CK(cudaStreamCreateWithFlags(&ctx->cap_stream, cudaStreamNonBlocking));
  TRY(alloc_all(ctx));
  TRY(is_bf16(ctx) ? setup_attrs<__nv_bfloat16>(ctx) : setup_attrs<__half>(ctx));
  TRY(setup_step_kernel(ctx));
  return 0;
}

int pi0_destroy(pi0_ctx* ctx) {
  if (!ctx) return 0;
  cudaSetDevice(ctx->device);
  for (auto& kv : ctx->graphs) cudaGraphExecDestroy(kv.second.first);
  for (auto& r : ctx->prof) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (auto e : ctx->ev_pool) cudaEventDestroy(e);
  if (ctx->cap_stream) cudaStreamDestroy(ctx->cap_stream);
  for (void* p : ctx->allocs) cudaFree(p);
  delete ctx;
  return 0;
}

const char* pi0_last_error(const pi0_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int pi0_num_params(const pi0_ctx* ctx) { return ctx ? (int)ctx->table.size() : -1; }

int pi0_param_info(const pi0_ctx* ctx, int i, const char** name, int* ndim, int64_t shape[2],
                   int* dtype) {
  if (!ctx || i < 0 || i >= (int)ctx->table.size()) return PI0_ERR_INVALID;
  const Entry& e = ctx->table[i];
  if (name) *name = e.name.c_str();
  if (ndim) *ndim = e.ndim;
  if (shape) {
    shape[0] = e.shape[0];
    shape[1] = e.shape[1];
  }
  if (dtype) *dtype = e.dtype;
  return 0;
}

int pi0_set_params(pi0_ctx* ctx, const void* const* params, int n, pi0_stream_t stream) {
  if (!ctx || !params) return PI0_ERR_INVALID;
  if (n != (int)ctx->table.size())
    return fail(ctx, PI0_ERR_INVALID, "expected " + std::to_string(ctx->table.size()) +
                                          " parameters, got " + std::to_string(n));
  CK(cudaSetDevice(ctx->device));
  int r = is_bf16(ctx) ? set_params_impl<__nv_bfloat16>(ctx, params, stream)
                       : set_params_impl<__half>(ctx, params, stream);
  if (r) return r;
  ctx->have_params = true;
  for (auto& kv : ctx->graphs) cudaGraphExecDestroy(kv.second.first);
  ctx->graphs.clear();
  return 0;
}

int pi0_prefill(pi0_ctx* ctx, int batch, const void* prefix_embs, const float* prefix_mask,
                float* keys, void* values, pi0_stream_t stream) {
  TRY(check_ready(ctx, batch));
  if (!prefix_embs || !prefix_mask || !keys || !values)
    return fail(ctx, PI0_ERR_INVALID, "null tensor argument");
  auto body = [&](cudaStream_t st) {
    if (is_bf16(ctx))
      return run_prefill<__nv_bfloat16>(ctx, batch, (const __nv_bfloat16*)prefix_embs, prefix_mask,
                                        keys, (__nv_bfloat16*)values, st);
    return run_prefill<__half>(ctx, batch, (const __half*)prefix_embs, prefix_mask, keys,
                               (__half*)values, st);
  };
  if (ctx->prof_on) return run_profiled(ctx, stream, body);
  return body(stream);
}

int pi0_denoise_step_kv(pi0_ctx* ctx, int batch, const float* keys, const void* values,
                        const void* x_t, const void* time_emb, const float* suffix_cos,
                        const float* suffix_sin, const float* prefix_mask, float* v_out,
                        pi0_stream_t stream) {
  TRY(check_ready(ctx, batch));
  if (!keys || !values || !x_t || !time_emb || !suffix_cos || !suffix_sin || !prefix_mask || !v_out)
    return fail(ctx, PI0_ERR_INVALID, "null tensor argument");
  auto body = [&](cudaStream_t st) {
    if (is_bf16(ctx))
      return run_step<__nv_bfloat16>(ctx, batch, keys, (const __nv_bfloat16*)values,
                                     (const __nv_bfloat16*)x_t, (const __nv_bfloat16*)time_emb,
                                     suffix_cos, suffix_sin, prefix_mask, v_out, st);
    return run_step<__half>(ctx, batch, keys, (const __half*)values, (const __half*)x_t,
                            (const __half*)time_emb, suffix_cos, suffix_sin, prefix_mask, v_out,
                            st);
  };
  if (ctx->prof_on) return run_profiled(ctx, stream, body);
  return body(stream);
}

int pi0_denoise_step(pi0_ctx* ctx, int batch, const void* prefix_embs, const void* x_t,
                     const void* time_emb, float* v_out, pi0_stream_t stream) {
  TRY(check_ready(ctx, batch));
  if (!prefix_embs || !x_t || !time_emb || !v_out)
    return fail(ctx, PI0_ERR_INVALID, "null tensor argument");
  auto body = [&](cudaStream_t st) {
    if (is_bf16(ctx)) {
      using T = __nv_bfloat16;
      TRY(run_prefill<T>(ctx, batch, (const T*)prefix_embs, ctx->m0_mask, ctx->m0_keys,
                         (T*)ctx->m0_values, st));
      return run_step<T>(ctx, batch, ctx->m0_keys, (const T*)ctx->m0_values, (const T*)x_t,
                         (const T*)time_emb, ctx->m0_cos, ctx->m0_sin, ctx->m0_mask, v_out, st);
    }
    using T = __half;
    TRY(run_prefill<T>(ctx, batch, (const T*)prefix_embs, ctx->m0_mask, ctx->m0_keys,
                       (T*)ctx->m0_values, st));
    return run_step<T>(ctx, batch, ctx->m0_keys, (const T*)ctx->m0_values, (const T*)x_t,
                       (const T*)time_emb, ctx->m0_cos, ctx->m0_sin, ctx->m0_mask, v_out, st);
  };
  if (ctx->prof_on) return run_profiled(ctx, stream, body);
  return body(stream);
}

int pi0_denoise_loop_kv(pi0_ctx* ctx, int batch, const float* keys, const void* values,
                        const float* x0, const void* time_embs, const float* suffix_cos,
                        const float* suffix_sin, const float* prefix_mask, float* x_out,
                        pi0_stream_t stream) {
  TRY(check_ready(ctx, batch));
  if (!keys || !values || !x0 || !time_embs || !suffix_cos || !suffix_sin || !prefix_mask || !x_out)
    return fail(ctx, PI0_ERR_INVALID, "null tensor argument");
  auto body = [&](cudaStream_t cs) {
    return is_bf16(ctx)
               ? run_loop_body<__nv_bfloat16>(ctx, batch, keys, (const __nv_bfloat16*)values, x0,
                                              (const __nv_bfloat16*)time_embs, suffix_cos,
                                              suffix_sin, prefix_mask, x_out, cs)
               : run_loop_body<__half>(ctx, batch, keys, (const __half*)values, x0,
                                       (const __half*)time_embs, suffix_cos, suffix_sin,
                                       prefix_mask, x_out, cs);
  };
  if (ctx->prof_on) return run_profiled(ctx, stream, body);
  GraphKey key{batch, {keys, values, x0, time_embs, suffix_cos, suffix_sin, prefix_mask, x_out,
                       nullptr}};
  auto it = ctx->graphs.find(key);
  if (it == ctx->graphs.end()) {
    cudaGraphExec_t exec = nullptr;
    int64_t nodes = 0;
    TRY(capture_graph(ctx, body, &exec, &nodes));
    if (ctx->graphs.size() > 64) {
      for (auto& kv : ctx->graphs) cudaGraphExecDestroy(kv.second.first);
      ctx->graphs.clear();
    }
    it = ctx->graphs.emplace(key, std::make_pair(exec, nodes)).first;
  }
  CK(cudaGraphLaunch(it->second.first, stream));
  ctx->launches += it->second.second;
  return 0;
}

int pi0_quantize_weight(int quant, int dtype, const void* w, int64_t n_out, int64_t k,
                        uint32_t* q_weight, void* q_scale, pi0_stream_t stream) {
  if (!w || !q_weight || !q_scale || n_out < 1 || k < 1) return PI0_ERR_INVALID;
  if (quant != PI0_QUANT_Q4 && quant != PI0_QUANT_Q3) return PI0_ERR_INVALID;
  const int G = quant == PI0_QUANT_Q3 ? 40 : 32, bits = quant == PI0_QUANT_Q3 ? 3 : 4;
  const int epw = quant == PI0_QUANT_Q3 ? 10 : 8, maxint = quant == PI0_QUANT_Q3 ? 3 : 7;
  int64_t n = n_out * ((k + G - 1) / G);
  int blocks = (int)((n + 255) / 256);
  if (dtype == PI0_F16)
    quantize_kernel<__half><<<blocks, 256, 0, stream>>>((const __half*)w, n_out, k, G, bits, epw,
                                                         maxint, q_weight, (__half*)q_scale);
  else if (dtype == PI0_BF16)
    quantize_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(
        (const __nv_bfloat16*)w, n_out, k, G, bits, epw, maxint, q_weight, (__nv_bfloat16*)q_scale);
  else
    return PI0_ERR_INVALID;
  return cudaGetLastError() == cudaSuccess ? 0 : PI0_ERR_CUDA;
}

int pi0_dequantize_weight(int quant, int dtype, const uint32_t* q_weight, const void* q_scale,
                          int64_t n_out, int64_t k, void* w, pi0_stream_t stream) {
  if (!w || !q_weight || !q_scale || n_out < 1 || k < 1) return PI0_ERR_INVALID;
  if (quant != PI0_QUANT_Q4 && quant != PI0_QUANT_Q3) return PI0_ERR_INVALID;
  const int G = quant == PI0_QUANT_Q3 ? 40 : 32, bits = quant == PI0_QUANT_Q3 ? 3 : 4;
  const int epw = quant == PI0_QUANT_Q3 ? 10 : 8, maxint = quant == PI0_QUANT_Q3 ? 3 : 7;
  int64_t n = n_out * k;
  int blocks = (int)((n + 255) / 256);
  if (dtype == PI0_F16)
    dequantize_kernel<__half><<<blocks, 256, 0, stream>>>(q_weight, (const __half*)q_scale, n_out,
                                                          k, G, bits, epw, maxint, (__half*)w);
  else if (dtype == PI0_BF16)
    dequantize_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(
        q_weight, (const __nv_bfloat16*)q_scale, n_out, k, G, bits, epw, maxint,
        (__nv_bfloat16*)w);
  else
    return PI0_ERR_INVALID;
  return cudaGetLastError() == cudaSuccess ? 0 : PI0_ERR_CUDA;
}

int64_t pi0_launch_count(const pi0_ctx* ctx) { return ctx ? ctx->launches : -1; }

int pi0_profile_enable(pi0_ctx* ctx, int on) {
  if (!ctx) return PI0_ERR_INVALID;
  CK(cudaSetDevice(ctx->device));
  for (auto& r : ctx->prof) {
    ctx->ev_pool.push_back(r.a);
    ctx->ev_pool.push_back(r.b);
  }
  ctx->prof.clear();
  ctx->prof_on = on != 0;
  return 0;
}

int pi0_profile_read(pi0_ctx* ctx, int n_families, int64_t* launches, double* total_ms) {
  if (!ctx || !launches || !total_ms) return PI0_ERR_INVALID;
  CK(cudaSetDevice(ctx->device));
  for (int f = 0; f < n_families; ++f) {
    launches[f] = 0;
    total_ms[f] = 0.0;
  }
  for (auto& r : ctx->prof) {
    CK(cudaEventSynchronize(r.b));
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, r.a, r.b));
    if (r.fam < n_families) {
      launches[r.fam] += 1;
      total_ms[r.fam] += ms;
    }
  }
  return 0;
}

int pi0_profile_families(void) { return F_NUM; }

int pi0_linear(pi0_ctx* ctx, const void* x, int M, int K, const void* w, int N, void* y,
               int engine, pi0_stream_t stream) {
  if (!ctx || !x || !w || !y || M < 1 || N < 2 || K < 8 || (N & 1) || (K % 8))
    return fail(ctx, PI0_ERR_INVALID, "pi0_linear: need M >= 1, even N, K a multiple of 8");
  if (engine == 2 && K % 32) return fail(ctx, PI0_ERR_INVALID, "warp-level engine needs K % 32 == 0");
  if (engine < 0 || engine > 5) return fail(ctx, PI0_ERR_INVALID, "pi0_linear: engine must be 0..5");
  CK(cudaSetDevice(ctx->device));
  if (is_bf16(ctx)) {
    using T = __nv_bfloat16;
    return gemm<T>(ctx, (const T*)x, K, (const T*)w, K, M, N, K, EpiStore<T>{(T*)y, N, nullptr},
                   stream, F_PRE_QKV, engine);
  }
  using T = __half;
  return gemm<T>(ctx, (const T*)x, K, (const T*)w, K, M, N, K, EpiStore<T>{(T*)y, N, nullptr},
                 stream, F_PRE_QKV, engine);
}

// One thread waits, through the same bounded mbarrier wait every kernel here uses, on a phase
// that completes only if `arrive` is nonzero: with no arrival the wait gives up after about a
// second and records ERR_TIMEOUT_EPI in *err, and the kernel returns normally.
__global__ void wait_check_kernel(int* err, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (arrive) tc::mbar_arrive(&bar);
    tc::mbar_wait(&bar, 0, err, tc::ERR_TIMEOUT_EPI, false);
  }
}

int pi0_wait_check(int* err, int arrive, pi0_stream_t stream) {
  if (!err) return PI0_ERR_INVALID;
  wait_check_kernel<<<1, 32, 0, stream>>>(err, arrive);
  return cudaGetLastError() == cudaSuccess ? 0 : PI0_ERR_CUDA;
}

int pi0_div_check(const float* a, const float* b, float* out, int64_t n, pi0_stream_t stream) {
  if (!a || !b || !out || n < 0) return PI0_ERR_INVALID;
  if (n == 0) return 0;
  div_check_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(a, b, out, n);
  return cudaGetLastError() == cudaSuccess ? 0 : PI0_ERR_CUDA;
}

int pi0_embed_language(int dtype, const void* table, int64_t vocab, int width,
                       const int32_t* input_ids, int n_tokens, void* out, int* err,
                       pi0_stream_t stream) {
  if (!table || !input_ids || !out || vocab < 1 || width < 8 || width % 8 || n_tokens < 0)
    return PI0_ERR_INVALID;
  // rows are moved in 16-byte vectors
  if ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15)
    return PI0_ERR_INVALID;
  if (n_tokens == 0) return 0;
  const int threads = std::min(256, std::max(32, width / 8));
  const double c = std::sqrt((double)width);
  if (dtype == PI0_F16) {
    embed_language_kernel<__half><<<n_tokens, threads, 0, stream>>>(
        (const __half*)table, vocab, width, input_ids, (__half*)out,
        __half2float(__float2half_rn((float)c)), err);
  } else if (dtype == PI0_BF16) {
    embed_language_kernel<__nv_bfloat16><<<n_tokens, threads, 0, stream>>>(
        (const __nv_bfloat16*)table, vocab, width, input_ids, (__nv_bfloat16*)out,
        __bfloat162float(__float2bfloat16_rn((float)c)), err);
  } else {
    return PI0_ERR_INVALID;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : PI0_ERR_CUDA;
}

int pi0_device_error(pi0_ctx* ctx) {
  if (!ctx) return PI0_ERR_INVALID;
  CK(cudaSetDevice(ctx->device));
  CK(cudaDeviceSynchronize());
  int h = 0;
  CK(cudaMemcpy(&h, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
  CK(cudaMemset(ctx->dev_err, 0, sizeof(int)));
  return h;
}

const char* pi0_profile_family_name(int family) {
  return family >= 0 && family < F_NUM ? kFamName[family] : "";
}

}  // extern "C"

// ---- allocation-free projection ----------------------------------------------------------
// y[M, N] = x[M, K] · w[N, K]^T on the warp-level split-K engine, with its split-K scratch in
// static device memory instead of a context's workspace, so that a call allocates nothing.
// The scratch is shared by every call on a device: calls that overlap in time (two streams,
// two host threads) race on it, so a caller must serialise them.
namespace {

constexpr size_t kNoAllocWsFloats = size_t(1) << 20;  // 4 MiB of fp32 split-K partials
constexpr int kNoAllocTickets = 4096;                  // output tiles of one call
constexpr int kNoAllocMaxDevices = 64;

// Tickets count the splits that have finished a tile; the last one resets its ticket to zero,
// so they are zero between calls that do not overlap. Static device memory starts zeroed. Two
// calls that overlap on the GPU can leave a ticket nonzero, and then every later call that uses
// that tile is wrong for the rest of the process: the caller must serialise the calls.
static __device__ __align__(256) float g_noalloc_ws[kNoAllocWsFloats];
static __device__ __align__(256) int g_noalloc_tickets[kNoAllocTickets];

struct NoAllocDev {
  float* ws = nullptr;
  int* tickets = nullptr;
  int num_sms = 0;
};
NoAllocDev g_noalloc[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current: the device addresses of the static scratch and
// the SM count. Neither call allocates.
int noalloc_setup(NoAllocDev* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PI0_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return PI0_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDev& d = g_noalloc[dev];
  if (!d.ws) {
    void* ws = nullptr;
    void* tk = nullptr;
    int sms = 0;
    if (cudaGetSymbolAddress(&ws, g_noalloc_ws) != cudaSuccess) return PI0_ERR_CUDA;
    if (cudaGetSymbolAddress(&tk, g_noalloc_tickets) != cudaSuccess) return PI0_ERR_CUDA;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return PI0_ERR_CUDA;
    d.tickets = static_cast<int*>(tk);
    d.num_sms = sms;
    d.ws = static_cast<float*>(ws);
  }
  *out = d;
  return 0;
}

template <typename T>
int linear_noalloc(const NoAllocDev& d, const T* x, int M, int K, const T* w, int N, T* y,
                   cudaStream_t st) {
  using C = GemmCfg<T, 64, 64, 32, 32, 4>;
  // the split rule of the context-owning warp-level engine (gemm(), M < 256)
  const int tiles = ((M + 63) / 64) * ((N + 63) / 64);
  int splits = std::max(1, (2 * d.num_sms + tiles - 1) / tiles);
  splits = std::min(splits, std::max(1, K / 128));
  const int ksteps = K / 32;
  splits = std::max(1, std::min(splits, ksteps));
  const int per = (ksteps + splits - 1) / splits;
  splits = (ksteps + per - 1) / per;
  if (splits > 1 && ((size_t)splits * M * N > kNoAllocWsFloats || tiles > kNoAllocTickets))
    return PI0_ERR_UNSUPPORTED;
  GemmArgs<T> g{x, K, w, K, M, N, K, per * 32, d.ws, d.tickets};
  dim3 grid((N + 63) / 64, (M + 63) / 64, splits);
  gemm_mma_kernel<T, 64, 64, 32, 32, 4, EpiStore<T>><<<grid, C::NT, C::SMEM, st>>>(
      g, EpiStore<T>{y, N, nullptr});
  return cudaGetLastError() == cudaSuccess ? 0 : PI0_ERR_CUDA;
}

}  // namespace

int pi0_linear_noalloc(int dtype, const void* x, int M, int K, const void* w, int N, void* y,
                       pi0_stream_t stream) {
  if (!x || !w || !y || M < 1 || N < 2 || (N & 1) || K < 32 || (K % 32)) return PI0_ERR_INVALID;
  if (dtype != PI0_F16 && dtype != PI0_BF16) return PI0_ERR_INVALID;
  // rows of x and w are read with 16-byte copies and y is written in pairs of elements: an
  // offset pointer is refused here instead of faulting in the kernel
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15 ||
      reinterpret_cast<uintptr_t>(y) & 3)
    return PI0_ERR_INVALID;
  NoAllocDev d;
  const int rc = noalloc_setup(&d);
  if (rc) return rc;
  if (dtype == PI0_BF16) {
    using T = __nv_bfloat16;
    return linear_noalloc<T>(d, (const T*)x, M, K, (const T*)w, N, (T*)y, stream);
  }
  using T = __half;
  return linear_noalloc<T>(d, (const T*)x, M, K, (const T*)w, N, (T*)y, stream);
}

#include "vision_api.cuh"
