// The vision stage of libpi0b200.so: vm["embed_image"] (python/mlc_vla/model/pi0/pi0_model.py:
// 97-99, spec :212-215; SigLIP So400m/14 + the PaliGemma projector, siglip.py:20-120) behind
// the pi0_vision_* C ABI of include/pi0b200.h. Included once by pi0_api.cu after its launch
// helpers: a vision context owns a pi0_ctx used only as launch plumbing (device, error text,
// error flag, SM count, launch counter, profiling records, graph cache).
//
// Per call, for n images of T = (image/patch)² patches (rows M = n·T):
//   patchify (zero-padded to kpad = round_up(p·p·C, 64) columns)
//   patch GEMM [M, kpad]·[W, kpad]^T  + bias + position embedding          -> x
//   per layer: LayerNorm -> q/k/v GEMM (bias; q·scale; head-padded model-dtype q, k and v)
//              -> attention (one CTA per 64 query rows of one image and head) -> out GEMM
//              over the head-padded context (+ bias, residual) -> LayerNorm -> fc1 GEMM (+ bias,
//              GELU-tanh) -> fc2 GEMM (+ bias, residual)
//   post LayerNorm -> projector GEMM (+ bias)                                -> out [M, proj]
// Heads of hd = 72 are padded to hdp = 80 columns (zero) so the attention's MMA shapes apply;
// the out-projection weight gets the matching zero input columns at bind time.
#pragma once

#include "vision.cuh"

namespace {

enum VRole {
  V_PATCH_W, V_PATCH_B, V_POS, V_Q_W, V_Q_B, V_K_W, V_K_B, V_V_W, V_V_B, V_O_W, V_O_B,
  V_FC1_W, V_FC1_B, V_FC2_W, V_FC2_B, V_LN1_W, V_LN1_B, V_LN2_W, V_LN2_B, V_POST_W, V_POST_B,
  V_PROJ_W, V_PROJ_B
};

struct VEntry {
  std::string name;
  int ndim;
  int64_t shape[2];
  VRole role;
  int layer;
};

struct VLayer {
  void *qkv_w, *qkv_b, *o_w, *o_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
  void *ln1_w, *ln1_b, *ln2_w, *ln2_b;
};

struct VisionKey {
  int n;
  const void* image;
  const void* out;
  bool operator<(const VisionKey& o) const {
    return std::tie(n, image, out) < std::tie(o.n, o.image, o.out);
  }
};

}  // namespace

struct pi0_vision_ctx {
  pi0_vision_config cfg{};
  pi0_ctx eng;  // launch plumbing only (its model config stays zero)
  std::vector<VEntry> table;
  int hd = 0, hdp = 0, np = 0, kpad = 0, pdim = 0;
  bool have_params = false;
  void *patch_w = nullptr, *patch_b = nullptr, *pos = nullptr;
  void *post_w = nullptr, *post_b = nullptr, *proj_w = nullptr, *proj_b = nullptr;
  std::vector<VLayer> layers;
  // workspaces for cfg.max_images images
  void *patches = nullptr, *x = nullptr, *xn = nullptr, *ctxo = nullptr, *h = nullptr;
  void *q = nullptr, *k = nullptr, *v = nullptr;  // model dtype, head-padded
  std::map<VisionKey, std::pair<cudaGraphExec_t, int64_t>> graphs;
};

namespace {

// the vision stage's parameter table in the reference's creation order (siglip.py:92-102,
// layers :78-83, attention :51-56, MLP :40-42)
void vision_table(pi0_vision_ctx* v) {
  const pi0_vision_config& c = v->cfg;
  const int W = c.hidden_size, F = c.intermediate_size;
  auto add = [&](const std::string& n, int64_t a, int64_t b, VRole r, int l) {
    v->table.push_back({n, b ? 2 : 1, {a, b}, r, l});
  };
  add("vision.patch_embedding.weight", W, v->pdim, V_PATCH_W, 0);
  add("vision.patch_embedding.bias", W, 0, V_PATCH_B, 0);
  add("vision.position_embedding", v->np, W, V_POS, 0);
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const std::string p = "vision.layers." + std::to_string(l) + ".";
    const char* projs[4] = {"q_proj", "k_proj", "v_proj", "out_proj"};
    const VRole rw[4] = {V_Q_W, V_K_W, V_V_W, V_O_W}, rb[4] = {V_Q_B, V_K_B, V_V_B, V_O_B};
    for (int i = 0; i < 4; ++i) {
      add(p + "self_attn." + projs[i] + ".weight", W, W, rw[i], l);
      add(p + "self_attn." + projs[i] + ".bias", W, 0, rb[i], l);
    }
    add(p + "mlp.fc1.weight", F, W, V_FC1_W, l);
    add(p + "mlp.fc1.bias", F, 0, V_FC1_B, l);
    add(p + "mlp.fc2.weight", W, F, V_FC2_W, l);
    add(p + "mlp.fc2.bias", W, 0, V_FC2_B, l);
    add(p + "layer_norm1.weight", W, 0, V_LN1_W, l);
    add(p + "layer_norm1.bias", W, 0, V_LN1_B, l);
    add(p + "layer_norm2.weight", W, 0, V_LN2_W, l);
    add(p + "layer_norm2.bias", W, 0, V_LN2_B, l);
  }
  add("vision.post_layernorm.weight", W, 0, V_POST_W, 0);
  add("vision.post_layernorm.bias", W, 0, V_POST_B, 0);
  add("vision.multi_modal_projector.weight", c.projection_dim, W, V_PROJ_W, 0);
  add("vision.multi_modal_projector.bias", c.projection_dim, 0, V_PROJ_B, 0);
}

int vision_validate(const pi0_vision_config& c, std::string& why) {
  auto bad = [&](const char* m) { why = m; return PI0_ERR_INVALID; };
  if (c.dtype != PI0_F16 && c.dtype != PI0_BF16) {
    why = "vision dtype must be float16 or bfloat16 on the GPU path";
    return PI0_ERR_UNSUPPORTED;
  }
  if (c.image_size < 1 || c.patch_size < 1 || c.num_channels < 1 || c.image_size % c.patch_size)
    return bad("image_size must be a positive multiple of patch_size");
  if (c.hidden_size < 8 || c.intermediate_size < 8 || c.projection_dim < 8 ||
      c.hidden_size % 8 || c.intermediate_size % 8 || c.projection_dim % 8)
    return bad("hidden_size, intermediate_size and projection_dim must be positive multiples of 8");
  if (c.hidden_size > 32 * 8 * LN_CHUNKS) {
    why = "hidden_size above 2048 is not supported";
    return PI0_ERR_UNSUPPORTED;
  }
  if (c.num_hidden_layers < 1 || c.num_attention_heads < 1 || c.hidden_size % c.num_attention_heads)
    return bad("num_hidden_layers >= 1 and hidden_size a multiple of num_attention_heads required");
  const int hd = c.hidden_size / c.num_attention_heads, hdp = (hd + 15) / 16 * 16;
  if (hd % 2 || !(hdp == 16 || hdp == 32 || hdp == 64 || hdp == 80 || hdp == 128)) {
    why = "head_dim must be even and pad to 16, 32, 64, 80 or 128";
    return PI0_ERR_UNSUPPORTED;
  }
  if (c.max_images < 1) return bad("max_images must be >= 1");
  if (!(c.layer_norm_eps > 0.f)) return bad("layer_norm_eps must be positive");
  return 0;
}

int vision_alloc(pi0_vision_ctx* v) {
  pi0_ctx* ctx = &v->eng;
  const pi0_vision_config& c = v->cfg;
  const size_t e = 2, W = c.hidden_size, F = c.intermediate_size, Pd = c.projection_dim;
  const size_t H = c.num_attention_heads, hdp = v->hdp, L = c.num_hidden_layers;
  const size_t M = (size_t)c.max_images * v->np;
  auto pad = [&](size_t elems) { return ((elems * e + 255) / 256) * 256; };
  size_t arena = pad(W * v->kpad) + pad(W) + pad((size_t)v->np * W) + 2 * pad(W) + pad(Pd * W) + pad(Pd);
  arena += L * (pad(3 * W * W) + pad(3 * W) + pad(W * H * hdp) + pad(W) + pad(F * W) + pad(F) +
                pad(W * F) + pad(W) + 4 * pad(W));
  TRY(dev_alloc(ctx, &ctx->arena, arena));
  ctx->arena_bytes = arena;
  CK(cudaMemset(ctx->arena, 0, arena));  // zero: the padded columns of the re-laid weights
  char* cur = (char*)ctx->arena;
  auto take = [&](size_t elems) {
    void* p = cur;
    cur += pad(elems);
    return p;
  };
  v->patch_w = take(W * v->kpad);
  v->patch_b = take(W);
  v->pos = take((size_t)v->np * W);
  v->post_w = take(W);
  v->post_b = take(W);
  v->proj_w = take(Pd * W);
  v->proj_b = take(Pd);
  v->layers.resize(L);
  for (auto& ly : v->layers) {
    ly.qkv_w = take(3 * W * W);
    ly.qkv_b = take(3 * W);
    ly.o_w = take(W * H * hdp);
    ly.o_b = take(W);
    ly.fc1_w = take(F * W);
    ly.fc1_b = take(F);
    ly.fc2_w = take(W * F);
    ly.fc2_b = take(W);
    ly.ln1_w = take(W);
    ly.ln1_b = take(W);
    ly.ln2_w = take(W);
    ly.ln2_b = take(W);
  }
  // workspaces; q, k and v keep their pad columns zero (the epilogue never writes them)
  TRY(dev_alloc(ctx, &v->patches, M * v->kpad * e));
  TRY(dev_alloc(ctx, &v->x, M * W * e));
  TRY(dev_alloc(ctx, &v->xn, M * W * e));
  for (void** p : {&v->q, &v->k, &v->v}) {
    TRY(dev_alloc(ctx, p, M * H * hdp * e));
    CK(cudaMemset(*p, 0, M * H * hdp * e));
  }
  TRY(dev_alloc(ctx, &v->ctxo, M * H * hdp * e));
  TRY(dev_alloc(ctx, &v->h, M * F * e));
  TRY(dev_alloc(ctx, (void**)&ctx->dev_err, sizeof(int)));
  CK(cudaMemset(ctx->dev_err, 0, sizeof(int)));
  return 0;
}

template <typename T, class Epi>
int attr_tc_all(pi0_ctx* ctx) {
  TRY((attr_tc<T, 256, 4, Epi>(ctx)));
  TRY((attr_tc<T, 256, 4, Epi, 2>(ctx)));
  TRY((attr_tc<T, 160, 5, Epi>(ctx)));
  TRY((attr_tc<T, 128, 6, Epi>(ctx)));
  TRY((attr_tc<T, 128, 6, Epi, 2>(ctx)));
  TRY((attr_tc<T, 256, pair_stages<256>(), Epi, 1, 2>(ctx)));
  return 0;
}

// Projection of the vision stage. The row count is small (256 per image), so a GEMM whose
// 128×128 tiles cover under half of the SMs (the N = hidden projections: 54 tiles for three
// images) splits K between the two CTAs of a cluster pair; otherwise the automatic tiling.
template <typename T, class Epi>
int vision_gemm(pi0_ctx* ctx, const T* A, int lda, const T* W, int ldw, int M, int N, int K,
                const Epi& epi, cudaStream_t st, int fam) {
  const int tiles128 = ((M + tc::BM - 1) / tc::BM) * ((N + 127) / 128);
  if (M > 128 && 2 * tiles128 <= ctx->num_sms && (K + tc::BK - 1) / tc::BK >= 8)
    return gemm_tc_pair_launch<T, Epi, 128, 6>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam);
  return gemm<T>(ctx, A, lda, W, ldw, M, N, K, epi, st, fam, M > 128 ? 0 : 1);
}

template <typename T, int HD>
int attr_vattn(pi0_ctx* ctx) {
  CK(cudaFuncSetAttribute(vattn_kernel<T, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          VattnSmem<HD>::BYTES));
  return 0;
}

template <typename T>
int vision_attrs(pi0_vision_ctx* v) {
  pi0_ctx* ctx = &v->eng;
  TRY((attr_tc_all<T, EpiBiasPos<T>>(ctx)));
  TRY((attr_tc_all<T, EpiVisionQkv<T>>(ctx)));
  TRY((attr_tc_all<T, EpiResidBias<T>>(ctx)));
  TRY((attr_tc_all<T, EpiBiasGelu<T>>(ctx)));
  TRY((attr_tc_all<T, EpiStore<T>>(ctx)));
  switch (v->hdp) {
    case 16: return attr_vattn<T, 16>(ctx);
    case 32: return attr_vattn<T, 32>(ctx);
    case 64: return attr_vattn<T, 64>(ctx);
    case 80: return attr_vattn<T, 80>(ctx);
    case 128: return attr_vattn<T, 128>(ctx);
  }
  return fail(ctx, PI0_ERR_UNSUPPORTED, "vision head_dim");
}

// Copies the caller's parameters (device pointers, table order) into the arena: q/k/v rows
// concatenated [q; k; v], the patch-embedding weight widened to kpad zero-padded columns and the
// out-projection weight to hdp columns per head.
int vision_set_params_impl(pi0_vision_ctx* v, const void* const* params, cudaStream_t st) {
  pi0_ctx* ctx = &v->eng;
  const pi0_vision_config& c = v->cfg;
  const size_t e = 2, W = c.hidden_size, F = c.intermediate_size, Pd = c.projection_dim;
  const int H = c.num_attention_heads;
  auto regroup = [&](void* dst, int dst_ld, const void* src, int src_ld, int rows, int groups,
                     int sg, int dg) -> int {
    const int64_t total = (int64_t)rows * groups * sg;
    regroup_cols_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
        (uint16_t*)dst, dst_ld, (const uint16_t*)src, src_ld, rows, groups, sg, dg);
    CKL();
    return 0;
  };
  for (size_t i = 0; i < v->table.size(); ++i) {
    const VEntry& en = v->table[i];
    const void* src = params[i];
    if (!src) return fail(ctx, PI0_ERR_INVALID, "null pointer for parameter " + en.name);
    VLayer* ly = en.role >= V_Q_W && en.role <= V_LN2_B ? &v->layers[en.layer] : nullptr;
    switch (en.role) {
      case V_PATCH_W:
        TRY(regroup(v->patch_w, v->kpad, src, v->pdim, (int)W, 1, v->pdim, v->kpad));
        break;
      case V_PATCH_B: TRY(copy(ctx, v->patch_b, src, W * e, st)); break;
      case V_POS: TRY(copy(ctx, v->pos, src, (size_t)v->np * W * e, st)); break;
      case V_Q_W: TRY(copy(ctx, ly->qkv_w, src, W * W * e, st)); break;
      case V_K_W: TRY(copy(ctx, (char*)ly->qkv_w + W * W * e, src, W * W * e, st)); break;
      case V_V_W: TRY(copy(ctx, (char*)ly->qkv_w + 2 * W * W * e, src, W * W * e, st)); break;
      case V_Q_B: TRY(copy(ctx, ly->qkv_b, src, W * e, st)); break;
      case V_K_B: TRY(copy(ctx, (char*)ly->qkv_b + W * e, src, W * e, st)); break;
      case V_V_B: TRY(copy(ctx, (char*)ly->qkv_b + 2 * W * e, src, W * e, st)); break;
      case V_O_W:
        TRY(regroup(ly->o_w, H * v->hdp, src, (int)W, (int)W, H, v->hd, v->hdp));
        break;
      case V_O_B: TRY(copy(ctx, ly->o_b, src, W * e, st)); break;
      case V_FC1_W: TRY(copy(ctx, ly->fc1_w, src, F * W * e, st)); break;
      case V_FC1_B: TRY(copy(ctx, ly->fc1_b, src, F * e, st)); break;
      case V_FC2_W: TRY(copy(ctx, ly->fc2_w, src, W * F * e, st)); break;
      case V_FC2_B: TRY(copy(ctx, ly->fc2_b, src, W * e, st)); break;
      case V_LN1_W: TRY(copy(ctx, ly->ln1_w, src, W * e, st)); break;
      case V_LN1_B: TRY(copy(ctx, ly->ln1_b, src, W * e, st)); break;
      case V_LN2_W: TRY(copy(ctx, ly->ln2_w, src, W * e, st)); break;
      case V_LN2_B: TRY(copy(ctx, ly->ln2_b, src, W * e, st)); break;
      case V_POST_W: TRY(copy(ctx, v->post_w, src, W * e, st)); break;
      case V_POST_B: TRY(copy(ctx, v->post_b, src, W * e, st)); break;
      case V_PROJ_W: TRY(copy(ctx, v->proj_w, src, Pd * W * e, st)); break;
      case V_PROJ_B: TRY(copy(ctx, v->proj_b, src, Pd * e, st)); break;
    }
  }
  return 0;
}

template <typename T>
int vision_layernorm(pi0_vision_ctx* v, const T* x, T* out, int rows, const void* w, const void* b,
                     cudaStream_t st) {
  pi0_ctx* ctx = &v->eng;
  Prof pr(ctx, F_VIS_NORM, st);
  return launch(ctx, layernorm_kernel<T>, dim3((rows + 7) / 8), dim3(256), 0, st, dim3(1, 1, 1), x,
                out, rows, v->cfg.hidden_size, v->cfg.layer_norm_eps, (const T*)w, (const T*)b);
}

template <typename T, int HD>
int vattn_launch(pi0_vision_ctx* v, int n, cudaStream_t st) {
  pi0_ctx* ctx = &v->eng;
  const int T_len = v->np, H = v->cfg.num_attention_heads;
  Prof pr(ctx, F_VIS_ATTN, st);
  return launch(ctx, vattn_kernel<T, HD>, dim3((T_len + VA_BQ - 1) / VA_BQ, 1, n * H), dim3(128),
                VattnSmem<HD>::BYTES, st, dim3(1, 1, 1), (const T*)v->q, (const T*)v->k,
                (const T*)v->v, (T*)v->ctxo, T_len, H);
}

template <typename T>
int vision_attention(pi0_vision_ctx* v, int n, cudaStream_t st) {
  switch (v->hdp) {
    case 16: return vattn_launch<T, 16>(v, n, st);
    case 32: return vattn_launch<T, 32>(v, n, st);
    case 64: return vattn_launch<T, 64>(v, n, st);
    case 80: return vattn_launch<T, 80>(v, n, st);
    case 128: return vattn_launch<T, 128>(v, n, st);
  }
  return fail(&v->eng, PI0_ERR_UNSUPPORTED, "vision head_dim");
}

template <typename T>
int run_embed_image(pi0_vision_ctx* v, int n, const T* image, T* out, cudaStream_t st) {
  pi0_ctx* ctx = &v->eng;
  const pi0_vision_config& c = v->cfg;
  const int W = c.hidden_size, F = c.intermediate_size, Pd = c.projection_dim;
  const int H = c.num_attention_heads, np = v->np, M = n * np, HP = H * v->hdp;
  T* x = (T*)v->x;
  T* xn = (T*)v->xn;
  {
    Prof pr(ctx, F_VIS_PATCH, st);
    const int64_t total = (int64_t)M * v->kpad;
    TRY(launch(ctx, patchify_kernel<T>, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st,
               dim3(1, 1, 1), image, (T*)v->patches, n, c.image_size, c.patch_size,
               c.num_channels, v->kpad));
  }
  TRY(vision_gemm<T>(ctx, (const T*)v->patches, v->kpad, (const T*)v->patch_w, v->kpad, M, W,
                     v->kpad, EpiBiasPos<T>{x, W, (const T*)v->patch_b, (const T*)v->pos, np}, st,
                     F_VIS_PATCH));
  // hd^-0.5 as a model-dtype constant (the scalar operand of q * scale takes q's dtype)
  const float s32 = (float)std::pow((double)v->hd, -0.5);
  const float qscale = Tr<T>::kBf16 ? __bfloat162float(__float2bfloat16_rn(s32))
                                    : __half2float(__float2half_rn(s32));
  for (const VLayer& ly : v->layers) {
    TRY(vision_layernorm<T>(v, x, xn, M, ly.ln1_w, ly.ln1_b, st));
    TRY(vision_gemm<T>(ctx, xn, W, (const T*)ly.qkv_w, W, M, 3 * W, W,
                       EpiVisionQkv<T>{(T*)v->q, (T*)v->k, (T*)v->v, (const T*)ly.qkv_b, np, H,
                                       v->hd, v->hdp, qscale},
                       st, F_VIS_QKV));
    TRY(vision_attention<T>(v, n, st));
    TRY(vision_gemm<T>(ctx, (const T*)v->ctxo, HP, (const T*)ly.o_w, HP, M, W, HP,
                       EpiResidBias<T>{x, W, (const T*)ly.o_b}, st, F_VIS_O));
    TRY(vision_layernorm<T>(v, x, xn, M, ly.ln2_w, ly.ln2_b, st));
    TRY(vision_gemm<T>(ctx, xn, W, (const T*)ly.fc1_w, W, M, F, W,
                       EpiBiasGelu<T>{(T*)v->h, F, (const T*)ly.fc1_b}, st, F_VIS_FC1));
    TRY(vision_gemm<T>(ctx, (const T*)v->h, F, (const T*)ly.fc2_w, F, M, W, F,
                       EpiResidBias<T>{x, W, (const T*)ly.fc2_b}, st, F_VIS_FC2));
  }
  TRY(vision_layernorm<T>(v, x, xn, M, v->post_w, v->post_b, st));
  return vision_gemm<T>(ctx, xn, W, (const T*)v->proj_w, W, M, Pd, W,
                        EpiStore<T>{out, Pd, (const T*)v->proj_b}, st, F_VIS_PROJ);
}

}  // namespace

// =============================================================================================
// C ABI of the vision stage
// =============================================================================================
extern "C" {

int pi0_vision_create(const pi0_vision_config* cfg, int device, pi0_vision_ctx** out) {
  if (!cfg || !out) return PI0_ERR_INVALID;
  pi0_vision_ctx* v = new pi0_vision_ctx();
  *out = v;
  v->cfg = *cfg;
  v->eng.device = device;
  pi0_ctx* ctx = &v->eng;
  std::string why;
  int r = vision_validate(*cfg, why);
  if (r) return fail(ctx, r, why);
  v->hd = cfg->hidden_size / cfg->num_attention_heads;
  v->hdp = (v->hd + 15) / 16 * 16;
  const int side = cfg->image_size / cfg->patch_size;
  v->np = side * side;
  v->pdim = cfg->patch_size * cfg->patch_size * cfg->num_channels;
  v->kpad = (v->pdim + 63) / 64 * 64;
  vision_table(v);
  CK(cudaSetDevice(device));
  int sms = 0;
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  ctx->num_sms = sms;
  if (const char* env = std::getenv("PI0_CTA_PAIR")) ctx->cta_pair = env[0] != '0';
  CK(cudaStreamCreateWithFlags(&ctx->cap_stream, cudaStreamNonBlocking));
  TRY(vision_alloc(v));
  return cfg->dtype == PI0_BF16 ? vision_attrs<__nv_bfloat16>(v) : vision_attrs<__half>(v);
}

int pi0_vision_destroy(pi0_vision_ctx* v) {
  if (!v) return 0;
  cudaSetDevice(v->eng.device);
  for (auto& kv : v->graphs) cudaGraphExecDestroy(kv.second.first);
  for (auto& r : v->eng.prof) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (auto e : v->eng.ev_pool) cudaEventDestroy(e);
  if (v->eng.cap_stream) cudaStreamDestroy(v->eng.cap_stream);
  for (void* p : v->eng.allocs) cudaFree(p);
  delete v;
  return 0;
}

const char* pi0_vision_last_error(const pi0_vision_ctx* v) {
  return v ? v->eng.err.c_str() : "null context";
}

int pi0_vision_num_params(const pi0_vision_ctx* v) { return v ? (int)v->table.size() : -1; }

int pi0_vision_param_info(const pi0_vision_ctx* v, int i, const char** name, int* ndim,
                          int64_t shape[2], int* dtype) {
  if (!v || i < 0 || i >= (int)v->table.size()) return PI0_ERR_INVALID;
  const VEntry& e = v->table[i];
  if (name) *name = e.name.c_str();
  if (ndim) *ndim = e.ndim;
  if (shape) {
    shape[0] = e.shape[0];
    shape[1] = e.shape[1];
  }
  if (dtype) *dtype = v->cfg.dtype;
  return 0;
}

int pi0_vision_set_params(pi0_vision_ctx* v, const void* const* params, int n,
                          pi0_stream_t stream) {
  if (!v || !params) return PI0_ERR_INVALID;
  pi0_ctx* ctx = &v->eng;
  if (n != (int)v->table.size())
    return fail(ctx, PI0_ERR_INVALID, "expected " + std::to_string(v->table.size()) +
                                          " parameters, got " + std::to_string(n));
  CK(cudaSetDevice(ctx->device));
  TRY(vision_set_params_impl(v, params, stream));
  v->have_params = true;
  return 0;
}

int pi0_embed_image(pi0_vision_ctx* v, int n_images, const void* image, void* out,
                    pi0_stream_t stream) {
  if (!v) return PI0_ERR_INVALID;
  pi0_ctx* ctx = &v->eng;
  if (!v->have_params) return fail(ctx, PI0_ERR_NO_PARAMS, "pi0_vision_set_params has not been called");
  if (n_images < 1 || n_images > v->cfg.max_images)
    return fail(ctx, PI0_ERR_INVALID, "n_images must be in [1, max_images]");
  if (!image || !out) return fail(ctx, PI0_ERR_INVALID, "null tensor argument");
  if ((reinterpret_cast<uintptr_t>(out) & 3) || (reinterpret_cast<uintptr_t>(image) & 1))
    return fail(ctx, PI0_ERR_INVALID, "image must be 2-byte and out 4-byte aligned");
  CK(cudaSetDevice(ctx->device));
  auto body = [&](cudaStream_t cs) {
    if (v->cfg.dtype == PI0_BF16)
      return run_embed_image<__nv_bfloat16>(v, n_images, (const __nv_bfloat16*)image,
                                            (__nv_bfloat16*)out, cs);
    return run_embed_image<__half>(v, n_images, (const __half*)image, (__half*)out, cs);
  };
  if (ctx->prof_on) return run_profiled(ctx, stream, body);
  VisionKey key{n_images, image, out};
  auto it = v->graphs.find(key);
  if (it == v->graphs.end()) {
    cudaGraphExec_t exec = nullptr;
    int64_t nodes = 0;
    TRY(capture_graph(ctx, body, &exec, &nodes));
    if (v->graphs.size() > 64) {
      for (auto& kv : v->graphs) cudaGraphExecDestroy(kv.second.first);
      v->graphs.clear();
    }
    it = v->graphs.emplace(key, std::make_pair(exec, nodes)).first;
  }
  CK(cudaGraphLaunch(it->second.first, stream));
  ctx->launches += it->second.second;
  return 0;
}

int64_t pi0_vision_launch_count(const pi0_vision_ctx* v) { return v ? v->eng.launches : -1; }

int pi0_vision_device_error(pi0_vision_ctx* v) { return v ? pi0_device_error(&v->eng) : PI0_ERR_INVALID; }

int pi0_vision_profile_enable(pi0_vision_ctx* v, int on) {
  return v ? pi0_profile_enable(&v->eng, on) : PI0_ERR_INVALID;
}

int pi0_vision_profile_read(pi0_vision_ctx* v, int n_families, int64_t* launches,
                            double* total_ms) {
  return v ? pi0_profile_read(&v->eng, n_families, launches, total_ms) : PI0_ERR_INVALID;
}

}  // extern "C"
