/*
 * pi0b200.h — C ABI of libpi0b200.so, the B200 (sm_100a) π0.5 M1 hot path.
 *
 * The reference compiles the π0.5 backbone with TVM and calls three exported functions
 * through a Relax VM, passing the packed parameter list as the last argument:
 *
 *   vm["prefill"](prefix_embs, prefix_mask, params)                -> (keys, values)
 *   vm["denoise_step_kv"](keys, values, x_t, time_emb, suffix_cos,
 *                         suffix_sin, prefix_mask, params)         -> v_t
 *   vm["denoise_loop_kv"](keys, values, x0, time_embs, suffix_cos,
 *                         suffix_sin, prefix_mask, params)         -> x
 *
 * (python/mlc_vla/model/pi0/pi0_model.py:128-194, spec :197-255; called from
 * python/mlc_vla/sample.py:128,158,184). This header is the C-level replacement of that
 * VM boundary: plain device pointers and sizes, one context per (GPU, host thread), every
 * call asynchronous on the caller's stream and returning a status code.
 *
 * Tensor layouts (row-major, batch B ≤ cfg.max_batch; the reference fixes B = 1):
 *   prefix_embs  [B, P, W0]            model dtype
 *   prefix_mask  [B, P]                fp32 additive (0 = valid, -1e9 = padding)
 *   keys         [L, B, KV, P, hd]     fp32 (post-RoPE)
 *   values       [L, B, KV, P, hd]     model dtype
 *   x_t          [B, S, D]             model dtype
 *   x0, x, v     [B, S, D]             fp32
 *   time_emb     [1, W1]               model dtype (shared by the batch)
 *   time_embs    [N, W1]               model dtype
 *   suffix_cos/sin [B, S, hd/2]        fp32 (per-request RoPE offset = #valid prefix)
 * where P = prefix_len, S = action_horizon, D = action_dim, W0/W1 = expert widths,
 * L = depth, KV = num_kv_heads, hd = head_dim, N = num_denoise_steps.
 */
#ifndef PI0B200_H_
#define PI0B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* pi0_stream_t; /* the same type as cudaStream_t */
typedef struct pi0_ctx pi0_ctx;

enum pi0_status {
  PI0_OK = 0,
  PI0_ERR_INVALID = 1,     /* bad argument, shape or configuration */
  PI0_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  PI0_ERR_NO_PARAMS = 3,   /* compute called before pi0_set_params */
  PI0_ERR_DEVICE = 4,      /* a kernel reported an error flag (bounded wait gave up) */
  PI0_ERR_UNSUPPORTED = 5  /* configuration this build does not implement */
};

enum pi0_dtype { PI0_F16 = 0, PI0_BF16 = 1, PI0_F32 = 2, PI0_U32 = 3 };

/* Weight formats: the reference's quantisation presets (python/mlc_vla/quant.py:370-387). */
enum pi0_quant { PI0_QUANT_NONE = 0, PI0_QUANT_Q4 = 1 /* q4f16_1 / q4bf16_1 */,
                 PI0_QUANT_Q3 = 2 /* q3f16_1 */ };

/* Operand type of the attention logits q·kᵀ: the reference's Pi0Config.attn_logits_dtype
 * (python/mlc_vla/model/pi0/pi0_config.py:97-102, gemma_dual.py:115), whose default is
 * "float32" (fp32 q and k); the model dtype casts q and k to fp16 / bf16 first. Either way the
 * product is accumulated in fp32. */
enum pi0_logits { PI0_LOGITS_F32 = 0, PI0_LOGITS_MODEL_DTYPE = 1 };

/* Model shape: the fields of Pi0Config / GemmaExpertConfig the backbone build reads
 * (python/mlc_vla/model/pi0/pi0_config.py:17-170). */
typedef struct pi0_config {
  int32_t vlm_width, vlm_mlp_dim;     /* W0, F0 */
  int32_t ae_width, ae_mlp_dim;       /* W1, F1 */
  int32_t depth, num_heads, num_kv_heads, head_dim;
  int32_t prefix_len, action_horizon, action_dim;
  int32_t num_denoise_steps;
  int32_t dtype;                      /* pi0_dtype: PI0_F16 or PI0_BF16 */
  int32_t quant;                      /* pi0_quant */
  int32_t max_batch;                  /* workspace sizing; calls may use any B ≤ this */
  float rms_norm_eps;                 /* 1e-6 */
  float rope_theta;                   /* 1e4 */
  int32_t attn_logits;                /* pi0_logits (zero: fp32, the reference's default) */
} pi0_config;

/* Replaces compile_model + relax.VirtualMachine (python/mlc_vla/sample.py:91-95,
 * compile.py:99-133): allocates the context, workspaces and the packed-weight arena on
 * `device`. */
int pi0_create(const pi0_config* cfg, int device, pi0_ctx** out);
int pi0_destroy(pi0_ctx* ctx);
/* Text of the last error on this context (valid until the next call on it). */
const char* pi0_last_error(const pi0_ctx* ctx);

/* The packed-parameter table, in the reference's export order (export_tvm named_params,
 * python/mlc_vla/compile.py:34-38): name, shape (ndim ≤ 2) and pi0_dtype of entry i. */
int pi0_num_params(const pi0_ctx* ctx);
int pi0_param_info(const pi0_ctx* ctx, int i, const char** name, int* ndim, int64_t shape[2],
                   int* dtype);

/* Replaces the per-call `params` argument of every VM function (sample.py:98-100,128): takes
 * the device pointers of all n = pi0_num_params() parameters, in table order, and repacks
 * them into the context's weight arena (the caller keeps ownership of its buffers). */
int pi0_set_params(pi0_ctx* ctx, const void* const* params, int n, pi0_stream_t stream);

/* vm["prefill"] (pi0_model.py:128-140): writes keys and values for B requests. */
int pi0_prefill(pi0_ctx* ctx, int batch, const void* prefix_embs, const float* prefix_mask,
                float* keys, void* values, pi0_stream_t stream);

/* vm["denoise_step_kv"] (pi0_model.py:142-163): one suffix-only step; v_out fp32. */
int pi0_denoise_step_kv(pi0_ctx* ctx, int batch, const float* keys, const void* values,
                        const void* x_t, const void* time_emb, const float* suffix_cos,
                        const float* suffix_sin, const float* prefix_mask, float* v_out,
                        pi0_stream_t stream);

/* vm["denoise_step"], the M0 joint step (pi0_model.py:111-125; gemma_dual.py:162-233): one
 * denoising step of both experts over [prefix; suffix] with the joint mask (all prefix tokens
 * valid; suffix RoPE positions P .. P+S-1). Computed as the prefix expert's pass into a K/V cache
 * the context owns, then the suffix step on it: the joint mask lets no prefix token see the
 * suffix, so this is the same function (the M1 ≡ M0 identity). prefix_embs [B, P, W0], x_t
 * [B, S, D] model dtype, time_emb [1, W1]; v_out [B, S, D] fp32. */
int pi0_denoise_step(pi0_ctx* ctx, int batch, const void* prefix_embs, const void* x_t,
                     const void* time_emb, float* v_out, pi0_stream_t stream);

/* vm["denoise_loop_kv"] (pi0_model.py:165-194): cfg.num_denoise_steps Euler steps
 * (dt = -1/N, x in fp32), replayed as one CUDA graph per distinct argument set. x_out may
 * alias x0. */
int pi0_denoise_loop_kv(pi0_ctx* ctx, int batch, const float* keys, const void* values,
                        const float* x0, const void* time_embs, const float* suffix_cos,
                        const float* suffix_sin, const float* prefix_mask, float* x_out,
                        pi0_stream_t stream);

/* Replaces GroupQuantize.quantize_weight (python/mlc_vla/quant.py:195-266) on the GPU:
 * w [n_out, k] model dtype -> q_weight [n_out, ceil(k/G)*G/epw] uint32 and
 * q_scale [n_out, ceil(k/G)] model dtype, for quant PI0_QUANT_Q4 (G=32, 8 codes per word)
 * or PI0_QUANT_Q3 (G=40, 10 codes per word). Context-free. */
int pi0_quantize_weight(int quant, int dtype, const void* w, int64_t n_out, int64_t k,
                        uint32_t* q_weight, void* q_scale, pi0_stream_t stream);

/* The inverse (quant.py:176-193): w = (code - max_int) * scale in the model dtype. */
int pi0_dequantize_weight(int quant, int dtype, const uint32_t* q_weight, const void* q_scale,
                          int64_t n_out, int64_t k, void* w, pi0_stream_t stream);

/* vm["embed_language"] (python/mlc_vla/model/pi0/pi0_model.py:101-104, spec :217-220; the prefix
 * expert's token embedding before prefix assembly): out[t, :] = table[input_ids[t], :] · sqrt(width)
 * in the model dtype (the constant rounded to that dtype, one rounding of the product).
 * table [vocab, width] (embed_tokens.weight, PaliGemma vocab 257152), input_ids [n_tokens] int32,
 * out [n_tokens, width]; width a multiple of 8, table and out 16-byte aligned (PI0_ERR_INVALID
 * otherwise). An id outside [0, vocab) yields a zero row and
 * sets the device int *err to 1 (err may be NULL). Context-free. */
int pi0_embed_language(int dtype, const void* table, int64_t vocab, int width,
                       const int32_t* input_ids, int n_tokens, void* out, int* err,
                       pi0_stream_t stream);

/* ---- the vision stage: vm["embed_image"] ---------------------------------------------------
 * The reference compiles each stage as its own engine with its own packed parameters
 * (python/mlc_vla/model/pi0/pi0_model.py:43-58 include_for, :76-77) and calls
 *   vm["embed_image"](image, params) -> image tokens
 * (pi0_model.py:97-99, spec :212-215: image [1, 224, 224, 3] model dtype, channels last). These
 * calls replace that engine: a vision context holds the SigLIP So400m/14 tower and the PaliGemma
 * projector (siglip.py:20-120). Layouts: image [n, S, S, C] model dtype (S = image_size, C =
 * num_channels), out [n, T, projection_dim] model dtype, T = (S / patch_size)². */
typedef struct pi0_vision_ctx pi0_vision_ctx;

/* SiglipConfig (python/mlc_vla/model/pi0/pi0_config.py:60-81) plus the model dtype and the
 * workspace size. */
typedef struct pi0_vision_config {
  int32_t image_size, patch_size, num_channels;   /* 224, 14, 3 */
  int32_t hidden_size, intermediate_size;         /* 1152, 4304 */
  int32_t num_hidden_layers, num_attention_heads; /* 27, 16 */
  int32_t projection_dim;                         /* 2048 (the prefix expert's width) */
  int32_t dtype;                                  /* pi0_dtype: PI0_F16 or PI0_BF16 */
  int32_t max_images;                             /* workspace sizing; calls use n ≤ this */
  float layer_norm_eps;                           /* 1e-6 */
} pi0_vision_config;

/* Replaces compiling and loading the vision engine (compile.py:99-133 with functions
 * ["embed_image"]). */
int pi0_vision_create(const pi0_vision_config* cfg, int device, pi0_vision_ctx** out);
int pi0_vision_destroy(pi0_vision_ctx* ctx);
const char* pi0_vision_last_error(const pi0_vision_ctx* ctx);
/* The vision engine's packed-parameter table (Pi0Model(include={"vision"}).named_params, creation
 * order of siglip.py:92-102): 3 + 16·layers + 4 entries, every one in the model dtype. */
int pi0_vision_num_params(const pi0_vision_ctx* ctx);
int pi0_vision_param_info(const pi0_vision_ctx* ctx, int i, const char** name, int* ndim,
                          int64_t shape[2], int* dtype);
int pi0_vision_set_params(pi0_vision_ctx* ctx, const void* const* params, int n,
                          pi0_stream_t stream);
/* vm["embed_image"] for n ≤ max_images images at once (the reference runs one image per call);
 * replayed as one CUDA graph per (n, image, out). image 2-byte and out 4-byte aligned. */
int pi0_embed_image(pi0_vision_ctx* ctx, int n_images, const void* image, void* out,
                    pi0_stream_t stream);
int64_t pi0_vision_launch_count(const pi0_vision_ctx* ctx);
int pi0_vision_device_error(pi0_vision_ctx* ctx);
/* pi0_profile_enable / pi0_profile_read for a vision context (families "vision.*"). */
int pi0_vision_profile_enable(pi0_vision_ctx* ctx, int on);
int pi0_vision_profile_read(pi0_vision_ctx* ctx, int n_families, int64_t* launches,
                            double* total_ms);

/* ---- building block and measurement hooks (no counterpart in the reference) --------------- */

/* y[M, N] = x[M, K] · w[N, K]^T in the context's model dtype (fp32 accumulation, one rounding):
 * the GEMM engine every projection of the path runs on, exposed for direct tests. engine: 0 =
 * automatic, 1 = tcgen05 tiles (M >= 128), 2 = warp-level mma, 3 = tcgen05 weight-streaming
 * split-K (M <= 128), 4 = tcgen05 128×256 tiles split over K between two CTAs of a cluster
 * (M >= 128, K > 64), 5 = tcgen05 256×256 tiles on a CTA pair (cta_group::2). Other engine
 * numbers: PI0_ERR_INVALID. */
int pi0_linear(pi0_ctx* ctx, const void* x, int M, int K, const void* w, int N, void* y,
               int engine, pi0_stream_t stream);

/* Allocation-free, context-free variant of pi0_linear's warp-level engine (engine 2); no
 * counterpart in the reference. For callers that must not allocate device memory after start-up
 * and may hold no pi0 context at all: a control loop with a fixed memory budget, or an embedder
 * that owns every allocation itself. Same arguments as pi0_linear plus the model dtype
 * (PI0_F16 / PI0_BF16); K must be a multiple of 32, N even, x and w 16-byte aligned and y 4-byte
 * aligned (PI0_ERR_INVALID otherwise; an out-of-range device index gives PI0_ERR_UNSUPPORTED).
 * It always uses the engine's small-M tiling (64 × 64 tiles, split over K), which for M < 256 is
 * exactly what pi0_linear's engine 2 runs; for M >= 256 engine 2 switches to 128 × 128 tiles
 * without a split, so the two then agree within rounding, not bit for bit.
 * The split-K partials and tile tickets live in static device memory of this library (4 MiB of
 * fp32 partials, 4096 tiles). The first call on a device looks up their addresses and the SM
 * count with that device current; with CUDA's lazy module loading (the default) that first call,
 * and the first call of each dtype, may also load this library's kernels and static arrays into
 * device memory. Make one call of each dtype you use at start-up, before any stream capture;
 * later calls allocate nothing. Returns PI0_ERR_UNSUPPORTED when a call would need more scratch
 * than that (splits·M·N > 2^20 floats or more than 4096 output tiles). The tickets must be zero
 * between calls: static memory starts zeroed and every call that runs alone leaves them zero.
 * The scratch is shared by all calls on a device, so calls that overlap in time (two streams or
 * two threads) race on it and must be serialised by the caller; one overlap can leave a ticket
 * nonzero, after which later calls on that device give wrong results for the rest of the
 * process. */
int pi0_linear_noalloc(int dtype, const void* x, int M, int K, const void* w, int N, void* y,
                       pi0_stream_t stream);

/* Reads and clears the device error flag (synchronises the context's device). Nonzero means a
 * bounded wait inside a kernel gave up. */
int pi0_device_error(pi0_ctx* ctx);

/* Bounded-wait check (no counterpart in the reference): one device thread waits on a barrier
 * phase with the bounded wait all kernels here use. The phase completes only when `arrive` is
 * nonzero; otherwise the wait gives up after about one second, stores 3 (timeout) into the
 * device int *err if it is still 0, and the kernel returns, leaving the context usable. Lets
 * tests exercise the failure path without faulting or hanging a GPU. Context-free. */
int pi0_wait_check(int* err, int arrive, pi0_stream_t stream);

/* out[i] = a[i] / b[i] (fp32, n elements, device pointers) computed by the reciprocal-and-
 * correction sequence the norm-fused projections use for x / sqrt(mean(x²) + eps); exposed so
 * tests can compare it with IEEE division bit for bit. Context-free. */
int pi0_div_check(const float* a, const float* b, float* out, int64_t n, pi0_stream_t stream);


/* Kernels this context has launched so far (a replayed graph counts its kernel nodes). */
int64_t pi0_launch_count(const pi0_ctx* ctx);

/* While enabled, every kernel launch is bracketed by CUDA events, and each call is captured into
 * a one-shot graph, replayed and synchronised, so per-kernel-family device times (without host
 * launch gaps) can be read back. Enabling clears earlier records. */
int pi0_profile_enable(pi0_ctx* ctx, int on);
/* Synchronises the recorded events and returns, per kernel family (index < pi0_profile_families),
 * its launch count and total device milliseconds. */
int pi0_profile_read(pi0_ctx* ctx, int n_families, int64_t* launches, double* total_ms);
int pi0_profile_families(void);
const char* pi0_profile_family_name(int family);

#ifdef __cplusplus
}
#endif
#endif /* PI0B200_H_ */
