/*
 * wam_b200 — C ABI of the B200-native GWP-0.5 Mixture-of-Transformers engine.
 *
 * The engine replaces the reference's ggml execution engine behind
 * wam::internal::gwp05::engine::Engine (src/models/gwp05/engine/engine.h:142-155,
 * factory engine::create at engine.h:202-203). Every entry point returns 0 on
 * success and a non-zero wam_b200_error code on failure; engine entry points also
 * fill an optional wam_b200_status whose message is malloc'd and released by
 * wam_b200_status_free (the convention of the reference's C ABI,
 * src/serving/c_api.cpp:18-55). wam_b200_last_error() returns the calling
 * thread's last message for the op-level entry points.
 *
 * The op-level entry points (wam_b200_op_*) take DEVICE pointers and a CUDA
 * stream (cudaStream_t passed as void*); they exist so that each kernel of the
 * path can be checked against a CPU restatement on identical inputs. They run
 * only on an sm_100a device and never fall back to another implementation.
 */
#ifndef WAM_B200_H
#define WAM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WAM_B200_ABI_VERSION 2u

#if defined(__GNUC__)
#define WAM_B200_API __attribute__((visibility("default")))
#else
#define WAM_B200_API
#endif

enum wam_b200_error {
  WAM_B200_OK = 0,
  WAM_B200_INVALID_ARGUMENT = 1,
  WAM_B200_CUDA_ERROR = 2,
  WAM_B200_UNSUPPORTED = 3,
  WAM_B200_ARTIFACT_ERROR = 4,
  WAM_B200_INFERENCE_FAILED = 5,
  WAM_B200_DEVICE_TIMEOUT = 6
};

/* ABI version of this library (WAM_B200_ABI_VERSION at build time). */
WAM_B200_API uint32_t wam_b200_abi_version(void);

/* Last error message of the calling thread ("" if none). */
WAM_B200_API const char* wam_b200_last_error(void);

/* ------------------------------------------------------------------ ops */

/* BF16 tcgen05 GEMM with fused epilogue (one linear layer).
 * y[m, n] = epilogue(sum_k x[m, k] * w[n, k]); x: [m, ldx] BF16, w: [n, k] BF16
 * (GGUF ne = {k, n}), out: [m, ldo] BF16 (F32 for epilogue 6).
 * epilogue: 0 bias, 1 bias+GELU(tanh), 2 bias+SiLU, 3 gated residual
 * (r + linear * gate), 4 residual (r + linear), 5 F32 accumulate + bias,
 * 6 raw F32 accumulator, 7 bias then GELU(tanh) of the rounded linear,
 * 8 bias then exact-erf GELU. Split-K partial tiles are reduced through
 * distributed shared memory inside a thread-block cluster when workspace is
 * NULL (1 to 8 splits), or through the caller's global workspace
 * (wam_b200_gemm_scratch_floats floats; counters zeroed before first use, the
 * kernel leaves them zero). force_splits <= 0 picks automatically. error:
 * device word receiving a non-zero code on a pipeline timeout. OR-ing
 * WAM_B200_GEMM_TILED_WEIGHTS into epilogue says w was written by
 * wam_b200_op_retile_weights (n a multiple of 256): each 256x64 weight tile is
 * then one contiguous 32 KB block fetched by a single bulk copy.
 * Replaces: linear / linear_with_activation / linear_gelu_with_activation
 * (src/models/gwp05/engine/weights.cpp:786-849) and gated_residual
 * (src/models/gwp05/engine/mot.cpp:161-173). */
WAM_B200_API int wam_b200_op_gemm(const void* x, int ldx, int m, const void* w, int n, int k,
                                  int epilogue, const void* bias, const float* gate,
                                  const void* residual, int ldr, void* out, int ldo,
                                  float* workspace, size_t workspace_floats, unsigned* counters,
                                  int counter_slots, unsigned* error, int force_splits,
                                  void* stream);

/* The same GEMM for callers that must not allocate device memory (no
 * counterpart in the reference). A robot control loop that calls the policy
 * every cycle cannot afford cudaMalloc/cudaFree (they may synchronize the device
 * and take unbounded time), and hosting frameworks that own the allocator may
 * forbid side allocations; wam_b200_op_gemm needs a caller-allocated workspace
 * for split-K, this entry point uses a fixed library-owned device array instead
 * (8 MiB of partials + 4096 tile counters, held on every GPU that loads the
 * library until exit) and calls no allocating routine. Shapes whose split-K
 * partials exceed it are rejected with WAM_B200_INVALID_ARGUMENT; unsplit and
 * persistent shapes need none of it, whatever their size. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make that
 * first call before any stream capture. All calls share the array: calls that
 * overlap on the GPU race and must be serialized by the caller. Arguments as
 * wam_b200_op_gemm, without the workspace and the error word (flags
 * WAM_B200_GEMM_TILED_WEIGHTS / _Q8_WEIGHTS / _PAIR accepted). */
WAM_B200_API int wam_b200_op_gemm_noalloc(const void* x, int ldx, int m, const void* w, int n,
                                          int k, int epilogue, const void* bias, const float* gate,
                                          const void* residual, int ldr, void* out, int ldo,
                                          int force_splits, void* stream);
/* Device error word of the last wam_b200_op_gemm_noalloc call on the current
 * device (0: no pipeline wait timed out; otherwise the code the kernel set).
 * Blocking: synchronises with that call through a device-to-host copy of one
 * word into *code. Allocates nothing. */
WAM_B200_API int wam_b200_op_gemm_noalloc_error(unsigned* code);

#define WAM_B200_GEMM_TILED_WEIGHTS 0x100
/* w holds Q8_0 weight tiles written by wam_b200_op_q8_retile (n % 256 == 0):
 * the GEMM streams 17 KB per 256 x 64 weight tile and converts it to BF16
 * (q * d rounded to BF16) in shared memory for the tensor cores. */
#define WAM_B200_GEMM_Q8_WEIGHTS 0x200
/* Run a GEMM of >= 256 token rows on CTA pairs (tcgen05.mma.cta_group::2: one
 * UMMA of 256 tokens x 256 features over two SMs, each holding 128 token rows
 * and 128 weight rows per k-block), split over 2 or 4 pairs of one cluster when
 * the output tiles are few and a workspace is given. BF16 weights only (row-major
 * or WAM_B200_GEMM_TILED_WEIGHTS); ignored with force_splits > 0 or Q8_0
 * weights. Without the flag, wam_b200_op_gemm and the engine choose CTA pairs
 * by themselves for GEMMs of >= 256 rows whose 256 x 256 tiles occupy at least
 * half of the GPU's resident pairs; the environment variable WAM_B200_GEMM_PAIR
 * set at load to 1 (every GEMM of >= 256 rows) or 0 (only where the flag asks)
 * overrides that choice. */
#define WAM_B200_GEMM_PAIR 0x400

/* Quantises n_elems BF16 weights (n_elems % 32 == 0, row-major [n][k]) to GGML
 * Q8_0 blocks (34 bytes per 32 values: fp16 scale d, 32 int8 q; value q * d)
 * with the gguf-py quantiser's rules: d = max|x| / 127 in F32, q = x * (1/d)
 * rounded half away from zero, d rounded to fp16. No counterpart in the
 * reference, whose artifacts are BF16/F32 only (src/models/gwp05/artifact.cpp:
 * 129-133); this is the Q8_0 policy of the build's config 5. */
WAM_B200_API int wam_b200_op_q8_quantize(const void* w, long long n_elems, void* blocks,
                                         void* stream);

/* Re-tiles row-major Q8_0 blocks of an [n][k] weight (n % 256 == 0, k % 64 ==
 * 0; the GGUF layout of a Q8_0 tensor with ne = {k, n}) into GEMM tiles
 * [n/256][k/64] of 17408 bytes: int8 [256][64], then fp16 scales [256][2]. */
WAM_B200_API int wam_b200_op_q8_retile(const void* blocks, void* tiles, int n, int k, void* stream);

/* Re-tiles a row-major BF16 weight w[n][k] (n % 256 == 0, k % 64 == 0, the
 * GGUF ne = {k, n} layout) into dst as contiguous 32 KB tiles
 * [n/256][k/64][256][64] with the tensor cores' 128-byte shared-memory swizzle
 * pre-applied (16-byte chunk c of tile row r stored at chunk c ^ (r % 8)). src
 * and dst must not overlap. No counterpart in the reference, which keeps GGUF's
 * row-major layout (src/models/gwp05/engine/weights.cpp:702-770 loads tensors
 * as stored); the engine applies it to every GEMM weight at load time. */
WAM_B200_API int wam_b200_op_retile_weights(const void* src, void* dst, int n, int k, void* stream);

/* Split-K scratch (floats) and output-tile count wam_b200_op_gemm needs for a shape. */
WAM_B200_API size_t wam_b200_gemm_scratch_floats(int m, int n, int k, int force_splits,
                                                 int* tiles_out);

/* Flash attention softmax(scale Q K^T) V over head-major BF16 tensors:
 * element (seq, head, row, d) of q at q[seq*q_seq_stride + head*q_head_stride +
 * row*128 + d], k/v likewise with kv strides; out row r of seq b at
 * out[(b*lq + r)*ldo + head*128 + d]. Replaces the cached joint attention
 * (src/models/gwp05/engine/mot.cpp:432-446) and cross attention (:299-321). */
WAM_B200_API int wam_b200_op_attention(const void* q, long long q_seq_stride,
                                       long long q_head_stride, const void* k, const void* v,
                                       long long kv_seq_stride, long long kv_head_stride, int lq,
                                       int lk, int heads, int batch, float scale, void* out,
                                       int ldo, void* stream);

/* LayerNorm + AdaLN modulation y = bf16(LN(x)(1 + scale) + shift) with F32
 * scale/shift (modulated_norm, mot.cpp:147-159) when affine == 0; affine
 * LayerNorm y = bf16(LN(x) w + b) with BF16 w/b (layer_norm, weights.cpp:919-930)
 * when affine != 0. */
WAM_B200_API int wam_b200_op_layernorm(const void* x, int rows, int cols, const void* a,
                                       const void* b, float eps, int affine, void* y,
                                       void* stream);

/* Q/K/V post-processing of a packed QKV projection and its scatter into the
 * head-major K/V cache (expert_qkv's RMSNorm + RoPE + cast, src/models/gwp05/
 * engine/mot.cpp:210-267, and the prefix cache write of engine/cache.cpp:
 * 441-469, in this engine's layout). For token row r (sequence b = r /
 * rows_per_seq, row i = r % rows_per_seq in it) and part x in {q, k, v} with a
 * source column >= 0: optional RMSNorm over the whole hidden width (F32,
 * x * rsqrt(mean(x^2) + eps) * norm; v is never normalised), optional RoPE
 * NORMAL on pairs (2j, 2j+1) at 1-D position pos_base + i (rope_mode 1) or at the
 * 3-D position pos_thw[i] = (t, h, w) over sections 44/42/42 (rope_mode 2;
 * v never roped), cast to BF16, and element (head, d) stored at
 *   q: q_out[b*q_seq_stride + head*q_head_stride + (q_row_offset + i)*128 + d]
 *   k/v: k_out/v_out[b*kv_seq_stride + head*kv_head_stride + (kv_row_offset + i)*128 + d].
 * The engine's cache is [heads][prefix rows + action rows][128] per request and
 * layer: row 0 the state token, rows 1..V the visual tokens, rows P..P+T-1 the
 * action tokens. inv_freq: a device copy of wam_b200_rope_inv_freq(rope_mode).
 * All pointers are device pointers; pos_thw is int32 [rows_per_seq][3]. */
typedef struct wam_b200_qkv_scatter_args {
  const void* src; /* BF16 [rows][ld_src] */
  int ld_src, rows, rows_per_seq, heads;
  int q_col, k_col, v_col; /* first source column of each part, -1 to skip it */
  const void* q_norm;      /* BF16 [heads*128] or NULL (no RMSNorm) */
  const void* k_norm;
  float eps;
  int rope_mode, pos_base;
  const int* pos_thw;
  const float* inv_freq;
  void* q_out;
  long long q_seq_stride, q_head_stride;
  int q_row_offset;
  void* k_out;
  void* v_out;
  long long kv_seq_stride, kv_head_stride;
  int kv_row_offset;
} wam_b200_qkv_scatter_args;
WAM_B200_API int wam_b200_op_qkv_scatter(const wam_b200_qkv_scatter_args* args, void* stream);
/* RoPE inverse frequencies [64] (mode 1: 1-D over 128 dims; mode 2: visual
 * sections 44/42/42 at [0..21], [22..42], [43..63]), as the engine uploads them
 * (ggml_rope_ext NORMAL, theta_scale = 10000^(-2/n_dims); mot.cpp:175-202). */
WAM_B200_API int wam_b200_rope_inv_freq(int mode, float* out64);

/* Deterministic synthetic BF16 tensor (the generator behind synthetic weights):
 * w[i] = bf16(f32(z_i) * f32(scale / sd) + f32(center)), z_i the Irwin-Hall(4)
 * sum of the 16-bit lanes of splitmix64(tensor_seed + (i + 1) * golden) minus
 * its mean. No reference counterpart (the reference loads trained weights). */
WAM_B200_API int wam_b200_op_synth(void* w, long long n, uint64_t tensor_seed, double scale,
                                   double center, void* stream);
/* Seed of a synthetic tensor: splitmix64(seed ^ fnv1a64(name)). */
WAM_B200_API uint64_t wam_b200_tensor_seed(uint64_t seed, const char* name);

/* ------------------------------------------------- host-side arithmetic */

/* Flow-match Euler schedule: timesteps [steps], sigmas [steps + 1]
 * (make_flow_match_euler_schedule, src/models/common/scheduler.cpp:26-55). */
WAM_B200_API int wam_b200_flow_schedule(int steps, float shift, float* timesteps, float* sigmas);
/* Visual RoPE positions [gh * gw][3] = (t, h, w) (visual_positions,
 * src/models/gwp05/semantics.cpp:235-257). */
WAM_B200_API int wam_b200_visual_positions(int gh, int gw, int* thw);
/* State normalisation to [-1, 1], zero-padded to `padded` (engine.cpp:249-253,
 * normalize_and_pad_state, semantics.cpp:154-172). */
WAM_B200_API int wam_b200_normalize_state(const float* state, int n, int padded, const float* q01,
                                          const float* q99, float* out);
/* Action de-normalisation plus delta dims 0-5 and 7-12 (engine.cpp:436-445,
 * postprocess_action, semantics.cpp:178-208): out [steps][real]. */
WAM_B200_API int wam_b200_postprocess_action(const float* action, int steps, int padded, int real,
                                             const float* q01, const float* q99,
                                             const float* raw_state, float* out);

/* --------------------------------------------------------------- engine */

typedef struct wam_b200_engine wam_b200_engine;

/* Error detail of an engine call; message is malloc'd (free with
 * wam_b200_status_free). Mirrors wam_rpc_result (src/serving/c_api.cpp:18-55). */
typedef struct wam_b200_status {
  int code;
  char* message;
} wam_b200_status;

/* Model geometry (the gwp05.* GGUF keys, src/models/gwp05/artifact.cpp:20-94),
 * plus prompt_tokens = cross-attention text length (the reference fixes it at
 * 64, src/models/gwp05/semantics.h:11) and text_dim = gwp05.t5_hidden. */
typedef struct wam_b200_geometry {
  int hidden, layers, heads, ffn, action_hidden, action_ffn, action_dim;
  int real_state_dim, real_action_dim, num_embodiments, embodiment_id;
  int grid_h, grid_w, vae_z, action_chunk, steps, prompt_tokens, text_dim;
  float norm_eps, flow_shift;
} wam_b200_geometry;

/* Engine options (struct_size-versioned like wam_rpc_model_options_v2,
 * include/wam/c_api.h). With artifact_path NULL the engine generates
 * deterministic synthetic weights from (synthetic_geometry, synthetic_seed). */
typedef struct wam_b200_options {
  uint32_t struct_size;
  const char* artifact_path;
  wam_b200_geometry synthetic_geometry;
  uint64_t synthetic_seed;
  float synthetic_bias_scale;
  int device_index;
  int max_batch;
  int use_cuda_graphs;
  int prompt_cache; /* reuse projected prompt K/V for an identical prompt */
  /* Added after the first layout (read only when struct_size covers it):
   * 0 BF16 weights; 1 Q8_0 linear weights (config 5: synthetic weights are
   * quantised on the device with the gguf-py Q8_0 rules; a GGUF artifact may
   * hold Q8_0 tensors). Linear layers then compute with q * d rounded to BF16. */
  int weight_format;
  /* Added with the single-block entry (read only when struct_size covers them).
   * ffn_kind: 0 GELU(tanh) FFN (the reference, mot.cpp:341-346), 1 SiLU-gated
   * FFN silu(x Wg + bg) * (x Wu + bu) with ffn.in holding [gate rows; up rows]
   * (2F x W); norm_kind: 0 LayerNorm inside the AdaLN modulated norms (the
   * reference, mot.cpp:147-159), 1 RMSNorm; block_mode != 0 creates an engine
   * for wam_b200_block_forward (synthetic weights, layers == 1, steps == 1,
   * max_batch == 1, prompt_cache == 0). The variants are BASELINE config 1's
   * literal block ("RMSNorm + AdaLN, SiLU-gated MLP"); synthetic weights only. */
  int ffn_kind;
  int norm_kind;
  int block_mode;
  /* Added with the vision front-end: 1 loads the Wan VAE encoder (the vae.*
   * tensors and gwp05.vae_latents_{mean,std} of the artifact, or synthetic
   * weights from synthetic_seed) so that requests may carry camera images. */
  int vae;
  /* 1 loads the UMT5 text encoder (the t5.* tensors and gwp05.t5_* geometry of
   * the artifact; synthetic: hidden = text_dim, 64-dim heads, max tokens =
   * prompt_tokens and the three sizes below) so that requests may carry prompt
   * token ids (the reference's resident language-encoder policy). */
  int t5;
  int t5_vocab, t5_ffn, t5_layers;
} wam_b200_options;

/* A camera view (ImageView, src/models/gwp05/engine/engine.h:82-89): host (or,
 * for wam_b200_op_preprocess, device) pixels, HWC RGB. */
#define WAM_B200_PIXEL_U8 0         /* 3 bytes per pixel (PixelFormat::U8) */
#define WAM_B200_PIXEL_F32_RGB_01 1 /* 3 floats per pixel in [0, 1] */
typedef struct wam_b200_image {
  const void* data;
  int w;
  int h;
  int format;
} wam_b200_image;

/* One request (EngineInputsView, src/models/gwp05/engine/engine.h:91-105, with
 * the precomputed prompt embedding the external_embedding policy uses, and
 * either the precomputed VAE latent or the three camera views). Host pointers,
 * borrowed for the call. */
typedef struct wam_b200_request {
  const float* state;      /* [state_n >= real_state_dim], un-normalised */
  int state_n;
  const float* noise;      /* [action_chunk * action_dim] or NULL (engine RNG) */
  const float* ref_latent; /* [vae_z * 2 grid_h * 2 grid_w] */
  long long ref_latent_n;
  const float* prompt_emb; /* [prompt_tokens_in * text_dim], zero-padded to prompt_tokens */
  int prompt_tokens;
  /* ABI 2: with ref_latent NULL, the views [n_images == 3] run the vision
   * front-end on the device (compose + VAE encoder, as run_vae, engine/
   * vae.cpp:279-388, when the reference gets no precomputed latent,
   * engine.cpp:260-270); needs an engine created with vae = 1. */
  const wam_b200_image* images;
  int n_images;
  /* ABI 2: with prompt_emb NULL, the prompt token ids [n_lang] (and optional
   * attention mask [attention_mask_n], a contiguous valid prefix of ones) run
   * the UMT5 encoder on the device (run_t5, engine/text_encoder.cpp:112-204);
   * needs an engine created with t5 = 1. */
  const int32_t* lang_tokens;
  int n_lang;
  const int32_t* attention_mask;
  int attention_mask_n;
} wam_b200_request;

typedef struct wam_b200_stats {
  float ms_total;
  float ms_device; /* prompt projection + prefix + denoise on the device */
  int prompt_cache_hit;
  int kernel_launches;
  uint64_t resident_device_bytes;
} wam_b200_stats;

WAM_B200_API void wam_b200_status_free(wam_b200_status* status);

/* engine::create (src/models/gwp05/engine/engine.h:202-203, impl engine.cpp:99-228). */
WAM_B200_API int wam_b200_create(const wam_b200_options* options, wam_b200_engine** engine,
                                 wam_b200_status* status);
WAM_B200_API void wam_b200_destroy(wam_b200_engine* engine);
/* Engine::reset (engine.h:146): drops the projected-prompt cache. */
WAM_B200_API int wam_b200_reset(wam_b200_engine* engine);
WAM_B200_API int wam_b200_geometry_of(const wam_b200_engine* engine, wam_b200_geometry* out);

/* Engine::predict (engine.h:145, impl engine.cpp:230-449): one action chunk.
 * action_out: [action_chunk * real_action_dim] de-normalised actions. */
WAM_B200_API int wam_b200_predict(wam_b200_engine* engine, const wam_b200_request* request,
                                  float* action_out, size_t action_out_n, wam_b200_stats* stats,
                                  wam_b200_status* status);
/* Batched predict (no reference counterpart; the reference is batch 1):
 * action_out: [batch][action_chunk][real_action_dim]. */
WAM_B200_API int wam_b200_predict_batch(wam_b200_engine* engine, const wam_b200_request* requests,
                                        int batch, float* action_out, size_t action_out_n,
                                        wam_b200_stats* stats, wam_b200_status* status);

/* max_batch of the engine's options (requests per predict_batch). */
WAM_B200_API int wam_b200_max_batch(const wam_b200_engine* engine);

/* Batch-capable serving surface (no reference counterpart: the reference
 * serialises predicts on a per-model mutex, src/models/gwp05/model.cpp:61,
 * and reports Capabilities::batch_inference = false, include/wam/types.h:236-237).
 * Any number of threads call wam_b200_batcher_predict concurrently; a worker
 * thread runs the queued requests in arrival order as predict_batch calls of
 * up to max_batch, waiting at most max_wait_us after the first request for
 * more. A failing batch is retried request by request, so a bad request fails
 * alone. batch_size reports the batch a request rode in. The engine must not
 * be used directly while a batcher serves it. */
typedef struct wam_b200_batcher wam_b200_batcher;
WAM_B200_API int wam_b200_batcher_create(wam_b200_engine* engine, int max_wait_us,
                                         wam_b200_batcher** batcher, wam_b200_status* status);
/* Drains the queue, stops the worker (the engine stays alive). */
WAM_B200_API void wam_b200_batcher_destroy(wam_b200_batcher* batcher);
WAM_B200_API int wam_b200_batcher_predict(wam_b200_batcher* batcher, const wam_b200_request* request,
                                          float* action_out, size_t action_out_n,
                                          wam_b200_stats* stats, int* batch_size,
                                          wam_b200_status* status);
/* Batches run and requests served so far. */
WAM_B200_API int wam_b200_batcher_counts(wam_b200_batcher* batcher, long long* batches,
                                         long long* requests);

/* One MoT layer over given hidden states: the layer body
 * of the reference's un-cached forward, run_mot_step (src/models/gwp05/engine/
 * mot.cpp:1008-1067), for layer 0 of a block-mode engine. The action stream
 * [state token; action tokens] runs through the action expert (state token at
 * timestep 0, action tokens at `timestep`; action_timesteps with the clean
 * state, semantics.cpp:224-233), the visual tokens through the visual expert
 * at 0; one joint self-attention where state and visual queries see the state
 * and visual keys and action queries see every key (the mask built at
 * mot.cpp:1147-1158); then each expert's cross attention over its text hidden
 * states (projected and normalised by the layer) and its FFN. Host pointers:
 * visual [V][H], action [1 + T][E], text_visual [N_t][H], text_action
 * [N_t][E] (F32, used as BF16 hidden states); outputs likewise. */
typedef struct wam_b200_block_inputs {
  const float* visual;
  const float* action;
  const float* text_visual;
  const float* text_action;
  float timestep;
} wam_b200_block_inputs;
WAM_B200_API int wam_b200_block_forward(wam_b200_engine* engine, const wam_b200_block_inputs* in,
                                        float* visual_out, size_t visual_out_n, float* action_out,
                                        size_t action_out_n, float* device_ms,
                                        wam_b200_status* status);

/* Split form of predict_batch for device-resident timing: stage (host->device
 * inputs), run (enqueue prompt projection, prefix and denoise on the engine's
 * stream, no host sync), fetch (sync, device->host, de-normalise). */
WAM_B200_API int wam_b200_stage(wam_b200_engine* engine, const wam_b200_request* requests,
                                int batch, wam_b200_status* status);
WAM_B200_API int wam_b200_run(wam_b200_engine* engine, int batch, wam_b200_status* status);
WAM_B200_API int wam_b200_fetch(wam_b200_engine* engine, const wam_b200_request* requests,
                                int batch, float* action_out, size_t action_out_n,
                                wam_b200_status* status);
/* The engine's CUDA stream (cudaStream_t) for event timing. */
WAM_B200_API void* wam_b200_stream(wam_b200_engine* engine);
/* Kernels one chunk launches at this batch (with / without prompt projection). */
WAM_B200_API int wam_b200_kernel_launches(wam_b200_engine* engine, int batch, int with_prompt);
/* Device time (ms) of the phases of the last run/predict: prompt projection
 * (0 when the projected-prompt cache hit), prefix cache, denoise. */
WAM_B200_API int wam_b200_phase_ms(wam_b200_engine* engine, float* prompt_ms, float* prefix_ms,
                                   float* denoise_ms);

/* Per-kernel profile of one chunk on the staged batch: runs every op eagerly
 * between CUDA events and fills up to max_ops records (phase 0 prompt /
 * 1 prefix / 2 denoise; kind 0 GEMM, 1 attention, 2 layer norm, 3 q/k/v
 * norm+RoPE scatter, 4 small linear, 5 elementwise; ms; algorithmic bytes and
 * FLOPs). Returns the number of ops, or a negative error code. */
typedef struct wam_b200_op_profile {
  int phase, kind, launches;
  float ms;
  double bytes, flops;
  int shape[4]; /* GEMM: m, n, k, split-K factor (negative: CTA-pair kernel, -splits) */
} wam_b200_op_profile;
WAM_B200_API int wam_b200_profile(wam_b200_engine* engine, int batch, wam_b200_op_profile* out,
                                  int max_ops, wam_b200_status* status);

/* Device time of one (phase, kind) of the staged batch's chunk inside a CUDA
 * graph: the ops of that phase and kind (e.g. phase 2, kind 0 = every denoise
 * GEMM) captured alone, in issue order, with the same launches and buffers as
 * the chunk's graphs, replayed `reps` times between CUDA events after one
 * warm-up replay. ms = device time per replay; bytes / flops = the ops'
 * algorithmic HBM bytes / FLOPs per replay; launches = kernels per replay.
 * Leaves the engine's activations overwritten (the next run recomputes them). */
typedef struct wam_b200_graph_profile {
  float ms;
  double bytes, flops;
  int launches;
} wam_b200_graph_profile;
WAM_B200_API int wam_b200_profile_graph(wam_b200_engine* engine, int batch, int phase, int kind,
                                        int reps, wam_b200_graph_profile* out,
                                        wam_b200_status* status);
/* The same restricted to the ops of one lane of the phase (lane 0: the main
 * stream, e.g. the prefix's 768 visual tokens; lane 1: the side stream, e.g.
 * the prefix state token's action-expert work; -1: every lane). */
WAM_B200_API int wam_b200_profile_graph_lane(wam_b200_engine* engine, int batch, int phase,
                                             int kind, int lane, int reps,
                                             wam_b200_graph_profile* out,
                                             wam_b200_status* status);

/* Stage dumps as F32 (the reference's WAM_GWP05_CACHE_DUMP_DIR stages,
 * engine/cache.cpp:441-469): "prefix_k"/"prefix_v" [heads][1+V][128],
 * "prompt_k"/"prompt_v" [heads][prompt_tokens][128] of one layer,
 * "velocity" [steps][action_chunk][action_dim] (layer ignored). */
WAM_B200_API int wam_b200_read_tensor(wam_b200_engine* engine, const char* name, int slot,
                                      int layer, float* out, size_t out_n,
                                      wam_b200_status* status);

/* ---------------------------------------------------------------- vision
 * Stage 1 of the vision front-end: compose three camera views onto the
 * image_width x image_height canvas (view 0 top half, views 1 / 2 bottom left /
 * right; each resized to cover its cell with a triangle filter and centre
 * cropped), patchify 2x2 and map to [-1, 1]. Output [12][h/2][w/2] F32 on the
 * device, packed channel (c * 2 + dx) * 2 + dy. Bit-identical to the reference's
 * CPU compose_and_patchify (src/models/gwp05/engine/vae.cpp:1-134); replaces its
 * CUDA preprocessor (src/models/gwp05/kernels/cuda_preprocess.h:6-14). Views are
 * wam_b200_image (above). */
typedef struct wam_b200_preprocessor wam_b200_preprocessor;

/* gwp05_cuda_preprocessor_create / _destroy (cuda_preprocess.cu:139-148): device
 * buffers for the three views on device_index, grown on demand. */
WAM_B200_API int wam_b200_preprocessor_create(int device_index, wam_b200_preprocessor** out,
                                              wam_b200_status* status);
WAM_B200_API void wam_b200_preprocessor_destroy(wam_b200_preprocessor* preprocessor);
/* gwp05_cuda_preprocess (cuda_preprocess.cu:150-198): host images (exactly 3,
 * U8 or F32_RGB_01, w, h > 0), copied to the device on `stream` (NULL: the
 * legacy default stream), composed into output_device; returns after the stream
 * has finished. output_width / output_height must be positive and even. */
WAM_B200_API int wam_b200_preprocess(wam_b200_preprocessor* preprocessor,
                                     const wam_b200_image* images, int image_count,
                                     int output_width, int output_height, float* output_device,
                                     void* stream, wam_b200_status* status);
/* The same kernel on views already on the device (asynchronous on `stream`). */
WAM_B200_API int wam_b200_op_preprocess(const wam_b200_image* device_images, int output_width,
                                        int output_height, float* output_device, void* stream);

/* Implicit-GEMM convolution of the VAE encoder on NHWC BF16 activations of one
 * image ([in_h][in_w][cin], cin >= 64 and a multiple of 8): mode 0 = 3x3 stride 1 padding
 * 1, 1 = 3x3 stride 2 after a one-pixel zero pad at the right and bottom (the
 * downsampler, vae.cpp:211-214), 2 = 1x1. Output [out_h][out_w][cout] BF16
 * (cout a multiple of 16). epilogue 0: out = bf16(bf16(conv) + bias);
 * 4: out = bf16(residual + bf16(bf16(conv) + bias)) (vae_conv + ggml_add,
 * vae.cpp:141-160, 178-191). w_laid comes from wam_b200_op_conv_weight_layout
 * of the [cout][cin][kh][kw] weight: [wam_b200_conv_cout_pad(cout)][taps]
 * [wam_b200_conv_cin_pad(cin)], zero padded.
 * `error` is a device word the kernel sets on a timed-out wait. */
WAM_B200_API int wam_b200_conv_cin_pad(int cin);
WAM_B200_API int wam_b200_conv_cout_pad(int cout);
WAM_B200_API int wam_b200_op_conv_weight_layout(const void* src, void* dst, int cout, int cin,
                                                int taps, void* stream);
WAM_B200_API int wam_b200_op_conv2d(const void* x, int in_w, int in_h, int cin, int mode,
                                    const void* w_laid, int cout, int epilogue, const void* bias,
                                    const void* residual, void* out, unsigned* error,
                                    void* stream);

/* Stage 2 of the vision front-end: the Wan VAE encoder (single frame), the
 * reference's run_vae (src/models/gwp05/engine/vae.cpp:279-388) on the B200
 * as one captured CUDA graph of implicit-GEMM convolutions. Weights: the vae.*
 * tensors of a GGUF artifact (BF16, policy mot-vae-bf16*) with
 * gwp05.vae_latents_mean / _std, or deterministic synthetic ones
 * (artifact_path NULL). image_width / image_height: the canvas (multiples of
 * 32); the latent is [z_dim][H / 16][W / 16] F32, (posterior mode - mean) / std. */
typedef struct wam_b200_vae wam_b200_vae;
typedef struct wam_b200_vae_options {
  uint32_t struct_size; /* sizeof(wam_b200_vae_options) */
  const char* artifact_path;
  uint64_t synthetic_seed;
  int image_width;
  int image_height;
  int z_dim;
  int device_index;
  int use_cuda_graph;
} wam_b200_vae_options;
/* The encoder's tensors (82, the reference's compact GGUF names): name and
 * shape ([cout, cin, kh, kw] or [c]) of tensor `index`; returns the rank, or
 * -1 past the last tensor. Host only. */
WAM_B200_API int wam_b200_vae_tensor_spec(int z_dim, int index, char* name, size_t name_n,
                                          long long* shape4);
WAM_B200_API int wam_b200_vae_create(const wam_b200_vae_options* options, wam_b200_vae** vae,
                                     wam_b200_status* status);
WAM_B200_API void wam_b200_vae_destroy(wam_b200_vae* vae);
/* Floats of one latent, kernel launches of one encode, FLOPs of one encode. */
WAM_B200_API int wam_b200_vae_info(const wam_b200_vae* vae, int* latent_count, int* launches,
                                   double* flops);
/* run_vae with host images: preprocess (stage 1) + encoder; latent to host.
 * Synchronous. */
WAM_B200_API int wam_b200_vae_encode(wam_b200_vae* vae, const wam_b200_image* images,
                                     int image_count, float* latent, size_t latent_n,
                                     wam_b200_status* status);
/* Encoder only, device pointers: pixels [12][H/2][W/2] F32 (stage 1 output),
 * latent [z][H/16][W/16] F32; asynchronous on `stream` (NULL: the legacy
 * default stream). */
WAM_B200_API int wam_b200_vae_encode_device(wam_b200_vae* vae, const float* pixels,
                                            float* latent, void* stream,
                                            wam_b200_status* status);
/* F32 copy of an intermediate NHWC activation ("conv_in", "down0".."down3",
 * "mid", "moments") of the last encode, for parity checks. */
WAM_B200_API int wam_b200_vae_read_stage(wam_b200_vae* vae, const char* name, float* out,
                                         size_t n, int* h, int* w, int* c);

/* ---------------------------------------------------------------- UMT5
 * The UMT5 text encoder (the reference's run_t5, src/models/gwp05/engine/
 * text_encoder.cpp:112-204): prompt token ids -> prompt embedding
 * [max_tokens][hidden] F32 (rows past the valid prompt zero), the input of the
 * prompt projection when the language encoder is resident. Weights: the t5.*
 * tensors of a GGUF artifact (BF16; geometry from gwp05.t5_*), or synthetic
 * from synthetic_seed and the geometry below. */
typedef struct wam_b200_t5 wam_b200_t5;
typedef struct wam_b200_t5_options {
  uint32_t struct_size; /* sizeof(wam_b200_t5_options) */
  const char* artifact_path;
  uint64_t synthetic_seed;
  int vocab, hidden, ffn, heads, head_dim, layers; /* synthetic geometry (head_dim 64) */
  int max_tokens;                                  /* n_lang (semantics: 512 at config 2) */
  int device_index;
  int use_cuda_graphs;
} wam_b200_t5_options;
WAM_B200_API int wam_b200_t5_create(const wam_b200_t5_options* options, wam_b200_t5** t5,
                                    wam_b200_status* status);
WAM_B200_API void wam_b200_t5_destroy(wam_b200_t5* t5);
/* Geometry actually loaded (from the artifact when one is given). */
WAM_B200_API int wam_b200_t5_geometry(const wam_b200_t5* t5, int* vocab, int* hidden, int* ffn,
                                      int* heads, int* layers, int* max_tokens);
/* run_t5 with the reference's input checks (validate_prompt_mask,
 * text_encoder.cpp:74-109): tokens [n_lang] with 1 <= n_lang <= max_tokens,
 * optional mask [mask_n == n_lang] of 0/1 forming a contiguous valid prefix;
 * the valid prefix is encoded. out: host [max_tokens * hidden]. Synchronous. */
WAM_B200_API int wam_b200_t5_encode(wam_b200_t5* t5, const int32_t* tokens, int n_lang,
                                    const int32_t* mask, int mask_n, float* out, size_t out_n,
                                    wam_b200_status* status);
/* The same into device memory, asynchronous on `stream` (NULL: the legacy
 * default stream). */
WAM_B200_API int wam_b200_t5_encode_device(wam_b200_t5* t5, const int32_t* tokens, int n_lang,
                                           const int32_t* mask, int mask_n, float* out_device,
                                           void* stream, wam_b200_status* status);
/* FLOPs and kernel launches of one encode of n valid tokens. */
WAM_B200_API int wam_b200_t5_info(wam_b200_t5* t5, int n, double* flops, int* launches);
/* relative_position_bucket (text_encoder.cpp:14-24), for parity checks. */
WAM_B200_API int wam_b200_t5_relative_bucket(int relative, int buckets, int max_distance);

#ifdef __cplusplus
}
#endif

#endif /* WAM_B200_H */
