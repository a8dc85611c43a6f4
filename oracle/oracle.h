/*
 * CPU oracle for the GWP-0.5 MoT forward pass — TEST INFRASTRUCTURE ONLY.
 *
 * A plain C++/OpenMP restatement of the reference's BF16 latency path
 * (GigaAI-research/wam.cpp, src/models/gwp05/engine/{mot,cache,weights,
 * text_encoder,engine}.cpp, src/models/common/scheduler.cpp,
 * src/models/gwp05/semantics.cpp). Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs load it, always as the checker
 * or the timed CPU baseline, never as part of the product path.
 *
 * Parity status: the reference's tensor arithmetic lives in the un-vendored
 * llama.cpp b9866 ggml, which cannot be built here, so the tensor math is
 * "parity unpinned" (restated from the reference's call sites and op
 * definitions). The host-side schedule, positions and state/action
 * (de)normalisation are pinned against the reference's own scheduler.cpp and
 * semantics.cpp compiled from source (oracle/Makefile, target ref).
 */
#ifndef WAM_ORACLE_H
#define WAM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oracle_geometry {
  int hidden;          /* H = heads * 128 (visual expert width, attention width) */
  int layers;          /* L */
  int heads;           /* H / 128 */
  int ffn;             /* visual expert FFN width */
  int action_hidden;   /* E */
  int action_ffn;      /* action expert FFN width */
  int action_dim;      /* padded action/state dim A */
  int real_state_dim;
  int real_action_dim;
  int num_embodiments;
  int embodiment_id;
  int grid_h, grid_w;  /* visual token grid; latent is [vae_z, 2 grid_h, 2 grid_w] */
  int vae_z;
  int action_chunk;    /* T */
  int steps;           /* S */
  int prompt_tokens;   /* N_t (cross-attention keys) */
  int text_dim;        /* D */
  float norm_eps;
  float flow_shift;
} oracle_geometry;

/* Creates a model over BF16 tensors given by compact GGUF name
 * (gwp.blk.<l>.<a|v>.sa.qkv.weight ...). Data is copied. Returns NULL and
 * writes err on failure. */
void* oracle_create(const oracle_geometry* g, int n_tensors, const char** names,
                    const uint16_t** data, const int64_t* numel, const float* state_q01,
                    const float* state_q99, const float* action_q01, const float* action_q99,
                    char* err, int errlen);
/* Model over the deterministic synthetic weights of oracle/synth.py (same bits),
 * generated in C++ for full-width CPU baselines. */
void* oracle_create_synthetic(const oracle_geometry* g, uint64_t seed, double bias_scale,
                              char* err, int errlen);
/* The same with a config-1 FFN variant: ffn_kind 0 GELU(tanh) (the
 * reference), 1 SiLU-gated (ffn.in weights hold [gate rows; up rows], 2F x W). */
void* oracle_create_synthetic_ex(const oracle_geometry* g, uint64_t seed, double bias_scale,
                                 int ffn_kind, char* err, int errlen);
void oracle_destroy(void* model);
/* Config 1: one MoT layer (layer 0) of the un-cached forward over given hidden
 * states. xv [V][H] visual tokens, xa [1 + T][E] state token then action
 * tokens, tv [Nt][H] / ta [Nt][E] text hidden states of the visual / action
 * experts, t the action tokens' timestep (the state token and the visual
 * tokens run at 0). norm_kind 0 LayerNorm inside AdaLN (the reference),
 * 1 RMSNorm. Outputs ov [V][H], oa [1 + T][E]. */
int oracle_block(void* model, int norm_kind, float t, const float* xv, const float* xa,
                 const float* tv, const float* ta, float* ov, float* oa);
/* Config-5 policy: replaces every linear weight whose rows are whole 32-value
 * blocks by its exact F32 Q8_0 dequantisation (no BF16 rounding of q * d). */
int oracle_quantize_q8(void* model);
/* GGML Q8_0 quantise + dequantise of n BF16 values (n % 32 == 0) into F32. */
void oracle_q8_roundtrip(const uint16_t* bf16, int64_t n, float* out);
/* uncached != 0: recompute the prefix at every step, as the reference's CPU
 * backend does (engine.cpp:334-337). Results are identical; only time differs. */
void oracle_set_uncached(void* model, int uncached);

/* One request. state: [real_state_dim] raw; latent: [vae_z][2gh][2gw];
 * prompt: [prompt_tokens][text_dim] (zero-padded by the caller);
 * noise: [T][A]. action_out: [T][real_action_dim].
 * Optional dumps (NULL to skip), element (layer, head, row, d):
 *   prefix_k / prefix_v: [L][heads][1 + V][128] after RoPE, BF16-rounded;
 *   prompt_k / prompt_v: [L][heads][N_t][128];
 *   velocity: [S][T][A] decoder outputs; actions: [S][T][A] Euler outputs. */
int oracle_predict(void* model, const float* state, const float* latent, const float* prompt,
                   const float* noise, float* action_out, float* prefix_k, float* prefix_v,
                   float* prompt_k, float* prompt_v, float* velocity, float* actions);

/* Flow-match Euler schedule: timesteps [steps], sigmas [steps + 1]. */
void oracle_schedule(int steps, float shift, float* timesteps, float* sigmas);
/* Sinusoidal timestep embedding [dim]: cos block then sin block. */
void oracle_timestep_embedding(float t, int dim, float* out);
/* Visual positions for a grid: time/height/width [gh * gw]. */
void oracle_visual_positions(int gh, int gw, int32_t* t, int32_t* h, int32_t* w);
/* Threads the oracle's parallel regions use. */
int oracle_threads(void);

/* Vision front-end stage 1 (vision.cpp): three views (format 0 U8 RGB, 1 F32
 * RGB in [0, 1]) composed onto an out_w x out_h canvas, patchified 2x2 into
 * out [12][out_h / 2][out_w / 2] in [-1, 1]. Returns non-zero on bad input. */
int oracle_compose_and_patchify(const void* const* data, const int* w, const int* h,
                                const int* format, int out_w, int out_h, float* out);

/* Vision front-end stage 2 (vae.cpp): the Wan VAE encoder on pixels
 * [12][height / 2][width / 2] (stage 1 output) with BF16 weights given by
 * compact name; latent [z][height / 16][width / 16]. With `stage` naming an
 * intermediate ("conv_in", "down0".."down3", "mid", "moments") its NHWC values
 * go to stage_out and its (h, w, c) to stage_dims. Returns non-zero on bad
 * input (2: a tensor is missing). */
/* UMT5 encoder (t5.cpp) over n valid tokens with BF16 weights by compact name;
 * out [max_tokens][hidden] (rows >= n zero). Non-zero on bad input. */
int oracle_t5_encode(const char* const* names, const uint16_t* const* tensors, int n_tensors,
                     int hidden, int heads, int head_dim, int ffn, int layers, int vocab,
                     const int32_t* tokens, int n, int max_tokens, float* out);

int oracle_vae_encode(const char* const* names, const uint16_t* const* tensors, int n_tensors,
                      const float* mean, const float* stdv, int z, const float* pixels, int width,
                      int height, float* latent, const char* stage, float* stage_out,
                      int* stage_dims);

#ifdef __cplusplus
}
#endif

#endif
