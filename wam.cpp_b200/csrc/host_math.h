// Host-side arithmetic of the action-chunk path (no device code): flow-match
// schedule, timestep embedding, visual positions, state normalisation and
// action post-processing.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace wamb {

// make_flow_match_euler_schedule (src/models/common/scheduler.cpp:26-55).
void flow_schedule(int steps, float shift, std::vector<float>* timesteps,
                   std::vector<float>* sigmas);
// timestep_embedding (src/models/gwp05/engine/text_encoder.cpp:1-12).
void timestep_embedding(float t, int dim, float* out);
// RoPE NORMAL inverse frequencies theta_scale^i, theta_scale = base^(-2/n_dims)
// (ggml_rope_ext as called by apply_rope_1d / apply_visual_rope,
// src/models/gwp05/engine/mot.cpp:175-202). mode 1: the 1-D action rope over
// 128 dims, out[0..63]; mode 2: the three visual sections 44/42/42 at
// out[0..21], out[22..42], out[43..63].
void rope_inv_freq(int mode, float* out64);
// visual_positions (src/models/gwp05/semantics.cpp:235-257), [gh*gw][3] = (t, h, w).
void visual_positions(int gh, int gw, int* thw);
// validate_prompt_mask (src/models/gwp05/engine/text_encoder.cpp:74-109) plus
// the token-count check of run_t5 (:117-121): the number of valid (leading)
// tokens of a prompt, or -1 with the reason.
int t5_valid_tokens(int n_lang, const int32_t* mask, int mask_n, int max_tokens, std::string* why);
// State normalisation (engine.cpp:249-253, semantics.cpp:154-172): the first
// n values map to [-1, 1] by the q01/q99 statistics, the rest of the padded
// vector is zero.
void normalize_state(const float* state, int n, int padded, const float* q01, const float* q99,
                     float* out);
// De-normalisation + delta actions (engine.cpp:436-445, semantics.cpp:178-208).
void postprocess_action(const float* action, int steps, int padded, int real, const float* q01,
                        const float* q99, const float* raw_state, float* out);

}  // namespace wamb
