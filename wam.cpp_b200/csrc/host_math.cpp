#include "host_math.h"

#include <algorithm>
#include <cmath>

#include "wam_b200.h"

namespace wamb {

void flow_schedule(int steps, float shift, std::vector<float>* ts, std::vector<float>* sig) {
  ts->assign(steps, 0.0f);
  sig->assign(steps + 1, 0.0f);
  // The endpoint comes from the F32 training schedule; linspace and the shift
  // transform run in F64, then round to F32.
  const float training_sigma = 1.0f / 1000.0f;
  const float smin = shift * training_sigma / (1.0f + (shift - 1.0f) * training_sigma);
  const double tmin = static_cast<double>(smin) * 1000.0;
  for (int s = 0; s < steps; ++s) {
    const double u = steps == 1 ? 1000.0 : 1000.0 + (tmin - 1000.0) * s / (steps - 1);
    const double sigma = u / 1000.0;
    const double sh =
        static_cast<double>(shift) * sigma / (1.0 + (static_cast<double>(shift) - 1.0) * sigma);
    (*sig)[s] = static_cast<float>(sh);
    (*ts)[s] = (*sig)[s] * 1000.0f;
  }
  (*sig)[steps] = 0.0f;
}

void timestep_embedding(float t, int dim, float* out) {
  const int half = dim / 2;
  for (int i = 0; i < half; ++i) {
    const float f =
        std::exp(-std::log(10000.0f) * static_cast<float>(i) / static_cast<float>(half));
    const float v = t * f;
    out[i] = std::cos(v);
    out[i + half] = std::sin(v);
  }
}

void rope_inv_freq(int mode, float* out) {
  for (int i = 0; i < 64; ++i) out[i] = 0.0f;
  if (mode == 1) {
    const float ts = std::pow(10000.0f, -2.0f / 128.0f);
    for (int i = 0; i < 64; ++i) out[i] = std::pow(ts, static_cast<float>(i));
    return;
  }
  const int sec[3] = {44, 42, 42}, base[3] = {0, 22, 43};
  for (int k = 0; k < 3; ++k) {
    const float t3 = std::pow(10000.0f, -2.0f / static_cast<float>(sec[k]));
    for (int i = 0; i < sec[k] / 2; ++i) out[base[k] + i] = std::pow(t3, static_cast<float>(i));
  }
}

void visual_positions(int gh, int gw, int* thw) {
  for (int y = 0; y < gh; ++y)
    for (int x = 0; x < gw; ++x) {
      const int t = y * gw + x;
      thw[t * 3 + 0] = 0;
      thw[t * 3 + 1] = y;
      thw[t * 3 + 2] = x;
    }
}

void normalize_state(const float* state, int n, int padded, const float* q01, const float* q99,
                     float* out) {
  for (int d = 0; d < padded; ++d) out[d] = 0.0f;
  for (int d = 0; d < n && d < padded; ++d) {
    const float range = std::max(q99[d] - q01[d], 1e-8f);
    out[d] = ((state[d] - q01[d]) / range) * 2.0f - 1.0f;
  }
}

void postprocess_action(const float* action, int steps, int padded, int real, const float* q01,
                        const float* q99, const float* raw_state, float* out) {
  for (int t = 0; t < steps; ++t)
    for (int d = 0; d < real; ++d) {
      const float range = std::max(q99[d] - q01[d], 1e-8f);
      float v = ((action[static_cast<size_t>(t) * padded + d] + 1.0f) * 0.5f) * range + q01[d];
      if (d < 6 || (d >= 7 && d < 13)) v += raw_state[d];
      out[static_cast<size_t>(t) * real + d] = v;
    }
}

int t5_valid_tokens(int n_lang, const int32_t* mask, int mask_n, int max_tokens, std::string* why) {
  if (n_lang < 1 || n_lang > max_tokens) {
    *why = "lang token count " + std::to_string(n_lang) + " outside [1," + std::to_string(max_tokens) + "]";
    return -1;
  }
  if (!mask && mask_n != 0) {
    *why = "T5 mask length is nonzero without a mask";
    return -1;
  }
  if (mask && mask_n != n_lang) {
    *why = "T5 mask length " + std::to_string(mask_n) + " does not match token count " +
           std::to_string(n_lang);
    return -1;
  }
  int valid = n_lang;
  if (mask) {
    valid = 0;
    bool padding = false;
    for (int i = 0; i < n_lang; ++i) {
      if (mask[i] != 0 && mask[i] != 1) {
        *why = "T5 mask values must be zero or one";
        return -1;
      }
      if (mask[i] == 1) {
        if (padding) {
          *why = "T5 mask must be a contiguous valid prefix";
          return -1;
        }
        ++valid;
      } else {
        padding = true;
      }
    }
  }
  if (valid == 0) {
    *why = "T5 mask contains no valid tokens";
    return -1;
  }
  return valid;
}

}  // namespace wamb

extern "C" {

WAM_B200_API int wam_b200_flow_schedule(int steps, float shift, float* timesteps, float* sigmas) {
  if (steps <= 0 || !(shift > 0.0f) || !std::isfinite(shift) || !timesteps || !sigmas)
    return WAM_B200_INVALID_ARGUMENT;
  std::vector<float> ts, sg;
  wamb::flow_schedule(steps, shift, &ts, &sg);
  std::copy(ts.begin(), ts.end(), timesteps);
  std::copy(sg.begin(), sg.end(), sigmas);
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_rope_inv_freq(int mode, float* out64) {
  if ((mode != 1 && mode != 2) || !out64) return WAM_B200_INVALID_ARGUMENT;
  wamb::rope_inv_freq(mode, out64);
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_visual_positions(int gh, int gw, int* thw) {
  if (gh <= 0 || gw <= 0 || !thw) return WAM_B200_INVALID_ARGUMENT;
  wamb::visual_positions(gh, gw, thw);
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_normalize_state(const float* state, int n, int padded, const float* q01,
                                          const float* q99, float* out) {
  if (!state || !q01 || !q99 || !out || n < 1 || n > padded) return WAM_B200_INVALID_ARGUMENT;
  for (int d = 0; d < n; ++d)
    if (!std::isfinite(state[d])) return WAM_B200_INVALID_ARGUMENT;
  wamb::normalize_state(state, n, padded, q01, q99, out);
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_postprocess_action(const float* action, int steps, int padded, int real,
                                             const float* q01, const float* q99,
                                             const float* raw_state, float* out) {
  if (!action || !q01 || !q99 || !raw_state || !out || steps < 1 || real < 1 || real > padded)
    return WAM_B200_INVALID_ARGUMENT;
  wamb::postprocess_action(action, steps, padded, real, q01, q99, raw_state, out);
  return WAM_B200_OK;
}

}  // extern "C"
