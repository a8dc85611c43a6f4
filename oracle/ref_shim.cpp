// C wrappers over the reference's own host-side code, compiled from its
// sources (src/models/common/scheduler.cpp, src/models/gwp05/semantics.cpp)
// by `make ref` into oracle/_ref/libwamref.so. TEST INFRASTRUCTURE ONLY: the
// tests use it to pin the oracle's and the engine's schedule, positions and
// state/action (de)normalisation to the reference's exact outputs.
#include <cstdint>
#include <cstring>
#include <vector>

#include "models/common/scheduler.h"
#include "models/gwp05/semantics.h"

namespace sem = wam::internal::gwp05::semantics;

extern "C" {

// make_flow_match_euler_schedule (scheduler.cpp:26-55).
int wamref_schedule(int steps, float shift, float* timesteps, float* sigmas) {
  try {
    auto s = wam::internal::make_flow_match_euler_schedule(steps, shift);
    std::memcpy(timesteps, s.timesteps.data(), sizeof(float) * s.timesteps.size());
    std::memcpy(sigmas, s.sigmas.data(), sizeof(float) * s.sigmas.size());
    return 0;
  } catch (...) {
    return 1;
  }
}

// visual_positions (semantics.cpp:235-257).
int wamref_visual_positions(int gh, int gw, int32_t* t, int32_t* h, int32_t* w) {
  try {
    auto p = sem::visual_positions(gh, gw);
    std::memcpy(t, p.time.data(), sizeof(int32_t) * p.time.size());
    std::memcpy(h, p.height.data(), sizeof(int32_t) * p.height.size());
    std::memcpy(w, p.width.data(), sizeof(int32_t) * p.width.size());
    return 0;
  } catch (...) {
    return 1;
  }
}

// action_positions (semantics.cpp:210-222).
int wamref_action_positions(int tokens, int include_state, int32_t* out) {
  try {
    auto p = sem::action_positions(tokens, include_state != 0);
    std::memcpy(out, p.data(), sizeof(int32_t) * p.size());
    return 0;
  } catch (...) {
    return 1;
  }
}

// normalize_and_pad_state (semantics.cpp:154-172).
int wamref_normalize_state(const float* state, int n, int padded, const float* q01,
                           const float* q99, float* out) {
  try {
    std::vector<float> s(state, state + n), a(q01, q01 + padded), b(q99, q99 + padded);
    auto r = sem::normalize_and_pad_state(s, padded, a, b);
    std::memcpy(out, r.data(), sizeof(float) * r.size());
    return 0;
  } catch (...) {
    return 1;
  }
}

// postprocess_action (semantics.cpp:178-208).
int wamref_postprocess(const float* action, int steps, int padded, int real, const float* q01,
                       const float* q99, const float* raw_state, int state_n, float* out) {
  try {
    std::vector<float> a(action, action + static_cast<size_t>(steps) * padded);
    std::vector<float> l(q01, q01 + padded), h(q99, q99 + padded), s(raw_state, raw_state + state_n);
    auto r = sem::postprocess_action(a, steps, padded, real, l, h, s);
    std::memcpy(out, r.data(), sizeof(float) * r.size());
    return 0;
  } catch (...) {
    return 1;
  }
}

}  // extern "C"
