// C wrappers over the reference's own timestep embedding and T5 relative
// position bucketing (src/models/gwp05/engine/text_encoder.cpp:1-24),
// compiled from its source by `make ref` into oracle/_ref/libwamref_text.so.
// TEST INFRASTRUCTURE ONLY. text_encoder.cpp is an include fragment whose
// remainder needs ggml; the Makefile streams its first part (everything before
// build_attention) into this file through WAMREF_TEXT_ENCODER, straight from
// the reference tree.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "models/gwp05/engine/engine.h"

namespace wam::internal::gwp05::engine {
#include WAMREF_TEXT_ENCODER
}  // namespace wam::internal::gwp05::engine

namespace eng = wam::internal::gwp05::engine;

extern "C" {

int wamref_relative_bucket(int relative, int buckets, int max_distance) {
  return eng::relative_position_bucket(relative, buckets, max_distance);
}

void wamref_timestep_embedding(float t, int dim, float* out) {
  const std::vector<float> v = eng::timestep_embedding(t, dim);
  std::memcpy(out, v.data(), sizeof(float) * v.size());
}

}  // extern "C"
