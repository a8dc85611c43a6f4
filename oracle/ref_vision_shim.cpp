// C wrapper over the reference's own image composition, compiled from its
// source by `make ref` into oracle/_ref/libwamref_vision.so. TEST
// INFRASTRUCTURE ONLY: pins the oracle's and the CUDA kernel's preprocess to
// the reference's exact outputs.
//
// src/models/gwp05/engine/vae.cpp is not a translation unit of its own (the
// reference includes it into engine.cpp:84 inside the engine namespace), and
// its second half needs ggml. The Makefile therefore streams the first half
// (resize_center_crop + compose_and_patchify, vae.cpp:1-134, everything before
// vae_bias) into this file through the WAMREF_VAE_PREPROCESS include, straight
// from the reference tree; nothing of it is written to disk.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <vector>

#include "models/gwp05/engine/engine.h"

namespace wam::internal::gwp05::engine {
#include WAMREF_VAE_PREPROCESS
}  // namespace wam::internal::gwp05::engine

namespace eng = wam::internal::gwp05::engine;

extern "C" {

// compose_and_patchify (vae.cpp:91-134) of three views; format 0 U8, 1 F32.
int wamref_compose_and_patchify(const void* const* data, const int* w, const int* h,
                                const int* format, int out_w, int out_h, float* out,
                                long long out_n) {
  eng::ImageView views[3];
  for (int i = 0; i < 3; ++i) {
    views[i].data = data[i];
    views[i].w = w[i];
    views[i].h = h[i];
    views[i].format = format[i] == 0 ? eng::PixelFormat::U8 : eng::PixelFormat::F32_RGB_01;
  }
  eng::EngineInputsView in;
  in.images = views;
  in.n_images = 3;
  eng::Config cfg;
  cfg.image_width = out_w;
  cfg.image_height = out_h;
  const std::vector<float> r = eng::compose_and_patchify(in, cfg);
  if (static_cast<long long>(r.size()) != out_n) return 1;
  std::memcpy(out, r.data(), sizeof(float) * r.size());
  return 0;
}

}  // extern "C"
