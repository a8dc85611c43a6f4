// Wan VAE encoder on the B200 (vae.cu): patchified image -> standardised
// latent, the reference's run_vae (src/models/gwp05/engine/vae.cpp:279-388)
// without ggml. One image of image_width x image_height per call; the whole
// encoder is one captured CUDA graph.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <string>
#include <vector>

#include "kernels.h"

namespace wamb {

struct VaeOptions {
  std::string artifact_path;  // GGUF with vae.* tensors + gwp05.vae_latents_{mean,std}; empty: synthetic
  uint64_t synthetic_seed = 0;
  int image_width = 0, image_height = 0;  // canvas; multiples of 32
  int z_dim = 48;
  int device_index = 0;
  bool use_cuda_graph = true;
};

// Tensor names and shapes ([cout][cin][kh][kw] for convolutions, [c] for
// gains and biases) of the encoder, in the reference's compact GGUF naming
// (weights.cpp:116-167, vae component): 82 tensors.
std::vector<std::pair<std::string, std::vector<int64_t>>> vae_tensor_specs(int z_dim);

class VaeEncoder {
 public:
  ~VaeEncoder();
  bool init(const VaeOptions& opt, std::string* err);
  // pixels: device [12][H/2][W/2] F32 (the preprocess output); latent: device
  // [z][H/16][W/16] F32, (posterior mode - mean) / std.
  bool encode(const float* pixels, float* latent, cudaStream_t stream, std::string* err);
  // run_vae from camera views in host memory (3 views; PreprocessView with host
  // data pointers): the views are copied into device buffers owned by the
  // encoder, composed (stage 1) into the pixel slot and encoded into `latent`
  // (device), all on `stream`.
  bool encode_images(const PreprocessView* host_views, int n_views, float* latent,
                     cudaStream_t stream, std::string* err);
  int latent_count() const { return opt_.z_dim * (opt_.image_height / 16) * (opt_.image_width / 16); }
  const VaeOptions& options() const { return opt_; }
  cudaStream_t stream() const { return stream_; }
  // Launches of one encode (kernels recorded in the program).
  int launches() const { return static_cast<int>(program_.size()); }
  // F32 copy of an intermediate NHWC activation by stage name ("conv_in",
  // "down0".."down3", "mid", "moments"), for parity tests.
  bool read_stage(const std::string& name, std::vector<float>* out, int* h, int* w, int* c);
  double flops() const { return flops_; }
  // The device buffers the captured program reads (pixels) and writes (latent):
  // writing the pixels there and reading the latent from there skips encode's copies.
  float* pixels_slot() const { return pixels_slot_; }
  float* latent_slot() const { return latent_slot_; }
  unsigned* error_word() const { return error_; }

 private:
  struct Act {
    bf16* p = nullptr;
    int h = 0, w = 0, c = 0;
  };
  Act act(int h, int w, int c, std::string* err);
  bool load_weights(std::string* err);
  bool build(std::string* err);
  bool conv(const Act& x, const std::string& wname, int mode, Act* out, const Act* residual,
            std::string* err, const std::string& bias_name = "");
  void rms(const Act& x, const std::string& gamma, bool silu, Act* out);
  bool resnet(const std::string& prefix, const Act& x, int cout, Act* out, std::string* err);
  bool down_block(int index, const Act& x, bool downsample, bool temporal, int cout, Act* out,
                  std::string* err);
  bool mid_attention(const Act& x, Act* out, std::string* err);
  bool gemm(const bf16* x, int ldx, int m, const bf16* w, int n, int k, int epi, const bf16* bias,
            const bf16* residual, void* out, std::string* err, bool weights_from_prev = false);

  VaeOptions opt_;
  cudaStream_t stream_ = nullptr;
  std::map<std::string, bf16*> w_;       // raw tensors
  std::map<std::string, bf16*> wconv_;   // convolution weights in the kernel layout
  std::vector<void*> allocs_;
  std::vector<float> mean_, std_;
  float* stats_dev_ = nullptr;  // [2][z]
  unsigned* error_ = nullptr;
  float* gemm_ws_ = nullptr;
  unsigned* gemm_counters_ = nullptr;
  size_t gemm_ws_floats_ = 0;
  const float* pixels_in_ = nullptr;
  void* view_buf_[3] = {nullptr, nullptr, nullptr};
  size_t view_cap_[3] = {0, 0, 0};
  float* pixels_slot_ = nullptr;  // device copy target the graph reads
  float* latent_slot_ = nullptr;
  std::vector<std::function<bool(cudaStream_t)>> program_;
  std::map<std::string, Act> stages_;
  cudaGraphExec_t graph_ = nullptr;
  double flops_ = 0.0;
};

}  // namespace wamb
