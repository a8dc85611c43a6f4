// UMT5 text encoder on the B200 (t5.cu): prompt token ids -> prompt embedding
// [n_lang][hidden] F32, the reference's run_t5
// (src/models/gwp05/engine/text_encoder.cpp:112-204) without ggml.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "kernels.h"

namespace wamb {

struct T5Geometry {
  int vocab = 256384, hidden = 4096, ffn = 10240, heads = 64, head_dim = 64, layers = 24;
  int max_tokens = 512;  // n_lang: the longest prompt and the output rows
};

struct T5Options {
  std::string artifact_path;  // GGUF with t5.* tensors (geometry from gwp05.t5_*); empty: synthetic
  uint64_t synthetic_seed = 0;
  T5Geometry geometry;        // synthetic geometry (max_tokens always from here)
  int device_index = 0;
  bool use_cuda_graph = true;
};

// relative_position_bucket (text_encoder.cpp:14-24): bidirectional, 32
// buckets, max distance 128; relative = key - query.
int t5_relative_bucket(int relative, int buckets, int max_distance);

// Tensor names and shapes (torch order) in the reference's compact naming
// (weights.cpp:146-153, t5 component): 2 + 10 per layer.
std::vector<std::pair<std::string, std::vector<int64_t>>> t5_tensor_specs(const T5Geometry& g);

class T5Encoder {
 public:
  ~T5Encoder();
  bool init(const T5Options& opt, std::string* err);
  // tokens: host ids of the valid prompt prefix (n in [1, max_tokens]); out:
  // device [max_tokens][hidden] F32, rows >= n zeroed. On `stream`.
  bool encode(const int32_t* tokens, int n, float* out, cudaStream_t stream, std::string* err);
  const T5Geometry& geometry() const { return g_; }
  cudaStream_t stream() const { return stream_; }
  double flops(int n) const;
  int launches(int n);

 private:
  struct Program {
    std::vector<std::function<bool(cudaStream_t)>> ops;
    cudaGraphExec_t graph = nullptr;
  };
  bool load_weights(std::string* err);
  Program* program(int n, std::string* err);
  bool gemm(Program* p, const bf16* x, int ldx, int m, const bf16* w, int n, int k, int epi,
            const bf16* residual, int ldr, void* out, int ldo, std::string* err);

  T5Options opt_;
  T5Geometry g_;
  cudaStream_t stream_ = nullptr;
  std::vector<void*> allocs_;
  std::map<std::string, bf16*> w_;
  bf16* qkv_w_ = nullptr;  // per layer [3 hidden][hidden], layers contiguous
  bf16* up_w_ = nullptr;   // per layer [2 ffn][hidden] (wi_0 rows, then wi_1 rows)
  // activations (max_tokens rows)
  float* h_ = nullptr;      // residual stream F32 [T][hidden]
  bf16* n_ = nullptr;       // normalised BF16 [T][hidden]
  bf16* qkv_ = nullptr;     // [T][3 hidden]
  bf16* att_ = nullptr;     // [T][hidden]
  bf16* tmp_ = nullptr;     // branch output [T][hidden]
  bf16* up_ = nullptr;      // [T][ffn]
  float* out_ = nullptr;    // [max_tokens][hidden]
  int32_t* ids_ = nullptr;  // [max_tokens]
  int8_t* buckets_ = nullptr;  // [2 max_tokens - 1] bucket of relative position d - (max_tokens - 1)
  float* ws_ = nullptr;
  unsigned* counters_ = nullptr;
  unsigned* error_ = nullptr;
  size_t ws_floats_ = 0;
  std::map<int, std::unique_ptr<Program>> programs_;
};

}  // namespace wamb
