// C ABI of the UMT5 text encoder (include/wam_b200.h, "UMT5").
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "c_api_util.h"
#include "host_math.h"
#include "t5.h"
#include "wam_b200.h"

struct wam_b200_t5 {
  wamb::T5Encoder enc;
  int device = 0;
};

namespace {

int tfail(wam_b200_status* st, int code, const std::string& msg) {
  wamb::set_last_error(msg);
  if (st) {
    st->code = code;
    st->message = static_cast<char*>(std::malloc(msg.size() + 1));
    if (st->message) std::memcpy(st->message, msg.c_str(), msg.size() + 1);
  }
  return code;
}

int tok(wam_b200_status* st) {
  if (st) {
    st->code = WAM_B200_OK;
    st->message = nullptr;
  }
  return WAM_B200_OK;
}

}  // namespace

extern "C" {

WAM_B200_API int wam_b200_t5_relative_bucket(int relative, int buckets, int max_distance) {
  return wamb::t5_relative_bucket(relative, buckets, max_distance);
}

WAM_B200_API int wam_b200_t5_create(const wam_b200_t5_options* o, wam_b200_t5** out,
                                    wam_b200_status* st) {
  if (!o || !out) return tfail(st, WAM_B200_INVALID_ARGUMENT, "options and encoder pointer are required");
  *out = nullptr;
  if (o->struct_size < sizeof(wam_b200_t5_options))
    return tfail(st, WAM_B200_INVALID_ARGUMENT, "wam_b200_t5_options.struct_size is too small");
  if (cudaSetDevice(o->device_index) != cudaSuccess)
    return tfail(st, WAM_B200_CUDA_ERROR, "cudaSetDevice failed");
  std::string why;
  const int rc = wamb::check_sm100(&why);
  if (rc != WAM_B200_OK) return tfail(st, rc, why);
  wamb::T5Options to;
  to.artifact_path = o->artifact_path ? o->artifact_path : "";
  to.synthetic_seed = o->synthetic_seed;
  to.geometry.vocab = o->vocab;
  to.geometry.hidden = o->hidden;
  to.geometry.ffn = o->ffn;
  to.geometry.heads = o->heads;
  to.geometry.head_dim = o->head_dim;
  to.geometry.layers = o->layers;
  to.geometry.max_tokens = o->max_tokens;
  to.device_index = o->device_index;
  to.use_cuda_graph = o->use_cuda_graphs != 0;
  auto* t = new wam_b200_t5();
  t->device = o->device_index;
  std::string err;
  if (!t->enc.init(to, &err)) {
    delete t;
    return tfail(st, err.find("artifact") != std::string::npos ? WAM_B200_ARTIFACT_ERROR
                                                               : WAM_B200_INVALID_ARGUMENT,
                 err);
  }
  *out = t;
  return tok(st);
}

WAM_B200_API void wam_b200_t5_destroy(wam_b200_t5* t) {
  if (!t) return;
  cudaSetDevice(t->device);
  delete t;
}

WAM_B200_API int wam_b200_t5_geometry(const wam_b200_t5* t, int* vocab, int* hidden, int* ffn,
                                      int* heads, int* layers, int* max_tokens) {
  if (!t) return WAM_B200_INVALID_ARGUMENT;
  const auto& g = t->enc.geometry();
  if (vocab) *vocab = g.vocab;
  if (hidden) *hidden = g.hidden;
  if (ffn) *ffn = g.ffn;
  if (heads) *heads = g.heads;
  if (layers) *layers = g.layers;
  if (max_tokens) *max_tokens = g.max_tokens;
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_t5_encode_device(wam_b200_t5* t, const int32_t* tokens, int n_lang,
                                           const int32_t* mask, int mask_n, float* out,
                                           void* stream, wam_b200_status* st) {
  if (!t || !tokens || !out) return tfail(st, WAM_B200_INVALID_ARGUMENT, "encoder, tokens and output are required");
  std::string why;
  const int valid = wamb::t5_valid_tokens(n_lang, mask, mask_n, t->enc.geometry().max_tokens, &why);
  if (valid < 0) return tfail(st, WAM_B200_INVALID_ARGUMENT, why);
  cudaSetDevice(t->device);
  std::string err;
  if (!t->enc.encode(tokens, valid, out, static_cast<cudaStream_t>(stream), &err))
    return tfail(st, err.find("vocabulary") != std::string::npos ? WAM_B200_INVALID_ARGUMENT
                                                                 : WAM_B200_CUDA_ERROR,
                 err);
  return tok(st);
}

WAM_B200_API int wam_b200_t5_encode(wam_b200_t5* t, const int32_t* tokens, int n_lang,
                                    const int32_t* mask, int mask_n, float* out, size_t out_n,
                                    wam_b200_status* st) {
  if (!t || !out) return tfail(st, WAM_B200_INVALID_ARGUMENT, "encoder and output are required");
  const auto& g = t->enc.geometry();
  const size_t need = static_cast<size_t>(g.max_tokens) * g.hidden;
  if (out_n < need) return tfail(st, WAM_B200_INVALID_ARGUMENT, "output buffer is too small");
  cudaSetDevice(t->device);
  float* dev = nullptr;
  if (cudaMalloc(&dev, need * sizeof(float)) != cudaSuccess)
    return tfail(st, WAM_B200_CUDA_ERROR, "output allocation failed");
  const int rc = wam_b200_t5_encode_device(t, tokens, n_lang, mask, mask_n, dev, t->enc.stream(), st);
  if (rc == WAM_B200_OK) {
    cudaError_t e = cudaStreamSynchronize(t->enc.stream());
    if (e == cudaSuccess) e = cudaMemcpy(out, dev, need * sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (e != cudaSuccess) return tfail(st, WAM_B200_CUDA_ERROR, cudaGetErrorString(e));
    return WAM_B200_OK;
  }
  cudaFree(dev);
  return rc;
}

WAM_B200_API int wam_b200_t5_info(wam_b200_t5* t, int n, double* flops, int* launches) {
  if (!t || n < 1 || n > t->enc.geometry().max_tokens) return WAM_B200_INVALID_ARGUMENT;
  if (flops) *flops = t->enc.flops(n);
  if (launches) *launches = t->enc.launches(n);
  return WAM_B200_OK;
}

}  // extern "C"
