// C ABI entry points (include/wam_b200.h). Op-level functions forward device
// pointers to the kernels; engine-level functions live in engine_api.cpp.
#include <cstring>
#include <string>

#include "c_api_util.h"
#include "engine.h"
#include "kernels.h"
#include "wam_b200.h"

namespace wamb {

thread_local std::string g_last_error;

void set_last_error(const std::string& msg) { g_last_error = msg; }

int num_sms_current() {
  static thread_local int dev = -1;
  static thread_local int sms = 0;
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return 148;
  if (d != dev) {
    dev = d;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess) sms = 148;
  }
  return sms;
}

int check_sm100(std::string* why) {
  int d = 0, major = 0, minor = 0;
  if (cudaGetDevice(&d) != cudaSuccess) {
    *why = "no CUDA device";
    return WAM_B200_CUDA_ERROR;
  }
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d);
  if (major != 10 || minor != 0) {
    *why = "wam_b200 kernels are built for sm_100a only (device is sm_" + std::to_string(major) +
           std::to_string(minor) + ")";
    return WAM_B200_UNSUPPORTED;
  }
  return WAM_B200_OK;
}

}  // namespace wamb

using namespace wamb;

extern "C" {

WAM_B200_API uint32_t wam_b200_abi_version(void) { return WAM_B200_ABI_VERSION; }

WAM_B200_API const char* wam_b200_last_error(void) { return g_last_error.c_str(); }

WAM_B200_API size_t wam_b200_gemm_scratch_floats(int m, int n, int k, int force_splits,
                                                 int* tiles_out) {
  return gemm_scratch_floats(m, n, k, num_sms_current(), force_splits, tiles_out);
}

WAM_B200_API int wam_b200_op_gemm(const void* x, int ldx, int m, const void* w, int n, int k,
                                  int epilogue, const void* bias, const float* gate,
                                  const void* residual, int ldr, void* out, int ldo,
                                  float* workspace, size_t workspace_floats, unsigned* counters,
                                  int counter_slots, unsigned* error, int force_splits,
                                  void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  if (gemm_init(dev) != cudaSuccess) {
    set_last_error("gemm_init failed");
    return WAM_B200_CUDA_ERROR;
  }
  GemmScratch scratch;
  scratch.workspace = workspace;
  scratch.workspace_floats = workspace_floats;
  scratch.counters = counters;
  scratch.counter_slots = counter_slots;
  scratch.error = error;
  const bool tiled = (epilogue & WAM_B200_GEMM_TILED_WEIGHTS) != 0;
  const bool q8 = (epilogue & WAM_B200_GEMM_Q8_WEIGHTS) != 0;
  const bool pair = (epilogue & WAM_B200_GEMM_PAIR) != 0;
  epilogue &= ~(WAM_B200_GEMM_TILED_WEIGHTS | WAM_B200_GEMM_Q8_WEIGHTS | WAM_B200_GEMM_PAIR);
  GemmOp op;
  const char* err = gemm_plan(&op, static_cast<const bf16*>(x), ldx, m, static_cast<const bf16*>(w),
                              n, k, epilogue, static_cast<const bf16*>(bias), gate,
                              static_cast<const bf16*>(residual), ldr, out, ldo, scratch,
                              num_sms_current(), force_splits, tiled, q8, pair);
  if (err) {
    set_last_error(err);
    return WAM_B200_INVALID_ARGUMENT;
  }
  cudaError_t ce = gemm_launch(op, static_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) {
    set_last_error(std::string("gemm launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_retile_weights(const void* src, void* dst, int n, int k,
                                            void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  if (!src || !dst || n <= 0 || k <= 0 || n % gemm_weight_tile_rows() || k % 64 ||
      (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 16) {
    set_last_error("retile_weights: n % 256, k % 64 and 16-byte aligned pointers required");
    return WAM_B200_INVALID_ARGUMENT;
  }
  const uintptr_t a = reinterpret_cast<uintptr_t>(src), b = reinterpret_cast<uintptr_t>(dst);
  const uintptr_t bytes = static_cast<uintptr_t>(n) * k * 2;
  if (a < b + bytes && b < a + bytes) {
    set_last_error("retile_weights: src and dst overlap");
    return WAM_B200_INVALID_ARGUMENT;
  }
  launch_retile_weights(static_cast<const bf16*>(src), static_cast<bf16*>(dst), n, k,
                        static_cast<cudaStream_t>(stream));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    set_last_error(std::string("retile_weights launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_q8_quantize(const void* w, long long n_elems, void* blocks,
                                         void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  if (!w || !blocks || n_elems <= 0 || n_elems % 32) {
    set_last_error("q8_quantize: n_elems must be a positive multiple of 32");
    return WAM_B200_INVALID_ARGUMENT;
  }
  launch_q8_quantize(static_cast<const bf16*>(w), n_elems, static_cast<uint8_t*>(blocks),
                     static_cast<cudaStream_t>(stream));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    set_last_error(std::string("q8_quantize launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_q8_retile(const void* blocks, void* tiles, int n, int k,
                                       void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  if (!blocks || !tiles || n <= 0 || k <= 0 || n % 256 || k % 64 ||
      reinterpret_cast<uintptr_t>(tiles) % 16) {
    set_last_error("q8_retile: n % 256, k % 64 and a 16-byte aligned destination required");
    return WAM_B200_INVALID_ARGUMENT;
  }
  launch_q8_retile(static_cast<const uint8_t*>(blocks), static_cast<uint8_t*>(tiles), n, k,
                   static_cast<cudaStream_t>(stream));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    set_last_error(std::string("q8_retile launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_attention(const void* q, long long q_seq_stride,
                                       long long q_head_stride, const void* k, const void* v,
                                       long long kv_seq_stride, long long kv_head_stride, int lq,
                                       int lk, int heads, int batch, float scale, void* out,
                                       int ldo, void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  if (lq < 1 || lk < 1 || heads < 1 || batch < 1 || ldo < heads * 128) {
    set_last_error("attention: bad shape");
    return WAM_B200_INVALID_ARGUMENT;
  }
  if (attention_init() != cudaSuccess) {
    set_last_error("attention_init failed");
    return WAM_B200_CUDA_ERROR;
  }
  AttnArgs a{};
  a.q = static_cast<const bf16*>(q);
  a.q_seq_stride = q_seq_stride;
  a.q_head_stride = q_head_stride;
  a.k = static_cast<const bf16*>(k);
  a.v = static_cast<const bf16*>(v);
  a.kv_seq_stride = kv_seq_stride;
  a.kv_head_stride = kv_head_stride;
  a.lq = lq;
  a.lk = lk;
  a.heads = heads;
  a.batch = batch;
  a.scale = scale;
  a.out = static_cast<bf16*>(out);
  a.ldo = ldo;
  launch_attention(a, static_cast<cudaStream_t>(stream));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    set_last_error(std::string("attention launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_layernorm(const void* x, int rows, int cols, const void* a,
                                       const void* b, float eps, int affine, void* y,
                                       void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  if (rows < 1 || cols < 8 || cols % 8) {
    set_last_error("layernorm: cols must be a positive multiple of 8");
    return WAM_B200_INVALID_ARGUMENT;
  }
  if (affine)
    launch_ln_affine(static_cast<const bf16*>(x), cols, rows, cols, static_cast<const bf16*>(a),
                     static_cast<const bf16*>(b), eps, static_cast<bf16*>(y), cols,
                     static_cast<cudaStream_t>(stream));
  else
    launch_ln_modulate(static_cast<const bf16*>(x), cols, rows, cols, static_cast<const float*>(a),
                       static_cast<const float*>(b), eps, static_cast<bf16*>(y), cols,
                       static_cast<cudaStream_t>(stream));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    set_last_error(std::string("layernorm launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_qkv_scatter(const wam_b200_qkv_scatter_args* p, void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  if (!p || !p->src || p->rows < 1 || p->rows_per_seq < 1 || p->rows % p->rows_per_seq ||
      p->heads < 1 || p->ld_src % 8 || p->rope_mode < 0 || p->rope_mode > 2 ||
      (p->rope_mode && !p->inv_freq) || (p->rope_mode == 2 && !p->pos_thw) ||
      (p->q_col >= 0 && !p->q_out) || (p->k_col >= 0 && !p->k_out) || (p->v_col >= 0 && !p->v_out)) {
    set_last_error("qkv_scatter: invalid arguments");
    return WAM_B200_INVALID_ARGUMENT;
  }
  const int H = p->heads * 128;
  for (int c : {p->q_col, p->k_col, p->v_col})
    if (c >= 0 && (c % 8 || c + H > p->ld_src)) {
      set_last_error("qkv_scatter: source columns must be multiples of 8 inside the row");
      return WAM_B200_INVALID_ARGUMENT;
    }
  QkvScatter q{};
  q.src = static_cast<const bf16*>(p->src);
  q.ld_src = p->ld_src;
  q.rows = p->rows;
  q.rows_per_seq = p->rows_per_seq;
  q.hidden = H;
  q.heads = p->heads;
  q.q_col = p->q_col;
  q.k_col = p->k_col;
  q.v_col = p->v_col;
  q.q_norm = static_cast<const bf16*>(p->q_norm);
  q.k_norm = static_cast<const bf16*>(p->k_norm);
  q.eps = p->eps;
  q.rope_mode = p->rope_mode;
  q.pos_base = p->pos_base;
  q.pos_thw = p->pos_thw;
  q.inv_freq = p->inv_freq;
  q.q_out = static_cast<bf16*>(p->q_out);
  q.q_seq_stride = p->q_seq_stride;
  q.q_head_stride = p->q_head_stride;
  q.q_row_offset = p->q_row_offset;
  q.k_out = static_cast<bf16*>(p->k_out);
  q.v_out = static_cast<bf16*>(p->v_out);
  q.kv_seq_stride = p->kv_seq_stride;
  q.kv_head_stride = p->kv_head_stride;
  q.kv_row_offset = p->kv_row_offset;
  launch_qkv_scatter(q, static_cast<cudaStream_t>(stream));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    set_last_error(std::string("qkv_scatter launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_synth(void* w, long long n, uint64_t seed, double scale,
                                   double center, void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  launch_synth_bf16(static_cast<bf16*>(w), n, seed, scale, center, static_cast<cudaStream_t>(stream));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    set_last_error(std::string("synth launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API uint64_t wam_b200_tensor_seed(uint64_t seed, const char* name) {
  return tensor_seed(seed, name ? name : "");
}

}  // extern "C"
