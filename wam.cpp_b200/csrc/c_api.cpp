// C ABI entry points (include/wam_b200.h). Op-level functions forward device
// pointers to the kernels; engine-level functions live in engine_api.cpp.
#include <cstring>
#include <string>

#include "c_api_util.h"
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
  GemmScratch scratch;
  scratch.workspace = workspace;
  scratch.workspace_floats = workspace_floats;
  scratch.counters = counters;
  scratch.counter_slots = counter_slots;
  scratch.error = error;
  GemmOp op;
  const char* err = gemm_plan(&op, static_cast<const bf16*>(x), ldx, m, static_cast<const bf16*>(w),
                              n, k, epilogue, static_cast<const bf16*>(bias), gate,
                              static_cast<const bf16*>(residual), ldr, out, ldo, scratch,
                              num_sms_current(), force_splits);
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

}  // extern "C"
