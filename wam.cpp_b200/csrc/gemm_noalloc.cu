// wam_b200_op_gemm_noalloc: the split-K GEMM with its scratch in a fixed,
// library-owned device array, for callers that are not allowed to allocate
// device memory.
//
// Who needs this: a robot control loop that calls the policy every cycle must
// keep each call's latency bounded, and cudaMalloc/cudaFree may synchronize the
// whole device and take unbounded time; plugins hosted by a framework that owns
// the device allocator (and forbids side allocations); code paths that run
// while another component records a CUDA graph. wam_b200_op_gemm asks its caller
// for a workspace (the caller must cudaMalloc it); this variant uses the
// library's own array instead and calls no allocating routine.
//
// The array is file-scope device memory: every GPU that loads the library holds
// kScratchFloats floats plus kScratchCounters counters until the process exits.
// All calls share it and it keeps the last call's contents, so the counters and
// the error word are cleared (cudaMemsetAsync, no allocation) before every
// launch; wam_b200_op_gemm_noalloc_error reads the error word back (the status
// of the last call on the current device). Calls that overlap on the GPU (two
// streams, or two host threads on the same device) race on the array and must
// be serialized by the caller.
#include <cstring>
#include <mutex>
#include <string>

#include "c_api_util.h"
#include "kernels.h"
#include "wam_b200.h"

namespace wamb {
namespace {

// Maximum split-K partial storage (floats): tiles x splits x token tile x 128.
constexpr size_t kScratchFloats = size_t(2) << 20;  // 8 MiB
constexpr int kScratchCounters = 4096;              // output tiles
constexpr int kMaxDevices = 64;

// [partials | counters + error word]; zero-initialised when the module loads.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchFloats * sizeof(float) +
                                                                  (kScratchCounters + 64) *
                                                                      sizeof(unsigned)];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Once per device, with that device current: the host-side name of the array
// is not a device address, so the address comes from cudaGetSymbolAddress.
cudaError_t scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return cudaSuccess;
}

}  // namespace
}  // namespace wamb

using namespace wamb;

extern "C" {

WAM_B200_API int wam_b200_op_gemm_noalloc(const void* x, int ldx, int m, const void* w, int n,
                                          int k, int epilogue, const void* bias, const float* gate,
                                          const void* residual, int ldr, void* out, int ldo,
                                          int force_splits, void* stream) {
  std::string why;
  int rc = check_sm100(&why);
  if (rc != WAM_B200_OK) {
    set_last_error(why);
    return rc;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error("gemm_noalloc: no usable current device");
    return WAM_B200_CUDA_ERROR;
  }
  if (gemm_init(dev) != cudaSuccess) {
    set_last_error("gemm_init failed");
    return WAM_B200_CUDA_ERROR;
  }
  void* base = nullptr;
  cudaError_t ce = scratch_address(dev, &base);
  if (ce != cudaSuccess) {
    set_last_error(std::string("gemm_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  GemmScratch scratch;
  scratch.workspace = static_cast<float*>(base);
  scratch.workspace_floats = kScratchFloats;
  scratch.counters = reinterpret_cast<unsigned*>(static_cast<float*>(base) + kScratchFloats);
  scratch.counter_slots = kScratchCounters;
  scratch.error = scratch.counters + kScratchCounters;
  const bool tiled = (epilogue & WAM_B200_GEMM_TILED_WEIGHTS) != 0;
  const bool q8 = (epilogue & WAM_B200_GEMM_Q8_WEIGHTS) != 0;
  const bool pair = (epilogue & WAM_B200_GEMM_PAIR) != 0;
  epilogue &= ~(WAM_B200_GEMM_TILED_WEIGHTS | WAM_B200_GEMM_Q8_WEIGHTS | WAM_B200_GEMM_PAIR);
  GemmOp op;
  // gemm_plan checks the exact scratch need of the mode it picks: unsplit,
  // persistent and cluster-split shapes need no counters whatever their tile
  // count; only split-K partials must fit the array.
  const char* err = gemm_plan(&op, static_cast<const bf16*>(x), ldx, m, static_cast<const bf16*>(w),
                              n, k, epilogue, static_cast<const bf16*>(bias), gate,
                              static_cast<const bf16*>(residual), ldr, out, ldo, scratch,
                              num_sms_current(), force_splits, tiled, q8, pair);
  if (err) {
    std::string msg(err);
    if (msg.find("scratch too small") != std::string::npos) {
      int tiles = 0;
      const size_t need = gemm_scratch_floats(m, n, k, num_sms_current(), force_splits, &tiles);
      msg = "gemm_noalloc: shape needs " + std::to_string(need) + " split-K floats and " +
            std::to_string(tiles) + " output tiles; the built-in scratch holds " +
            std::to_string(kScratchFloats) + " floats and " + std::to_string(kScratchCounters) +
            " tile counters (use wam_b200_op_gemm with a workspace)";
    }
    set_last_error(msg);
    return WAM_B200_INVALID_ARGUMENT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: counters and error word must
  // start at zero for this launch.
  ce = cudaMemsetAsync(scratch.counters, 0, (kScratchCounters + 1) * sizeof(unsigned), s);
  if (ce == cudaSuccess) ce = gemm_launch(op, s);
  if (ce != cudaSuccess) {
    set_last_error(std::string("gemm_noalloc launch: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_op_gemm_noalloc_error(unsigned* code) {
  if (!code) {
    set_last_error("gemm_noalloc_error: null output");
    return WAM_B200_INVALID_ARGUMENT;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error("gemm_noalloc_error: no usable current device");
    return WAM_B200_CUDA_ERROR;
  }
  void* base = nullptr;
  cudaError_t ce = scratch_address(dev, &base);
  if (ce == cudaSuccess)
    ce = cudaMemcpy(code, reinterpret_cast<unsigned*>(static_cast<float*>(base) + kScratchFloats) +
                              kScratchCounters,
                    sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) {
    set_last_error(std::string("gemm_noalloc_error: ") + cudaGetErrorString(ce));
    return WAM_B200_CUDA_ERROR;
  }
  return WAM_B200_OK;
}

}  // extern "C"
