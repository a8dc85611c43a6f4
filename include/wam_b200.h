/*
 * wam_b200 — C ABI of the B200-native GWP-0.5 Mixture-of-Transformers engine.
 *
 * The engine replaces the reference's ggml execution engine behind
 * wam::internal::gwp05::engine::Engine (src/models/gwp05/engine/engine.h:142-155,
 * factory engine::create at engine.h:202-203). Every entry point returns 0 on
 * success and a non-zero wam_b200_error code on failure; engine entry points also
 * fill an optional wam_b200_status whose message is malloc'd and released by
 * wam_b200_status_free (the convention of the reference's C ABI,
 * src/serving/c_api.cpp:18-55). wam_b200_last_error() returns the calling
 * thread's last message for the op-level entry points.
 *
 * The op-level entry points (wam_b200_op_*) take DEVICE pointers and a CUDA
 * stream (cudaStream_t passed as void*); they exist so that each kernel of the
 * path can be checked against a CPU restatement on identical inputs. They run
 * only on an sm_100a device and never fall back to another implementation.
 */
#ifndef WAM_B200_H
#define WAM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WAM_B200_ABI_VERSION 1u

#if defined(__GNUC__)
#define WAM_B200_API __attribute__((visibility("default")))
#else
#define WAM_B200_API
#endif

enum wam_b200_error {
  WAM_B200_OK = 0,
  WAM_B200_INVALID_ARGUMENT = 1,
  WAM_B200_CUDA_ERROR = 2,
  WAM_B200_UNSUPPORTED = 3,
  WAM_B200_ARTIFACT_ERROR = 4,
  WAM_B200_INFERENCE_FAILED = 5,
  WAM_B200_DEVICE_TIMEOUT = 6
};

/* ABI version of this library (WAM_B200_ABI_VERSION at build time). */
WAM_B200_API uint32_t wam_b200_abi_version(void);

/* Last error message of the calling thread ("" if none). */
WAM_B200_API const char* wam_b200_last_error(void);

/* ------------------------------------------------------------------ ops */

/* BF16 tcgen05 GEMM with fused epilogue (one linear layer).
 * y[m, n] = epilogue(sum_k x[m, k] * w[n, k]); x: [m, ldx] BF16, w: [n, k] BF16
 * (GGUF ne = {k, n}), out: [m, ldo] BF16 (F32 for epilogue 6).
 * epilogue: 0 bias, 1 bias+GELU(tanh), 2 bias+SiLU, 3 gated residual
 * (r + linear * gate), 4 residual (r + linear), 5 F32 accumulate + bias,
 * 6 raw F32 accumulator. workspace/counters: split-K scratch (counters zeroed
 * before first use; the kernel leaves them zero). force_splits <= 0 picks
 * automatically. error: device word receiving a non-zero code on a pipeline
 * timeout.
 * Replaces: linear / linear_with_activation / linear_gelu_with_activation
 * (src/models/gwp05/engine/weights.cpp:786-849) and gated_residual
 * (src/models/gwp05/engine/mot.cpp:161-173). */
WAM_B200_API int wam_b200_op_gemm(const void* x, int ldx, int m, const void* w, int n, int k,
                                  int epilogue, const void* bias, const float* gate,
                                  const void* residual, int ldr, void* out, int ldo,
                                  float* workspace, size_t workspace_floats, unsigned* counters,
                                  int counter_slots, unsigned* error, int force_splits,
                                  void* stream);

/* Split-K scratch (floats) and output-tile count wam_b200_op_gemm needs for a shape. */
WAM_B200_API size_t wam_b200_gemm_scratch_floats(int m, int n, int k, int force_splits,
                                                 int* tiles_out);

#ifdef __cplusplus
}
#endif

#endif /* WAM_B200_H */
