// GEMM / convolution epilogue of one output row: CNT consecutive features of
// token (pixel) m from F32 accumulators to the kernel's output, with the
// reference's BF16 rounding points per epilogue kind (kernels.h, Epilogue).
// Shared by the linear GEMMs (gemm.cu) and the implicit-GEMM convolutions
// (conv.cu).
#pragma once

#include <cuda_bf16.h>

#include "kernels.h"
#include "mathops.cuh"

namespace wamb {
namespace {

// Epilogue of CNT consecutive features n0.. of token m (CNT = 8 or 16; the
// epilogue kind is a compile-time constant so each run is straight-line code).
template <int EPI, int CNT>
__device__ __forceinline__ void epi_run_t(const GemmArgs& a, int m, int n0, const float* v,
                                          const float* bias, const float* gate) {
  float o[CNT];
  float r[CNT];
  if constexpr (EPI == EPI_GATED_RES || EPI == EPI_RES || EPI == EPI_MUL) {
    const uint4* rp =
        reinterpret_cast<const uint4*>(a.residual + static_cast<long long>(m) * a.ldr + n0);
#pragma unroll
    for (int q = 0; q < CNT / 8; ++q) {
      const uint4 u = rp[q];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        r[q * 8 + 2 * j] = __uint_as_float(w[j] << 16);
        r[q * 8 + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  }
  const bool hb = a.bias != nullptr;
#pragma unroll
  for (int j = 0; j < CNT; ++j) {
    const float acc = v[j];
    const float b = bias[j];
    if constexpr (EPI == EPI_BIAS) {
      float t = bf16_round(acc);
      if (hb) t = t + b;
      o[j] = t;
    } else if constexpr (EPI == EPI_BIAS_GELU) {
      o[j] = gelu_tanh(bf16_round(acc) + b);
    } else if constexpr (EPI == EPI_BIAS_SILU) {
      float t = bf16_round(acc);
      if (hb) t = bf16_round(t + b);
      o[j] = silu(t);
    } else if constexpr (EPI == EPI_GATED_RES) {
      float t = bf16_round(acc);
      if (hb) t = bf16_round(t + b);
      o[j] = fmaf(t, gate[j], r[j]);
    } else if constexpr (EPI == EPI_RES) {
      float t = bf16_round(acc);
      if (hb) t = bf16_round(t + b);
      o[j] = r[j] + t;
    } else if constexpr (EPI == EPI_MUL) {
      float t = bf16_round(acc);
      if (hb) t = bf16_round(t + b);
      o[j] = r[j] * t;
    } else if constexpr (EPI == EPI_F32_BIAS) {
      o[j] = acc + b;
    } else if constexpr (EPI == EPI_BIAS_GELU_R) {
      float t = bf16_round(acc);
      if (hb) t = bf16_round(t + b);
      o[j] = gelu_tanh(t);
    } else if constexpr (EPI == EPI_BIAS_GELU_ERF) {
      float t = bf16_round(acc);
      if (hb) t = bf16_round(t + b);
      o[j] = gelu_erf(t);
    } else {
      o[j] = acc;
    }
  }
  if constexpr (EPI == EPI_F32_OUT) {
    float4* op = reinterpret_cast<float4*>(static_cast<float*>(a.out) +
                                           static_cast<long long>(m) * a.ldo + n0);
#pragma unroll
    for (int q = 0; q < CNT / 4; ++q)
      op[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
  } else {
    uint4* op = reinterpret_cast<uint4*>(static_cast<bf16*>(a.out) +
                                         static_cast<long long>(m) * a.ldo + n0);
#pragma unroll
    for (int q = 0; q < CNT / 8; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(o[q * 8 + 2 * j], o[q * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      op[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Dispatches the epilogue once per run (a per-element switch over nine
// inlined epilogues made every store wait on instruction fetch).
template <int CNT>
__device__ __forceinline__ void epi_run(const GemmArgs& a, int m, int n0, const float* v,
                                        const float* bias, const float* gate) {
  if (n0 >= a.n) return;
  switch (a.epilogue) {
    case EPI_BIAS: epi_run_t<EPI_BIAS, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_BIAS_GELU: epi_run_t<EPI_BIAS_GELU, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_BIAS_SILU: epi_run_t<EPI_BIAS_SILU, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_GATED_RES: epi_run_t<EPI_GATED_RES, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_RES: epi_run_t<EPI_RES, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_MUL: epi_run_t<EPI_MUL, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_F32_BIAS: epi_run_t<EPI_F32_BIAS, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_BIAS_GELU_R: epi_run_t<EPI_BIAS_GELU_R, CNT>(a, m, n0, v, bias, gate); break;
    case EPI_BIAS_GELU_ERF: epi_run_t<EPI_BIAS_GELU_ERF, CNT>(a, m, n0, v, bias, gate); break;
    default: epi_run_t<EPI_F32_OUT, CNT>(a, m, n0, v, bias, gate); break;
  }
}

}  // namespace
}  // namespace wamb
