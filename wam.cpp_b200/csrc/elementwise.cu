// HBM-bound row and elementwise kernels of the MoT forward pass: LayerNorm +
// AdaLN modulation, affine LayerNorm, q/k RMSNorm + RoPE + scatter, the small
// encoder/decoder projections, modulation tables, patchify, the Euler update
// and the deterministic synthetic-weight generator. Rows are processed by one
// warp each with 16-byte vector loads; reductions use warp shuffles.
#include <cmath>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"
#include "mathops.cuh"
#include "ptx.cuh"

namespace wamb {

namespace {

struct alignas(16) Bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  const Bf16x8 x = *reinterpret_cast<const Bf16x8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(x.v[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  Bf16x8 x;
#pragma unroll
  for (int i = 0; i < 4; ++i) x.v[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<Bf16x8*>(p) = x;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}


constexpr int kRowThreads = 128;  // threads cooperating on one row

// Sum over the 128 threads of a block (4 warps) via shared memory.
__device__ __forceinline__ float block128_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  return red[0] + red[1] + red[2] + red[3];
}

// One 128-thread block per row; each thread holds up to MAXC 8-wide chunks of
// the row and of its parameters in registers, loaded in one batch so the row
// costs a single memory round trip.
// mode 0: AdaLN  y = bf16(n * (1 + scale) + shift), scale/shift F32
// mode 1: affine y = bf16(n * w + b), w/b BF16
// mode 2: AdaLN over RMSNorm (n = x * rsqrt(mean(x^2) + eps), no mean
//         subtraction; the config-1 variant), scale/shift F32
template <int MODE, int MAXC>
__global__ void __launch_bounds__(kRowThreads)
    ln_kernel(const bf16* __restrict__ x, int ldx, int rows, int cols, const void* pa,
              const void* pb, float eps, bf16* __restrict__ y, int ldy) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[4];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const bf16* xr = x + static_cast<long long>(row) * ldx;
  bf16* yr = y + static_cast<long long>(row) * ldy;
  const int chunks = cols >> 3;
  float v[MAXC][8], p0[MAXC][8], p1[MAXC][8];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kRowThreads;
    if (c < chunks) {
      load8(xr + c * 8, v[i]);
      if (MODE != 1) {
        const float4* sc = reinterpret_cast<const float4*>(static_cast<const float*>(pa) + c * 8);
        const float4* sh = reinterpret_cast<const float4*>(static_cast<const float*>(pb) + c * 8);
        const float4 s0 = sc[0], s1 = sc[1], h0 = sh[0], h1 = sh[1];
        p0[i][0] = s0.x; p0[i][1] = s0.y; p0[i][2] = s0.z; p0[i][3] = s0.w;
        p0[i][4] = s1.x; p0[i][5] = s1.y; p0[i][6] = s1.z; p0[i][7] = s1.w;
        p1[i][0] = h0.x; p1[i][1] = h0.y; p1[i][2] = h0.z; p1[i][3] = h0.w;
        p1[i][4] = h1.x; p1[i][5] = h1.y; p1[i][6] = h1.z; p1[i][7] = h1.w;
      } else {
        load8(static_cast<const bf16*>(pa) + c * 8, p0[i]);
        load8(static_cast<const bf16*>(pb) + c * 8, p1[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[i][j];
    }
  }
  const float mean = MODE == 2 ? 0.0f : block128_sum(s, red) / cols;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i)
    if (tid + i * kRowThreads < chunks) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[i][j] - mean;
        q += d * d;
      }
    }
  const float inv_std = rsqrtf(block128_sum(q, red) / cols + eps);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kRowThreads;
    if (c < chunks) {
      float f[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        f[j] = MODE != 1 ? fmaf((v[i][j] - mean) * inv_std, 1.0f + p0[i][j], p1[i][j])
                         : fmaf((v[i][j] - mean) * inv_std, p0[i][j], p1[i][j]);
      store8(yr + c * 8, f);
    }
  }
}

// The same LayerNorm for many rows (batched prefix / prompt, >= 1024 rows):
// the row stays packed as BF16 in registers and the parameters are read in
// the output pass (they stay in L1 / L2 across rows), so twelve blocks fit per
// SM instead of five and three times the row bytes are in flight. Same
// arithmetic and summation order as ln_kernel: bit-identical outputs.
template <int MODE, int MAXC>
__global__ void __launch_bounds__(kRowThreads, 12)
    ln_stream_kernel(const bf16* __restrict__ x, int ldx, int rows, int cols, const void* pa,
                     const void* pb, float eps, bf16* __restrict__ y, int ldy) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[4];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const bf16* xr = x + static_cast<long long>(row) * ldx;
  bf16* yr = y + static_cast<long long>(row) * ldy;
  const int chunks = cols >> 3;
  uint4 raw[MAXC];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kRowThreads;
    if (c < chunks) raw[i] = *reinterpret_cast<const uint4*>(xr + c * 8);
  }
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i)
    if (tid + i * kRowThreads < chunks) {
      float v[8];
      load8(reinterpret_cast<const bf16*>(&raw[i]), v);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[j];
    }
  const float mean = MODE == 2 ? 0.0f : block128_sum(s, red) / cols;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i)
    if (tid + i * kRowThreads < chunks) {
      float v[8];
      load8(reinterpret_cast<const bf16*>(&raw[i]), v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[j] - mean;
        q += d * d;
      }
    }
  const float inv_std = rsqrtf(block128_sum(q, red) / cols + eps);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kRowThreads;
    if (c < chunks) {
      float v[8], p0[8], p1[8];
      load8(reinterpret_cast<const bf16*>(&raw[i]), v);
      if (MODE != 1) {
        const float4* sc = reinterpret_cast<const float4*>(static_cast<const float*>(pa) + c * 8);
        const float4* sh = reinterpret_cast<const float4*>(static_cast<const float*>(pb) + c * 8);
        const float4 s0 = __ldg(sc), s1 = __ldg(sc + 1), h0 = __ldg(sh), h1 = __ldg(sh + 1);
        p0[0] = s0.x; p0[1] = s0.y; p0[2] = s0.z; p0[3] = s0.w;
        p0[4] = s1.x; p0[5] = s1.y; p0[6] = s1.z; p0[7] = s1.w;
        p1[0] = h0.x; p1[1] = h0.y; p1[2] = h0.z; p1[3] = h0.w;
        p1[4] = h1.x; p1[5] = h1.y; p1[6] = h1.z; p1[7] = h1.w;
      } else {
        load8(static_cast<const bf16*>(pa) + c * 8, p0);
        load8(static_cast<const bf16*>(pb) + c * 8, p1);
      }
      float f[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        f[j] = MODE != 1 ? fmaf((v[j] - mean) * inv_std, 1.0f + p0[j], p1[j])
                         : fmaf((v[j] - mean) * inv_std, p0[j], p1[j]);
      store8(yr + c * 8, f);
    }
  }
}

// Generic fallback for rows wider than 128 * 8 * 4 columns: one warp per row,
// three passes over the row.
template <int MODE>
__global__ void __launch_bounds__(256)
    ln_wide_kernel(const bf16* __restrict__ x, int ldx, int rows, int cols, const void* pa,
                   const void* pb, float eps, bf16* __restrict__ y, int ldy) {
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bf16* xr = x + static_cast<long long>(row) * ldx;
  bf16* yr = y + static_cast<long long>(row) * ldy;
  const int chunks = cols >> 3;
  float s = 0.0f;
  for (int c = lane; c < chunks; c += 32) {
    float f[8];
    load8(xr + c * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += f[i];
  }
  const float mean = MODE == 2 ? 0.0f : warp_sum(s) / cols;
  float q = 0.0f;
  for (int c = lane; c < chunks; c += 32) {
    float f[8];
    load8(xr + c * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = f[i] - mean;
      q += d * d;
    }
  }
  const float inv_std = rsqrtf(warp_sum(q) / cols + eps);
  for (int c = lane; c < chunks; c += 32) {
    float f[8], p0[8], p1[8];
    load8(xr + c * 8, f);
    if (MODE != 1) {
      for (int i = 0; i < 8; ++i) {
        p0[i] = static_cast<const float*>(pa)[c * 8 + i];
        p1[i] = static_cast<const float*>(pb)[c * 8 + i];
      }
    } else {
      load8(static_cast<const bf16*>(pa) + c * 8, p0);
      load8(static_cast<const bf16*>(pb) + c * 8, p1);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      f[i] = MODE != 1 ? fmaf((f[i] - mean) * inv_std, 1.0f + p0[i], p1[i])
                       : fmaf((f[i] - mean) * inv_std, p0[i], p1[i]);
    store8(yr + c * 8, f);
  }
}

// RoPE inverse frequency and position of the pair starting at head dim `dim`.
__device__ __forceinline__ float rope_theta(const QkvScatter& a, int dim, int pos1, int pt, int ph,
                                            int pw) {
  if (a.rope_mode == 1) return static_cast<float>(pos1) * __ldg(a.inv_freq + (dim >> 1));
  if (dim < 44) return static_cast<float>(pt) * __ldg(a.inv_freq + (dim >> 1));
  if (dim < 86) return static_cast<float>(ph) * __ldg(a.inv_freq + 22 + ((dim - 44) >> 1));
  return static_cast<float>(pw) * __ldg(a.inv_freq + 43 + ((dim - 86) >> 1));
}

// One block per token row, threadIdx.y = part (0 q, 1 k, 2 v), 128 threads per
// part; each thread holds up to MAXC 8-wide chunks of its part in registers
// (the norm weights, 12 KB shared by every row, are read again from L1 / L2
// when the chunk is written), so that three blocks fit an SM and more of the
// rows' bytes are in flight. MAXC = 0: generic loop.
template <int MAXC>
__global__ void __launch_bounds__(3 * kRowThreads, 3) qkv_scatter_kernel(const __grid_constant__ QkvScatter a) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[3][4];
  const int row = blockIdx.x;
  const int layer = blockIdx.y;
  const int which = threadIdx.y + (3 - static_cast<int>(blockDim.y));  // blocks without q: parts 1, 2
  const int tid = threadIdx.x;
  const int col = which == 0 ? a.q_col : (which == 1 ? a.k_col : a.v_col);
  const bf16* src = a.src + layer * a.src_layer_stride + static_cast<long long>(row) * a.ld_src +
                    (col < 0 ? 0 : col);
  const int seq = row / a.rows_per_seq;
  const int rin = row - seq * a.rows_per_seq;
  const int chunks = a.hidden >> 3;
  bf16* dst_base = nullptr;
  long long head_stride = 0;
  if (col >= 0) {
    if (which == 0) {
      dst_base = a.q_out + layer * a.out_layer_stride + seq * a.q_seq_stride +
                 static_cast<long long>(a.q_row_offset + rin) * 128;
      head_stride = a.q_head_stride;
    } else {
      dst_base = (which == 1 ? a.k_out : a.v_out) + layer * a.out_layer_stride +
                 seq * a.kv_seq_stride + static_cast<long long>(a.kv_row_offset + rin) * 128;
      head_stride = a.kv_head_stride;
    }
  }
  const bf16* nw = which == 0 ? a.q_norm
                              : (which == 1 ? (a.k_norms ? a.k_norms[layer] : a.k_norm) : nullptr);
  int pt = 0, ph = 0, pw = 0;
  if (a.rope_mode == 2 && which < 2 && col >= 0) {
    pt = a.pos_thw[rin * 3 + 0];
    ph = a.pos_thw[rin * 3 + 1];
    pw = a.pos_thw[rin * 3 + 2];
  }
  const int pos1 = a.pos_base + rin;
  const bool rope = a.rope_mode != 0 && which < 2;
  auto emit = [&](int c, float (&f)[8], float inv) {
    const int d = c * 8;
    const int hd = d & 127;
    if (nw) {
      float w[8];
      load8(nw + c * 8, w);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = f[i] * inv * w[i];
    }
    if (rope) {
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        float sn, cs;
        sincosf(rope_theta(a, hd + 2 * p, pos1, pt, ph, pw), &sn, &cs);
        const float x0 = f[2 * p], x1 = f[2 * p + 1];
        f[2 * p] = x0 * cs - x1 * sn;
        f[2 * p + 1] = x0 * sn + x1 * cs;
      }
    }
    store8(dst_base + (d >> 7) * head_stride + hd, f);
  };
  if constexpr (MAXC > 0) {
    float v[MAXC][8];
    float ss = 0.0f;
    if (col >= 0) {
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kRowThreads;
        if (c < chunks) {
          load8(src + c * 8, v[i]);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
      }
    }
    // block-wide sum for this part (all parts take part in the barriers)
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[which][tid >> 5] = ss;
    __syncthreads();
    const float tot = red[which][0] + red[which][1] + red[which][2] + red[which][3];
    if (col < 0) return;
    const float inv = nw ? rsqrtf(tot / a.hidden + a.eps) : 1.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * kRowThreads;
      if (c < chunks) emit(c, v[i], inv);
    }
  } else {
    float ss = 0.0f;
    if (col >= 0 && nw) {
      for (int c = tid; c < chunks; c += kRowThreads) {
        float f[8];
        load8(src + c * 8, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
      }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[which][tid >> 5] = ss;
    __syncthreads();
    const float tot = red[which][0] + red[which][1] + red[which][2] + red[which][3];
    if (col < 0) return;
    const float inv = nw ? rsqrtf(tot / a.hidden + a.eps) : 1.0f;
    for (int c = tid; c < chunks; c += kRowThreads) {
      float f[8];
      load8(src + c * 8, f);
      emit(c, f, inv);
    }
  }
}

// One warp per output element.
__global__ void small_linear_kernel(const bf16* __restrict__ x, int ldx, int m, int k,
                                    const bf16* __restrict__ w, long long w_sn, long long w_sk,
                                    const bf16* __restrict__ b, int n, int act,
                                    bf16* __restrict__ y, int ldy) {
  griddep_wait();
  griddep_launch_dependents();
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (long long o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
       o < static_cast<long long>(m) * n; o += warps) {
    const int mi = static_cast<int>(o / n);
    const int ni = static_cast<int>(o - static_cast<long long>(mi) * n);
    const bf16* xr = x + static_cast<long long>(mi) * ldx;
    const bf16* wr = w + ni * w_sn;
    float acc = 0.0f;
    for (int kk = lane; kk < k; kk += 32)
      acc += __bfloat162float(xr[kk]) * __bfloat162float(wr[kk * w_sk]);
    acc = warp_sum(acc);
    if (lane == 0) {
      float v = bf16_round(acc);
      if (b) v = bf16_round(v + __bfloat162float(b[ni]));
      if (act == ACT_GELU_ERF) v = gelu_erf(v);
      y[static_cast<long long>(mi) * ldy + ni] = __float2bfloat16_rn(v);
    }
  }
}

__global__ void modulation_add_kernel(const bf16* __restrict__ mod, int ld_mod, int period,
                                      int steps, const bf16* const* __restrict__ tables,
                                      int layers, int width, float* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = static_cast<long long>(steps) * layers * width;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(i % width);
    const long long sl = i / width;
    const int l = static_cast<int>(sl % layers);
    const int s = static_cast<int>(sl / layers);
    out[i] = __bfloat162float(mod[static_cast<long long>(s) * ld_mod + (j % period)]) +
             __bfloat162float(tables[l][j]);
  }
}

__global__ void silu_kernel(const bf16* __restrict__ x, bf16* __restrict__ y, int n) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(silu(__bfloat162float(x[i])));
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, bf16* __restrict__ y, long long n) {
  griddep_wait();
  griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

__global__ void bf16_to_f32_kernel(const bf16* __restrict__ x, float* __restrict__ y, long long n) {
  griddep_wait();
  griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

__global__ void patchify_kernel(const float* __restrict__ lat, int batch, int ch, int gh, int gw,
                                bf16* __restrict__ cols) {
  griddep_wait();
  griddep_launch_dependents();
  const int kk = ch * 4;
  const long long total = static_cast<long long>(batch) * gh * gw * kk;
  const int lh = 2 * gh, lw = 2 * gw;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int q = static_cast<int>(i % kk);
    const long long bt = i / kk;
    const int t = static_cast<int>(bt % (gh * gw));
    const int b = static_cast<int>(bt / (gh * gw));
    const int c = q >> 2, dy = (q >> 1) & 1, dx = q & 1;
    const int y = t / gw, x = t - (t / gw) * gw;
    const float v = lat[((static_cast<long long>(b) * ch + c) * lh + 2 * y + dy) * lw + 2 * x + dx];
    cols[i] = __float2bfloat16_rn(v);
  }
}

// ggml_add(action, ggml_mul(velocity, dt)) in F32, stored BF16 (weights.cpp:897-901).
__global__ void euler_kernel(bf16* __restrict__ a, const bf16* __restrict__ v, int n,
                             const float* __restrict__ dt) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float prod = __fmul_rn(__bfloat162float(v[i]), *dt);
    a[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(a[i]), prod));
  }
}

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void synth_kernel(bf16* __restrict__ w, long long n, unsigned long long seed, float k,
                             float center) {
  griddep_wait();
  griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const unsigned long long h =
        mix64(seed + static_cast<unsigned long long>(i + 1) * 0x9E3779B97F4A7C15ull);
    const int z = static_cast<int>((h & 0xFFFFull) + ((h >> 16) & 0xFFFFull) +
                                   ((h >> 32) & 0xFFFFull) + (h >> 48)) -
                  131070;
    const float v = __fadd_rn(__fmul_rn(static_cast<float>(z), k), center);
    w[i] = __float2bfloat16_rn(v);
  }
}

inline int grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

}  // namespace

template <int MODE>
void launch_ln(const bf16* x, int ldx, int rows, int cols, const void* pa, const void* pb,
               float eps, bf16* y, int ldy, cudaStream_t s) {
  const int per = (cols / 8 + kRowThreads - 1) / kRowThreads;
  const dim3 grid(rows), block(kRowThreads);
  if (rows >= 1024 && per <= 4) {  // many rows: bandwidth shape
    if (per <= 1)
      launch_pdl(ln_stream_kernel<MODE, 1>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
    else if (per <= 2)
      launch_pdl(ln_stream_kernel<MODE, 2>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
    else if (per <= 3)
      launch_pdl(ln_stream_kernel<MODE, 3>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
    else
      launch_pdl(ln_stream_kernel<MODE, 4>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
    return;
  }
  if (per <= 1)
    launch_pdl(ln_kernel<MODE, 1>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
  else if (per <= 2)
    launch_pdl(ln_kernel<MODE, 2>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
  else if (per <= 3)
    launch_pdl(ln_kernel<MODE, 3>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
  else if (per <= 4)
    launch_pdl(ln_kernel<MODE, 4>, grid, block, 0, s, x, ldx, rows, cols, pa, pb, eps, y, ldy);
  else
    launch_pdl(ln_wide_kernel<MODE>, dim3((rows + 7) / 8), dim3(256), 0, s, x, ldx, rows, cols,
               pa, pb, eps, y, ldy);
}

void launch_ln_modulate(const bf16* x, int ldx, int rows, int cols, const float* scale,
                        const float* shift, float eps, bf16* y, int ldy, cudaStream_t s) {
  launch_ln<0>(x, ldx, rows, cols, scale, shift, eps, y, ldy, s);
}

void launch_ln_affine(const bf16* x, int ldx, int rows, int cols, const bf16* w, const bf16* b,
                      float eps, bf16* y, int ldy, cudaStream_t s) {
  launch_ln<1>(x, ldx, rows, cols, w, b, eps, y, ldy, s);
}

void launch_rms_modulate(const bf16* x, int ldx, int rows, int cols, const float* scale,
                         const float* shift, float eps, bf16* y, int ldy, cudaStream_t s) {
  launch_ln<2>(x, ldx, rows, cols, scale, shift, eps, y, ldy, s);
}

void launch_qkv_scatter(const QkvScatter& a, cudaStream_t s) {
  const int per = (a.hidden / 8 + kRowThreads - 1) / kRowThreads;
  const dim3 grid(a.rows, a.layers), block(kRowThreads, a.q_col < 0 ? 2 : 3);
  if (per <= 1)
    launch_pdl(qkv_scatter_kernel<1>, grid, block, 0, s, a);
  else if (per <= 2)
    launch_pdl(qkv_scatter_kernel<2>, grid, block, 0, s, a);
  else if (per <= 3)
    launch_pdl(qkv_scatter_kernel<3>, grid, block, 0, s, a);
  else if (per <= 4)
    launch_pdl(qkv_scatter_kernel<4>, grid, block, 0, s, a);
  else
    launch_pdl(qkv_scatter_kernel<0>, grid, block, 0, s, a);
}

void launch_small_linear(const bf16* x, int ldx, int m, int k, const bf16* w, long long w_sn,
                         long long w_sk, const bf16* b, int n, int act, bf16* y, int ldy,
                         cudaStream_t s) {
  const long long outs = static_cast<long long>(m) * n;
  launch_pdl(small_linear_kernel, dim3(grid_for(outs * 32, 256)), dim3(256), 0, s, x, ldx, m, k, w,
             w_sn, w_sk, b, n, act, y, ldy);
}

void launch_modulation_add(const bf16* mod, int ld_mod, int period, int steps,
                           const bf16* const* tables, int layers, int width, float* combined,
                           cudaStream_t s) {
  const long long n = static_cast<long long>(steps) * layers * width;
  launch_pdl(modulation_add_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, mod, ld_mod, period,
             steps, tables, layers, width, combined);
}

void launch_silu(const bf16* x, bf16* y, int n, cudaStream_t s) {
  launch_pdl(silu_kernel, dim3((n + 255) / 256), dim3(256), 0, s, x, y, n);
}

void launch_f32_to_bf16(const float* x, bf16* y, long long n, cudaStream_t s) {
  launch_pdl(f32_to_bf16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, x, y, n);
}

void launch_bf16_to_f32(const bf16* x, float* y, long long n, cudaStream_t s) {
  launch_pdl(bf16_to_f32_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, x, y, n);
}

void launch_patchify(const float* latent, int batch, int channels, int gh, int gw, bf16* cols,
                     cudaStream_t s) {
  const long long n = static_cast<long long>(batch) * gh * gw * channels * 4;
  launch_pdl(patchify_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, latent, batch, channels, gh,
             gw, cols);
}

void launch_euler(bf16* action, const bf16* velocity, int n, const float* dt, cudaStream_t s) {
  launch_pdl(euler_kernel, dim3((n + 255) / 256), dim3(256), 0, s, action, velocity, n, dt);
}

void launch_synth_bf16(bf16* w, long long n, unsigned long long seed, double scale, double center,
                       cudaStream_t s) {
  // Unit-variance scaling of the Irwin-Hall(4) sum of 16-bit uniforms, rounded
  // to F32 once so host (numpy) and device apply the same constant.
  const double ih4_std = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  const float k = static_cast<float>(scale / ih4_std);
  launch_pdl(synth_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, w, n, seed, k,
             static_cast<float>(center));
}

}  // namespace wamb
