// Flash attention for the MoT's joint self-attention over the prefix K/V
// cache and its cross-attention over the prompt K/V cache.
//
// softmax(scale * Q K^T) V per (sequence, head): F32 scores, online softmax in
// F32 (running max / sum), probabilities rounded to BF16 for the P·V product,
// F32 accumulation, BF16 output. One CTA = 4 warps = 64 query rows of one
// (sequence, head); K/V tiles of 64 keys stream through a double-buffered
// cp.async pipeline into XOR-swizzled shared memory.
//
// Reference: the cached joint attention (src/models/gwp05/engine/mot.cpp:432-446,
// scores at GGML_PREC_F32, ggml_soft_max_ext with scale 1/sqrt(128), no mask),
// the prefix attention (engine/cache.cpp:274-287) and the cached cross attention
// (mot.cpp:299-321).
#include "kernels.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace wamb {

namespace {

constexpr int kBQ = 64;
constexpr int kBKey = 64;
constexpr int kD = 128;
constexpr int kTileBytes = kBKey * kD * 2;  // 16 KB
constexpr int kSmem = kTileBytes * 5;       // Q + 2 x (K, V)

// Byte offset of (row, 16-byte chunk) in a [64][128] BF16 tile with the chunk
// index XOR-swizzled by the row (conflict-free ldmatrix).
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void load_tile(uint32_t smem, const bf16* g, int rows_valid, int tid) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = tid + i * 128;
    const int row = idx >> 4;
    const int chunk = idx & 15;
    const bool ok = row < rows_valid;
    const bf16* src = g + (ok ? row : 0) * kD + chunk * 8;
    cp_async_16(smem + swz(row, chunk), src, ok);
  }
}

__global__ void __launch_bounds__(128) attention_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t s_q = smem_u32(smem);
  const uint32_t s_k[2] = {s_q + kTileBytes, s_q + 3 * kTileBytes};
  const uint32_t s_v[2] = {s_q + 2 * kTileBytes, s_q + 4 * kTileBytes};

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int q0 = blockIdx.x * kBQ;
  const int head = blockIdx.y;
  const int seq = blockIdx.z;

  griddep_wait();
  griddep_launch_dependents();
  const bf16* qg = a.q + seq * a.q_seq_stride + head * a.q_head_stride + static_cast<long long>(q0) * kD;
  const bf16* kg = a.k + seq * a.kv_seq_stride + head * a.kv_head_stride;
  const bf16* vg = a.v + seq * a.kv_seq_stride + head * a.kv_head_stride;

  const int n_kb = (a.lk + kBKey - 1) / kBKey;
  load_tile(s_q, qg, a.lq - q0, tid);
  load_tile(s_k[0], kg, a.lk, tid);
  load_tile(s_v[0], vg, a.lk, tid);
  cp_async_commit();

  // Q fragments for this warp's 16 rows, 8 k-steps of 16 dims.
  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  const float sl2 = a.scale * 1.4426950408889634f;

  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      const int nb = buf ^ 1;
      load_tile(s_k[nb], kg + static_cast<long long>(kb + 1) * kBKey * kD, a.lk - (kb + 1) * kBKey, tid);
      load_tile(s_v[nb], vg + static_cast<long long>(kb + 1) * kBKey * kD, a.lk - (kb + 1) * kBKey, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int row = warp * 16 + (lane & 15);
        const int chunk = kk * 2 + (lane >> 4);
        ldmatrix_x4(s_q + swz(row, chunk), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys.
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        const int key = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int chunk = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(s_k[buf] + swz(key, chunk), b0, b1, b2, b3);
        mma_bf16_16816(s[2 * jp], qf[kk], b0, b1);
        mma_bf16_16816(s[2 * jp + 1], qf[kk], b2, b3);
      }
    }
    // Mask keys beyond lk.
    const int kbase = kb * kBKey;
    if (kbase + kBKey > a.lk) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = kbase + j * 8 + (lane & 3) * 2;
        if (c >= a.lk) s[j][0] = s[j][2] = -INFINITY;
        if (c + 1 >= a.lk) s[j][1] = s[j][3] = -INFINITY;
      }
    }
    // Online softmax over rows g (regs 0,1) and g+8 (regs 2,3).
    float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], rs[2] = {0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < 2; ++r) corr[r] = exp2f((m_run[r] - mx[r]) * sl2);
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f((s[j][0] - mx[0]) * sl2);
      const float p1 = exp2f((s[j][1] - mx[0]) * sl2);
      const float p2 = exp2f((s[j][2] - mx[1]) * sl2);
      const float p3 = exp2f((s[j][3] - mx[1]) * sl2);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int kk = j >> 1;
      if ((j & 1) == 0) {
        pf[kk][0] = pack_bf16(p0, p1);
        pf[kk][1] = pack_bf16(p2, p3);
      } else {
        pf[kk][2] = pack_bf16(p0, p1);
        pf[kk][3] = pack_bf16(p2, p3);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * corr[r] + rs[r];
      m_run[r] = mx[r];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // O += P V: 4 k-steps of 16 keys, 16 n-tiles of 8 dims.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int chunk = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(s_v[buf] + swz(key, chunk), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * dp], pf[kk], b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();
  }

  // Normalise and store BF16 rows.
  const float inv[2] = {1.0f / l_run[0], 1.0f / l_run[1]};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = q0 + warp * 16 + (lane >> 2) + r * 8;
    if (row >= a.lq) continue;
    bf16* dst;
    if (a.split_first) {
      dst = row == 0 ? a.out_first + static_cast<long long>(seq) * a.ldo_first
                     : a.out + (static_cast<long long>(seq) * (a.lq - 1) + row - 1) * a.ldo;
    } else {
      dst = a.out + (static_cast<long long>(seq) * a.lq + row) * a.ldo;
    }
    dst += head * kD + (lane & 3) * 2;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t v = pack_bf16(o[i][2 * r] * inv[r], o[i][2 * r + 1] * inv[r]);
      *reinterpret_cast<uint32_t*>(dst + i * 8) = v;
    }
  }
}

}  // namespace

cudaError_t attention_init() {
  return cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
}

void launch_attention(const AttnArgs& a, cudaStream_t s) {
  dim3 grid((a.lq + kBQ - 1) / kBQ, a.heads, a.batch);
  launch_pdl(attention_kernel, grid, dim3(128), kSmem, s, a);
}

}  // namespace wamb
