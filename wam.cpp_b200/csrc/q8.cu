// Q8_0 weights (GGML block format: 32 weights = fp16 scale d + 32 int8 q,
// value q * d; 34 bytes). Two device kernels:
//  * quantisation of BF16 weights to Q8_0 blocks with the semantics of the
//    gguf-py package's Q8_0 quantiser (the format's reference codec, used by the
//    build's test fixtures): d = max|x| / 127 in F32, q = round-half-away(x * (1/d)),
//    d stored as fp16 (round to nearest even);
//  * re-tiling of row-major Q8_0 blocks [n][k/32][34 B] into the GEMM's weight
//    tiles: per (256-row tile, 64-wide k-block) 16 KB of int8 [256][64] followed
//    by 1 KB of fp16 scales [256][2], 17408 contiguous bytes (one bulk copy).
#include <cuda_fp16.h>

#include "kernels.h"
#include "launch.cuh"

namespace wamb {
namespace {

constexpr int kQ8Block = 32;
constexpr int kQ8Bytes = 34;

// Round half away from zero of a non-negative a, exactly: floor(a) plus one
// when the fraction is >= 1/2 (2 * fraction is exact in F32).
__device__ __forceinline__ float round_half_away_pos(float a) {
  const float fl = floorf(a);
  return fl + floorf(2.0f * (a - fl));
}

// One warp per Q8_0 block; lane i holds weight i.
__global__ void q8_quantize_kernel(const bf16* __restrict__ w, long long blocks,
                                   uint8_t* __restrict__ out) {
  const long long warp0 = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (long long b = warp0; b < blocks; b += nwarps) {
    const float x = __bfloat162float(w[b * kQ8Block + lane]);
    float amax = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
    const float t = __fmul_rn(x, id);
    const float r = round_half_away_pos(fabsf(t));
    const int q = static_cast<int>(t < 0.0f ? -r : r);
    uint8_t* blk = out + b * kQ8Bytes;
    // Blocks start at even byte offsets (34 * b): the scale is one 16-bit store.
    if (lane == 0) *reinterpret_cast<unsigned short*>(blk) = __half_as_ushort(__float2half_rn(d));
    blk[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
  }
}

// One thread per Q8_0 block of the source.
__global__ void q8_retile_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int n,
                                 int k) {
  const int bpr = k / kQ8Block;  // blocks per row
  const long long total = static_cast<long long>(n) * bpr;
  const int kbs = k / 64;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / bpr);
    const int blk = static_cast<int>(i % bpr);
    const int kb = blk >> 1, half = blk & 1;
    const int nt = row >> 8, r = row & 255;
    uint8_t* tile = dst + (static_cast<size_t>(nt) * kbs + kb) * kQ8TileBytes;
    const uint8_t* s = src + i * kQ8Bytes;
    uint8_t* q = tile + r * 64 + half * 32;
#pragma unroll
    for (int j = 0; j < 32; ++j) q[j] = s[2 + j];
    tile[16384 + r * 4 + half * 2] = s[0];
    tile[16384 + r * 4 + half * 2 + 1] = s[1];
  }
}

// One thread per weight: value = q * d (exact in F32), rounded to BF16.
__global__ void q8_dequantize_kernel(const uint8_t* __restrict__ blocks, long long n,
                                     bf16* __restrict__ w) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint8_t* blk = blocks + (i / kQ8Block) * kQ8Bytes;
    const unsigned short hb = static_cast<unsigned short>(blk[0] | (blk[1] << 8));
    const float d = __half2float(__ushort_as_half(hb));
    const int q = static_cast<int8_t>(blk[2 + (i % kQ8Block)]);
    w[i] = __float2bfloat16_rn(static_cast<float>(q) * d);
  }
}

int grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

}  // namespace

void launch_q8_quantize(const bf16* w, long long n_elems, uint8_t* out, cudaStream_t s) {
  const long long blocks = n_elems / kQ8Block;
  q8_quantize_kernel<<<grid_for(blocks * 32, 256), 256, 0, s>>>(w, blocks, out);
}

void launch_q8_dequantize(const uint8_t* blocks, long long n_elems, bf16* w, cudaStream_t s) {
  q8_dequantize_kernel<<<grid_for(n_elems, 256), 256, 0, s>>>(blocks, n_elems, w);
}

void launch_q8_retile(const uint8_t* src, uint8_t* dst, int n, int k, cudaStream_t s) {
  const long long total = static_cast<long long>(n) * (k / kQ8Block);
  q8_retile_kernel<<<grid_for(total, 256), 256, 0, s>>>(src, dst, n, k);
}

}  // namespace wamb
