// Implicit-GEMM 2-D convolution on tcgen05 for the Wan VAE encoder (the
// reference runs these as cuDNN IMPLICIT_PRECOMP_GEMM convolutions,
// patches/llama-b9866-native-bf16.patch:202-248, reached from vae_conv,
// src/models/gwp05/engine/vae.cpp:141-160).
//
// Activations are NHWC BF16 ([H][W][C], one image). The GEMM view: M = output
// pixels, N = output channels, K = taps x input channels. A tile is 8 rows x
// 16 columns of output pixels (M = 128 = the TMEM lanes); its k-block
// (tap, 64-channel block) is ONE tiled TMA load of the input window shifted
// by the tap, so im2col never touches memory:
//   3x3 stride 1, padding 1: 3-D map {C, W, H}, box {64, 16, 8} at
//     (cb * 64, x0 + dx - 1, y0 + dy - 1); the padding ring is the TMA
//     out-of-bounds zero fill;
//   3x3 stride 2 after a zero pad of one column / row at the end (the
//     downsampler, vae.cpp:211-214): 5-D map {C, 2, W/2, 2, H/2} (pixel
//     parities split out), box {64, 1, 16, 1, 8} at (cb * 64, dx & 1,
//     x0 + dx / 2, dy & 1, y0 + dy / 2);
//   1x1: the 3-D map with one tap at (cb * 64, x0, y0).
// Channel blocks past C read zeros, so C need not be a multiple of 64. The
// innermost coordinate (the channel) is always a multiple of 64 elements.
// Weights are re-laid out at load to [Cout rounded up to 256][tap][C rounded
// up to 64] (zero padded) and read with a 2-D map, box {64, 256}.
//
// Pipeline as the persistent linear GEMM: warp 0 TMA producer, warp 1 TMEM
// allocator + single-thread UMMA issuer (M = 128, N = 160 or 256, K = 16), warps 2-5
// epilogue (bias, residual, BF16 rounding as the reference's
// conv -> BF16, + bias -> BF16, + shortcut -> BF16), two TMEM accumulators so
// one tile's epilogue overlaps the next tile's mainloop; CTAs loop over tiles.
#include <cstdio>
#include <mutex>

#include "epilogue.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace wamb {
namespace {

constexpr int kTileW = 16, kTileH = 8;  // output pixels per tile (M = 128)
constexpr int kCM = 128, kCN = 256, kCK = 64;  // kCN: the widest N tile (padding unit)
constexpr int kCThreads = 192;
constexpr uint32_t kCA = kCM * kCK * 2;   // 16 KB
// N tile of the kernel: 256 output channels, or 160 when Cout is a multiple of
// 160 (the VAE's 160 / 320 / 640): a UMMA's time is linear in N, so a 256-wide
// tile over 160 channels would spend 37.5 % of the tensor time on padding.
template <int WN>
struct ConvTile {
  static constexpr uint32_t kB = WN * kCK * 2;  // 32 / 20 KB per stage
  static constexpr int kStages = 196608 / (kCA + kB) > 6 ? 6 : 196608 / (kCA + kB);
  static constexpr int kSmem = kStages * (kCA + kB) + 1024 + 256 + 2 * kCN * 4;
};

__device__ __forceinline__ void conv_load_a(const CUtensorMap* tm, uint8_t* dst, uint64_t* bar,
                                            const ConvParams& p, int kb, int x0, int y0,
                                            uint64_t pol) {
  const int tap = kb / p.cblocks, cb = kb - tap * p.cblocks;
  const int c0 = cb * kCK;
  if (p.mode == 1) {
    const int dy = tap / 3, dx = tap - dy * 3;
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(dx & 1),
        "r"(x0 + (dx >> 1)), "r"(dy & 1), "r"(y0 + (dy >> 1)), "l"(pol)
        : "memory");
  } else {
    int xs = x0, ys = y0;
    if (p.mode == 0) {
      const int dy = tap / 3, dx = tap - dy * 3;
      xs += dx - 1;
      ys += dy - 1;
    }
    tma_load_3d(dst, tm, bar, c0, xs, ys, pol);
  }
}

template <int WN>
__global__ void __launch_bounds__(kCThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ ConvParams p, const __grid_constant__ GemmArgs args) {
  constexpr int kS = ConvTile<WN>::kStages;
  constexpr uint32_t kBw = ConvTile<WN>::kB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + kS * kCA;
  uint8_t* tail = smem_w + kS * kBw;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + kS;
  uint64_t* acc_full = empty + kS;  // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* bias_s = reinterpret_cast<float*>(tail + 256);
  float* gate_s = bias_s + kCN;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = p.tiles_x * p.tiles_y;
  const int tiles = tiles_m * p.tiles_n;
  const int nkb = p.taps * p.cblocks;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
    for (int s = 0; s < kS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 1);
    }
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kCN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_last();  // every pixel tile reads the same weights
      const uint64_t pol_x = policy_evict_last();  // the 9 taps re-read each window
      int g = 0;
      bool waited = false, good = true;
      for (int t = blockIdx.x; t < tiles && good; t += gridDim.x) {
        const int tm = t % tiles_m, tn = t / tiles_m;
        const int x0 = (tm % p.tiles_x) * kTileW, y0 = (tm / p.tiles_x) * kTileH;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kS;
          if (g >= kS && !mbar_wait(&empty[s], ((g / kS) & 1) ^ 1)) {
            atomicCAS(args.error, 0u, static_cast<unsigned>(kErrProducerTimeout));
            good = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kCA + kBw);
          tma_load_2d(smem_w + s * kBw, &tm_w, &full[s], kb * kCK, tn * WN, pol_w);
          if (!waited) {  // the input comes from the preceding kernel
            griddep_wait();
            waited = true;
          }
          conv_load_a(&tm_x, smem_a + s * kCA, &full[s], p, kb, x0, y0, pol_x);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kCM, WN);
      int g = 0, j = 0;
      bool good = true;
      for (int t = blockIdx.x; t < tiles && good; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&acc_empty[b], ((j >> 1) - 1) & 1)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + static_cast<uint32_t>(b * WN);
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kS;
          if (!mbar_wait(&full[s], (g / kS) & 1)) {
            atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
            good = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_kmajor_desc(smem_u32(smem_a + s * kCA));
          const uint64_t db = sw128_kmajor_desc(smem_u32(smem_w + s * kBw));
#pragma unroll
          for (int k = 0; k < kCK / 16; ++k)
            umma_bf16_ss(acc, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (good) umma_commit(&acc_full[b]);
      }
    }
  } else {
    griddep_wait();
    const int et = threadIdx.x - 64;
    const int q = warp & 3;
    const int row = q * 32 + lane;  // pixel of the tile: (row % 16, row / 16)
    int j = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int b = j & 1;
      const int tm = t % tiles_m, tn = t / tiles_m;
      const int x = (tm % p.tiles_x) * kTileW + (row % kTileW);
      const int y = (tm / p.tiles_x) * kTileH + (row / kTileW);
      const int n_base = tn * WN;
      named_bar_sync(1, 128);  // the previous tile's bias is no longer read
      for (int jj = et; jj < WN; jj += 128) {
        const int n = n_base + jj;
        bias_s[jj] = (args.bias && n < args.n) ? __bfloat162float(args.bias[n]) : 0.0f;
        gate_s[jj] = 0.0f;
      }
      named_bar_sync(1, 128);
      const bool ok = mbar_wait(&acc_full[b], (j >> 1) & 1);
      if (!ok) atomicCAS(args.error, 0u, static_cast<unsigned>(kErrEpilogueTimeout));
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(b * WN) + (static_cast<uint32_t>(q * 32) << 16);
      const bool valid = ok && x < p.out_w && y < p.out_h;
#pragma unroll 1
      for (int c = 0; c < WN && n_base + c < args.n; c += 16) {
        uint32_t r[16];
        tmem_ld_x16(taddr + c, r);
        tmem_ld_wait();
        if (valid)
          epi_run<16>(args, y * p.out_w + x, n_base + c, reinterpret_cast<const float*>(r),
                      bias_s + c, gate_s + c);
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (et == 0) mbar_arrive(&acc_empty[b]);
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kCN);
  }
}

__global__ void conv_weight_layout_kernel(const bf16* __restrict__ src, bf16* __restrict__ dst,
                                          int cout, int cin, int taps, int cin_pad, int cout_pad) {
  const long long total = static_cast<long long>(cout_pad) * taps * cin_pad;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cin_pad);
    const long long r = i / cin_pad;
    const int tap = static_cast<int>(r % taps);
    const int o = static_cast<int>(r / taps);
    dst[i] = (c < cin && o < cout) ? src[(static_cast<long long>(o) * cin + c) * taps + tap]
                                   : __float2bfloat16_rn(0.0f);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) ==
            cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(q);
  });
  return fn;
}

bool encode(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
            const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides,
            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int conv_cin_pad(int cin) { return (cin + kCK - 1) / kCK * kCK; }
int conv_cout_pad(int cout) { return (cout + kCN - 1) / kCN * kCN; }

void launch_conv_weight_layout(const bf16* src, bf16* dst, int cout, int cin, int taps,
                               cudaStream_t stream) {
  const long long total = static_cast<long long>(conv_cout_pad(cout)) * taps * conv_cin_pad(cin);
  const int blocks = static_cast<int>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  conv_weight_layout_kernel<<<blocks, 256, 0, stream>>>(src, dst, cout, cin, taps,
                                                        conv_cin_pad(cin), conv_cout_pad(cout));
}

const char* conv_plan(ConvOp* op, const bf16* x, int in_w, int in_h, int cin, int mode,
                      const bf16* w_laid, int cout, int epilogue, const bf16* bias,
                      const bf16* residual, bf16* out, int num_sms) {
  if (mode < 0 || mode > 2) return "conv: mode must be 0 (3x3), 1 (3x3 stride 2) or 2 (1x1)";
  if (in_w <= 0 || in_h <= 0 || cin <= 0 || cout <= 0) return "conv: empty shape";
  // Every TMA box lies within the tensor's extent in the channel dimension
  // (boxes may overhang the far edge, never exceed the whole extent).
  if (cin < kCK) return "conv: at least 64 input channels (pad the input)";
  if ((cin * 2) % 16 != 0) return "conv: input channels must be a multiple of 8";
  if (cout % 16 != 0) return "conv: output channels must be a multiple of 16";
  if (mode == 1 && (in_w % 2 || in_h % 2)) return "conv: stride 2 needs an even input size";
  if (epilogue != EPI_BIAS && epilogue != EPI_RES)
    return "conv: epilogue must be EPI_BIAS or EPI_RES";
  if (epilogue == EPI_RES && !residual) return "conv: EPI_RES needs a residual";
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_laid) |
       reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) % 16)
    return "conv: operands must be 16-byte aligned";
  ConvParams& p = op->params;
  p.mode = mode;
  p.taps = mode == 2 ? 1 : 9;
  p.cblocks = conv_cin_pad(cin) / kCK;
  p.out_w = mode == 1 ? in_w / 2 : in_w;
  p.out_h = mode == 1 ? in_h / 2 : in_h;
  p.tiles_x = (p.out_w + kTileW - 1) / kTileW;
  p.tiles_y = (p.out_h + kTileH - 1) / kTileH;
  op->wn = cout % 160 == 0 ? 160 : kCN;
  p.tiles_n = (cout + op->wn - 1) / op->wn;
  const cuuint64_t c = static_cast<cuuint64_t>(cin);
  if (mode == 1) {
    const cuuint64_t dims[5] = {c, 2, static_cast<cuuint64_t>(in_w / 2), 2,
                                static_cast<cuuint64_t>(in_h / 2)};
    const cuuint64_t strides[4] = {c * 2, c * 4, static_cast<cuuint64_t>(in_w) * c * 2,
                                   static_cast<cuuint64_t>(in_w) * c * 4};
    const cuuint32_t box[5] = {kCK, 1, kTileW, 1, kTileH};
    if (!encode(&op->tm_x, x, 5, dims, strides, box)) return "conv: input tensor map";
  } else {
    const cuuint64_t dims[3] = {c, static_cast<cuuint64_t>(in_w), static_cast<cuuint64_t>(in_h)};
    const cuuint64_t strides[2] = {c * 2, static_cast<cuuint64_t>(in_w) * c * 2};
    const cuuint32_t box[3] = {kCK, kTileW, kTileH};
    if (!encode(&op->tm_x, x, 3, dims, strides, box)) return "conv: input tensor map";
  }
  const int kpad = p.taps * conv_cin_pad(cin);
  const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(kpad),
                               static_cast<cuuint64_t>(conv_cout_pad(cout))};
  const cuuint64_t wstr[1] = {static_cast<cuuint64_t>(kpad) * 2};
  const cuuint32_t wbox[2] = {kCK, static_cast<cuuint32_t>(op->wn)};
  if (!encode(&op->tm_w, w_laid, 2, wdims, wstr, wbox)) return "conv: weight tensor map";
  GemmArgs& a = op->args;
  a = GemmArgs{};
  a.m = p.out_w * p.out_h;
  a.n = cout;
  a.k = kpad;
  a.num_kb = p.taps * p.cblocks;
  a.epilogue = epilogue;
  a.bias = bias;
  a.residual = residual;
  a.ldr = cout;
  a.out = out;
  a.ldo = cout;
  const int tiles = p.tiles_x * p.tiles_y * p.tiles_n;
  op->grid = tiles < num_sms ? tiles : num_sms;
  return nullptr;
}

template <int WN>
bool conv_launch_t(const ConvOp& op, unsigned* error, cudaStream_t stream, bool pdl) {
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(conv_tc_kernel<WN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         ConvTile<WN>::kSmem);
  });
  GemmArgs a = op.args;
  a.error = error;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.grid);
  cfg.blockDim = dim3(kCThreads);
  cfg.dynamicSmemBytes = ConvTile<WN>::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, conv_tc_kernel<WN>, op.tm_w, op.tm_x, op.params, a) == cudaSuccess;
}

bool conv_launch(const ConvOp& op, unsigned* error, cudaStream_t stream, bool pdl) {
  return op.wn == 160 ? conv_launch_t<160>(op, error, stream, pdl)
                      : conv_launch_t<256>(op, error, stream, pdl);
}

}  // namespace wamb
