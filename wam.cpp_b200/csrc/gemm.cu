// BF16 tcgen05 GEMM for every linear layer of the MoT forward pass.
//
// Orientation: the token tile is the UMMA "A" operand (M = 128 token rows =
// the 128 TMEM lanes) and the weight tile is "B" (N = 256 output features =
// 256 TMEM columns). One tcgen05.mma of M = 128, K = 16 occupies the tensor
// core for about the same ~130 cycles for every N up to 256 (measured on
// B200), so 256 weight rows per instruction double the weight bytes an SM can
// consume per cycle compared with putting the weights on the M side, which is
// what bounds the batch-1 denoise GEMMs (48 tokens: HBM/weight streaming).
// Token tiles shorter than 128 rows load only the rows that exist; the
// accumulator rows of the missing tokens are never read.
//
// Pipeline: warp 0 = TMA / bulk-copy producer, warp 1 = TMEM allocator +
// single-thread UMMA issuer, warps 2-5 = epilogue (warp w reads TMEM lanes
// 32*(w%4).., i.e. one token per thread, 16 features per tcgen05.ld, and
// stores them as 16-byte vectors along the feature axis).
// Split-K: the splits of one output tile form a thread-block cluster and
// reduce their F32 partial tiles through distributed shared memory, or go
// through a caller-provided global workspace (the last CTA reduces).
//
// Reference: every ggml_mul_mat / ggml_mul_mat_out_type of the BF16 latency
// path (src/models/gwp05/engine/weights.cpp:786-849; cuBLAS route in
// patches/llama-b9866-native-bf16.patch:259-313).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "kernels.h"
#include "epilogue.cuh"
#include "mathops.cuh"
#include "ptx.cuh"
#include <cuda_fp16.h>

namespace wamb {

namespace {

constexpr int kTM = 128;              // token rows per tile (UMMA M, TMEM lanes)
constexpr int kWN = 256;              // weight rows per tile (UMMA N, TMEM columns)
constexpr int kBK = 64;               // K per stage: one 128-byte swizzle row of BF16
constexpr int kBBytes = kWN * kBK * 2;  // weight tile per stage (32 KB)
constexpr int kThreads = 256;  // warp 0 copies, 1 MMA, 2-5 epilogue
// gemm_tc_kernel with Q8_0 weights: warps 2-11 convert the stages to BF16.
constexpr int kThreadsQ8 = 384;
#ifndef WAM_GEMM_STAGE_BUDGET_KB
#define WAM_GEMM_STAGE_BUDGET_KB 200
#endif
constexpr int kStageBudget = WAM_GEMM_STAGE_BUDGET_KB * 1024;
constexpr int kMaxStages = 8;
#ifndef WAM_GEMM_WEIGHT_EVICT_FIRST
#define WAM_GEMM_WEIGHT_EVICT_FIRST 1
#endif
constexpr int kPartLd = kWN + 4;      // padded F32 row of a staged partial tile
constexpr int kSmemTail = 256 + 2 * kWN * 4;  // barriers + staged bias / gate
constexpr uint32_t kTmemCols = kWN;

// Token rows a tile loads: all 128 when the GEMM has that many, else the
// token count rounded up to 16.
int a_rows_for(int m) { return m >= kTM ? kTM : ((m + 15) / 16) * 16; }

// Pipeline stages: one weight k-block (32 KB) and one token k-block per
// stage, as many stages as the shared-memory budget holds (the weight stream
// is latency bound, so the bytes in flight per SM set its rate).
// Q8_0 weights add a raw 17 KB buffer per stage (converted into the BF16 stage).
int stage_bytes(int a_rows, bool q8) { return a_rows * kBK * 2 + kBBytes + (q8 ? kQ8TileBytes : 0); }
int stages_for(int a_rows, bool q8 = false) {
  const int st = kStageBudget / stage_bytes(a_rows, q8);
  return st > kMaxStages ? kMaxStages : st;
}
int smem_for(int a_rows, bool q8 = false) {
  return stages_for(a_rows, q8) * stage_bytes(a_rows, q8) + 1024 + kSmemTail;
}

// epi_run / epi_run_t (one token row, CNT features): epilogue.cuh.

// Unsplit tiles leave TMEM in two passes. Pass 1 (one token per thread):
// bias / activation of 16 features, written to a shared-memory staging tile
// [token][256] (BF16 rows of 528 bytes, or F32 rows of 1040 bytes for the raw
// accumulator epilogue; the padding keeps the 16-byte writes of a warp on
// distinct banks). Pass 2 (8 features per thread, lanes along the feature
// axis): residual / gate and coalesced 16-byte stores to the output rows.
constexpr int kStageLdB = kWN + 8;  // BF16 staging row (elements)

template <int EPI>
__device__ __forceinline__ void stage16_t(const GemmArgs& a, uint8_t* stg, int row, int c,
                                          const float* v, const float* bias) {
  const bool hb = a.bias != nullptr;
  if constexpr (EPI == EPI_F32_OUT) {
    float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(stg) + row * kPartLd + c);
#pragma unroll
    for (int q = 0; q < 4; ++q) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
    float o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float acc = v[j], b = bias[j];
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
      } else if constexpr (EPI == EPI_GATED_RES || EPI == EPI_RES || EPI == EPI_MUL) {
        // The residual is added (multiplied) in pass 2 to this BF16-exact linear output.
        float t = bf16_round(acc);
        if (hb) t = bf16_round(t + b);
        o[j] = t;
      } else if constexpr (EPI == EPI_F32_BIAS) {
        o[j] = acc + b;
      } else if constexpr (EPI == EPI_BIAS_GELU_R) {
        float t = bf16_round(acc);
        if (hb) t = bf16_round(t + b);
        o[j] = gelu_tanh(t);
      } else {  // EPI_BIAS_GELU_ERF
        float t = bf16_round(acc);
        if (hb) t = bf16_round(t + b);
        o[j] = gelu_erf(t);
      }
    }
    uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(stg) + row * kStageLdB + c);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(o[q * 8 + 2 * j], o[q * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      d[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

__device__ __forceinline__ void stage16(const GemmArgs& a, uint8_t* stg, int row, int c,
                                        const float* v, const float* bias) {
  switch (a.epilogue) {
    case EPI_BIAS: stage16_t<EPI_BIAS>(a, stg, row, c, v, bias); break;
    case EPI_BIAS_GELU: stage16_t<EPI_BIAS_GELU>(a, stg, row, c, v, bias); break;
    case EPI_BIAS_SILU: stage16_t<EPI_BIAS_SILU>(a, stg, row, c, v, bias); break;
    case EPI_GATED_RES: stage16_t<EPI_GATED_RES>(a, stg, row, c, v, bias); break;
    case EPI_RES: stage16_t<EPI_RES>(a, stg, row, c, v, bias); break;
    case EPI_MUL: stage16_t<EPI_MUL>(a, stg, row, c, v, bias); break;
    case EPI_F32_BIAS: stage16_t<EPI_F32_BIAS>(a, stg, row, c, v, bias); break;
    case EPI_BIAS_GELU_R: stage16_t<EPI_BIAS_GELU_R>(a, stg, row, c, v, bias); break;
    case EPI_BIAS_GELU_ERF: stage16_t<EPI_BIAS_GELU_ERF>(a, stg, row, c, v, bias); break;
    default: stage16_t<EPI_F32_OUT>(a, stg, row, c, v, bias); break;
  }
}

// Pass 2 over rows x (256 / 8) items, 8 consecutive features each.
template <int EPI>
__device__ __forceinline__ void copy_out_t(const GemmArgs& a, const uint8_t* stg, int rows,
                                           int m_base, int n_base, const float* gate, int t0,
                                           int nthreads) {
  const int items = rows * (kWN / 8);
  for (int it = t0; it < items; it += nthreads) {
    const int r = it / (kWN / 8), g = it % (kWN / 8);
    const int n0 = n_base + g * 8;
    if (n0 >= a.n) continue;
    const long long m = m_base + r;
    if constexpr (EPI == EPI_F32_OUT) {
      const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(stg) +
                                                          r * kPartLd + g * 8);
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + m * a.ldo + n0);
      dst[0] = src[0];
      dst[1] = src[1];
    } else {
      uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(stg) +
                                                r * kStageLdB + g * 8);
      if constexpr (EPI == EPI_GATED_RES || EPI == EPI_RES || EPI == EPI_MUL) {
        const uint4 rv = *reinterpret_cast<const uint4*>(a.residual + m * a.ldr + n0);
        uint32_t tw[4] = {u.x, u.y, u.z, u.w};
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float t0v = __uint_as_float(tw[j] << 16), t1v = __uint_as_float(tw[j] & 0xFFFF0000u);
          const float r0v = __uint_as_float(rw[j] << 16), r1v = __uint_as_float(rw[j] & 0xFFFF0000u);
          float o0, o1;
          if constexpr (EPI == EPI_GATED_RES) {
            o0 = fmaf(t0v, gate[g * 8 + 2 * j], r0v);
            o1 = fmaf(t1v, gate[g * 8 + 2 * j + 1], r1v);
          } else if constexpr (EPI == EPI_MUL) {
            o0 = r0v * t0v;
            o1 = r1v * t1v;
          } else {
            o0 = r0v + t0v;
            o1 = r1v + t1v;
          }
          const __nv_bfloat162 h = __floats2bfloat162_rn(o0, o1);
          tw[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
        u = make_uint4(tw[0], tw[1], tw[2], tw[3]);
      }
      *reinterpret_cast<uint4*>(static_cast<bf16*>(a.out) + m * a.ldo + n0) = u;
    }
  }
}

__device__ __forceinline__ void copy_out(const GemmArgs& a, const uint8_t* stg, int rows,
                                         int m_base, int n_base, const float* gate, int t0,
                                         int nthreads) {
  switch (a.epilogue) {
    case EPI_GATED_RES:
      copy_out_t<EPI_GATED_RES>(a, stg, rows, m_base, n_base, gate, t0, nthreads);
      break;
    case EPI_RES: copy_out_t<EPI_RES>(a, stg, rows, m_base, n_base, gate, t0, nthreads); break;
    case EPI_MUL: copy_out_t<EPI_MUL>(a, stg, rows, m_base, n_base, gate, t0, nthreads); break;
    case EPI_F32_OUT:
      copy_out_t<EPI_F32_OUT>(a, stg, rows, m_base, n_base, gate, t0, nthreads);
      break;
    default: copy_out_t<EPI_BIAS>(a, stg, rows, m_base, n_base, gate, t0, nthreads); break;
  }
}

// Output tile t of a persistent GEMM -> (token tile, weight tile). Token
// tiles go in groups of group_m, and a group runs through all weight tiles
// before the next group starts: a wave of CTAs then covers a few token tiles x
// many weight tiles, so both operands of the wave stay in L2. (With the token
// tile fastest over all tiles, every token tile is read from HBM again for
// each weight tile once the tokens exceed L2.) group_m >= tiles_m is that
// plain order.
__device__ __forceinline__ void tile_coords(const GemmArgs& a, int t, int& tile_m, int& tile_n) {
  const int g = a.group_m > 0 && a.group_m < a.tiles_m ? a.group_m : a.tiles_m;
  const int span = g * a.tiles_n;
  const int grp = t / span;
  const int first = grp * g;
  const int gsize = a.tiles_m - first < g ? a.tiles_m - first : g;
  const int local = t - grp * span;
  tile_m = first + local % gsize;
  tile_n = local / gsize;
}

// Persistent variant for GEMMs with more output tiles than SMs (prefix,
// batched denoise; no split-K, BF16 weights): CTA c takes tiles c, c + grid,
// ... The copy ring runs on across tiles, and two TMEM accumulators (2 x 256
// columns) let the epilogue of one tile overlap the mainloop of the next; the
// epilogue stores straight from registers (its time is hidden).
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_persistent_kernel(const __grid_constant__ CUtensorMap tm_w,
                              const __grid_constant__ CUtensorMap tm_x,
                              const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = args.stages;
  const uint32_t a_bytes = static_cast<uint32_t>(args.a_rows) * kBK * 2;
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + S * a_bytes;
  uint8_t* tail = smem_w + S * kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* bias_s = reinterpret_cast<float*>(tail + 256);
  float* gate_s = bias_s + kWN;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = args.tiles_m * args.tiles_n;
  const int nkb = args.num_kb;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
    for (int s = 0; s < S; ++s) {
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
    tmem_alloc(tmem_slot, 2 * kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = WAM_GEMM_WEIGHT_EVICT_FIRST ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_x = policy_evict_last();
      const uint32_t stage_tx = a_bytes + kBBytes;
      int g = 0;  // stages issued so far
      bool waited = false, good = true;
      for (int t = blockIdx.x; t < tiles && good; t += gridDim.x) {
        int tile_m, tile_n;
        tile_coords(args, t, tile_m, tile_n);
        const bf16* w_tiles =
            args.w_tiled ? args.w_tiled + static_cast<size_t>(tile_n) * nkb * (kWN * kBK) : nullptr;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % S;
          if (g >= S && !mbar_wait(&empty[s], ((g / S) & 1) ^ 1)) {
            atomicCAS(args.error, 0u, static_cast<unsigned>(kErrProducerTimeout));
            good = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], stage_tx);
          if (w_tiles)
            bulk_load(smem_w + s * kBBytes, w_tiles + static_cast<size_t>(kb) * (kWN * kBK),
                      kBBytes, &full[s], pol_w);
          else
            tma_load_2d(smem_w + s * kBBytes, &tm_w, &full[s], kb * kBK, tile_n * kWN, pol_w);
          if (!waited) {  // weights first; the tokens come from the preceding kernel
            griddep_wait();
            waited = true;
          }
          tma_load_2d(smem_a + s * a_bytes, &tm_x, &full[s], kb * kBK, tile_m * kTM, pol_x);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kTM, kWN);
      int g = 0, j = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&acc_empty[b], ((j >> 1) - 1) & 1)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + static_cast<uint32_t>(b * kWN);
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % S;
          if (!mbar_wait(&full[s], (g / S) & 1)) {
            atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
            kb = nkb;
            t = tiles;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_kmajor_desc(smem_u32(smem_a + s * a_bytes));
          const uint64_t db = sw128_kmajor_desc(smem_u32(smem_w + s * kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16_ss(acc, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
      }
    }
  } else if (warp < 6) {
    griddep_wait();
    const int et = threadIdx.x - 64;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int j = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int b = j & 1;
      int tile_m, tile_n;
      tile_coords(args, t, tile_m, tile_n);
      const int m_base = tile_m * kTM, n_base = tile_n * kWN;
      const int rows = args.m - m_base < kTM ? args.m - m_base : kTM;
      named_bar_sync(1, 128);  // the previous tile's bias / gate are no longer read
      for (int jj = et; jj < kWN; jj += 128) {
        const int n = n_base + jj;
        bias_s[jj] = (args.bias && n < args.n) ? __bfloat162float(args.bias[n]) : 0.0f;
        gate_s[jj] = (args.gate && n < args.n) ? args.gate[n] : 0.0f;
      }
      named_bar_sync(1, 128);
      const bool ok = mbar_wait(&acc_full[b], (j >> 1) & 1);
      if (!ok) atomicCAS(args.error, 0u, static_cast<unsigned>(kErrEpilogueTimeout));
      tc_fence_after();
      if (q * 32 < rows) {
        const uint32_t taddr =
            tmem_base + static_cast<uint32_t>(b * kWN) + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < kWN; c += 16) {
          uint32_t r[16];
          tmem_ld_x16(taddr + c, r);
          tmem_ld_wait();
          if (ok && row < rows)
            epi_run<16>(args, m_base + row, n_base + c, reinterpret_cast<const float*>(r),
                        bias_s + c, gate_s + c);
        }
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (et == 0) mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kTmemCols);
  }
}

// CTA x = (tile, split) with the split index fastest (one cluster = the splits
// of one output tile) and the token tile next, so the CTAs that share a weight
// tile run side by side and the weight tile is read from HBM once.
__global__ void __launch_bounds__(kThreadsQ8, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = args.stages;
  const uint32_t a_bytes = static_cast<uint32_t>(args.a_rows) * kBK * 2;
  // Token stages first: a UMMA reads 128 token rows from every stage, so the
  // rows past a short tile must land in (unused) shared memory that follows.
  const bool q8 = args.w_q8 != nullptr;
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + S * a_bytes;
  uint8_t* smem_q8 = smem_w + S * kBBytes;  // Q8_0 stages (q8 only)
  uint8_t* tail = smem_q8 + (q8 ? S * kQ8TileBytes : 0);
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + S;
  uint64_t* conv = empty + S;  // q8: BF16 weights of the stage are ready
  uint64_t* accum = conv + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* ok_flag = last_flag + 1;
  float* bias_s = reinterpret_cast<float*>(tail + 256);
  float* gate_s = bias_s + kWN;
  float* partial = reinterpret_cast<float*>(smem);  // reuses the stages after the mainloop

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x % args.splits;
  const int tile = blockIdx.x / args.splits;
  const int tile_m = tile % args.tiles_m;
  const int tile_n = tile / args.tiles_m;
  const int kb0 = static_cast<int>((static_cast<long long>(split) * args.num_kb) / args.splits);
  const int kb1 =
      static_cast<int>((static_cast<long long>(split + 1) * args.num_kb) / args.splits);
  const int nkb = kb1 - kb0;
  const int m_base = tile_m * kTM;
  const int rows = args.m - m_base < kTM ? args.m - m_base : kTM;  // valid token rows
  const bool m64 = args.a_rows <= 64;  // token tile of <= 64 rows: M = 64 UMMAs
  const int n_base = tile_n * kWN;
  const bool cluster_mode = args.splits > 1 && args.split_mode != SPLIT_WORKSPACE;
  const bool global_xchg = args.split_mode == SPLIT_CLUSTER_GLOBAL;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Let the next kernel in the stream start its own set-up now; it waits for
  // this grid's completion before touching anything this grid writes.
  griddep_launch_dependents();

  bool ok = true;
  // Q8_0 -> BF16 of every stage of the mainloop by warps 2.. (ct = 0 ..
  // conv_threads - 1; the Q8_0 launch has kThreadsQ8 threads):
  // 16 weights (half a Q8_0 block, one scale) per thread and step, two 16-byte
  // swizzled chunks of the UMMA operand row. value = q * d exactly: the byte
  // becomes the float 2^23 + (q + 128) through a byte permute; subtracting
  // 2^23 + 128 leaves q (exact, integers below 2^24), and q * d is exact in F32
  // (8 + 11 significant bits); then rounded to BF16.
  const int conv_threads = static_cast<int>(blockDim.x) - 64;
  auto q8_convert_stages = [&](int ct) {
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!mbar_wait(&full[s], ph)) {
        atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
        break;
      }
      const uint8_t* raw = smem_q8 + s * kQ8TileBytes;
      uint8_t* wst = smem_w + s * kBBytes;
#pragma unroll 2
      for (int it = ct; it < kWN * 4; it += conv_threads) {
        const int r = it >> 2, c2 = it & 3;
        const uint4 qv = *reinterpret_cast<const uint4*>(raw + r * 64 + c2 * 16);
        const float d = __half2float(
            *reinterpret_cast<const __half*>(raw + 16384 + r * 4 + (c2 >> 1) * 2));
        const uint32_t qw[4] = {qv.x ^ 0x80808080u, qv.y ^ 0x80808080u, qv.z ^ 0x80808080u,
                                qv.w ^ 0x80808080u};
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t word = qw[j >> 1];
          const uint32_t sel0 = 0x7540u | (2 * (j & 1));
          const uint32_t sel1 = 0x7540u | (2 * (j & 1) + 1);
          const float f0 = __uint_as_float(__byte_perm(word, 0x4B000000u, sel0));
          const float f1 = __uint_as_float(__byte_perm(word, 0x4B000000u, sel1));
          // (f - (2^23 + 128)) * d for both values with packed F32 pairs (each
          // lane rounds as the scalar subtract and multiply would)
          const float2 qd = __fmul2_rn(__fadd2_rn(make_float2(f0, f1), make_float2(-8388736.0f, -8388736.0f)),
                                       make_float2(d, d));
          const __nv_bfloat162 h = __floats2bfloat162_rn(qd.x, qd.y);
          o[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
        const int ca = 2 * c2, cb = 2 * c2 + 1;
        *reinterpret_cast<uint4*>(wst + r * 128 + ((ca ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(wst + r * 128 + ((cb ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();  // generic-proxy writes -> the tensor cores' async proxy
      named_bar_sync(2, conv_threads);
      if (ct == 0) mbar_arrive(&conv[s]);
    }
  };
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = WAM_GEMM_WEIGHT_EVICT_FIRST ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_x = policy_evict_last();
      const uint32_t stage_tx = a_bytes + (q8 ? kQ8TileBytes : kBBytes);
      const bf16* w_tiles =
          args.w_tiled ? args.w_tiled + static_cast<size_t>(tile_n) * args.num_kb * (kWN * kBK)
                       : nullptr;
      auto load_w = [&](int stage, int kb) {
        if (q8)
          bulk_load(smem_q8 + stage * kQ8TileBytes,
                    args.w_q8 + (static_cast<size_t>(tile_n) * args.num_kb + kb) * kQ8TileBytes,
                    kQ8TileBytes, &full[stage], pol_w);
        else if (w_tiles)
          bulk_load(smem_w + stage * kBBytes, w_tiles + static_cast<size_t>(kb) * (kWN * kBK),
                    kBBytes, &full[stage], pol_w);
        else
          tma_load_2d(smem_w + stage * kBBytes, &tm_w, &full[stage], kb * kBK, n_base, pol_w);
      };
      const int pre = nkb < S ? nkb : S;
      // Weights never depend on the preceding kernel: the first pre_w stages'
      // weight copies start before waiting for it (programmatic dependent
      // launch). The copies of one SM complete roughly in issue order, so the
      // remaining first-round copies alternate token / weight by stage.
      const int pre_w = pre < args.pre_w ? pre : args.pre_w;
      for (int i = 0; i < pre_w; ++i) {
        mbar_arrive_expect_tx(&full[i], stage_tx);
        load_w(i, kb0 + i);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i) {
        if (i >= pre_w) mbar_arrive_expect_tx(&full[i], stage_tx);
        tma_load_2d(smem_a + i * a_bytes, &tm_x, &full[i], (kb0 + i) * kBK, m_base, pol_x);
        if (i >= pre_w) load_w(i, kb0 + i);
      }
      for (int i = pre; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrProducerTimeout));
          break;
        }
        mbar_arrive_expect_tx(&full[s], stage_tx);
        load_w(s, kb0 + i);
        tma_load_2d(smem_a + s * a_bytes, &tm_x, &full[s], (kb0 + i) * kBK, m_base, pol_x);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Token tiles of <= 64 rows run M = 64 UMMAs: half the tensor-core work
      // per weight k-block of an M = 128 instruction on the same 256 features.
      const uint32_t idesc = umma_idesc_bf16(m64 ? 64 : kTM, kWN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(q8 ? &conv[s] : &full[s], ph)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
          break;
        }
        tc_fence_after();
        const uint64_t da = sw128_kmajor_desc(smem_u32(smem_a + s * a_bytes));
        const uint64_t db = sw128_kmajor_desc(smem_u32(smem_w + s * kBBytes));
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          // +32 bytes along K inside the swizzle row = +2 in the 16-byte address field.
          umma_bf16_ss(tmem_base, da + 2 * k, db + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else if (warp >= 6) {
    if (q8) q8_convert_stages(threadIdx.x - 64);
  } else {
    // Epilogue warps 2..5. Per-feature bias / gate of this tile go to shared
    // memory while the mainloop runs.
    griddep_wait();  // residual / gate / outputs are touched only after the preceding kernel
    const int et = threadIdx.x - 64;
    for (int j = et; j < kWN; j += 128) {
      const int n = n_base + j;
      bias_s[j] = (args.bias && n < args.n) ? __bfloat162float(args.bias[n]) : 0.0f;
      gate_s[j] = (args.gate && n < args.n) ? args.gate[n] : 0.0f;
    }
    named_bar_sync(1, 128);
    if (q8) q8_convert_stages(threadIdx.x - 64);
    ok = mbar_wait(accum, 0);
    if (!ok) atomicCAS(args.error, 0u, static_cast<unsigned>(kErrEpilogueTimeout));
    tc_fence_after();
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    // M = 128: token q*32 + lane in lane q*32 + lane. M = 64: tokens 16q..16q+15
    // in lanes 32q..32q+15 of the quadrant (lanes 16-31 hold nothing).
    const int row = m64 ? q * 16 + (lane & 15) : q * 32 + lane;
    const bool lane_ok = !m64 || lane < 16;
    const bool warp_rows = (m64 ? q * 16 : q * 32) < rows;  // warp-uniform: tcgen05.ld is warp-collective
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    if (args.splits == 1) {
      uint8_t* stg = smem;  // the stages are free once the accumulator is complete
      if (warp_rows) {
        // The TMEM load of the next 16 columns is in flight while this chunk
        // is staged.
        const bool st = lane_ok && row < rows;
        uint32_t r0[16], r1[16];
        tmem_ld_x16(taddr, r0);
        tmem_ld_wait();
#pragma unroll 1
        for (int c = 0; c < kWN; c += 32) {
          tmem_ld_x16(taddr + c + 16, r1);
          if (st) stage16(args, stg, row, c, reinterpret_cast<const float*>(r0), bias_s + c);
          tmem_ld_wait();
          if (c + 32 < kWN) tmem_ld_x16(taddr + c + 32, r0);
          if (st)
            stage16(args, stg, row, c + 16, reinterpret_cast<const float*>(r1), bias_s + c + 16);
          tmem_ld_wait();
        }
      }
      named_bar_sync(1, 128);
      if (ok) copy_out(args, stg, rows, m_base, n_base, gate_s, et, 128);
    } else if (cluster_mode && global_xchg) {
      // Partial tile as [16-feature chunk][token][16] F32 in the workspace. Full
      // 128-token tiles stage it in shared memory (the stages are free once the
      // accumulator is complete) and write it with one bulk copy (768 x 3072 x
      // 3072: 26.3 -> 24.8 us); short tiles store straight from the TMEM loads
      // (a warp writes 2 KB contiguous), which measured faster for them.
      const size_t tile_floats = static_cast<size_t>(args.a_rows) * kWN;
      float* ws = args.workspace + (static_cast<size_t>(tile) * args.splits + split) * tile_floats;
      const bool staged = args.a_rows == kTM;
      float* dst_base = staged ? reinterpret_cast<float*>(smem) : ws;
      if (warp_rows) {
        const bool st = lane_ok && row < rows;
#pragma unroll 1
        for (int c = 0; c < kWN; c += 32) {
          uint32_t r[32];
          tmem_ld_x32(taddr + c, r);
          tmem_ld_wait();
          if (st) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float4* d = reinterpret_cast<float4*>(
                  dst_base + (static_cast<size_t>(c / 16 + h) * args.a_rows + row) * 16);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                d[j] = make_float4(__uint_as_float(r[16 * h + 4 * j]), __uint_as_float(r[16 * h + 4 * j + 1]),
                                   __uint_as_float(r[16 * h + 4 * j + 2]), __uint_as_float(r[16 * h + 4 * j + 3]));
            }
          }
        }
      }
      if (staged) {
        fence_proxy_async_smem();  // the staged tile (generic writes) is read by the bulk copy
        named_bar_sync(1, 128);
      }
      if (threadIdx.x == 64) {
        if (staged) {
          bulk_store(ws, dst_base, static_cast<uint32_t>(tile_floats * 4));
          bulk_commit();
          bulk_wait_all();
          fence_proxy_async_global();  // before the cluster barrier's release
        }
        *ok_flag = ok ? 1 : 0;
      }
    } else if (cluster_mode) {
      // Stage this split's F32 partial tile [token][feature] in shared memory.
      if (warp_rows) {
#pragma unroll 1
        for (int c = 0; c < kWN; c += 16) {
          uint32_t r[16];
          tmem_ld_x16(taddr + c, r);
          tmem_ld_wait();
          if (lane_ok && row < rows) {
            float4* dst = reinterpret_cast<float4*>(partial + row * kPartLd + c);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          }
        }
      }
    } else {
      // Workspace mode: partial tile to global memory; the last CTA of the tile
      // to arrive reduces all partials in split order and runs the epilogue.
      const size_t tile_floats = static_cast<size_t>(args.a_rows) * kWN;
      float* ws_tile = args.workspace + static_cast<size_t>(tile) * args.splits * tile_floats;
      float* ws = ws_tile + static_cast<size_t>(split) * tile_floats;
      if (warp_rows) {
#pragma unroll 1
        for (int c = 0; c < kWN; c += 16) {
          uint32_t r[16];
          tmem_ld_x16(taddr + c, r);
          tmem_ld_wait();
          if (lane_ok && row < rows) {
            float4* dst = reinterpret_cast<float4*>(ws + row * kWN + c);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          }
        }
      }
      __threadfence();
      named_bar_sync(1, 128);
      if (et == 0) {
        const unsigned prev = atomicAdd(&args.counters[tile], 1u);
        *last_flag = (prev == static_cast<unsigned>(args.splits - 1)) ? 1 : 0;
      }
      named_bar_sync(1, 128);
      if (*last_flag) {
        __threadfence();
        const int items = rows * (kWN / 8);
        for (int it = et; it < items; it += 128) {
          const int rr = it / (kWN / 8), g = it % (kWN / 8);
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
          for (int sp = 0; sp < args.splits; ++sp) {
            const float4* src = reinterpret_cast<const float4*>(
                ws_tile + sp * tile_floats + static_cast<size_t>(rr) * kWN + g * 8);
            const float4 x0 = __ldcg(src), x1 = __ldcg(src + 1);
            acc[0] += x0.x; acc[1] += x0.y; acc[2] += x0.z; acc[3] += x0.w;
            acc[4] += x1.x; acc[5] += x1.y; acc[6] += x1.z; acc[7] += x1.w;
          }
          if (ok) epi_run<8>(args, m_base + rr, n_base + g * 8, acc, bias_s + g * 8, gate_s + g * 8);
        }
        if (et == 0) args.counters[tile] = 0u;
      }
    }
  }

  __syncwarp();
  if (cluster_mode && global_xchg) {
    // Every split's partial tile is in the workspace: each CTA reduces a
    // slice of (16-feature chunk, token) items over all splits, in split
    // order; consecutive threads read consecutive 64-byte token rows.
    cluster_sync_all();
    {
      // All threads: one (16-feature chunk, token, half) item each pass.
      const bool ok_all = *ok_flag != 0;
      const int sp_n = args.splits;
      const int items = rows * (kWN / 8);
      const int i0 = static_cast<int>((static_cast<long long>(split) * items) / sp_n);
      const int i1 = static_cast<int>((static_cast<long long>(split + 1) * items) / sp_n);
      const size_t tile_floats = static_cast<size_t>(args.a_rows) * kWN;
      const float* ws_tile = args.workspace + static_cast<size_t>(tile) * sp_n * tile_floats;
      for (int it = i0 + static_cast<int>(threadIdx.x); it < i1; it += static_cast<int>(blockDim.x)) {
        const int c = it / (2 * rows), rem = it % (2 * rows);
        const int rr = rem >> 1, h = rem & 1;
        const float* src0 = ws_tile + (static_cast<size_t>(c) * args.a_rows + rr) * 16 + h * 8;
        float4 x[8][2];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          if (p < sp_n) {
            const float4* src = reinterpret_cast<const float4*>(src0 + p * tile_floats);
            x[p][0] = __ldcg(src);
            x[p][1] = __ldcg(src + 1);
          }
        }
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          if (p < sp_n) {
            acc[0] += x[p][0].x; acc[1] += x[p][0].y; acc[2] += x[p][0].z; acc[3] += x[p][0].w;
            acc[4] += x[p][1].x; acc[5] += x[p][1].y; acc[6] += x[p][1].z; acc[7] += x[p][1].w;
          }
        }
        const int f = c * 16 + h * 8;
        if (ok_all) epi_run<8>(args, m_base + rr, n_base + f, acc, bias_s + f, gate_s + f);
      }
    }
  } else if (cluster_mode) {
    // All partial tiles of this output tile are in the cluster's shared memory.
    cluster_sync_all();
    if (warp >= 2 && warp < 6) {
      const int et = threadIdx.x - 64;
      const int sp_n = args.splits;
      const int items = rows * (kWN / 8);
      const int i0 = static_cast<int>((static_cast<long long>(split) * items) / sp_n);
      const int i1 = static_cast<int>((static_cast<long long>(split + 1) * items) / sp_n);
      const uint32_t base = smem_u32(partial);
      for (int it = i0 + et; it < i1; it += 128) {
        const int rr = it / (kWN / 8), g = it % (kWN / 8);
        const uint32_t off = static_cast<uint32_t>(rr * kPartLd + g * 8) * 4u;
        // All peers' loads are issued before any is summed (each DSMEM load
        // is a round trip); the sum runs in split order.
        float4 x[8][2];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          if (p < sp_n) {
            const uint32_t pa = mapa_shared(base + off, static_cast<uint32_t>(p));
            x[p][0] = ld_shared_cluster_f32x4(pa);
            x[p][1] = ld_shared_cluster_f32x4(pa + 16);
          }
        }
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          if (p < sp_n) {
            acc[0] += x[p][0].x; acc[1] += x[p][0].y; acc[2] += x[p][0].z; acc[3] += x[p][0].w;
            acc[4] += x[p][1].x; acc[5] += x[p][1].y; acc[6] += x[p][1].z; acc[7] += x[p][1].w;
          }
        }
        if (ok) epi_run<8>(args, m_base + rr, n_base + g * 8, acc, bias_s + g * 8, gate_s + g * 8);
      }
    }
    // No CTA leaves while a peer may still read its shared memory.
    cluster_sync_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------ streaming GEMM
// Token tiles of <= 64 rows (the batch-1 denoise step and the prefix state
// token): every CTA owns NT = 32, 64 or 128 output features (a divisor of the
// 256-row weight tile) over the whole K, so no CTA's partial sums ever leave
// it. Each pipeline stage holds KB consecutive k-blocks of both operands,
// fetched by one 3-D TMA box each: weights from the re-tiled layout viewed as
// [N/256][K/64][256][64] (rows n0 % 256 .. + NT of tile n0 / 256, pre-swizzled,
// copied verbatim) or a row-major [N][K] weight with the 128-byte swizzle;
// tokens as [K/64][rows][64] with the 128-byte swizzle. UMMA M = 64 (token
// rows in TMEM lanes 0-15 of each quadrant), N = NT, K = 16. The epilogue
// applies the fused bias / activation / residual per row straight from TMEM.
constexpr int kStreamBudget = 200 * 1024;

int stream_stage_bytes(int a_rows, int nt, int kb) { return kb * (a_rows + nt) * kBK * 2; }

__global__ void __launch_bounds__(kThreads, 1)
    gemm_stream_kernel(const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = args.stages, NT = args.nt, KB = args.kb;
  const uint32_t a_bytes = static_cast<uint32_t>(KB * args.a_rows * kBK * 2);
  const uint32_t w_bytes = static_cast<uint32_t>(KB * NT * kBK * 2);
  const uint32_t stage = a_bytes + w_bytes;
  uint8_t* tail = smem + S * stage;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  float* bias_s = reinterpret_cast<float*>(tail + 256);
  float* gate_s = bias_s + 128;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * NT;
  const int rows = args.m < 64 ? args.m : 64;
  const int nst = args.num_kb / KB;  // stages of work (num_kb % KB == 0)
  const uint32_t tcols = NT < 32 ? 32 : NT;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = WAM_GEMM_WEIGHT_EVICT_FIRST ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_x = policy_evict_last();
      const bool tiled = args.w_tiled != nullptr;
      auto load_w = [&](int s, int j) {
        uint8_t* dst = smem + s * stage + a_bytes;
        if (tiled)
          tma_load_4d(dst, &tm_w, &full[s], 0, n0 % kWN, j * KB, n0 / kWN, pol_w);
        else
          tma_load_3d(dst, &tm_w, &full[s], 0, n0, j * KB, pol_w);
      };
      const int pre = nst < S ? nst : S;
      const int pre_w = pre < args.pre_w ? pre : args.pre_w;
      for (int j = 0; j < pre_w; ++j) {
        mbar_arrive_expect_tx(&full[j], stage);
        load_w(j, j);
      }
      griddep_wait();  // tokens come from the preceding kernel
      for (int j = 0; j < pre; ++j) {
        if (j >= pre_w) mbar_arrive_expect_tx(&full[j], stage);
        tma_load_3d(smem + j * stage, &tm_x, &full[j], 0, 0, j * KB, pol_x);
        if (j >= pre_w) load_w(j, j);
      }
      for (int j = pre; j < nst; ++j) {
        const int s = j % S;
        if (!mbar_wait(&empty[s], ((j / S) & 1) ^ 1)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrProducerTimeout));
          break;
        }
        mbar_arrive_expect_tx(&full[s], stage);
        load_w(s, j);
        tma_load_3d(smem + s * stage, &tm_x, &full[s], 0, 0, j * KB, pol_x);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(64, NT);
      for (int j = 0; j < nst; ++j) {
        const int s = j % S;
        if (!mbar_wait(&full[s], (j / S) & 1)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
          break;
        }
        tc_fence_after();
        for (int b = 0; b < KB; ++b) {
          const uint64_t da = sw128_kmajor_desc(smem_u32(smem + s * stage + b * args.a_rows * 128));
          const uint64_t db = sw128_kmajor_desc(smem_u32(smem + s * stage + a_bytes + b * NT * 128));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16_ss(tmem_base, da + 2 * k, db + 2 * k, idesc, (j | b | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else if (warp < 6) {
    griddep_wait();  // residual / gate / outputs are touched only after the preceding kernel
    const int et = threadIdx.x - 64;
    for (int jj = et; jj < NT; jj += 128) {
      const int n = n0 + jj;
      bias_s[jj] = (args.bias && n < args.n) ? __bfloat162float(args.bias[n]) : 0.0f;
      gate_s[jj] = (args.gate && n < args.n) ? args.gate[n] : 0.0f;
    }
    named_bar_sync(1, 128);
    const bool ok = mbar_wait(accum, 0);
    if (!ok) atomicCAS(args.error, 0u, static_cast<unsigned>(kErrEpilogueTimeout));
    tc_fence_after();
    const int q = warp & 3;
    const int row = q * 16 + (lane & 15);  // M = 64: rows 16q.. in lanes 32q..32q+15
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    if (q * 16 < rows) {
#pragma unroll 1
      for (int c = 0; c < NT; c += 16) {
        uint32_t r[16];
        tmem_ld_x16(taddr + c, r);
        tmem_ld_wait();
        if (ok && lane < 16 && row < rows)
          epi_run<16>(args, row, n0 + c, reinterpret_cast<const float*>(r), bias_s + c, gate_s + c);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
}

// ------------------------------------------------------------ CTA-pair GEMM
// Tensor-bound GEMMs (>= 256 token rows: the prefix, prompt and batched
// GEMMs) run on CTA pairs with tcgen05.mma.cta_group::2: one UMMA covers 256
// tokens x 256 features, each CTA holding 128 token rows and 128 of the 256
// weight rows of every k-block (16 + 16 KB per stage instead of 16 + 32 KB).
// At the same shared memory that is six stages instead of four and a third
// less data per SM per UMMA. The one-CTA kernel measured at 45% tensor-pipe
// activity with the L2 -> SM crossbar at a third of its peak: its copies are
// latency bound (bytes in flight per SM), which this layout relieves.
//
// Roles as in gemm_tc_persistent_kernel; in addition the leader (even CTA)
// issues every UMMA of the pair, both CTAs' copies complete on the leader's
// stage barriers (cta_group::2 TMA), and the leader's commits arrive on the
// stage / accumulator barriers of both CTAs (multicast commit). The leader's
// accumulator-empty barriers count both CTAs' epilogues.
// Clusters of 2 * splits CTAs: rank = split * 2 + half. splits == 1: the
// cluster (one pair) loops over pair tiles (persistent). splits > 1: one pair
// tile per cluster; each pair sums a K range and the partial tiles meet in
// the caller's workspace, as in the SPLIT_CLUSTER_GLOBAL mode of gemm_tc_kernel.
constexpr int kPairRows = 128;                              // token rows per CTA
constexpr uint32_t kPairA = kPairRows * kBK * 2;            // 16 KB
constexpr uint32_t kPairB = (kWN / 2) * kBK * 2;            // 16 KB
constexpr uint32_t kPairStage = kPairA + kPairB;
constexpr uint32_t kPairTmemCols = 2 * kWN;                 // two accumulators

int pair_stages() {
  const int st = kStageBudget / static_cast<int>(kPairStage);
  return st > kMaxStages ? kMaxStages : st;
}
int pair_smem() { return pair_stages() * static_cast<int>(kPairStage) + 1024 + kSmemTail; }

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = args.stages;
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + S * kPairA;
  uint8_t* tail = smem_w + S * kPairB;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);  // leader's count both CTAs' copies
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;      // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2], leader's: both CTAs' epilogues
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* ok_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* bias_s = reinterpret_cast<float*>(tail + 256);
  float* gate_s = bias_s + kWN;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int half = static_cast<int>(crank & 1u);
  const int split = static_cast<int>(crank >> 1);
  const bool leader = half == 0;
  const uint32_t lead_rank = crank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << lead_rank);
  const int csize = 2 * args.splits;
  const int cl = blockIdx.x / csize, ncl = gridDim.x / csize;
  const int tiles = args.tiles_m * args.tiles_n;  // pair tiles (256 tokens x 256 features)
  const int kb0 = static_cast<int>((static_cast<long long>(split) * args.num_kb) / args.splits);
  const int kb1 = static_cast<int>((static_cast<long long>(split + 1) * args.num_kb) / args.splits);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2);
    }
    *ok_flag = 1;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kPairTmemCols);
    tmem_relinquish_pair();
  }
  __syncwarp();  // warp 0 reconverges after thread 0's set-up: the cluster barrier is .aligned
  tc_fence_before();
  cluster_sync_all();  // the peer's barriers exist before any copy or commit reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = WAM_GEMM_WEIGHT_EVICT_FIRST ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_x = policy_evict_last();
      const uint32_t full_lead = mapa_shared(smem_u32(full), lead_rank);
      int g = 0;
      bool waited = false, good = true;
      for (int t = cl; t < tiles && good; t += ncl) {
        int tile_m, tile_n;
        tile_coords(args, t, tile_m, tile_n);
        const int m_row = tile_m * (2 * kPairRows) + half * kPairRows;
        for (int i = 0; i < nkb; ++i, ++g) {
          const int s = g % S;
          if (g >= S && !mbar_wait(&empty[s], ((g / S) & 1) ^ 1)) {
            atomicCAS(args.error, 0u, static_cast<unsigned>(kErrProducerTimeout));
            good = false;
            break;
          }
          const uint32_t fb = full_lead + static_cast<uint32_t>(s) * 8u;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * kPairStage);
          const int kb = kb0 + i;
          // Re-tiled weights: row ((tile_n * K/64 + kb) * 256 + half * 128) of the
          // [N * K / 64][64] view, 128 pre-swizzled rows copied verbatim.
          if (args.w_tiled)
            tma_load_2d_pair(smem_w + s * kPairB, &tm_w, fb, 0,
                             (tile_n * args.num_kb + kb) * kWN + half * (kWN / 2), pol_w);
          else
            tma_load_2d_pair(smem_w + s * kPairB, &tm_w, fb, kb * kBK,
                             tile_n * kWN + half * (kWN / 2), pol_w);
          if (!waited) {  // weights first; the tokens come from the preceding kernel
            griddep_wait();
            waited = true;
          }
          tma_load_2d_pair(smem_a + s * kPairA, &tm_x, fb, kb * kBK, m_row, pol_x);
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(2 * kPairRows, kWN);
      int g = 0, j = 0;
      bool good = true;
      for (int t = cl; t < tiles && good; t += ncl, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait_cluster(&acc_empty[b], ((j >> 1) - 1) & 1)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + static_cast<uint32_t>(b * kWN);
        for (int i = 0; i < nkb; ++i, ++g) {
          const int s = g % S;
          if (!mbar_wait(&full[s], (g / S) & 1)) {
            atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
            good = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_kmajor_desc(smem_u32(smem_a + s * kPairA));
          const uint64_t db = sw128_kmajor_desc(smem_u32(smem_w + s * kPairB));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16_ss_pair(acc, da + 2 * k, db + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
          umma_commit_pair_mc(&empty[s], pair_mask);
        }
        if (good) umma_commit_pair_mc(&acc_full[b], pair_mask);
      }
    }
  } else if (warp < 6) {
    griddep_wait();  // residual / gate / outputs are touched only after the preceding kernel
    const int et = threadIdx.x - 64;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t acc_empty_lead = mapa_shared(smem_u32(acc_empty), lead_rank);
    int j = 0;
    for (int t = cl; t < tiles; t += ncl, ++j) {
      const int b = j & 1;
      int tile_m, tile_n;
      tile_coords(args, t, tile_m, tile_n);
      const int m_base = tile_m * (2 * kPairRows) + half * kPairRows, n_base = tile_n * kWN;
      int rows = args.m - m_base;
      rows = rows < 0 ? 0 : (rows > kPairRows ? kPairRows : rows);
      named_bar_sync(1, 128);  // the previous tile's bias / gate are no longer read
      for (int jj = et; jj < kWN; jj += 128) {
        const int n = n_base + jj;
        bias_s[jj] = (args.bias && n < args.n) ? __bfloat162float(args.bias[n]) : 0.0f;
        gate_s[jj] = (args.gate && n < args.n) ? args.gate[n] : 0.0f;
      }
      named_bar_sync(1, 128);
      const bool ok = mbar_wait(&acc_full[b], (j >> 1) & 1);
      if (!ok) atomicCAS(args.error, 0u, static_cast<unsigned>(kErrEpilogueTimeout));
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(b * kWN) + (static_cast<uint32_t>(q * 32) << 16);
      if (args.splits == 1) {
        if (q * 32 < rows) {
#pragma unroll 1
          for (int c = 0; c < kWN; c += 16) {
            uint32_t r[16];
            tmem_ld_x16(taddr + c, r);
            tmem_ld_wait();
            if (ok && row < rows)
              epi_run<16>(args, m_base + row, n_base + c, reinterpret_cast<const float*>(r),
                          bias_s + c, gate_s + c);
          }
        }
      } else {
        // Partial tile [16-feature chunk][token][16] of (pair tile, half, split).
        const size_t tile_floats = static_cast<size_t>(kPairRows) * kWN;
        float* ws = args.workspace +
                    ((static_cast<size_t>(t) * 2 + half) * args.splits + split) * tile_floats;
        if (q * 32 < rows) {
#pragma unroll 1
          for (int c = 0; c < kWN; c += 32) {
            uint32_t r[32];
            tmem_ld_x32(taddr + c, r);
            tmem_ld_wait();
            if (row < rows) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                float4* d = reinterpret_cast<float4*>(
                    ws + (static_cast<size_t>(c / 16 + h) * kPairRows + row) * 16);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
                  d[jj] = make_float4(__uint_as_float(r[16 * h + 4 * jj]),
                                      __uint_as_float(r[16 * h + 4 * jj + 1]),
                                      __uint_as_float(r[16 * h + 4 * jj + 2]),
                                      __uint_as_float(r[16 * h + 4 * jj + 3]));
              }
            }
          }
        }
        if (!ok && et == 0) *ok_flag = 0;
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (et == 0) mbar_arrive_cluster(acc_empty_lead + static_cast<uint32_t>(b) * 8u);
      if (!ok) break;
    }
  }

  __syncwarp();
  if (args.splits > 1) {
    // Every split's partial tile is in the workspace (cluster barrier =
    // release / acquire): each CTA reduces its slice of its half's items over
    // the splits, in split order, and runs the epilogue.
    cluster_sync_all();
    const int t = cl;
    if (t < tiles) {
      int tile_m, tile_n;
      tile_coords(args, t, tile_m, tile_n);
      const int m_base = tile_m * (2 * kPairRows) + half * kPairRows, n_base = tile_n * kWN;
      int rows = args.m - m_base;
      rows = rows < 0 ? 0 : (rows > kPairRows ? kPairRows : rows);
      const bool ok_all = *ok_flag != 0;
      const int sp_n = args.splits;
      const int items = rows * (kWN / 8);
      const int i0 = static_cast<int>((static_cast<long long>(split) * items) / sp_n);
      const int i1 = static_cast<int>((static_cast<long long>(split + 1) * items) / sp_n);
      const size_t tile_floats = static_cast<size_t>(kPairRows) * kWN;
      const float* ws_tile =
          args.workspace + (static_cast<size_t>(t) * 2 + half) * sp_n * tile_floats;
      for (int it = i0 + static_cast<int>(threadIdx.x); it < i1; it += kThreads) {
        const int c = it / (2 * rows), rem = it % (2 * rows);
        const int rr = rem >> 1, h = rem & 1;
        const float* src0 = ws_tile + (static_cast<size_t>(c) * kPairRows + rr) * 16 + h * 8;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int p = 0; p < sp_n; ++p) {
          const float4* src = reinterpret_cast<const float4*>(src0 + p * tile_floats);
          const float4 x0 = __ldcg(src), x1 = __ldcg(src + 1);
          acc[0] += x0.x; acc[1] += x0.y; acc[2] += x0.z; acc[3] += x0.w;
          acc[4] += x1.x; acc[5] += x1.y; acc[6] += x1.z; acc[7] += x1.w;
        }
        const int f = c * 16 + h * 8;
        if (ok_all) epi_run<8>(args, m_base + rr, n_base + f, acc, bias_s + f, gate_s + f);
      }
    }
  }

  // No CTA frees its TMEM while its peer's UMMAs or epilogue may still use it.
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kPairTmemCols);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D BF16 tensor map over a row-major [rows, cols] matrix with row stride ld
// (elements), box = 64 x box_rows, 128-byte swizzle, zero fill out of bounds.
bool encode_bf16_2d(CUtensorMap* map, const void* base, int cols, int rows, int ld,
                    int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Resident CTA slots for a split-K cluster size s (index s = 1..8): clusters
// are placed inside one GPC, so s-wide clusters of one-CTA-per-SM kernels fit
// floor(SMs per GPC / s) times per GPC. Filled by gemm_init from
// cudaOccupancyMaxActiveClusters.
int g_cluster_slots[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};

// Split-K factor (1..8 = cluster size). Output tiles that fill less than
// three quarters of the SMs split K as far as one wave of clusters allows
// (>= 2 k-blocks per split): the batch-1 denoise GEMMs (48 tokens, 12..56
// tiles of 256 features) stream their weights from 96..144 SMs instead of
// 12..56.
int pick_splits(int tiles, int nkb, int num_sms) {
  if (tiles * 4 >= num_sms * 3) return 1;
  int best = 1;
  for (int s = 2; s <= 8; ++s) {
    const int slots = g_cluster_slots[s] > 0 ? g_cluster_slots[s] : num_sms;
    if (tiles * s <= slots && nkb / s >= 2) best = s;
  }
  return best;
}

bool g_pdl = [] {
  const char* v = std::getenv("WAM_B200_DISABLE_PDL");
  return !(v && *v && *v != '0');
}();

// CTA-pair kernel choice (WAM_B200_GEMM_PAIR): unset = automatic, for GEMMs
// of >= 256 token rows whose 256 x 256 pair tiles occupy at least half of the
// resident pairs (measured in CUDA-graph replay: 768 x 14336 x 3072 61.4 vs
// 62.7 us, 768 x 9216 x 3072 43.0 vs 44.1, the 64-request prefix 471 vs 495 ms;
// fewer tiles leave SMs idle that the one-CTA kernel's split-K fills:
// 768 x 3072 x 14336 87.9 vs 62.7 us); 1 = every GEMM of >= 256 rows; 0 =
// never. A caller can also ask for it per GEMM (gemm_plan's pair argument).
int g_pair_mode = [] {
  const char* v = std::getenv("WAM_B200_GEMM_PAIR");
  if (v && *v == '1') return 1;
  if (v && *v == '0') return 0;
  return 2;
}();
// Streaming GEMM (no split-K) for token tiles of <= 64 rows and N >= 1536
// (default); WAM_B200_GEMM_STREAM=0 keeps such GEMMs on the split-K kernel,
// WAM_B200_GEMM_STREAM_NT=32|64|128 fixes the features per CTA.
bool g_stream = [] {
  const char* v = std::getenv("WAM_B200_GEMM_STREAM");
  return !(v && *v == '0');
}();
int g_stream_nt = [] {
  const char* v = std::getenv("WAM_B200_GEMM_STREAM_NT");
  const int n = v ? std::atoi(v) : 0;
  return n == 32 || n == 64 || n == 128 ? n : 0;
}();
// Stages whose weight copies a GEMM CTA issues before waiting for the
// preceding kernel (WAM_B200_GEMM_PREW, default 2).
int g_pre_w = [] {
  const char* v = std::getenv("WAM_B200_GEMM_PREW");
  const int n = v ? std::atoi(v) : 2;
  return n < 0 ? 0 : (n > kMaxStages ? kMaxStages : n);
}();

// Kernel and split-K choice of one GEMM shape. Pair tiles (256 tokens x 256
// features) that leave more than a quarter of the resident pairs idle split K
// over 2 or 4 pairs of one cluster (one wave of clusters, >= 4 k-blocks each)
// when the caller gives a workspace.
struct ShapeChoice {
  bool pair = false;
  int splits = 1;
  int tiles = 0;  // output tiles of the chosen kernel (pair tiles for the pair kernel)
};

ShapeChoice choose_shape(int m, int n, int k, int num_sms, int force_splits, bool w_q8,
                         bool workspace, bool want_pair) {
  ShapeChoice c;
  const int nkb = k / kBK;
  const int pair_tiles = ((m + 2 * kTM - 1) / (2 * kTM)) * ((n + kWN - 1) / kWN);
  const int pairs = g_cluster_slots[2] > 0 ? g_cluster_slots[2] / 2 : num_sms / 2;
  const bool pair_auto = g_pair_mode == 2 && 2 * pair_tiles >= pairs;
  if ((g_pair_mode == 1 || want_pair || pair_auto) && !w_q8 && force_splits <= 0 &&
      m >= 2 * kTM) {
    c.pair = true;
    c.tiles = pair_tiles;
    if (workspace && c.tiles * 4 < pairs * 3) {
      for (int s = 2; s <= 4; s *= 2) {
        const int clusters = g_cluster_slots[2 * s] > 0 ? g_cluster_slots[2 * s] / (2 * s)
                                                        : num_sms / (2 * s);
        if (c.tiles <= clusters && nkb / s >= 4) c.splits = s;
      }
    }
    return c;
  }
  c.tiles = ((m + kTM - 1) / kTM) * ((n + kWN - 1) / kWN);
  c.splits = force_splits > 0 ? force_splits : pick_splits(c.tiles, nkb, num_sms);
  if (c.splits > nkb) c.splits = nkb;
  return c;
}

// Token tiles per group of the persistent tile order (tile_coords): the
// group's token rows (tile_rows x K BF16) stay within 32 MB of L2, 1 to 16 tiles.
int group_m_for(int tile_rows, int k) {
  const long long tile_bytes = static_cast<long long>(tile_rows) * k * 2;
  long long g = (32ll << 20) / (tile_bytes > 0 ? tile_bytes : 1);
  return static_cast<int>(g < 1 ? 1 : (g > 16 ? 16 : g));
}

// One thread per 16-byte chunk: chunk c of row r of tile (nt, kb) goes to
// chunk c ^ (r & 7) of that row in the tile's contiguous 32 KB block.
__global__ void retile_weights_kernel(const bf16* __restrict__ src, bf16* __restrict__ dst, int n,
                                      int k) {
  griddep_wait();
  const int kbs = k / kBK;
  const long long total = static_cast<long long>(n) * (k / 8);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / (k / 8));
    const int cg = static_cast<int>(i % (k / 8));  // 8-element chunk along k
    const int kb = cg >> 3, c = cg & 7;
    const int nt = row / kWN, r = row % kWN;
    const size_t tile = (static_cast<size_t>(nt) * kbs + kb) * (kWN * kBK);
    const uint4 v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(row) * k + cg * 8);
    *reinterpret_cast<uint4*>(dst + tile + r * kBK + ((c ^ (r & 7)) * 8)) = v;
  }
}

}  // namespace

int gemm_weight_tile_rows() { return kWN; }

void launch_retile_weights(const bf16* src, bf16* dst, int n, int k, cudaStream_t s) {
  const long long total = static_cast<long long>(n) * (k / 8);
  long long grid = (total + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  retile_weights_kernel<<<static_cast<int>(grid), 256, 0, s>>>(src, dst, n, k);
}

size_t gemm_scratch_floats(int m, int n, int k, int num_sms, int force_splits, int* tiles_out) {
  const ShapeChoice c = choose_shape(m, n, k, num_sms, force_splits, false, true, false);
  if (tiles_out) *tiles_out = c.tiles;
  if (c.splits <= 1) return 0;
  if (c.pair) return static_cast<size_t>(c.tiles) * 2 * c.splits * kPairRows * kWN;
  return static_cast<size_t>(c.tiles) * c.splits * a_rows_for(m) * kWN;
}

namespace {

// Tensor map over re-tiled weights viewed as [N * K / 64][64] BF16 rows (the
// 128-byte swizzle is already in the data): box = 128 rows copied verbatim,
// half of one 256 x 64 tile.
bool encode_tiled_rows(CUtensorMap* map, const void* base, long long rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kBK), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kBK) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(kWN / 2)};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [N/256][K/64][256][64] view of re-tiled weights (pre-swizzled, copied
// verbatim): box = 64 x nt rows x kb k-blocks of one 256-row tile.
bool encode_tiled_stream(CUtensorMap* map, const void* base, int n, int k, int nt, int kb) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kBK), static_cast<cuuint64_t>(kWN),
                              static_cast<cuuint64_t>(k / kBK), static_cast<cuuint64_t>(n / kWN)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kBK) * 2,
                                 static_cast<cuuint64_t>(kWN) * kBK * 2,
                                 static_cast<cuuint64_t>(k / kBK) * kWN * kBK * 2};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(nt),
                             static_cast<cuuint32_t>(kb), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major [rows][ld] BF16 viewed as [cols / 64][rows][64] (128-byte swizzle):
// box = 64 x box_rows x kb k-blocks.
bool encode_kblocks(CUtensorMap* map, const void* base, int cols, int rows, int ld, int box_rows,
                    int kb) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kBK), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(cols / kBK)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, static_cast<cuuint64_t>(kBK) * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows),
                             static_cast<cuuint32_t>(kb)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Streaming plan: NT = 128 features per CTA when that still gives >= 96 CTAs
// (enough weight streams to fill HBM) and K <= 4096 (every CTA reads all of the
// token rows from L2); KB k-blocks per stage so a stage moves >= 24 KB, as many
// stages as the budget holds (>= 2). Measured on B200 (op cases, µs, streaming
// vs split-K): 48x14336x3072 19.7 vs 21.7 (NT 128, used); 48x3072x3072 14.2 vs
// 10.9 (NT 32), 48x9216x3072 18.7 vs 16.9 (NT 64), 48x3072x14336 49.7 vs 20.9
// (NT 32): narrower tiles lose to split-K, so they are not planned.
const char* plan_stream(GemmOp* op, const bf16* x, int ldx, int m, const bf16* w, int n, int k,
                        int epilogue, const bf16* bias, const float* gate, const bf16* residual,
                        int ldr, void* out, int ldo, const GemmScratch& scratch, int num_sms,
                        bool w_tiled) {
  (void)num_sms;
  int nt = 128;
  if (g_stream_nt > 0) {
    if (n % g_stream_nt != 0) return "stream: not applicable";
    nt = g_stream_nt;
  } else if (n % 128 != 0 || n / 128 < 96 || k > 4096) {
    return "stream: not applicable";
  }
  const int a_rows = a_rows_for(m);
  const int nkb = k / kBK;
  int kb = 1;
  while (kb < 8 && stream_stage_bytes(a_rows, nt, kb) < 24 * 1024 && nkb % (kb * 2) == 0) kb *= 2;
  int stages = kStreamBudget / stream_stage_bytes(a_rows, nt, kb);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2 || nkb % kb != 0) return "stream: not applicable";
  if (w_tiled) {
    if (!encode_tiled_stream(&op->tm_w, w, n, k, nt, kb)) return "gemm: weight tensor map encode failed";
  } else if (!encode_kblocks(&op->tm_w, w, k, n, k, nt, kb)) {
    return "gemm: weight tensor map encode failed";
  }
  if (!encode_kblocks(&op->tm_x, x, k, m, ldx, a_rows, kb))
    return "gemm: activation tensor map encode failed";
  GemmArgs& a = op->args;
  a.m = m;
  a.n = n;
  a.k = k;
  a.num_kb = nkb;
  a.splits = 1;
  a.split_mode = SPLIT_CLUSTER;
  a.a_rows = a_rows;
  a.stages = stages;
  a.pre_w = stages < g_pre_w ? stages : g_pre_w;
  a.nt = nt;
  a.kb = kb;
  a.w_tiled = w_tiled ? w : nullptr;
  a.w_q8 = nullptr;
  a.tiles_m = 1;
  a.tiles_n = n / nt;
  a.epilogue = epilogue;
  a.bias = bias;
  a.gate = gate;
  a.residual = residual;
  a.ldr = ldr;
  a.out = out;
  a.ldo = ldo;
  a.workspace = scratch.workspace;
  a.counters = scratch.counters;
  a.error = scratch.error;
  op->stream = true;
  op->grid = n / nt;
  op->smem_bytes = stages * stream_stage_bytes(a_rows, nt, kb) + 1024 + kSmemTail;
  return nullptr;
}

const char* plan_pair(GemmOp* op, const bf16* x, int ldx, int m, const bf16* w, int n, int k,
                      int epilogue, const bf16* bias, const float* gate, const bf16* residual,
                      int ldr, void* out, int ldo, const GemmScratch& scratch, int num_sms,
                      const ShapeChoice& c, bool w_tiled) {
  const int nkb = k / kBK;
  if (w_tiled) {
    if (!encode_tiled_rows(&op->tm_w, w, static_cast<long long>(n) * nkb))
      return "gemm: weight tensor map encode failed";
  } else if (!encode_bf16_2d(&op->tm_w, w, k, n, k, kWN / 2)) {
    return "gemm: weight tensor map encode failed";
  }
  if (!encode_bf16_2d(&op->tm_x, x, k, m, ldx, kPairRows))
    return "gemm: activation tensor map encode failed";
  GemmArgs& a = op->args;
  a.m = m;
  a.n = n;
  a.k = k;
  a.num_kb = nkb;
  a.splits = c.splits;
  a.split_mode = SPLIT_CLUSTER_GLOBAL;
  a.a_rows = kPairRows;
  a.stages = pair_stages();
  a.w_tiled = w_tiled ? w : nullptr;
  a.w_q8 = nullptr;
  a.tiles_m = (m + 2 * kTM - 1) / (2 * kTM);
  a.tiles_n = (n + kWN - 1) / kWN;
  a.group_m = group_m_for(2 * kTM, k);
  a.epilogue = epilogue;
  a.bias = bias;
  a.gate = gate;
  a.residual = residual;
  a.ldr = ldr;
  a.out = out;
  a.ldo = ldo;
  a.workspace = scratch.workspace;
  a.counters = scratch.counters;
  a.error = scratch.error;
  op->pair = true;
  op->cluster = 2 * c.splits;
  int clusters = c.tiles;
  if (c.splits == 1) {  // persistent: at most one wave of pairs
    const int pairs = g_cluster_slots[2] > 0 ? g_cluster_slots[2] / 2 : num_sms / 2;
    if (clusters > pairs) clusters = pairs;
  }
  op->grid = clusters * op->cluster;
  op->smem_bytes = pair_smem();
  return nullptr;
}

}  // namespace

const char* gemm_plan(GemmOp* op, const bf16* x, int ldx, int m, const bf16* w, int n, int k,
                      int epilogue, const bf16* bias, const float* gate, const bf16* residual,
                      int ldr, void* out, int ldo, const GemmScratch& scratch, int num_sms,
                      int force_splits, bool w_tiled, bool w_q8, bool pair) {
  if (m <= 0 || n <= 0 || k <= 0) return "gemm: empty shape";
  if (w_q8 && (n % kWN != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0))
    return "gemm: Q8_0 weight tiles need N a multiple of 256 and a 16-byte aligned pointer";
  if (w_tiled && (n % kWN != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0))
    return "gemm: re-tiled weights need N a multiple of 256 and a 16-byte aligned pointer";
  if (k % kBK != 0) return "gemm: K must be a multiple of 64";
  if (n % 16 != 0) return "gemm: N must be a multiple of 16";
  if (ldx % 8 != 0 || ldx < k) return "gemm: activation row stride must be >= K and a multiple of 8";
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return "gemm: operands must be 16-byte aligned";
  if ((epilogue == EPI_GATED_RES && (!gate || !residual)) ||
      ((epilogue == EPI_RES || epilogue == EPI_MUL) && !residual))
    return "gemm: residual epilogue needs its inputs";
  if (epilogue < 0 || epilogue > EPI_MUL) return "gemm: unknown epilogue";
  const int out_align = epilogue == EPI_F32_OUT ? 4 : 8;
  if (ldo < n || ldo % out_align != 0 || (reinterpret_cast<uintptr_t>(out) & 15))
    return "gemm: output must be 16-byte aligned with a row stride >= N in 16-byte units";
  if ((epilogue == EPI_GATED_RES || epilogue == EPI_RES || epilogue == EPI_MUL) &&
      (ldr < n || ldr % 8 != 0 || (reinterpret_cast<uintptr_t>(residual) & 15)))
    return "gemm: residual must be 16-byte aligned with a row stride >= N in 16-byte units";
  std::memset(op, 0, sizeof(*op));
  {
    ShapeChoice c =
        choose_shape(m, n, k, num_sms, force_splits, w_q8, scratch.workspace != nullptr, pair);
    if (c.pair) {
      if (c.splits > 1 &&
          static_cast<size_t>(c.tiles) * 2 * c.splits * kPairRows * kWN > scratch.workspace_floats)
        c.splits = 1;
      return plan_pair(op, x, ldx, m, w, n, k, epilogue, bias, gate, residual, ldr, out, ldo,
                       scratch, num_sms, c, w_tiled);
    }
  }
  if (g_stream && m <= 64 && !w_q8 && !pair && force_splits <= 0 && n % 32 == 0 && n >= 1536) {
    const char* e = plan_stream(op, x, ldx, m, w, n, k, epilogue, bias, gate, residual, ldr, out,
                                ldo, scratch, num_sms, w_tiled);
    if (!e || std::strcmp(e, "stream: not applicable") != 0) return e;
  }
  const int a_rows = a_rows_for(m);
  // The epilogue stages a [token][feature] tile (F32 rows of kPartLd floats at
  // most) in the pipeline stages' shared memory.
  if (static_cast<long long>(a_rows) * kPartLd * 4 >
      static_cast<long long>(stages_for(a_rows, w_q8)) * (a_rows * kBK * 2 + kBBytes))
    return "gemm: stage budget too small for the epilogue tile";
  const int tiles_m = (m + kTM - 1) / kTM;
  const int tiles_n = (n + kWN - 1) / kWN;
  const int nkb = k / kBK;
  int splits = force_splits > 0 ? force_splits : pick_splits(tiles_m * tiles_n, nkb, num_sms);
  if (splits > nkb) splits = nkb;
  // Split-K partials: with a workspace, the splits of a tile (a cluster of up
  // to 8 CTAs) exchange them through global memory / L2; without one, through
  // distributed shared memory; more than 8 splits need a workspace and tile
  // counters (the last CTA of a tile reduces).
  int mode = SPLIT_CLUSTER;
  if (scratch.workspace) mode = splits <= 8 ? SPLIT_CLUSTER_GLOBAL : SPLIT_WORKSPACE;
  if (splits > 8 && mode == SPLIT_CLUSTER)
    return "gemm: cluster split-K takes at most 8 splits (or a workspace)";
  if (splits > 1 && mode != SPLIT_CLUSTER) {
    const size_t need = static_cast<size_t>(tiles_m) * tiles_n * splits * a_rows * kWN;
    if (need > scratch.workspace_floats ||
        (mode == SPLIT_WORKSPACE && (!scratch.counters || tiles_m * tiles_n > scratch.counter_slots)))
      return "gemm: split-K scratch too small";
  }
  if (!w_tiled && !w_q8 && !encode_bf16_2d(&op->tm_w, w, k, n, k, kWN))
    return "gemm: weight tensor map encode failed";
  if (!encode_bf16_2d(&op->tm_x, x, k, m, ldx, a_rows))
    return "gemm: activation tensor map encode failed";
  GemmArgs& a = op->args;
  a.m = m;
  a.n = n;
  a.k = k;
  a.num_kb = nkb;
  a.splits = splits;
  a.split_mode = mode;
  a.a_rows = a_rows;
  a.stages = stages_for(a_rows, w_q8);
  a.pre_w = g_pre_w;
  a.w_tiled = w_tiled && !w_q8 ? w : nullptr;
  a.w_q8 = w_q8 ? reinterpret_cast<const uint8_t*>(w) : nullptr;
  a.tiles_m = tiles_m;
  a.tiles_n = tiles_n;
  a.epilogue = epilogue;
  a.bias = bias;
  a.gate = gate;
  a.residual = residual;
  a.ldr = ldr;
  a.out = out;
  a.ldo = ldo;
  a.workspace = scratch.workspace;
  a.counters = scratch.counters;
  a.error = scratch.error;
  op->grid = tiles_m * tiles_n * splits;
  op->smem_bytes = smem_for(a_rows, w_q8);
  // More than a wave of unsplit tiles: persistent CTAs (one per SM).
  op->persistent = splits == 1 && !w_q8 && tiles_m * tiles_n > num_sms;
  if (op->persistent) op->grid = num_sms;
  a.group_m = group_m_for(kTM, k);
  return nullptr;
}

cudaError_t gemm_init(int device) {
  // Opt-in shared memory once per device, before any launch (so that launches
  // can be captured into CUDA graphs), and the cluster occupancy per split.
  static std::mutex mu;
  static std::vector<int> done;
  std::lock_guard<std::mutex> lock(mu);
  for (int d : done)
    if (d == device) return cudaSuccess;
  const int smem = kStageBudget + 1024 + kSmemTail;  // every stage count stays within the budget
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(gemm_tc_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(gemm_tc_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           pair_smem());
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(gemm_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kStreamBudget + 1024 + kSmemTail);
  if (e != cudaSuccess) return e;
  int sms = 0;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
    return e;
  for (int s = 1; s <= 8; ++s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(s * sms, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = s;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_kernel, &cfg) == cudaSuccess)
      g_cluster_slots[s] = clusters * s;
    else
      cudaGetLastError();
  }
  done.push_back(device);
  return cudaSuccess;
}

cudaError_t gemm_launch(const GemmOp& op, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = op.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = (g_pdl && !op.weights_from_prev) ? 1 : 0;
  ++na;
  if (op.args.splits > 1 && op.args.split_mode != SPLIT_WORKSPACE) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = op.args.splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (op.pair) {
    na = 1;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = op.cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (op.pair) return cudaLaunchKernelEx(&cfg, gemm_tc_pair_kernel, op.tm_w, op.tm_x, op.args);
  if (op.stream) return cudaLaunchKernelEx(&cfg, gemm_stream_kernel, op.tm_w, op.tm_x, op.args);
  if (op.persistent) return cudaLaunchKernelEx(&cfg, gemm_tc_persistent_kernel, op.tm_w, op.tm_x, op.args);
  if (op.args.w_q8) cfg.blockDim = dim3(kThreadsQ8, 1, 1);
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, op.tm_w, op.tm_x, op.args);
}

}  // namespace wamb
