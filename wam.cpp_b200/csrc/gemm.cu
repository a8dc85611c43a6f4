// BF16 tcgen05 GEMM for every linear layer of the MoT forward pass.
//
// Orientation: the weight tile is the UMMA "A" operand (128 output features =
// the 128 TMEM lanes) and the token tile is "B" (UMMA N = BT tokens). The
// accumulator tile D[feature][token] lives in TMEM; each epilogue thread owns
// one feature (one TMEM lane), so per-feature bias / gate values are register
// constants and the stores of a warp cover 32 consecutive features.
// This keeps one kernel efficient for both regimes of the forward pass:
//   * denoise at batch 1 (48 tokens): weight streaming, HBM bound; split-K over
//     CTAs fills all 148 SMs and the last CTA to finish a tile reduces the F32
//     partials (deterministic order) and runs the epilogue;
//   * prefix / batched denoise (768..49152 tokens): tensor-core bound.
// Pipeline: warp 0 = TMA producer, warp 1 = TMEM allocator + single-thread
// UMMA issuer, warps 2-5 = epilogue. Shared-memory stages hold one 128 x 64
// weight tile and one BT x 64 token tile, both K-major with 128-byte swizzle.
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
#include "mathops.cuh"
#include "ptx.cuh"

namespace wamb {

namespace {

constexpr int kBN = 128;  // weight rows per tile (UMMA M, TMEM lanes)
constexpr int kBK = 64;   // K per stage: one 128-byte swizzle row of BF16
constexpr int kThreads = 192;

template <int BT>
struct Cfg {
  static constexpr int A_BYTES = kBN * kBK * 2;
  static constexpr int B_BYTES = BT * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // Small token tiles (the weight-streaming regime) keep ~96 KB of stages so
  // that two CTAs share an SM; large tiles keep a deep single-CTA pipeline.
  static constexpr int MIN_BLOCKS = BT <= 64 ? 2 : 1;
  static constexpr int BUDGET = BT <= 64 ? 96 * 1024 : 200 * 1024;
  static constexpr int STAGES_RAW = BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int TMEM_COLS = BT <= 32 ? 32 : (BT <= 64 ? 64 : (BT <= 128 ? 128 : 256));
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int PARTIAL_BYTES = BT * kBN * 4;  // F32 split-K partial tile
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "UMMA N for M=128");
  static_assert(STAGES >= 2, "pipeline depth");
  static_assert(PARTIAL_BYTES <= STAGES * STAGE_BYTES, "partial tile reuses the stage buffers");
};

__device__ __forceinline__ void store_out(const GemmArgs& a, int m, int n, float acc, float b,
                                          float g) {
  const long long o = static_cast<long long>(m) * a.ldo + n;
  bf16* out = static_cast<bf16*>(a.out);
  switch (a.epilogue) {
    case EPI_BIAS: {
      float v = bf16_round(acc);
      if (a.bias) v = v + b;
      out[o] = __float2bfloat16_rn(v);
      break;
    }
    case EPI_BIAS_GELU: {
      const float v = bf16_round(acc) + b;
      out[o] = __float2bfloat16_rn(gelu_tanh(v));
      break;
    }
    case EPI_BIAS_SILU: {
      float v = bf16_round(acc);
      if (a.bias) v = bf16_round(v + b);
      out[o] = __float2bfloat16_rn(silu(v));
      break;
    }
    case EPI_GATED_RES: {
      float v = bf16_round(acc);
      if (a.bias) v = bf16_round(v + b);
      const float r = __bfloat162float(a.residual[static_cast<long long>(m) * a.ldr + n]);
      out[o] = __float2bfloat16_rn(fmaf(v, g, r));
      break;
    }
    case EPI_RES: {
      float v = bf16_round(acc);
      if (a.bias) v = bf16_round(v + b);
      const float r = __bfloat162float(a.residual[static_cast<long long>(m) * a.ldr + n]);
      out[o] = __float2bfloat16_rn(r + v);
      break;
    }
    case EPI_F32_BIAS: {
      out[o] = __float2bfloat16_rn(acc + b);
      break;
    }
    case EPI_BIAS_GELU_R: {
      float v = bf16_round(acc);
      if (a.bias) v = bf16_round(v + b);
      out[o] = __float2bfloat16_rn(gelu_tanh(v));
      break;
    }
    case EPI_BIAS_GELU_ERF: {
      float v = bf16_round(acc);
      if (a.bias) v = bf16_round(v + b);
      out[o] = __float2bfloat16_rn(gelu_erf(v));
      break;
    }
    default: {
      static_cast<float*>(a.out)[o] = acc;
      break;
    }
  }
}

// CTA x = (tile, split) with the split index fastest, so that in cluster mode
// one thread-block cluster holds exactly the splits of one output tile.
template <int BT>
__global__ void __launch_bounds__(kThreads, Cfg<BT>::MIN_BLOCKS)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x, const GemmArgs args) {
  using C = Cfg<BT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_b + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
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
  const bool cluster_mode = args.splits > 1 && args.split_mode == SPLIT_CLUSTER;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
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
  const int q = warp & 3;
  const int row = q * 32 + lane;
  const int n = tile_n * kBN + row;
  const bool n_ok = n < args.n;
  const int m_base = tile_m * BT;
  float bias_v = 0.0f, gate_v = 0.0f;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      const int pre = nkb < C::STAGES ? nkb : C::STAGES;
      // Weights never depend on the preceding kernel: start streaming them
      // before waiting for it (programmatic dependent launch).
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
        tma_load_2d(smem_a + i * C::A_BYTES, &tm_w, &full[i], (kb0 + i) * kBK, tile_n * kBN, pol_w);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem_b + i * C::B_BYTES, &tm_x, &full[i], (kb0 + i) * kBK, tile_m * BT, pol_x);
      for (int i = pre; i < nkb; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrProducerTimeout));
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
        const int kc = (kb0 + i) * kBK;
        tma_load_2d(smem_a + s * C::A_BYTES, &tm_w, &full[s], kc, tile_n * kBN, pol_w);
        tma_load_2d(smem_b + s * C::B_BYTES, &tm_x, &full[s], kc, tile_m * BT, pol_x);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBN, BT);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (!mbar_wait(&full[s], ph)) {
          atomicCAS(args.error, 0u, static_cast<unsigned>(kErrMmaTimeout));
          break;
        }
        tc_fence_after();
        const uint64_t da = sw128_kmajor_desc(smem_u32(smem_a + s * C::A_BYTES));
        const uint64_t db = sw128_kmajor_desc(smem_u32(smem_b + s * C::B_BYTES));
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          // +32 bytes along K inside the swizzle row = +2 in the 16-byte address field.
          umma_bf16_ss(tmem_base, da + 2 * k, db + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    // Epilogue warps 2..5; the TMEM lane quadrant is fixed by warp % 4.
    griddep_wait();  // residual / gate / outputs are touched only after the preceding kernel
    bias_v = (args.bias && n_ok) ? __bfloat162float(args.bias[n]) : 0.0f;
    gate_v = (args.gate && n_ok) ? args.gate[n] : 0.0f;
    ok = mbar_wait(accum, 0);
    if (!ok) atomicCAS(args.error, 0u, static_cast<unsigned>(kErrEpilogueTimeout));
    tc_fence_after();
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    if (args.splits == 1) {
#pragma unroll 1
      for (int c = 0; c < BT; c += 16) {
        uint32_t r[16];
        tmem_ld_x16(taddr + c, r);
        tmem_ld_wait();
        if (ok && n_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m_base + c + j;
            if (m < args.m) store_out(args, m, n, __uint_as_float(r[j]), bias_v, gate_v);
          }
        }
      }
    } else if (cluster_mode) {
      // Stage this split's F32 partial tile [column][row] in shared memory.
#pragma unroll 1
      for (int c = 0; c < BT; c += 16) {
        uint32_t r[16];
        tmem_ld_x16(taddr + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) partial[(c + j) * kBN + row] = __uint_as_float(r[j]);
      }
    } else {
      // Workspace mode: partial tile to global memory; the last CTA of the tile
      // to arrive reduces all partials in split order and runs the epilogue.
      const int tile_id = tile;
      float* ws_tile = args.workspace + static_cast<size_t>(tile_id) * args.splits * BT * kBN;
      float* ws = ws_tile + static_cast<size_t>(split) * BT * kBN;
#pragma unroll 1
      for (int c = 0; c < BT; c += 16) {
        uint32_t r[16];
        tmem_ld_x16(taddr + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) ws[(c + j) * kBN + row] = __uint_as_float(r[j]);
      }
      __threadfence();
      named_bar_sync(1, 128);
      if (threadIdx.x == 64) {
        const unsigned prev = atomicAdd(&args.counters[tile_id], 1u);
        *last_flag = (prev == static_cast<unsigned>(args.splits - 1)) ? 1 : 0;
      }
      named_bar_sync(1, 128);
      if (*last_flag) {
        __threadfence();
        if (ok && n_ok) {
#pragma unroll 1
          for (int c0 = 0; c0 < BT; c0 += 8) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
            for (int s = 0; s < args.splits; ++s) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                acc[j] += __ldcg(ws_tile + (static_cast<size_t>(s) * BT + c0 + j) * kBN + row);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int m = m_base + c0 + j;
              if (m < args.m) store_out(args, m, n, acc[j], bias_v, gate_v);
            }
          }
        }
        if (threadIdx.x == 64) args.counters[tile_id] = 0u;
      }
    }
  }

  __syncwarp();
  if (cluster_mode) {
    // All partial tiles of this output tile are in the cluster's shared memory.
    cluster_sync_all();
    if (warp >= 2) {
      const int S = args.splits;
      const int cols = (BT + S - 1) / S;
      const int c0 = split * cols;
      const int c1 = c0 + cols < BT ? c0 + cols : BT;
      const uint32_t base = smem_u32(partial) + static_cast<uint32_t>(row) * 4u;
      uint32_t peer[8];
#pragma unroll
      for (int p = 0; p < 8; ++p) peer[p] = mapa_shared(base, p < S ? p : 0);
#pragma unroll 1
      for (int c = c0; c < c1; c += 4) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          if (p < S) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (c + j < c1)
                acc[j] += ld_shared_cluster_f32(peer[p] + static_cast<uint32_t>((c + j) * kBN) * 4u);
          }
        }
        if (ok && n_ok) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int m = m_base + c + j;
            if (c + j < c1 && m < args.m) store_out(args, m, n, acc[j], bias_v, gate_v);
          }
        }
      }
    }
    // No CTA leaves while a peer may still read its shared memory.
    cluster_sync_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
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

// Token tile: the largest tile for up to 256 tokens; beyond that the tile that
// minimises (waves x resident CTAs per SM x tile width), i.e. the per-SM
// tensor work of the slowest SM, preferring larger tiles on ties.
int pick_bt(int m, int n, int num_sms) {
  static const int small[] = {16, 32, 48, 64, 96, 128, 192, 256};
  if (m <= 256) {
    for (int o : small)
      if (o >= m) return o;
  }
  static const int big[] = {256, 192, 128, 96};
  const int tiles_n = (n + 127) / 128;
  int best = 256;
  long long best_cost = -1;
  for (int bt : big) {
    const long long tiles = static_cast<long long>((m + bt - 1) / bt) * tiles_n;
    const long long waves = (tiles + num_sms - 1) / num_sms;
    const long long cost = waves * bt;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bt;
    }
  }
  return best;
}

// Split-K factor in {1, 2, 4, 8} (cluster sizes). When the output tiles fill
// less than ~3/4 of the resident CTA slots (two per SM for token tiles <= 64),
// the K range is split as far as the slots allow, keeping >= 4 k-blocks
// (256 of K) per split.
int pick_splits(int tiles, int nkb, int num_sms, int bt) {
  // Large token tiles are tensor bound: splitting K only adds partial traffic.
  if (bt > 64) return 1;
  const int slots = num_sms * 2;
  if (tiles * 4 >= slots * 3) return 1;
  int best = 1;
  for (int s = 2; s <= 8; s *= 2)
    if (tiles * s <= slots && nkb / s >= 4) best = s;
  return best;
}

bool g_pdl = [] {
  const char* v = std::getenv("WAM_B200_DISABLE_PDL");
  return !(v && *v && *v != '0');
}();

template <int BT>
cudaError_t set_attr_bt() {
  return cudaFuncSetAttribute(gemm_bf16_tc_kernel<BT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Cfg<BT>::SMEM);
}

template <int BT>
cudaError_t launch_bt(const GemmOp& op, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg<BT>::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = g_pdl ? 1 : 0;
  ++na;
  if (op.args.splits > 1 && op.args.split_mode == SPLIT_CLUSTER) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = op.args.splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemm_bf16_tc_kernel<BT>, op.tm_w, op.tm_x, op.args);
}

int smem_for_bt(int bt) {
  switch (bt) {
    case 16: return Cfg<16>::SMEM;
    case 32: return Cfg<32>::SMEM;
    case 48: return Cfg<48>::SMEM;
    case 64: return Cfg<64>::SMEM;
    case 96: return Cfg<96>::SMEM;
    case 128: return Cfg<128>::SMEM;
    case 192: return Cfg<192>::SMEM;
    default: return Cfg<256>::SMEM;
  }
}

}  // namespace

size_t gemm_scratch_floats(int m, int n, int k, int num_sms, int force_splits, int* tiles_out) {
  const int bt = pick_bt(m, n, num_sms);
  const int tiles = ((m + bt - 1) / bt) * ((n + kBN - 1) / kBN);
  const int nkb = k / kBK;
  const int splits = force_splits > 0 ? force_splits : pick_splits(tiles, nkb, num_sms, bt);
  if (tiles_out) *tiles_out = tiles;
  if (splits <= 1) return 0;
  return static_cast<size_t>(tiles) * splits * bt * kBN;
}

const char* gemm_plan(GemmOp* op, const bf16* x, int ldx, int m, const bf16* w, int n, int k,
                      int epilogue, const bf16* bias, const float* gate, const bf16* residual,
                      int ldr, void* out, int ldo, const GemmScratch& scratch, int num_sms,
                      int force_splits) {
  if (m <= 0 || n <= 0 || k <= 0) return "gemm: empty shape";
  if (k % kBK != 0) return "gemm: K must be a multiple of 64";
  if (ldx % 8 != 0 || ldx < k) return "gemm: activation row stride must be >= K and a multiple of 8";
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return "gemm: operands must be 16-byte aligned";
  if ((epilogue == EPI_GATED_RES && (!gate || !residual)) || (epilogue == EPI_RES && !residual))
    return "gemm: residual epilogue needs its inputs";
  if (epilogue < 0 || epilogue > EPI_BIAS_GELU_ERF) return "gemm: unknown epilogue";
  std::memset(op, 0, sizeof(*op));
  const int bt = pick_bt(m, n, num_sms);
  const int tiles_m = (m + bt - 1) / bt;
  const int tiles_n = (n + kBN - 1) / kBN;
  const int nkb = k / kBK;
  int splits = force_splits > 0 ? force_splits : pick_splits(tiles_m * tiles_n, nkb, num_sms, bt);
  if (splits > nkb) splits = nkb;
  // Split-K partials are reduced through distributed shared memory inside a
  // thread-block cluster unless the caller hands in a global workspace.
  const int mode = scratch.workspace ? SPLIT_WORKSPACE : SPLIT_CLUSTER;
  if (splits > 1 && mode == SPLIT_CLUSTER && splits != 2 && splits != 4 && splits != 8)
    return "gemm: cluster split-K needs 2, 4 or 8 splits (or a workspace)";
  if (splits > 1 && mode == SPLIT_WORKSPACE) {
    const size_t need = static_cast<size_t>(tiles_m) * tiles_n * splits * bt * kBN;
    if (need > scratch.workspace_floats || !scratch.counters ||
        tiles_m * tiles_n > scratch.counter_slots)
      return "gemm: split-K scratch too small";
  }
  if (!encode_bf16_2d(&op->tm_w, w, k, n, k, kBN)) return "gemm: weight tensor map encode failed";
  if (!encode_bf16_2d(&op->tm_x, x, k, m, ldx, bt)) return "gemm: activation tensor map encode failed";
  GemmArgs& a = op->args;
  a.m = m;
  a.n = n;
  a.k = k;
  a.num_kb = nkb;
  a.splits = splits;
  a.split_mode = mode;
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
  op->bt = bt;
  op->grid = tiles_m * tiles_n * splits;
  op->smem_bytes = smem_for_bt(bt);
  return nullptr;
}

cudaError_t gemm_init(int device) {
  // Opt-in shared memory per instantiation, once per device, before any
  // launch (so that launches can be captured into CUDA graphs).
  static std::mutex mu;
  static std::vector<int> done;
  std::lock_guard<std::mutex> lock(mu);
  for (int d : done)
    if (d == device) return cudaSuccess;
  cudaError_t e;
  if ((e = set_attr_bt<16>()) != cudaSuccess) return e;
  if ((e = set_attr_bt<32>()) != cudaSuccess) return e;
  if ((e = set_attr_bt<48>()) != cudaSuccess) return e;
  if ((e = set_attr_bt<64>()) != cudaSuccess) return e;
  if ((e = set_attr_bt<96>()) != cudaSuccess) return e;
  if ((e = set_attr_bt<128>()) != cudaSuccess) return e;
  if ((e = set_attr_bt<192>()) != cudaSuccess) return e;
  if ((e = set_attr_bt<256>()) != cudaSuccess) return e;
  done.push_back(device);
  return cudaSuccess;
}

cudaError_t gemm_launch(const GemmOp& op, cudaStream_t stream) {
  switch (op.bt) {
    case 16: return launch_bt<16>(op, stream);
    case 32: return launch_bt<32>(op, stream);
    case 48: return launch_bt<48>(op, stream);
    case 64: return launch_bt<64>(op, stream);
    case 96: return launch_bt<96>(op, stream);
    case 128: return launch_bt<128>(op, stream);
    case 192: return launch_bt<192>(op, stream);
    case 256: return launch_bt<256>(op, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace wamb
