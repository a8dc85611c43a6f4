// tcgen05 attention for the denoise step: <= 64 queries per (sequence, head)
// over <= 896 keys (the 48 action queries over the joint keys, prefix + action,
// 817 at config 2, and over the 512 prompt keys), taken when the (sequence,
// head) grid fills the SMs (batched requests; see dec_tc_mode below).
//
// One CTA per (sequence, head) holds every key of the head, so there is no key
// split and no merge of partial rows. The scores are computed transposed,
// S^T = K Q^T (M = 128 keys of a tile, N = 64 query slots, K = 128 dims), each
// key tile into its own 64 TMEM columns (7 tiles + O^T = 512 columns): a TMEM
// lane is a key, so the exponentials of a tile are spread over all four lane
// quadrants whatever the query count. With every score resident the softmax
// is exact in two passes (the per-query max over all keys, then the
// probabilities; no rescaling of O). O^T = V^T P^T (M = 128 dims, N = 64
// queries, K = 128 keys per tile): the tensor core reads V as an MN-major A
// operand straight from its TMA tile (dims contiguous), and P^T, written by
// the softmax threads as an MN-major B operand (queries contiguous), from one
// of two shared-memory buffers.
//
// Roles (320 threads): warp 0 issues the TMA copies (Q once; K tiles then V
// tiles through a ring of 5 slots; tiles whose rows the preceding kernel does
// not write start before waiting for it), warp 1 owns TMEM and issues the
// MMAs, warps 2-9 = the softmax: warp w reads TMEM lane quadrant w % 4 (32
// keys of a tile, or 32 dims of O^T) and query half (w - 2) / 4, i.e. the
// 8-column chunks 16c + 8h .. 16c + 8h + 7 (c = 0..3) of the 64 query slots.
//
// Arithmetic: F32 scores, softmax(scale * S) with the max over every key,
// probabilities rounded to BF16 for P V, F32 accumulation, BF16 output, as the
// other attention kernels. Reference: the action self-attention over the
// cached prefix K/V and the cross attention over the prompt K/V
// (src/models/gwp05/engine/mot.cpp:683-724, mot.cpp:299-321), ggml_soft_max_ext
// with scale 1/sqrt(128) at GGML_PREC_F32 (mot.cpp:432-446).
#include <cmath>
#include <cstdlib>

#include "kernels.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace wamb {

namespace {

constexpr int kKeys = 128;                // keys per tile (UMMA M of S^T, TMEM lanes)
constexpr int kSlots = 64;                // query slots (UMMA N)
constexpr int kMaxTiles = 7;              // 7 x 64 S^T columns + 64 O^T columns = 512
constexpr int kRing = 5;                  // K / V tile slots
constexpr int kSoftWarps = 8;
constexpr int kSoft = 32 * kSoftWarps;
constexpr int kThreads = 64 + kSoft;
constexpr int kHalf = kKeys * 64 * 2;     // 128 rows x 64 dims, swizzled: 16 KB
constexpr int kTile = 2 * kHalf;          // one K or V tile: 32 KB
constexpr int kQHalf = kSlots * 64 * 2;   // 64 query rows x 64 dims: 8 KB
constexpr int kPBuf = kKeys * kSlots * 2; // P^T [128 keys][64 queries] BF16: 16 KB
constexpr int kOffQ = 0;
constexpr int kOffRing = kOffQ + 2 * kQHalf;
constexpr int kOffP = kOffRing + kRing * kTile;
constexpr int kOffBar = kOffP + 2 * kPBuf;
constexpr int kNumBars = 1 + 2 * kRing + kMaxTiles + 2 + 2 + 1;
constexpr int kOffRed = kOffBar + 8 * 32;  // [2 (max, sum)][4 quadrants][2 halves][32] F32
constexpr int kSmem = kOffRed + 2 * 4 * 2 * 32 * 4 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = kMaxTiles * kSlots;  // O^T columns

static_assert(kNumBars + 1 <= 32, "barrier area");
static_assert(kSmem <= 227 * 1024, "shared memory");

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

__device__ __forceinline__ void fail(const AttnArgs& a, unsigned code) {
  if (a.error) atomicCAS(a.error, 0u, code);
}

// Reduce-scatter of 32 values over a warp: lane l returns the max (MAX) or the
// sum of value l over the 32 lanes. Halving exchanges (31 shuffles); the
// combination order is fixed, so sums are deterministic.
template <bool MAX>
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = up ? v[i] : v[i + w];
      const float keep = up ? v[i + w] : v[i];
      const float recv = __shfl_xor_sync(0xffffffffu, send, w);
      v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
    }
  }
  return v[0];
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_dec_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem + kOffQ;
  uint8_t* ring = smem + kOffRing;
  uint8_t* pbuf = smem + kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* slot_full = bars + 1;                 // [kRing]
  uint64_t* slot_free = bars + 1 + kRing;         // [kRing]
  uint64_t* s_full = bars + 1 + 2 * kRing;        // [kMaxTiles], one phase each
  uint64_t* p_full = s_full + kMaxTiles;          // [2]
  uint64_t* p_free = p_full + 2;                  // [2]
  uint64_t* o_full = p_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  float* red = reinterpret_cast<float*>(smem + kOffRed);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.x, seq = blockIdx.y;
  const int nk = (a.lk + kKeys - 1) / kKeys;  // 1 .. kMaxTiles (checked by the host)

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], 1);
    mbar_init(&p_full[0], kSoftWarps);
    mbar_init(&p_full[1], kSoftWarps);
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
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------- copy producer
      // Item i < nk is K tile i, item nk + t is V tile t; item i goes to slot
      // i % kRing.
      const uint64_t pol = policy_evict_first();
      const int items = 2 * nk;
      auto load = [&](int i) {
        const int slot = i % kRing;
        const int t = i < nk ? i : i - nk;
        const CUtensorMap* m = i < nk ? &tm_k : &tm_v;
        uint8_t* dst = ring + slot * kTile;
        mbar_arrive_expect_tx(&slot_full[slot], kTile);
        tma_load_4d(dst, m, &slot_full[slot], 0, t * kKeys, head, seq, pol);
        tma_load_4d(dst + kHalf, m, &slot_full[slot], 64, t * kKeys, head, seq, pol);
      };
      int issued = 0;
      // K / V rows the preceding kernel does not write start before waiting for it.
      while (issued < items && issued < kRing) {
        const int t = issued < nk ? issued : issued - nk;
        const int end = (t + 1) * kKeys < a.lk ? (t + 1) * kKeys : a.lk;
        if (end > a.static_keys) break;
        load(issued++);
      }
      griddep_wait();
      griddep_launch_dependents();
      mbar_arrive_expect_tx(q_full, 2 * kQHalf);
      tma_load_4d(sq, &tm_q, q_full, 0, 0, head, seq, pol);
      tma_load_4d(sq + kQHalf, &tm_q, q_full, 64, 0, head, seq, pol);
      bool ok = true;
      for (; issued < items; ++issued) {
        if (issued >= kRing &&
            !mbar_wait(&slot_free[issued % kRing], ((issued / kRing) - 1) & 1)) {
          ok = false;
          break;
        }
        load(issued);
      }
      if (!ok) fail(a, kErrProducerTimeout);
      // Every issued copy lands before the CTA leaves.
      mbar_wait(q_full, 0);
      for (int i = issued - kRing > 0 ? issued - kRing : 0; i < issued; ++i)
        mbar_wait(&slot_full[i % kRing], (i / kRing) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------- MMA issuer
      // S^T: A = K tile (K-major, 128 keys x 2 x 64 dims), B = Q (K-major, 64
      // query slots x 2 x 64 dims). O^T: A = V tile read MN-major (dims
      // contiguous: two 64-dim atoms 16 KB apart, 8-key groups 1024 bytes
      // apart, 16 keys = 2048 bytes per step), B = P^T MN-major (one 64-query
      // atom, 8-key groups 1024 bytes apart).
      // S^T over the query slots in use (N = lq rounded up to 16; its columns
      // >= lq see the zero-filled Q rows)
      const uint32_t idesc_s = umma_idesc_bf16(kKeys, ((a.lq + 15) / 16) * 16);
      constexpr uint32_t idesc_o = umma_idesc_bf16_mn(128, kSlots);
      bool ok = mbar_wait(q_full, 0);
      for (int t = 0; t < nk && ok; ++t) {
        const int slot = t % kRing;
        if (!mbar_wait(&slot_full[slot], (t / kRing) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint64_t da = sw128_kmajor_desc(smem_u32(ring + slot * kTile + c * kHalf));
          const uint64_t db = sw128_kmajor_desc(smem_u32(sq + c * kQHalf));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_ss(tmem + static_cast<uint32_t>(t * kSlots), da + 2 * kk, db + 2 * kk, idesc_s,
                         (c | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
        umma_commit(&slot_free[slot]);
      }
      for (int t = 0; t < nk && ok; ++t) {
        const int i = nk + t, slot = i % kRing, b = t & 1;
        if (!mbar_wait(&slot_full[slot], (i / kRing) & 1) || !mbar_wait(&p_full[b], (t >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t v_base = smem_u32(ring + slot * kTile);
        const uint32_t p_base = smem_u32(pbuf + b * kPBuf);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t da = sw128_mnmajor_desc(v_base + static_cast<uint32_t>(kk * 2048), kHalf, 1024);
          const uint64_t dp = sw128_mnmajor_desc(p_base + static_cast<uint32_t>(kk * 2048), kPBuf, 1024);
          umma_bf16_ss(tmem + kTmemO, da, dp, idesc_o, (t | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&p_free[b]);
        umma_commit(&slot_free[slot]);
      }
      if (!ok) fail(a, kErrMmaTimeout);
      umma_commit(o_full);  // arrives once every MMA issued above has completed
      mbar_wait(o_full, 0);
    }
  } else {
    // ------------------------------------------------- softmax / P / output
    const int quad = warp & 3;              // TMEM lane quadrant: keys / dims 32 quad ..
    const int half = (warp - 2) >> 2;       // query chunks 16 c + 8 half (c = 0..3)
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int lq = a.lq;
    const float sl2 = a.scale * 1.4426950408889634f;
    float* red_m = red;                     // [4][2][32]
    float* red_l = red + 4 * 2 * 32;
    bool chunk_ok[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) chunk_ok[c] = 16 * c + 8 * half < lq;
    bool ok = true;

    // Pass 1: per-query max over this thread's keys (one per tile).
    float m[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) m[i] = -INFINITY;
    for (int t = 0; t < nk; ++t) {
      if (!mbar_wait(&s_full[t], 0)) ok = false;
      tc_fence_after();
      const int key = t * kKeys + quad * 32 + lane;
      if (t * kKeys + quad * 32 >= a.lk) continue;  // warp-uniform: no key of this warp
      uint32_t r[4][8];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (chunk_ok[c])
          tmem_ld_x8(tmem + lane_off + static_cast<uint32_t>(t * kSlots + 16 * c + 8 * half), r[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (!chunk_ok[c] || key >= a.lk) continue;
#pragma unroll
        for (int i = 0; i < 8; ++i) m[8 * c + i] = fmaxf(m[8 * c + i], u2f(r[c][i]));
      }
    }
    red_m[(quad * 2 + half) * 32 + lane] = warp_reduce_scatter32<true>(m, lane);
    ok = named_bar_and(1, kSoft, ok);
    // the max over all keys of this thread's 32 query columns, pre-scaled:
    // lane i combines the quadrants of column i, then every lane takes all 32
    float mb[32];
    {
      float v = red_m[half * 32 + lane];
#pragma unroll
      for (int q = 1; q < 4; ++q) v = fmaxf(v, red_m[(q * 2 + half) * 32 + lane]);
      v *= sl2;
#pragma unroll
      for (int i = 0; i < 32; ++i) mb[i] = __shfl_sync(0xffffffffu, v, i);
    }

    // Pass 2: probabilities -> P^T buffers, per-query sums.
    float l[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) l[i] = 0.0f;
    const int prow = quad * 32 + lane;  // key row of the P^T tile
    for (int t = 0; t < nk && ok; ++t) {
      const int b = t & 1;
      const int key = t * kKeys + prow;
      const bool warp_keys = t * kKeys + quad * 32 < a.lk;
      uint4 pk[4];
      uint32_t r[4][8];
      if (warp_keys) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (chunk_ok[c])
            tmem_ld_x8(tmem + lane_off + static_cast<uint32_t>(t * kSlots + 16 * c + 8 * half), r[c]);
        tmem_ld_wait();
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        pk[c] = make_uint4(0u, 0u, 0u, 0u);
        if (!chunk_ok[c] || !warp_keys || key >= a.lk) continue;
        float p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          p[i] = ex2_approx(u2f(r[c][i]) * sl2 - mb[8 * c + i]);
          l[8 * c + i] += p[i];
        }
        pk[c] = make_uint4(pack_bf16(p[0], p[1]), pack_bf16(p[2], p[3]), pack_bf16(p[4], p[5]),
                           pack_bf16(p[6], p[7]));
      }
      // The buffer is free once the P V that read it two tiles ago completed.
      // Warp-uniform outcome: the warp's lanes leave (or stay) together.
      if (t >= 2 && !__all_sync(0xffffffffu, mbar_wait(&p_free[b], ((t >> 1) - 1) & 1))) {
        ok = false;
        break;
      }
      uint8_t* dst = pbuf + b * kPBuf + prow * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int chunk = 2 * c + half;
        *reinterpret_cast<uint4*>(dst + ((chunk ^ (prow & 7)) << 4)) = pk[c];
      }
      fence_proxy_async_smem();  // generic-proxy writes -> the tensor core's async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    if (!ok) fail(a, kErrEpilogueTimeout);
    red_l[(quad * 2 + half) * 32 + lane] = warp_reduce_scatter32<false>(l, lane);
    if (ok) ok = mbar_wait(o_full, 0);
    if (named_bar_and(1, kSoft, ok)) {
      tc_fence_after();
      // 1 / (sum over all keys) of column `lane` (quadrants in order), shared
      // over the warp by shuffles
      float lsum = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) lsum += red_l[(q * 2 + half) * 32 + lane];
      const float inv = 1.0f / lsum;
      // O^T: lane = dim 32 quad + lane, columns = query slots
      const int d = quad * 32 + lane;
      uint32_t r[4][8];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (chunk_ok[c]) tmem_ld_x8(tmem + lane_off + kTmemO + static_cast<uint32_t>(16 * c + 8 * half), r[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (!chunk_ok[c]) continue;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float f = __shfl_sync(0xffffffffu, inv, 8 * c + i);
          const int qr = 16 * c + 8 * half + i;
          if (qr >= lq) continue;
          bf16* dst;
          if (a.split_first) {
            dst = qr == 0 ? a.out_first + static_cast<long long>(seq) * a.ldo_first
                          : a.out + (static_cast<long long>(seq) * (lq - 1) + qr - 1) * a.ldo;
          } else {
            dst = a.out + (static_cast<long long>(seq) * lq + qr) * a.ldo;
          }
          dst[head * 128 + d] = __float2bfloat16_rn(u2f(r[c][i]) * f);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// WAM_B200_ATTN_DEC_TC: 0 = never, 1 = every eligible launch, unset = when
// the (sequence, head) grid fills the SMs. With fewer CTAs the mma.sync kernel
// (attention.cu), which splits each head's keys over up to 8 CTAs, is faster:
// one CTA feeds the tensor core all of its head's K and V from shared memory,
// and the tensor core's operand reads (~52 bytes per cycle per SM measured)
// bound it at ~3.4 us for 817 keys (batch 1: 10.9 against 9.3 us per launch;
// batch 8: 24.4 against 25.0; batch 64: 140.4 against 142.1).
int dec_tc_mode() {
  static const int mode = [] {
    const char* v = std::getenv("WAM_B200_ATTN_DEC_TC");
    if (v && v[0] == '0') return 0;
    if (v && v[0] == '1') return 1;
    return 2;
  }();
  return mode;
}

int sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return sms;
}

}  // namespace

cudaError_t attention_dec_tc_init() {
  return cudaFuncSetAttribute(attention_dec_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
}

bool attention_dec_tc_eligible(const AttnArgs& a) {
  const int mode = dec_tc_mode();
  if (mode == 0 || (mode == 2 && static_cast<long long>(a.heads) * a.batch < sm_count())) return false;
  return a.lq >= 1 && a.lq <= kSlots && a.lk >= 1 && a.lk <= kMaxTiles * kKeys &&
         a.q_begin == 0 && a.q_end == 0 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.k) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.v) & 15) == 0 &&
         a.q_head_stride % 8 == 0 && a.q_seq_stride % 8 == 0 && a.kv_head_stride % 8 == 0 &&
         a.kv_seq_stride % 8 == 0 && a.batch <= 65535;
}

cudaError_t launch_attention_dec_tc(const AttnArgs& a, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (!attn_encode_rows(&mq, a.q, a.lq, a.heads, a.batch, a.q_head_stride, a.q_seq_stride, kSlots) ||
      !attn_encode_rows(&mk, a.k, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride, kKeys) ||
      !attn_encode_rows(&mv, a.v, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride, kKeys))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.heads, a.batch, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_dec_tc_kernel, mq, mk, mv, a);
}

}  // namespace wamb
