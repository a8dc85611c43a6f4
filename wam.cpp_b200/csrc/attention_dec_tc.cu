// tcgen05 attention for the denoise step: <= 64 queries per (sequence, head)
// over <= 896 keys (the 48 action queries over the joint keys, prefix + action,
// 817 at config 2, and over the 512 prompt keys).
//
// One CTA per (sequence, head) holds all of its keys, or, while the grid is
// smaller than the SMs, a cluster of 2 or 4 CTAs splits them by 128-key tiles
// (each CTA with its own max; the partial O^T, max and sum are published in
// shared memory and every CTA merges a quarter / half of the query slots from
// its peers' through distributed shared memory). The scores are computed transposed,
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
constexpr int kRing = 4;                  // K / V tile slots
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
constexpr int kNumBars = 1 + 2 * kRing + kMaxTiles + 2 + 2 + 1 + 2;
constexpr int kOffRed = kOffBar + 8 * 32;  // [2 (max, sum)][4 quadrants][2 halves][32] F32
// Key splits: receive area of the query slots this CTA merges, written by
// every split of its cluster: (scaled max, sum) [64][2] and unnormalised O
// [64][128] F32, each indexed [split * cols + slot] (splits * cols <= 64).
constexpr int kOffX = kOffRed + 2 * 4 * 2 * 32 * 4;
constexpr int kOffXO = kOffX + 2 * 64 * 4;
constexpr int kSmem = kOffXO + 64 * 128 * 4 + 1024;
constexpr int kMaxSplits = 4;
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

// Key-split merge of this CTA's query slots [split cols, (split + 1) cols)
// from its receive area (every split's scaled max, sum and unnormalised O),
// in split order.
template <int SPL>
__device__ __forceinline__ void merge_slots(const AttnArgs& a, const float* xml, const float* xo, int split,
                                            int cols, int wt, int nq, int q0, int seq, int head) {
  for (int it = wt; it < cols * 16; it += kSoft) {
    const int jl = it / 16, g = it % 16, j = split * cols + jl;
    if (j >= nq) break;
    float mp[SPL], lp[SPL];
    float4 o0[SPL], o1[SPL];
#pragma unroll
    for (int p = 0; p < SPL; ++p) {
      mp[p] = xml[2 * (p * cols + jl)];
      lp[p] = xml[2 * (p * cols + jl) + 1];
      const float4* ob = reinterpret_cast<const float4*>(xo + (p * cols + jl) * 128 + g * 8);
      o0[p] = ob[0];
      o1[p] = ob[1];
    }
    float mx = mp[0];
#pragma unroll
    for (int p = 1; p < SPL; ++p) mx = fmaxf(mx, mp[p]);
    float den = 0.0f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < SPL; ++p) {
      const float w = ex2_approx(mp[p] - mx);
      den += w * lp[p];
      acc[0] += w * o0[p].x; acc[1] += w * o0[p].y; acc[2] += w * o0[p].z; acc[3] += w * o0[p].w;
      acc[4] += w * o1[p].x; acc[5] += w * o1[p].y; acc[6] += w * o1[p].z; acc[7] += w * o1[p].w;
    }
    const float f = 1.0f / den;
    const int row = q0 + j;  // query row of the sequence
    bf16* dst;
    if (a.split_first) {
      dst = row == 0 ? a.out_first + static_cast<long long>(seq) * a.ldo_first
                     : a.out + (static_cast<long long>(seq) * (a.lq - 1) + row - 1) * a.ldo;
    } else {
      dst = a.out + (static_cast<long long>(seq) * a.lq + row) * a.ldo;
    }
    *reinterpret_cast<uint4*>(dst + head * 128 + g * 8) =
        make_uint4(pack_bf16(acc[0] * f, acc[1] * f), pack_bf16(acc[2] * f, acc[3] * f),
                   pack_bf16(acc[4] * f, acc[5] * f), pack_bf16(acc[6] * f, acc[7] * f));
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_dec_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ AttnArgs a,
                            int splits) {
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
  uint64_t* x_ready = o_full + 1;  // key splits: every split's partials have arrived
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* xml = reinterpret_cast<float*>(smem + kOffX);  // receive area (key splits)
  float* xo = reinterpret_cast<float*>(smem + kOffXO);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // With key splits the CTAs of a (sequence, head) form a cluster along x;
  // split r takes key tiles [r nk_all / splits, (r + 1) nk_all / splits).
  const int split = splits > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int head = static_cast<int>(blockIdx.x) / splits, seq = blockIdx.y;
  const int nk_all = (a.lk + kKeys - 1) / kKeys;  // 1 .. kMaxTiles (checked by the host)
  const int t_begin = split * nk_all / splits;
  const int nk = (split + 1) * nk_all / splits - t_begin;  // >= 1: splits <= nk_all

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], 1);
    mbar_init(&p_full[0], kSoftWarps);
    mbar_init(&p_full[1], kSoftWarps);
    fence_barrier_init();
    if (splits > 1) {
      // every split sends (scaled max, sum) and 128 O values of each of this
      // CTA's query slots below nq: 520 bytes per slot and split
      const int nq = (a.q_end > 0 ? a.q_end : a.lq) - a.q_begin;
      const int cols = (nq + splits - 1) / splits;
      const int mine = nq - split * cols < cols ? nq - split * cols : cols;
      mbar_init(x_ready, 1);
      fence_barrier_init();
      mbar_arrive_expect_tx(x_ready, static_cast<uint32_t>(splits * (mine > 0 ? mine : 0) * 520));
    }
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Every peer's mbarriers exist before anyone arrives on them remotely (all
  // threads converged here, right after the CTA barrier).
  if (splits > 1) cluster_sync_all();
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
        const int t = t_begin + (i < nk ? i : i - nk);
        const CUtensorMap* m = i < nk ? &tm_k : &tm_v;
        uint8_t* dst = ring + slot * kTile;
        mbar_arrive_expect_tx(&slot_full[slot], kTile);
        tma_load_4d(dst, m, &slot_full[slot], 0, t * kKeys, head, seq, pol);
        tma_load_4d(dst + kHalf, m, &slot_full[slot], 64, t * kKeys, head, seq, pol);
      };
      int issued = 0;
      // K / V rows the preceding kernel does not write start before waiting for it.
      while (issued < items && issued < kRing) {
        const int t = t_begin + (issued < nk ? issued : issued - nk);
        const int end = (t + 1) * kKeys < a.lk ? (t + 1) * kKeys : a.lk;
        if (end > a.static_keys) break;
        load(issued++);
      }
      griddep_wait();
      griddep_launch_dependents();
      mbar_arrive_expect_tx(q_full, 2 * kQHalf);
      tma_load_4d(sq, &tm_q, q_full, 0, a.q_begin, head, seq, pol);
      tma_load_4d(sq + kQHalf, &tm_q, q_full, 64, a.q_begin, head, seq, pol);
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
      // S^T over the query slots in use (N = the launch's rows rounded up to
      // 16; the columns past them are discarded)
      const int nq = (a.q_end > 0 ? a.q_end : a.lq) - a.q_begin;
      const uint32_t idesc_s = umma_idesc_bf16(kKeys, ((nq + 15) / 16) * 16);
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
    // query rows [q0, q0 + nq) of the sequence are this launch's slots 0 .. nq - 1
    const int q0 = a.q_begin;
    const int nq = (a.q_end > 0 ? a.q_end : a.lq) - q0;
    const float sl2 = a.scale * 1.4426950408889634f;
    float* red_m = red;                     // [4][2][32]
    float* red_l = red + 4 * 2 * 32;
    bool chunk_ok[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) chunk_ok[c] = 16 * c + 8 * half < nq;
    bool ok = true;

    // Pass 1: per-query max over this thread's keys (one per tile).
    float m[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) m[i] = -INFINITY;
    for (int t = 0; t < nk; ++t) {
      if (!mbar_wait(&s_full[t], 0)) ok = false;
      tc_fence_after();
      const int key = (t_begin + t) * kKeys + quad * 32 + lane;
      if ((t_begin + t) * kKeys + quad * 32 >= a.lk) continue;  // warp-uniform: no key of this warp
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
    float mb_lane;  // column `lane`'s, kept for the merge of key splits
    {
      float v = red_m[half * 32 + lane];
#pragma unroll
      for (int q = 1; q < 4; ++q) v = fmaxf(v, red_m[(q * 2 + half) * 32 + lane]);
      mb_lane = v * sl2;
#pragma unroll
      for (int i = 0; i < 32; ++i) mb[i] = __shfl_sync(0xffffffffu, mb_lane, i);
    }

    // Pass 2: probabilities -> P^T buffers, per-query sums.
    float l[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) l[i] = 0.0f;
    const int prow = quad * 32 + lane;  // key row of the P^T tile
    for (int t = 0; t < nk && ok; ++t) {
      const int b = t & 1;
      const int key = (t_begin + t) * kKeys + prow;
      const bool warp_keys = (t_begin + t) * kKeys + quad * 32 < a.lk;
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
    const bool all_ok = named_bar_and(1, kSoft, ok);
    if (splits > 1) {
      // ----------------------------------------------- merge of key splits
      // CTA r of the cluster merges query slots [r cols, (r + 1) cols). Every
      // split sends its scaled max, sum and unnormalised O^T of those slots
      // into the owner's receive area with st.async from registers, counted
      // in bytes on the owner's x_ready (which expects them since kernel
      // start); an owner merges from its own shared memory once all have
      // landed. No CTA reads another's memory and nothing is written into a
      // CTA after its x_ready has completed, so each may leave once merged.
      // The sends happen whatever went before (outputs only when every wait
      // succeeded).
      tc_fence_after();
      const int cols = (nq + splits - 1) / splits;
      float lsum = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) lsum += red_l[(q * 2 + half) * 32 + lane];
      if (quad == 0) {
        const int col = 16 * (lane >> 3) + 8 * half + (lane & 7);
        if (col < nq) {
          const uint32_t own = static_cast<uint32_t>(col / cols);
          const int jl = col - static_cast<int>(own) * cols;
          st_async_v2_b32(mapa_shared(smem_u32(xml + 2 * (split * cols + jl)), own), __float_as_uint(mb_lane),
                          __float_as_uint(lsum), mapa_shared(smem_u32(x_ready), own));
        }
      }
      {
        uint32_t r[4][8];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (chunk_ok[c]) tmem_ld_x8(tmem + lane_off + kTmemO + static_cast<uint32_t>(16 * c + 8 * half), r[c]);
        tmem_ld_wait();
        // 4 x 4 transposes within groups of 4 lanes: lane 4m + s then holds
        // query slot 4k + s of the chunk for dims 4m .. 4m + 3 (one 16-byte
        // store)
        const int s0 = lane & 1, s1 = (lane >> 1) & 1;
        const int dbase = quad * 32 + (lane & ~3);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (!chunk_ok[c]) continue;  // warp-uniform
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            uint32_t t[4] = {r[c][4 * k], r[c][4 * k + 1], r[c][4 * k + 2], r[c][4 * k + 3]};
#pragma unroll
            for (int jj = 0; jj < 4; jj += 2) {
              const uint32_t recv = __shfl_xor_sync(0xffffffffu, s0 ? t[jj] : t[jj + 1], 1);
              if (s0) t[jj] = recv; else t[jj + 1] = recv;
            }
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const uint32_t recv = __shfl_xor_sync(0xffffffffu, s1 ? t[jj] : t[jj + 2], 2);
              if (s1) t[jj] = recv; else t[jj + 2] = recv;
            }
            const int j = 16 * c + 8 * half + 4 * k + (lane & 3);
            if (j >= nq) continue;
            const uint32_t own = static_cast<uint32_t>(j / cols);
            const int jl = j - static_cast<int>(own) * cols;
            st_async_v4_b32(mapa_shared(smem_u32(xo + (split * cols + jl) * 128 + dbase), own), t[0], t[1], t[2],
                            t[3], mapa_shared(smem_u32(x_ready), own));
          }
        }
      }
      const bool xok = mbar_wait_cluster(x_ready, 0);
      const int wt = static_cast<int>(threadIdx.x) - 64;
      if (xok && all_ok) {
        if (splits == 4)
          merge_slots<4>(a, xml, xo, split, cols, wt, nq, q0, seq, head);
        else
          merge_slots<2>(a, xml, xo, split, cols, wt, nq, q0, seq, head);
      } else if (!xok) {
        fail(a, kErrEpilogueTimeout);
      }
    } else if (all_ok) {
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
          if (qr >= nq) continue;
          const int row = q0 + qr;
          bf16* dst;
          if (a.split_first) {
            dst = row == 0 ? a.out_first + static_cast<long long>(seq) * a.ldo_first
                           : a.out + (static_cast<long long>(seq) * (a.lq - 1) + row - 1) * a.ldo;
          } else {
            dst = a.out + (static_cast<long long>(seq) * a.lq + row) * a.ldo;
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

// WAM_B200_ATTN_DEC_TC=0 sends these shapes to the mma.sync kernel
// (attention.cu). Measured in the engine's graph, us per launch, this kernel
// against that one: batch 1 9.30 / 9.33 (4 key splits), batch 8 24.4 / 25.0,
// batch 64 140.4 / 142.1.
bool dec_tc_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("WAM_B200_ATTN_DEC_TC");
    return !(v && v[0] == '0');
  }();
  return on;
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
  const int rows = (a.q_end > 0 ? a.q_end : a.lq) - a.q_begin;
  return dec_tc_enabled() && rows >= 1 && rows <= kSlots && a.q_begin >= 0 && a.lk >= 1 &&
         a.lk <= kMaxTiles * kKeys && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.k) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.v) & 15) == 0 &&
         a.q_head_stride % 8 == 0 && a.q_seq_stride % 8 == 0 && a.kv_head_stride % 8 == 0 &&
         a.kv_seq_stride % 8 == 0 && a.batch <= 65535;
}

// Key splits (CTAs per (sequence, head), a cluster): the most of 1 / 2 / 4,
// at most one per key tile, whose CTAs still fit the SMs in one wave.
int dec_tc_splits(const AttnArgs& a) {
  const int nk = (a.lk + kKeys - 1) / kKeys;
  const long long ctas = static_cast<long long>(a.heads) * a.batch;
  int best = 1;
  for (int c = 2; c <= kMaxSplits; c *= 2)
    if (c <= nk && ctas * c <= sm_count()) best = c;
  return best;
}

cudaError_t launch_attention_dec_tc(const AttnArgs& a, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (!attn_encode_rows(&mq, a.q, a.lq, a.heads, a.batch, a.q_head_stride, a.q_seq_stride, kSlots) ||
      !attn_encode_rows(&mk, a.k, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride, kKeys) ||
      !attn_encode_rows(&mv, a.v, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride, kKeys))
    return cudaErrorInvalidValue;
  const int splits = dec_tc_splits(a);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.heads * splits, a.batch, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = splits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = splits > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, attention_dec_tc_kernel, mq, mk, mv, a, splits);
}

}  // namespace wamb
