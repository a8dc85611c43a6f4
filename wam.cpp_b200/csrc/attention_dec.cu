// tcgen05 flash attention for short query blocks: the denoise step's 48 action
// queries per (request, head) over the joint self-attention keys (state +
// visual prefix + action rows, 817 at config 2) and over the prompt's
// cross-attention keys (512), and the prefix state token's cross attention.
//
// One CTA = up to 64 query rows of one (sequence, head) and one contiguous
// range of its keys; the key ranges of a (sequence, head) are split over the
// CTAs of a thread-block cluster. Per key tile of 128:
//   S = Q K^T   (tcgen05.mma M = 64 queries, N = 128 keys, K = 128 dims, TMEM)
//   softmax     (one thread per query row reads its S row from TMEM; online
//                max with lazy rescaling of O, F32, P rounded to BF16)
//   O += P V^T  (M = 64 queries, N = 128 dims, K = 128 keys, TMEM)
// Q, K and V arrive by TMA (4-D boxes, 128-byte swizzle, rows past the end
// zero-filled); V is transposed to K-major in shared memory (ldmatrix.trans /
// stmatrix) into K's buffer once S is done, and P is written into V's. The
// splits then merge: each CTA writes its unnormalised O rows with their
// running max and sum to the caller's workspace (L2), the cluster meets at one
// barrier, and each CTA combines the rows it owns over all splits in split
// order and stores BF16. Without a workspace the rows move by one bulk copy
// per peer into the owner's shared memory (counted in bytes on its mbarrier).
//
// Arithmetic as attention.cu: F32 scores, softmax(scale * S) with F32 max and
// sum, probabilities rounded to BF16 for P V, F32 accumulation, BF16 output.
// Reference: the cached joint attention (src/models/gwp05/engine/mot.cpp:
// 432-446, scores at GGML_PREC_F32, ggml_soft_max_ext with scale 1/sqrt(128),
// no mask) and the cached cross attention (mot.cpp:299-321).
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "kernels.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace wamb {

namespace {

constexpr int kThreads = 192;          // warps 0-3 softmax (TMEM quadrants 0-3), 4 copies, 5 MMAs
constexpr int kSoftThreads = 128;
constexpr int kRows = 64;              // queries per CTA (UMMA M = 64)
constexpr int kKeys = 128;             // keys per tile
constexpr int kQHalf = kRows * 128;    // 64 rows x 64 dims, swizzled: 8 KB
constexpr int kKHalf = kKeys * 128;    // 128 rows x 64 dims (or keys): 16 KB
constexpr int kOffQ = 0;               // Q [2 halves of dims]
constexpr int kOffK = 2 * kQHalf;      // K [2 halves of dims], then V^T [2 halves of keys]
constexpr int kOffV = kOffK + 2 * kKHalf;  // V [2 halves of dims], then P [2 halves of keys]
constexpr int kOffRecv = kOffV + 2 * kKHalf;
constexpr int kRowRec = 132;           // floats per merged row record: O[128], max, sum, pad
constexpr int kMaxSplits = 8;
constexpr uint32_t kTmemCols = 256;    // S (128) + O (128)

// Query rows [row_begin(s), row_begin(s + 1)) of `rows` are merged by split s.
__host__ __device__ inline int row_begin(int s, int rows, int splits) {
  return (s * rows + splits - 1) / splits;
}
__host__ __device__ inline int recv_bytes(int rows, int splits) {
  return splits <= 1 ? 0 : splits * ((rows + splits - 1) / splits) * kRowRec * 4;
}
inline int smem_bytes(int rows, int splits) {
  return kOffRecv + recv_bytes(rows, splits) + 128 /* barriers */ + 1024 /* alignment */;
}

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

__device__ __forceinline__ void fail(const AttnArgs& a, unsigned code) {
  if (a.error) atomicCAS(a.error, 0u, code);
}

// blockIdx.x = key split (cluster rank), blockIdx.y = head, blockIdx.z = sequence.
// Warps 0-3 run the softmax and the merge (warp w reads TMEM lanes 32w..), warp
// 4 lane 0 issues the copies, warp 5 owns TMEM and its lane 0 issues the MMAs.
__global__ void __launch_bounds__(kThreads, 2)
    attention_dec_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ AttnArgs a,
                         int splits, int use_ws) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem + kOffQ;
  uint8_t* sk = smem + kOffK;  // K, then V^T
  uint8_t* sv = smem + kOffV;  // V, then P
  const int rows = a.lq < kRows ? a.lq : kRows;  // valid query rows (lq <= 64)
  uint8_t* recv = smem + kOffRecv;
  uint64_t* bars = reinterpret_cast<uint64_t*>(recv + recv_bytes(rows, use_ws ? 1 : splits));
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* p_full = bars + 4;
  uint64_t* pv_done = bars + 5;
  uint64_t* recv_bar = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, head = blockIdx.y, seq = blockIdx.z;
  const int nkt_all = (a.lk + kKeys - 1) / kKeys;
  const int kt0 = (split * nkt_all) / splits, kt1 = ((split + 1) * nkt_all) / splits;
  const int nk = kt1 - kt0;  // key tiles of this split (may be 0)
  const int rb0 = row_begin(split, rows, splits), rb1 = row_begin(split + 1, rows, splits);
  const int maxown = (rows + splits - 1) / splits;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    for (int i = 0; i < 7; ++i) mbar_init(&bars[i], 1);
    if (splits > 1 && !use_ws)  // armed with every byte the peers will copy here
      mbar_arrive_expect_tx(recv_bar,
                            static_cast<uint32_t>((splits - 1) * (rb1 - rb0) * kRowRec * 4));
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (splits > 1) cluster_arrive_aligned();  // this CTA's receive barrier is armed
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_o = tmem + 128;

  if (warp == 4) {
    if (lane == 0) {
    // ---------------------------------------------------- copy producer
    const uint64_t pol_kv = policy_evict_last();
    const uint64_t pol_q = policy_evict_first();
    auto load_kv = [&](int j) {
      const int key = (kt0 + j) * kKeys;
      mbar_arrive_expect_tx(k_full, 2 * kKHalf);
      tma_load_4d(sk, &tm_k, k_full, 0, key, head, seq, pol_kv);
      tma_load_4d(sk + kKHalf, &tm_k, k_full, 64, key, head, seq, pol_kv);
      mbar_arrive_expect_tx(v_full, 2 * kKHalf);
      tma_load_4d(sv, &tm_v, v_full, 0, key, head, seq, pol_kv);
      tma_load_4d(sv + kKHalf, &tm_v, v_full, 64, key, head, seq, pol_kv);
    };
    // K / V rows the preceding kernel does not write (cached prefix rows,
    // prompt K/V) start loading before waiting for it.
    int issued = 0;
    if (nk > 0 && (kt0 + 1) * kKeys <= a.static_keys) {
      load_kv(0);
      issued = 1;
    }
    griddep_launch_dependents();  // the next kernel may start its own pre-wait work
    griddep_wait();
    mbar_arrive_expect_tx(q_full, 2 * kQHalf);
    tma_load_4d(sq, &tm_q, q_full, 0, 0, head, seq, pol_q);
    tma_load_4d(sq + kQHalf, &tm_q, q_full, 64, 0, head, seq, pol_q);
    bool ok = true;
    for (int j = issued; j < nk && ok; ++j) {
      // K's buffer holds V^T and V's holds P until tile j - 1's P V is done.
      if (j >= 1 && !mbar_wait(pv_done, (j - 1) & 1)) {
        ok = false;
        break;
      }
      load_kv(j);
    }
    if (!ok) fail(a, kErrProducerTimeout);
    // Every issued copy lands before the CTA moves on.
    mbar_wait(q_full, 0);
    }
  } else if (warp == 5) {
    if (lane == 0) {
    // ------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = umma_idesc_bf16(kRows, kKeys);  // N = 128 keys, or 128 dims
    bool ok = mbar_wait(q_full, 0);
    for (int j = 0; j < nk && ok; ++j) {
      if (!mbar_wait(k_full, j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint64_t da = sw128_kmajor_desc(smem_u32(sq + c * kQHalf));
        const uint64_t db = sw128_kmajor_desc(smem_u32(sk + c * kKHalf));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16_ss(t_s, da + 2 * kk, db + 2 * kk, idesc, (c | kk) != 0 ? 1u : 0u);
      }
      umma_commit(s_full);
      if (!mbar_wait(p_full, j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint64_t da = sw128_kmajor_desc(smem_u32(sv + c * kQHalf));  // P half: 64 rows x 64 keys
        const uint64_t db = sw128_kmajor_desc(smem_u32(sk + c * kKHalf));  // V^T half: 128 dims x 64 keys
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16_ss(t_o, da + 2 * kk, db + 2 * kk, idesc, (j > 0 || c != 0 || kk != 0) ? 1u : 0u);
      }
      umma_commit(pv_done);
    }
    if (!ok) fail(a, kErrMmaTimeout);
    }
  }
  __syncwarp();
  if (warp >= 4) {
    // the copy / MMA warps complete both phases of the split cluster barrier
    if (splits > 1) {
      cluster_wait_aligned();
      cluster_sync_all();
    }
  } else {
  // ------------------------------------------ softmax / V^T / P (warps 0-3)
  // M = 64: query row r's accumulators sit in TMEM lane 32 (r / 16) + r % 16,
  // so lanes 0-15 of warp q own rows 16q..16q+15; every thread helps with V^T.
  const int qd = warp;
  const int row = qd * 16 + (lane & 15);
  const bool row_thread = lane < 16;
  const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
  const float sl2 = a.scale * 1.4426950408889634f;
  float m_used = -INFINITY, l = 0.0f;
  bool ok = true;
  for (int j = 0; j < nk; ++j) {
    ok = mbar_wait(s_full, j & 1);
    tc_fence_after();
    const int key0 = (kt0 + j) * kKeys;
    const int valid = a.lk - key0 < kKeys ? a.lk - key0 : kKeys;
    uint32_t pk[64];
    float mt = -INFINITY;
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      uint32_t r[32];
      tmem_ld_x32(t_s + lane_off + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c + i < valid) mt = fmaxf(mt, u2f(r[i]));
    }
    const float m_new = fmaxf(m_used, mt);
    const bool rescale = j == 0 || (m_new - m_used) * sl2 > 8.0f;
    const float mb = (rescale ? m_new : m_used) * sl2;
    float ls = 0.0f;
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      uint32_t r[32];
      tmem_ld_x32(t_s + lane_off + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const int k = c + i;
        const float p0 = k < valid ? exp2f(u2f(r[i]) * sl2 - mb) : 0.0f;
        const float p1 = k + 1 < valid ? exp2f(u2f(r[i + 1]) * sl2 - mb) : 0.0f;
        ls += p0 + p1;
        pk[(c + i) >> 1] = pack_bf16(p0, p1);
      }
    }
    // V of tile j lands; K's buffer is free once S is complete (s_full).
    if (ok) ok = mbar_wait(v_full, j & 1);
    if (!named_bar_and(1, kSoftThreads, ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    // O holds tiles 0..j-1 (their P V completed before this iteration began);
    // a rescale brings a row to its new max. The TMEM loads / stores are
    // warp-collective, so the warp runs them when any of its rows rescales
    // and the other rows scale by 1.
    if (__any_sync(0xffffffffu, rescale && row_thread) && j > 0) {
      const float corr = row_thread ? exp2f((m_used - m_new) * sl2) : 1.0f;
      const float f = rescale ? corr : 1.0f;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t r[32];
        tmem_ld_x32(t_o + lane_off + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(u2f(r[i]) * f);
        tmem_st_x32(t_o + lane_off + c, r);
      }
      tmem_st_wait();
      if (rescale) l *= corr;
    }
    if (rescale) m_used = m_new;
    l += ls;
    // V (rows = keys) -> V^T (rows = dims, K-major over keys) into K's buffer:
    // warp w transposes key groups 4w..4w+3 (8 keys each) x 16 dim groups.
    {
      const int m = lane >> 3, i8 = lane & 7;
#pragma unroll
      for (int kgi = 0; kgi < 4; ++kgi) {
        const int kg = warp * 4 + kgi;
        const int key = 8 * kg + i8;
#pragma unroll
        for (int dq = 0; dq < 16; dq += 4) {
          const int dg = dq + m;
          const uint32_t src = smem_u32(sv) + (dg >> 3) * kKHalf + key * 128 +
                               ((((dg & 7) ^ (key & 7))) << 4);
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4_trans(src, r0, r1, r2, r3);
          const int dr = 8 * dg + i8;  // row i8 of destination matrix m
          const uint32_t dst = smem_u32(sk) + (kg >> 3) * kKHalf + dr * 128 +
                               ((((kg & 7) ^ (dr & 7))) << 4);
          stmatrix_x4(dst, r0, r1, r2, r3);
        }
      }
    }
    named_bar_sync(1, kSoftThreads);  // V read by every warp before P overwrites it
    // this row's 128 probabilities -> P (K-major over keys) in V's buffer
    if (row_thread) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t off = h * kQHalf + row * 128 + ((i ^ (row & 7)) << 4);
          const int b = h * 32 + i * 4;
          *reinterpret_cast<uint4*>(sv + off) = make_uint4(pk[b], pk[b + 1], pk[b + 2], pk[b + 3]);
        }
    }
    fence_proxy_async_smem();  // P and V^T (generic stores) are read by the tensor core
    tc_fence_before();
    named_bar_sync(1, kSoftThreads);
    if (threadIdx.x == 0) mbar_arrive(p_full);
    // the next tile's S overwrites TMEM S only after this tile's P was read
    // from it (above), and its copies need this tile's P V done (producer)
    if (j + 1 < nk) {
      ok = mbar_wait(pv_done, j & 1);
      if (!named_bar_and(1, kSoftThreads, ok)) {
        ok = false;
        break;
      }
    }
  }
  if (!ok) fail(a, kErrEpilogueTimeout);
  if (nk > 0 && ok) ok = mbar_wait(pv_done, (nk - 1) & 1);
  ok = named_bar_and(1, kSoftThreads, ok);
  tc_fence_after();

  // ---------------------------------------------------------- output / merge
  bf16* dst = nullptr;
  auto out_row = [&](int r) -> bf16* {
    if (r >= a.lq) return nullptr;
    bf16* d = a.split_first
                  ? (r == 0 ? a.out_first + static_cast<long long>(seq) * a.ldo_first
                            : a.out + (static_cast<long long>(seq) * (a.lq - 1) + r - 1) * a.ldo)
                  : a.out + (static_cast<long long>(seq) * a.lq + r) * a.ldo;
    return d + head * 128;
  };
  if (splits == 1) {
    if (row_thread && row < rows) dst = out_row(row);
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      uint32_t r[32];
      if (nk > 0) {
        tmem_ld_x32(t_o + lane_off + c, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (dst && ok) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(dst + c + q * 8) =
              make_uint4(pack_bf16(u2f(r[8 * q]) * inv, u2f(r[8 * q + 1]) * inv),
                         pack_bf16(u2f(r[8 * q + 2]) * inv, u2f(r[8 * q + 3]) * inv),
                         pack_bf16(u2f(r[8 * q + 4]) * inv, u2f(r[8 * q + 5]) * inv),
                         pack_bf16(u2f(r[8 * q + 6]) * inv, u2f(r[8 * q + 7]) * inv));
      }
    }
  } else if (use_ws) {
    // [row][O 128 | max | sum | pad] of every split to the workspace (L2); one
    // cluster barrier (release / acquire) and each owner merges its rows.
    cluster_wait_aligned();  // first phase of the split barrier (armed at start)
    float* wsb = a.ws + (static_cast<size_t>(seq) * a.heads + head) * splits * kRows * kRowRec;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      uint32_t r[32];
      if (nk > 0) {
        tmem_ld_x32(t_o + lane_off + c, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (row_thread && row < rows) {
        float4* d = reinterpret_cast<float4*>(wsb + (split * kRows + row) * kRowRec + c);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          d[q] = make_float4(u2f(r[4 * q]), u2f(r[4 * q + 1]), u2f(r[4 * q + 2]), u2f(r[4 * q + 3]));
      }
    }
    if (row_thread && row < rows)
      *reinterpret_cast<float2*>(wsb + (split * kRows + row) * kRowRec + 128) = make_float2(m_used, l);
    __syncwarp();
    cluster_sync_all();  // every split's rows are in the workspace
    const int items = (rb1 - rb0) * 8;
    for (int it = threadIdx.x; it < items; it += kSoftThreads) {
      const int jr = it >> 3, dc = (it & 7) * 16;
      const int r = rb0 + jr;
      float mv[kMaxSplits], lv[kMaxSplits];
      float mx = -INFINITY;
#pragma unroll
      for (int p = 0; p < kMaxSplits; ++p) {
        mv[p] = -INFINITY;
        lv[p] = 0.0f;
        if (p < splits) {
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(wsb + (p * kRows + r) * kRowRec + 128));
          mv[p] = ml.x;
          lv[p] = ml.y;
          mx = fmaxf(mx, ml.x);
        }
      }
      float acc[16], den = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int p = 0; p < kMaxSplits; ++p) {
        if (p >= splits) continue;
        const float w = mv[p] != -INFINITY ? exp2f((mv[p] - mx) * sl2) : 0.0f;
        den += w * lv[p];
        const float4* src = reinterpret_cast<const float4*>(wsb + (p * kRows + r) * kRowRec + dc);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 v = __ldcg(src + i);
          acc[4 * i] = fmaf(w, v.x, acc[4 * i]);
          acc[4 * i + 1] = fmaf(w, v.y, acc[4 * i + 1]);
          acc[4 * i + 2] = fmaf(w, v.z, acc[4 * i + 2]);
          acc[4 * i + 3] = fmaf(w, v.w, acc[4 * i + 3]);
        }
      }
      const float inv = den > 0.0f ? 1.0f / den : 0.0f;
      bf16* d = out_row(r);
      if (d && ok) {
        d += dc;
#pragma unroll
        for (int q = 0; q < 2; ++q)
          *reinterpret_cast<uint4*>(d + q * 8) =
              make_uint4(pack_bf16(acc[8 * q] * inv, acc[8 * q + 1] * inv),
                         pack_bf16(acc[8 * q + 2] * inv, acc[8 * q + 3] * inv),
                         pack_bf16(acc[8 * q + 4] * inv, acc[8 * q + 5] * inv),
                         pack_bf16(acc[8 * q + 6] * inv, acc[8 * q + 7] * inv));
      }
    }
  } else {
    // Stage [row][O 128 | max | sum | pad] in Q/K's buffers (every MMA is done),
    // then one bulk copy per peer of the rows it owns.
    cluster_wait_aligned();  // every peer's receive barrier is armed
    float* stg = reinterpret_cast<float*>(smem);
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      uint32_t r[32];
      if (nk > 0) {
        tmem_ld_x32(t_o + lane_off + c, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (row_thread && row < rows) {
        float4* d = reinterpret_cast<float4*>(stg + row * kRowRec + c);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          d[q] = make_float4(u2f(r[4 * q]), u2f(r[4 * q + 1]), u2f(r[4 * q + 2]), u2f(r[4 * q + 3]));
      }
    }
    if (row_thread && row < rows) {
      stg[row * kRowRec + 128] = m_used;
      stg[row * kRowRec + 129] = l;
    }
    fence_proxy_async_smem();
    named_bar_sync(1, kSoftThreads);
    if (threadIdx.x == 0) {
      const uint32_t recv_u32 = smem_u32(recv), bar_u32 = smem_u32(recv_bar);
      for (int o = 0; o < splits; ++o) {
        if (o == split) continue;
        const int o0 = row_begin(o, rows, splits), o1 = row_begin(o + 1, rows, splits);
        if (o1 <= o0) continue;
        bulk_copy_to_peer(
            mapa_shared(recv_u32 + static_cast<uint32_t>(split * maxown * kRowRec * 4),
                        static_cast<uint32_t>(o)),
            smem_u32(stg + o0 * kRowRec), static_cast<uint32_t>((o1 - o0) * kRowRec * 4),
            mapa_shared(bar_u32, static_cast<uint32_t>(o)));
      }
    }
    const bool got = rb1 > rb0 ? mbar_wait_cluster(recv_bar, 0) : true;
    if (!got) fail(a, kErrEpilogueTimeout);
    // Owned rows: 16-dim chunks, one per thread and pass; splits in order.
    const int items = (rb1 - rb0) * 8;
    for (int it = threadIdx.x; it < items; it += kSoftThreads) {
      const int jr = it >> 3, dc = (it & 7) * 16;
      const int r = rb0 + jr;
      auto rec = [&](int p) -> const float* {
        return p == split ? stg + r * kRowRec
                          : reinterpret_cast<const float*>(recv) + (p * maxown + jr) * kRowRec;
      };
      float mx = -INFINITY;
      for (int p = 0; p < splits; ++p) mx = fmaxf(mx, rec(p)[128]);
      float acc[16], den = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
      for (int p = 0; p < splits; ++p) {
        const float* rp = rec(p);
        const float w = rp[128] != -INFINITY ? exp2f((rp[128] - mx) * sl2) : 0.0f;
        den += w * rp[129];
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(rp + dc + i);
          acc[i] = fmaf(w, v.x, acc[i]);
          acc[i + 1] = fmaf(w, v.y, acc[i + 1]);
          acc[i + 2] = fmaf(w, v.z, acc[i + 2]);
          acc[i + 3] = fmaf(w, v.w, acc[i + 3]);
        }
      }
      const float inv = den > 0.0f ? 1.0f / den : 0.0f;
      bf16* d = out_row(r);
      if (d && ok && got) {
        d += dc;
#pragma unroll
        for (int q = 0; q < 2; ++q)
          *reinterpret_cast<uint4*>(d + q * 8) =
              make_uint4(pack_bf16(acc[8 * q] * inv, acc[8 * q + 1] * inv),
                         pack_bf16(acc[8 * q + 2] * inv, acc[8 * q + 3] * inv),
                         pack_bf16(acc[8 * q + 4] * inv, acc[8 * q + 5] * inv),
                         pack_bf16(acc[8 * q + 6] * inv, acc[8 * q + 7] * inv));
      }
    }
    // no CTA leaves while a bulk copy out of its shared memory may be running
    __syncwarp();
    cluster_sync_all();
  }
  }  // softmax warps

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [batch][heads][rows][128] BF16 with the given strides (elements), boxes of
// box_rows rows x 64 dims with the 128-byte swizzle; rows past `rows` read as zero.
bool encode_rows(CUtensorMap* m, const void* base, int rows, int heads, int batch,
                 long long head_stride, long long seq_stride, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if (batch == 1) seq_stride = head_stride * heads;
  const cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[3] = {256, static_cast<cuuint64_t>(head_stride) * 2,
                                 static_cast<cuuint64_t>(seq_stride) * 2};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool dec_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("WAM_B200_ATTN_DEC");
    return !(v && v[0] == '0');
  }();
  return on;
}

}  // namespace

cudaError_t attention_dec_init() {
  return cudaFuncSetAttribute(attention_dec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              smem_bytes(kRows, kMaxSplits));
}

bool attention_dec_eligible(const AttnArgs& a) {
  return dec_enabled() && a.lq >= 1 && a.lq <= kRows && a.lk >= 1 &&
         (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.k) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.v) & 15) == 0 && a.q_head_stride % 8 == 0 &&
         a.q_seq_stride % 8 == 0 && a.kv_head_stride % 8 == 0 && a.kv_seq_stride % 8 == 0 &&
         a.ldo % 8 == 0 && (!a.split_first || a.ldo_first % 8 == 0);
}

// Key splits: as many CTAs per (sequence, head) as keep the launch within the
// resident CTAs (two per SM), each with at least one key tile, at most 8.
int attention_dec_splits(const AttnArgs& a, int num_sms) {
  const int ctas = a.heads * a.batch;
  const int tiles = (a.lk + kKeys - 1) / kKeys;
  int best = 1;
  for (int s = 2; s <= kMaxSplits; ++s)
    if (ctas * s <= 2 * num_sms && s <= tiles) best = s;
  return best;
}

cudaError_t launch_attention_dec(const AttnArgs& a, int num_sms, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (!encode_rows(&mq, a.q, a.lq, a.heads, a.batch, a.q_head_stride, a.q_seq_stride, kRows) ||
      !encode_rows(&mk, a.k, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride, kKeys) ||
      !encode_rows(&mv, a.v, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride, kKeys))
    return cudaErrorInvalidValue;
  const int splits = attention_dec_splits(a, num_sms);
  const int rows = a.lq < kRows ? a.lq : kRows;
  // The splits merge through the caller's workspace when it holds every
  // split's rows, else through the cluster's shared memory.
  const int use_ws = splits > 1 && a.ws &&
                     a.ws_floats >= static_cast<size_t>(a.batch) * a.heads * splits * kRows * kRowRec;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, a.heads, a.batch);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes(rows, use_ws ? 1 : splits);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = splits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, attention_dec_kernel, mq, mk, mv, a, splits, use_ws);
}

}  // namespace wamb
