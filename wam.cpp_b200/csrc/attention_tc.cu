// tcgen05 flash attention for query blocks of 128 rows: the prefix joint
// self-attention and visual cross-attention (769 / 768 queries) and the
// attention microbench (816 queries over 1280-16384 cached keys).
//
// One CTA = 128 query rows of one (sequence, head); keys stream in tiles of
// 128. Both products run on the tensor cores with accumulators in TMEM:
// S = Q K^T (M = 128 queries, N = 128 keys, K = 128 dims) into one of two S
// buffers, O += P V^T (M = 128 queries, N = 128 dims, K = 128 keys) into O.
// Roles (576 threads): warp 0 issues the TMA copies (4-D boxes of 128 rows x
// 64 dims with the 128-byte swizzle; rows past the end are zero-filled),
// warp 1 owns TMEM and issues the MMAs (S of tile j + 1 before P V of tile j,
// so the tensor core runs while the softmax works), warps 2-17 = four threads
// per query row, each over a quarter of the keys / dims (the row max and sum
// are exchanged through shared memory): softmax from S in TMEM (one pass, the
// thread's scores held in registers), P as BF16 written back into the first
// 64 columns of its own S buffer in TMEM (the A operand of P V), lazy
// rescaling of O in TMEM (only when the running max grows by more than 2^8),
// and the final normalised BF16 rows. Q and K use the K-major swizzled layout
// of the GEMM (csrc/gemm.cu); V tiles (double-buffered) are read by the tensor
// core as they land, as an MN-major operand (dims contiguous), with no
// transpose.
//
// Arithmetic as attention.cu's kernel: F32 scores, softmax(scale * S) with an
// online max, probabilities rounded to BF16 for P V, F32 accumulation, BF16
// output. Reference: the prefix attention (src/models/gwp05/engine/cache.cpp:274-287),
// the cached cross attention (mot.cpp:299-321) and ggml_soft_max_ext with scale
// 1/sqrt(128) at GGML_PREC_F32 (mot.cpp:432-446).
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "kernels.h"
#include "launch.cuh"
#include "ptx.cuh"

namespace wamb {

namespace {

constexpr int kParts = 4;                 // softmax threads per query row
constexpr int kCols = 128 / kParts;       // keys (of S) and dims (of O) per softmax thread
constexpr int kSoftmax = 128 * kParts;    // softmax threads
constexpr int kThreads = 64 + kSoftmax;   // warp 0 copies, 1 MMA, 2.. softmax
constexpr int kRows = 128;                // queries per CTA (UMMA M, TMEM lanes)
constexpr int kKeys = 128;                // keys per tile
constexpr int kHalf = 128 * 64 * 2;       // 128 rows x 64 dims (or keys), swizzled: 16 KB
constexpr int kTile = 2 * kHalf;          // 32 KB
constexpr int kOffQ = 0;                  // Q [2 halves of dims]
constexpr int kOffK = kTile;              // K ring [2][2 halves]
constexpr int kOffV = 3 * kTile;          // V ring [2][2 halves of dims], rows = keys
constexpr int kOffBar = 5 * kTile;
constexpr int kOffXch = kOffBar + 256;    // row max / sum exchange between a row's kParts threads
constexpr int kSmem = 5 * kTile + 256 + 2 * 4 * 128 * kParts + 1024 + 256;
constexpr uint32_t kTmemCols = 512;       // S[0], S[1], O (128 columns each)

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

__device__ __forceinline__ void fail(const AttnArgs& a, unsigned code) {
  if (a.error) atomicCAS(a.error, 0u, code);
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sq = smem + kOffQ;
  uint8_t* sk = smem + kOffK;
  uint8_t* sv = smem + kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_free = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;
  uint64_t* pv_done = bars + 14;
  uint64_t* o_full = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = a.q_begin + blockIdx.x * kRows, head = blockIdx.y, seq = blockIdx.z;
  const int q_end = a.q_end > 0 ? a.q_end : a.lq;
  const int nk = (a.lk + kKeys - 1) / kKeys;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    for (int i = 0; i < 16; ++i) mbar_init(&bars[i], 1);
    // P is published by every softmax warp (an S buffer is freed by the
    // commit of the P V that read the P written into it)
    mbar_init(p_full, kSoftmax / 32);
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
  const uint32_t t_s[2] = {tmem, tmem + 128};
  const uint32_t t_o = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------- copy producer
      const uint64_t pol_kv = policy_evict_last();  // K / V are read by every query tile of the head
      const uint64_t pol_q = policy_evict_first();
      auto load_k = [&](int j) {
        const int b = j & 1;
        mbar_arrive_expect_tx(&k_full[b], kTile);
        tma_load_4d(sk + b * kTile, &tm_k, &k_full[b], 0, j * kKeys, head, seq, pol_kv);
        tma_load_4d(sk + b * kTile + kHalf, &tm_k, &k_full[b], 64, j * kKeys, head, seq, pol_kv);
      };
      auto load_v = [&](int j) {
        const int b = j & 1;
        mbar_arrive_expect_tx(&v_full[b], kTile);
        tma_load_4d(sv + b * kTile, &tm_v, &v_full[b], 0, j * kKeys, head, seq, pol_kv);
        tma_load_4d(sv + b * kTile + kHalf, &tm_v, &v_full[b], 64, j * kKeys, head, seq, pol_kv);
      };
      int nk_issued = 0, nv_issued = 0;
      // K / V the preceding kernel does not write start before waiting for it.
      if (nk > 0 && (a.lk < kKeys ? a.lk : kKeys) <= a.static_keys) {
        load_k(0);
        load_v(0);
        nk_issued = nv_issued = 1;
      }
      griddep_wait();
      griddep_launch_dependents();
      mbar_arrive_expect_tx(q_full, kTile);
      tma_load_4d(sq, &tm_q, q_full, 0, q0, head, seq, pol_q);
      tma_load_4d(sq + kHalf, &tm_q, q_full, 64, q0, head, seq, pol_q);
      bool ok = true;
      for (int j = 0; j < nk && ok; ++j) {
        if (j >= nk_issued) {
          if (j >= 2 && !mbar_wait(&k_empty[j & 1], ((j >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          load_k(j);
          nk_issued = j + 1;
        }
        if (j >= nv_issued) {
          if (j >= 2 && !mbar_wait(&v_empty[j & 1], ((j >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          load_v(j);
          nv_issued = j + 1;
        }
      }
      if (!ok) fail(a, kErrProducerTimeout);
      // Every issued copy lands before the CTA leaves.
      mbar_wait(q_full, 0);
      for (int j = nk_issued - 2 > 0 ? nk_issued - 2 : 0; j < nk_issued; ++j)
        mbar_wait(&k_full[j & 1], (j >> 1) & 1);
      for (int j = nv_issued - 2 > 0 ? nv_issued - 2 : 0; j < nv_issued; ++j)
        mbar_wait(&v_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16(kRows, kKeys);
      constexpr uint32_t idesc_pv = umma_idesc_bf16_bmn(kRows, 128);  // V MN-major
      bool ok = mbar_wait(q_full, 0);
      for (int j = 0; j <= nk && ok; ++j) {
        if (j < nk) {
          const int b = j & 1;
          if (!mbar_wait(&k_full[b], (j >> 1) & 1) ||
              (j >= 2 && !mbar_wait(&s_free[b], ((j >> 1) - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint64_t da = sw128_kmajor_desc(smem_u32(sq + c * kHalf));
            const uint64_t db = sw128_kmajor_desc(smem_u32(sk + b * kTile + c * kHalf));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_ss(t_s[b], da + 2 * kk, db + 2 * kk, idesc, (c | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&s_full[b]);
          umma_commit(&k_empty[b]);
        }
        if (j >= 1) {
          const int jj = j - 1;
          const int vb = jj & 1;
          if (!mbar_wait(p_full, jj & 1) || !mbar_wait(&v_full[vb], (jj >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // O += P V: P in TMEM (the first 64 columns of S buffer jj % 2, two
          // BF16 keys per column: 8 columns per 16-key step); V as landed,
          // [keys][dims] in two 64-dim halves 16 KB apart (MN atoms), 8-key
          // groups 1024 bytes apart (K atoms): 16 keys = 2048 bytes per step.
          const uint32_t v_base = smem_u32(sv + vb * kTile);
          const uint32_t p_tmem = t_s[jj & 1];
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t db = sw128_mnmajor_desc(v_base + static_cast<uint32_t>(kk * 2048), kHalf, 1024);
            umma_bf16_ts(t_o, p_tmem + static_cast<uint32_t>(kk * 8), db, idesc_pv,
                         (jj > 0 || kk != 0) ? 1u : 0u);
          }
          umma_commit(pv_done);
          umma_commit(&v_empty[vb]);
          umma_commit(&s_free[jj & 1]);  // its P has been read
        }
      }
      if (!ok) fail(a, kErrMmaTimeout);
      umma_commit(o_full);  // arrives once every MMA issued above has completed
      mbar_wait(o_full, 0);
    }
  } else {
    // ------------------------------------------------- softmax / P / output
    // kParts threads per query row (warps w, w + 4, ... share a TMEM lane
    // quadrant); thread part p owns key columns and output dims
    // kCols p .. kCols (p + 1) - 1.
    const int wt = threadIdx.x - 64;
    const int qd = warp & 3;  // TMEM lane quadrant
    const int part = (warp - 2) >> 2;
    const int row = qd * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const int c0 = part * kCols;
    float* xch_base = reinterpret_cast<float*>(smem + kOffXch);  // [2][kParts][128]
    const float sl2 = a.scale * 1.4426950408889634f;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    // One CTA-wide barrier per tile (the row max exchange; its buffer
    // alternates by tile parity, so a thread that passes it cannot overwrite
    // what a slower one still reads). S buffers and P are released per warp.
    // Every wait's outcome is AND-ed over the softmax threads at that barrier,
    // so they all leave the loop together (a thread giving up alone would
    // strand the others at the barrier).
    for (int j = 0; j < nk; ++j) {
      const int b = j & 1;
      float* xch = xch_base + b * kParts * 128;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1)) ok = false;
      tc_fence_after();
      const int valid = a.lk - j * kKeys < kKeys ? a.lk - j * kKeys : kKeys;
      // This thread's kCols scores of the row, read from TMEM once; row max
      // over its valid keys, combined with the row's other parts.
      uint32_t sc[kCols];
      tmem_ld_x32(t_s[b] + lane_off + c0, sc);
      tmem_ld_wait();
      float mt = -INFINITY;
#pragma unroll
      for (int i = 0; i < kCols; ++i)
        if (c0 + i < valid) mt = fmaxf(mt, u2f(sc[i]));
      xch[part * 128 + row] = mt;
      if (!named_bar_and(1, kSoftmax, ok)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int q = 0; q < kParts; ++q) mt = fmaxf(mt, xch[q * 128 + row]);
      const float m_new = fmaxf(m_used, mt);
      const bool rescale = j == 0 || (m_new - m_used) * sl2 > 8.0f;
      const float mb = (rescale ? m_new : m_used) * sl2;
      // probabilities relative to the max in use, BF16-packed
      uint32_t pk[kCols / 2];
      float ls = 0.0f;
#pragma unroll
      for (int i = 0; i < kCols; i += 2) {
        const int k = c0 + i;
        const float p0 = k < valid ? ex2_approx(u2f(sc[i]) * sl2 - mb) : 0.0f;
        const float p1 = k + 1 < valid ? ex2_approx(u2f(sc[i + 1]) * sl2 - mb) : 0.0f;
        ls += p0 + p1;
        pk[i >> 1] = pack_bf16(p0, p1);
      }
      // P and O are free once the previous tile's P V has completed.
      if (j >= 1 && !mbar_wait(pv_done, (j - 1) & 1)) ok = false;
      tc_fence_after();
      // The TMEM loads / stores are warp-collective: the warp runs them when
      // any of its rows rescales, and the other rows scale by 1.
      if (__any_sync(0xffffffffu, rescale) && j > 0) {
        const float corr = exp2f((m_used - m_new) * sl2);
        const float f = rescale ? corr : 1.0f;
        uint32_t r[kCols];
        tmem_ld_x32(t_o + lane_off + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < kCols; ++i) r[i] = __float_as_uint(u2f(r[i]) * f);
        tmem_st_x32(t_o + lane_off + c0, r);
        tmem_st_wait();
        if (rescale) l *= corr;
      }
      if (rescale) m_used = m_new;
      l += ls;
      // this thread's kCols keys of the P row -> TMEM columns kCols/2 * part ..
      // of its S buffer (every thread's scores were read before the row-max
      // barrier, so no part overwrites scores another part still needs)
      tmem_st_x16(t_s[b] + lane_off + static_cast<uint32_t>(part * (kCols / 2)), pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (!ok) fail(a, kErrEpilogueTimeout);
    // row sum = the parts' sums
    {
      float* xch = xch_base + (nk & 1) * kParts * 128;
      xch[part * 128 + row] = l;
      named_bar_sync(1, kSoftmax);
      l = 0.0f;
#pragma unroll
      for (int q = 0; q < kParts; ++q) l += xch[q * 128 + row];
    }
    if (ok) ok = mbar_wait(o_full, 0);
    if (named_bar_and(1, kSoftmax, ok)) {
      tc_fence_after();
      const int qr = q0 + row;
      bf16* dst = nullptr;
      if (qr < q_end) {
        if (a.split_first) {
          dst = qr == 0 ? a.out_first + static_cast<long long>(seq) * a.ldo_first
                        : a.out + (static_cast<long long>(seq) * (a.lq - 1) + qr - 1) * a.ldo;
        } else {
          dst = a.out + (static_cast<long long>(seq) * a.lq + qr) * a.ldo;
        }
        dst += head * 128 + c0;
      }
      const float inv = 1.0f / l;
      uint32_t r[kCols];
      tmem_ld_x32(t_o + lane_off + c0, r);
      tmem_ld_wait();
      if (dst) {
#pragma unroll
        for (int q = 0; q < kCols / 8; ++q)
          *reinterpret_cast<uint4*>(dst + q * 8) =
              make_uint4(pack_bf16(u2f(r[8 * q]) * inv, u2f(r[8 * q + 1]) * inv),
                         pack_bf16(u2f(r[8 * q + 2]) * inv, u2f(r[8 * q + 3]) * inv),
                         pack_bf16(u2f(r[8 * q + 4]) * inv, u2f(r[8 * q + 5]) * inv),
                         pack_bf16(u2f(r[8 * q + 6]) * inv, u2f(r[8 * q + 7]) * inv));
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

}  // namespace

// [batch][heads][rows][128] BF16 with the given strides (elements), boxes of
// box_rows rows x 64 dims with the 128-byte swizzle; rows past `rows` read as
// zero.
bool attn_encode_rows(CUtensorMap* m, const void* base, int rows, int heads, int batch,
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

namespace {

bool encode_rows(CUtensorMap* m, const void* base, int rows, int heads, int batch,
                 long long head_stride, long long seq_stride) {
  return attn_encode_rows(m, base, rows, heads, batch, head_stride, seq_stride, 128);
}

bool tc_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("WAM_B200_ATTN_TC");
    return !(v && v[0] == '0');
  }();
  return on;
}

}  // namespace

cudaError_t attention_tc_init() {
  return cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
}

bool attention_tc_eligible(const AttnArgs& a) {
  return tc_enabled() && a.lq >= kRows && a.lk >= 1 &&
         (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.k) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.v) & 15) == 0 && a.q_head_stride % 8 == 0 &&
         a.q_seq_stride % 8 == 0 && a.kv_head_stride % 8 == 0 && a.kv_seq_stride % 8 == 0 &&
         a.ldo % 8 == 0 && (!a.split_first || a.ldo_first % 8 == 0);
}

cudaError_t launch_attention_tc(const AttnArgs& a, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (!encode_rows(&mq, a.q, a.lq, a.heads, a.batch, a.q_head_stride, a.q_seq_stride) ||
      !encode_rows(&mk, a.k, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride) ||
      !encode_rows(&mv, a.v, a.lk, a.heads, a.batch, a.kv_head_stride, a.kv_seq_stride))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  const int rows = (a.q_end > 0 ? a.q_end : a.lq) - a.q_begin;
  cfg.gridDim = dim3((rows + kRows - 1) / kRows, a.heads, a.batch);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_tc_kernel, mq, mk, mv, a);
}

}  // namespace wamb
