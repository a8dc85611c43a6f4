// Persistent denoise-step kernel: all action-expert layers of one
// flow-matching Euler step for up to 128 action tokens (batch 1-2 at the
// GWP-0.5 chunk of 48), one CTA per SM.
//
// Why: at batch 1 every denoise linear is a weight stream of 18.9-88 MB, and
// run as separate kernels each one pays a drain (last copies, split-K
// exchange, kernel exit) and a refill (launch, set-up, first copies) in which
// HBM idles; with 13 kernels per layer that latency, not bandwidth, set the
// step time. Here the program of one step (about 14 ops per layer) runs
// inside one grid: ops are separated by grid-wide phase counters, and the
// copy warp of every CTA streams the weights of its next GEMM slices into the
// shared-memory ring across those phase boundaries (weights never depend on
// an earlier op), so the HBM stream only waits where the ring is full.
//
// Roles (224 threads): warp 0 = copy producer (bulk copies of pre-swizzled
// 32 KB weight tiles and of the token k-blocks), warp 1 = TMEM owner and
// single-thread tcgen05.mma issuer (M = 128 token lanes, N = 256 weight rows,
// two 256-column accumulators), warps 2-5 = workers: they drain accumulators
// into F32 partials and run the row and attention ops; warp 6 = poller: it
// follows the grid phase counters and tells the copy thread (through shared
// memory) when a GEMM's token operand is complete, so that the copy thread
// never stalls on a global load while weight copies could be issued.
//
// GEMM ops are split stream-K: the tiles x k-blocks of a GEMM are divided into
// gridDim.x equal contiguous ranges, CTA c takes range c (at most two tiles),
// and writes one F32 partial tile per (CTA, tile) it touches. The op after a
// GEMM sums the partials of each output element in ascending CTA order
// (deterministic) and applies the GEMM's epilogue there: bias, GELU, gated
// residual, then LayerNorm / RMSNorm + RoPE / head-major scatter as the
// following op needs, so no separate normalisation kernels remain.
//
// Reference (GigaAI-research/wam.cpp): build_cached_action_body,
// src/models/gwp05/engine/mot.cpp:358-496 (one step), with expert_qkv
// (mot.cpp:210-267), joint attention (mot.cpp:432-446), expert_cross_ffn
// (mot.cpp:284-347), modulated_norm / gated_residual (mot.cpp:147-173) and the
// linear rounding points of weights.cpp:786-849. The arithmetic and rounding
// points are those of the multi-kernel path (gemm.cu, elementwise.cu,
// attention.cu); only the F32 summation order of the split-K partials differs.
#include <cmath>
#include <cstdint>

#include "kernels.h"
#include "mathops.cuh"
#include "ptx.cuh"

namespace wamb {

namespace {

constexpr int kThreads = 224;  // warps 0 copy, 1 MMA, 2-5 workers, 6 poller
constexpr int kWT = 256;                // weight rows per tile (UMMA N): one 32 KB copy per stage
constexpr int kBK = 64;                 // K per k-block (one 128-byte swizzle row)
constexpr int kWBytes = kWT * kBK * 2;  // 16 KB weight k-block
constexpr int kAttTile = 64 * 128 * 2;  // 16 KB attention tile (64 rows x 128 dims)
constexpr int kAttBytes = 5 * kAttTile; // Q + 2 x (K, V)
constexpr int kTailBytes = 2048;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kMaxStages = 8;
constexpr int kQ = 8;                   // pending token-load queue (>= stages)
constexpr int kMaxChunks = 4;           // 8-wide chunks per worker thread: widths <= 4096
constexpr int kBlockChunks = 6;         // chunks per thread of a GELU / RES unit (6144 features)
constexpr int kMaxSplits = 8;           // attention key splits
constexpr int kRowCounters = 128;       // per-row join counters (rows <= 128)

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_acquire_cta_shared(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_cta_shared(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ long long sk_start(int c, long long total, int grid) {
  return static_cast<long long>(c) * total / grid;
}

__device__ __forceinline__ bool aborted(const unsigned* flag) {
  return *reinterpret_cast<const volatile unsigned*>(flag) != 0u;
}

__device__ __forceinline__ void raise_abort(unsigned* flag, unsigned* err, unsigned code) {
  atomicCAS(err, 0u, code);
  atomicExch(flag, 1u);
}

// Bounded spin until *ctr >= target (acquire). False on timeout or abort.
__device__ __forceinline__ bool wait_counter(const unsigned* ctr, unsigned target, unsigned* abort_flag,
                             unsigned* err) {
  const long long t0 = clock64();
  int n = 0;
  while (ld_acquire_u32(ctr) < target) {
    if ((++n & 31) == 0) {
      if (aborted(abort_flag)) return false;
      if (clock64() - t0 > kWaitLimitCycles) {
        raise_abort(abort_flag, err, kErrStepPhaseTimeout);
        return false;
      }
    }
  }
  return true;
}

// Bounded mbarrier wait that also gives up when another role aborted.
__device__ __forceinline__ bool mbar_wait_ab(uint64_t* bar, uint32_t parity, unsigned* abort_flag, unsigned* err,
                             unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  int n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 255) == 0) {
      if (aborted(abort_flag)) return false;
      if (clock64() - t0 > kWaitLimitCycles) {
        raise_abort(abort_flag, err, code);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the 128 worker threads (named barrier 1; warps 0-1 are elsewhere).
__device__ __forceinline__ float workers_sum(float v, float* red, int wt) {
  v = warp_sum(v);
  named_bar_sync(1, 128);
  if ((wt & 31) == 0) red[wt >> 5] = v;
  named_bar_sync(1, 128);
  return red[0] + red[1] + red[2] + red[3];
}

__device__ __forceinline__ void load8_bf16(const bf16* p, float (&f)[8]) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 pack8_bf16(const float (&f)[8]) {
  return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]),
                    pack_bf16(f[6], f[7]));
}

// 8 consecutive features (n0 % 8 == 0) of row m in the token-tile layout
// [K/64][mr][64] with the 128-byte swizzle (16-byte chunk c of row r at c ^ (r % 8)).
__device__ __forceinline__ bf16* a_tile_at(bf16* base, int mr, int m, int n0) {
  const int kb = n0 >> 6, c = (n0 & 63) >> 3;
  return base + (static_cast<size_t>(kb) * mr + m) * 64 + ((c ^ (m & 7)) << 3);
}

// Partial-slot list of the tile holding feature n0 of a GEMM: seg[] = slots
// (cta * 2 + slot) in ascending CTA order, -1 past the last (at most NSEG).
// Constant for the launch, so it is read before the phase wait.
template <int NSEG>
__device__ __forceinline__ void load_seg(const int* segs, int n0, int (&seg)[NSEG]) {
  const int4* tb = reinterpret_cast<const int4*>(segs + (n0 / kWT) * 8);
  const int4 s0 = __ldg(tb);
  seg[0] = s0.x; seg[1] = s0.y; seg[2] = s0.z; seg[3] = s0.w;
  if constexpr (NSEG > 4) {
    const int4 s1 = __ldg(tb + 1);
    seg[4] = s1.x; seg[5] = s1.y; seg[6] = s1.z; seg[7] = s1.w;
  }
}

// Row ops stage the stream-K partials in shared memory (the attention tiles,
// idle during row ops) with cp.async instead of holding them in registers:
// record (chunk i, slot u) of worker thread wt is 32 bytes at
// ((i * NSEG + u) * 128 + wt) * 32. gather issues the copies of one chunk,
// reduce sums them in list order (deterministic) after cp.async.wait.
template <int NSEG>
__device__ __forceinline__ void gather(const StepArgs& a, uint32_t stage, const int (&seg)[NSEG],
                                       int m, int n0, int i, int wt) {
  const int f = n0 % kWT;
  const size_t slot_floats = static_cast<size_t>(a.mr) * kWT;
  const size_t off = (static_cast<size_t>(f >> 4) * a.mr + m) * 16 + (f & 15);
#pragma unroll
  for (int u = 0; u < NSEG; ++u) {
    if (seg[u] >= 0) {
      const float* p = a.ws + static_cast<size_t>(seg[u]) * slot_floats + off;
      const uint32_t d = stage + static_cast<uint32_t>(((i * NSEG + u) * 128 + wt) * 32);
      cp_async_16(d, p, true);
      cp_async_16(d + 16, p + 4, true);
    }
  }
}

template <int NSEG>
__device__ __forceinline__ void reduce(const uint8_t* stage, const int (&seg)[NSEG], int i, int wt,
                                       float (&acc)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
#pragma unroll
  for (int u = 0; u < NSEG; ++u) {
    if (seg[u] >= 0) {
      const float4* x = reinterpret_cast<const float4*>(stage + ((i * NSEG + u) * 128 + wt) * 32);
      const float4 x0 = x[0], x1 = x[1];
      acc[0] += x0.x; acc[1] += x0.y; acc[2] += x0.z; acc[3] += x0.w;
      acc[4] += x1.x; acc[5] += x1.y; acc[6] += x1.z; acc[7] += x1.w;
    }
  }
}

__device__ __forceinline__ void unpack8(uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ void load8_f32(const float* p, float (&f)[8]) {
  const float4 a0 = __ldg(reinterpret_cast<const float4*>(p));
  const float4 a1 = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a0.x; f[1] = a0.y; f[2] = a0.z; f[3] = a0.w;
  f[4] = a1.x; f[5] = a1.y; f[6] = a1.z; f[7] = a1.w;
}

// Linear output of 8 features with the op's epilogue (gemm.cu epi_run_t):
// EPI_BIAS: bf16(bf16(acc) + b); EPI_BIAS_GELU: gelu_tanh(bf16(acc) + b);
// EPI_GATED_RES / EPI_RES: residual + bf16(bf16(acc) + b) [* gate]. b = 0 when
// the op has no bias; the result is rounded to BF16 (what the multi-kernel
// path stores).
__device__ __forceinline__ void epilogue8(int epi, bool hb, const float (&acc)[8],
                                          const float (&b)[8], const float (&gt)[8],
                                          const float (&r)[8], float (&v)[8]) {
  if (epi == EPI_BIAS_GELU) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = bf16_round(gelu_tanh(bf16_round(acc[j]) + b[j]));
  } else if (epi == EPI_BIAS) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = bf16_round(bf16_round(acc[j]) + b[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t = bf16_round(acc[j]);
      if (hb) t = bf16_round(t + b[j]);
      v[j] = epi == EPI_GATED_RES ? bf16_round(fmaf(t, gt[j], r[j])) : bf16_round(r[j] + t);
    }
  }
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits (one thread polls with acquire loads, the others wait at the named
// barrier) until every CTA has finished op p. False if the wait gave up.
__device__ __forceinline__ bool phase_wait(const StepArgs& a, int p, int wt, int* flag) {
  if (wt == 0)
    *flag = wait_counter(a.counters + p, static_cast<unsigned>(gridDim.x),
                         a.counters + a.num_ops + a.attn_counters + kRowCounters + 1, a.error)
                ? 1 : 0;
  named_bar_sync(1, 128);
  const bool r = *flag != 0;
  named_bar_sync(1, 128);
  return r;
}

// Row barrier of a row op split over op.nblk column blocks (one CTA each, all
// resident): every block publishes its two statistics, then waits until all
// blocks of the row have (per-row counters, cumulative targets within one
// launch). Returns false if the wait gave up.
__device__ __forceinline__ bool row_join(const StepArgs& a, const StepOp& op, int m, int j, float s0, float s1,
                         int wt, int* flag) {
  float* st = a.stats + (static_cast<size_t>(m) * 8 + j) * 2;
  if (wt == 0) {
    *reinterpret_cast<float2*>(st) = make_float2(s0, s1);
    unsigned* ctr = a.counters + a.num_ops + a.attn_counters + m;
    red_release_add(ctr, 1u);  // publishes the statistics
    *flag = wait_counter(ctr, static_cast<unsigned>(op.sync_base + op.nblk),
                         a.counters + a.num_ops + a.attn_counters + kRowCounters + 1, a.error)
                ? 1 : 0;
  }
  named_bar_sync(1, 128);
  return *flag != 0;
}

// ---------------------------------------------------------------- row ops
// Every row op loads its constant operands (partial-slot lists, bias, gate,
// norm parameters, RoPE angles) before waiting for the op before it
// (wait_p >= 0); after the wait the partials are staged in shared memory by
// cp.async and the residual is loaded, in one round of loads. CH: 8-wide
// chunks per thread, NSEG: partial slots per tile of the GEMM before
// (CH * NSEG <= 20: the staging fits the 80 KB attention tiles).

// LayerNorm row op (STEP_LN), unit = (row m, column block j of op.nblk): the
// new residual (epilogue of the previous GEMM's partials, or the residual as
// is) into resid, LayerNorm statistics (two-pass mean / centred sum of squares
// per block, blocks combined in order with the parallel-variance formula; one
// block = elementwise.cu ln_kernel exactly), AdaLN modulation (ln 0:
// n * (1 + scale) + shift, F32 params) or affine (ln 1: BF16 w, b), BF16 into
// the token-tile layout of the next GEMM.
template <int CH, int NSEG>
__device__ __forceinline__ void row_ln(const StepArgs& a, const StepOp& op, int m, int j, int wt,
                                    uint8_t* stage, float* red, int* flag, int wait_p) {
  static_assert(CH * NSEG <= 20, "partial staging exceeds the attention tiles");
  const int* g = op.segs;  // partial slots of the GEMM before, or null
  const int bw = op.width / op.nblk;
  const int chunks = bw >> 3;
  const int c0 = j * chunks;
  const bool hb = op.bias != nullptr;
  int seg[CH][NSEG];
  float b[CH][8], gt[CH][8], pa[CH][8], pb[CH][8];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) {
      const int n0 = (c0 + c) * 8;
      if (g) {
        load_seg<NSEG>(g, n0, seg[i]);
        if (hb) unpack8(__ldg(reinterpret_cast<const uint4*>(op.bias + n0)), b[i]);
        else
#pragma unroll
          for (int k = 0; k < 8; ++k) b[i][k] = 0.0f;
        if (op.epi == EPI_GATED_RES) load8_f32(op.gate + n0, gt[i]);
      }
      if (op.ln == 0) {
        load8_f32(static_cast<const float*>(op.p0) + n0, pa[i]);
        load8_f32(static_cast<const float*>(op.p1) + n0, pb[i]);
      } else {
        unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const bf16*>(op.p0) + n0)), pa[i]);
        unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const bf16*>(op.p1) + n0)), pb[i]);
      }
    }
  }
  if (wait_p >= 0 && !phase_wait(a, wait_p, wt, flag)) return;
  const uint32_t st_addr = smem_u32(stage);
  uint4 rr[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) {
      const int n0 = (c0 + c) * 8;
      if (g) gather<NSEG>(a, st_addr, seg[i], m, n0, i, wt);
      rr[i] = __ldcg(reinterpret_cast<const uint4*>(op.resid + static_cast<size_t>(m) * op.ldr + n0));
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  float v[CH][8];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) {
      float r[8];
      unpack8(rr[i], r);
      if (g) {
        float acc[8];
        reduce<NSEG>(stage, seg[i], i, wt, acc);
        epilogue8(op.epi, hb, acc, b[i], gt[i], r, v[i]);
        *reinterpret_cast<uint4*>(op.resid + static_cast<size_t>(m) * op.ldr + (c0 + c) * 8) =
            pack8_bf16(v[i]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = r[k];
      }
    }
  }
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < CH; ++i)
    if (wt + i * 128 < chunks) {
#pragma unroll
      for (int k = 0; k < 8; ++k) s += v[i][k];
    }
  const float bmean = workers_sum(s, red, wt) / bw;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < CH; ++i)
    if (wt + i * 128 < chunks) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float d = v[i][k] - bmean;
        q += d * d;
      }
    }
  const float bm2 = workers_sum(q, red, wt);
  float mean = bmean, m2 = bm2;
  if (op.nblk > 1) {
    if (!row_join(a, op, m, j, bmean, bm2, wt, flag)) return;
    float n_a = 0.0f;
    mean = 0.0f;
    m2 = 0.0f;
    for (int bk = 0; bk < op.nblk; ++bk) {
      const float2 st = __ldcg(reinterpret_cast<const float2*>(a.stats + (static_cast<size_t>(m) * 8 + bk) * 2));
      const float n_b = static_cast<float>(bw), n = n_a + n_b;
      const float d = st.x - mean;
      mean += d * (n_b / n);
      m2 += st.y + d * d * (n_a * n_b / n);
      n_a = n;
    }
  }
  const float inv_std = rsqrtf(m2 / op.width + op.eps);
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) {
      float f[8];
      if (op.ln == 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = fmaf((v[i][k] - mean) * inv_std, 1.0f + pa[i][k], pb[i][k]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) f[k] = fmaf((v[i][k] - mean) * inv_std, pa[i][k], pb[i][k]);
      }
      *reinterpret_cast<uint4*>(a_tile_at(op.out_a, a.mr, m, (c0 + c) * 8)) = pack8_bf16(f);
    }
  }
}

// q / k / v row op (STEP_QKV, STEP_CQ), unit = (row m, part, column block j
// of op.nblk): linear output (EPI_BIAS) of the part (width H), RMSNorm over H
// with its weight (q, k; block sums of squares added in block order), 1-D RoPE
// (q, k of the self attention), BF16 scatter into the head-major attention
// buffers (elementwise.cu qkv_scatter_kernel).
template <int CH, int NSEG>
__device__ __forceinline__ void row_qkv(const StepArgs& a, const StepOp& op, int m, int part, int j,
                                     int wt, uint8_t* stage, float* red, int* flag, int wait_p) {
  static_assert(CH * NSEG <= 20, "partial staging exceeds the attention tiles");
  const int H = op.width;
  const int bw = H / op.nblk;
  const int chunks = bw >> 3;
  const int c0 = j * chunks;
  const int seq = m / a.rows_per_seq, rin = m - seq * a.rows_per_seq;
  const bf16* nw = part == 0 ? op.q_norm : (part == 1 ? op.k_norm : nullptr);
  const bool rope = op.rope != 0 && part < 2;
  const int pos1 = op.pos_base + rin;
  int seg[CH][NSEG];
  float b[CH][8], w[CH][8], cs[CH][4], sn[CH][4];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) {
      const int d = (c0 + c) * 8, n0 = part * H + d;
      load_seg<NSEG>(op.segs, n0, seg[i]);
      unpack8(__ldg(reinterpret_cast<const uint4*>(op.bias + n0)), b[i]);
      if (nw) unpack8(__ldg(reinterpret_cast<const uint4*>(nw + d)), w[i]);
      if (rope) {
        const float4 fr = __ldg(reinterpret_cast<const float4*>(a.inv_freq + ((d & 127) >> 1)));
        const float fq[4] = {fr.x, fr.y, fr.z, fr.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) sincosf(static_cast<float>(pos1) * fq[p], &sn[i][p], &cs[i][p]);
      }
    }
  }
  bf16* dst_base;
  long long head_stride;
  if (part == 0) {
    dst_base = op.q_out + seq * op.q_seq_stride + static_cast<long long>(rin) * 128;
    head_stride = op.q_head_stride;
  } else {
    dst_base = (part == 1 ? op.k_out : op.v_out) + seq * op.kv_seq_stride +
               static_cast<long long>(op.kv_row_offset + rin) * 128;
    head_stride = op.kv_head_stride;
  }
  if (wait_p >= 0 && !phase_wait(a, wait_p, wt, flag)) return;
  const uint32_t st_addr = smem_u32(stage);
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) gather<NSEG>(a, st_addr, seg[i], m, part * H + (c0 + c) * 8, i, wt);
  }
  cp_async_commit();
  cp_async_wait<0>();
  float v[CH][8];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) {
      float acc[8];
      reduce<NSEG>(stage, seg[i], i, wt, acc);
      epilogue8(EPI_BIAS, true, acc, b[i], b[i], b[i], v[i]);
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < CH; ++i)
    if (wt + i * 128 < chunks) {
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[i][k] * v[i][k];
    }
  float tot = workers_sum(ss, red, wt);
  if (op.nblk > 1 && nw) {
    if (!row_join(a, op, m, j, tot, 0.0f, wt, flag)) return;
    tot = 0.0f;
    for (int bk = 0; bk < op.nblk; ++bk) tot += __ldcg(a.stats + (static_cast<size_t>(m) * 8 + bk) * 2);
  }
  const float inv = nw ? rsqrtf(tot / H + op.eps) : 1.0f;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = wt + i * 128;
    if (c < chunks) {
      const int d = (c0 + c) * 8, hd = d & 127;
      float f[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = nw ? v[i][k] * inv * w[i][k] : v[i][k];
      if (rope) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float x0 = f[2 * p], x1 = f[2 * p + 1];
          f[2 * p] = x0 * cs[i][p] - x1 * sn[i][p];
          f[2 * p + 1] = x0 * sn[i][p] + x1 * cs[i][p];
        }
      }
      *reinterpret_cast<uint4*>(dst_base + (d >> 7) * head_stride + hd) = pack8_bf16(f);
    }
  }
}

// Column-block row op without a row reduction (STEP_GELU: FFN-up output into
// the token-tile layout of the FFN-down GEMM; STEP_RES: the step's last gated
// residual into the residual stream). Unit = (row m, block j of op.nblk, each
// CH * 1024 features).
// RES: the op may be STEP_RES (gated residual, resid read); false: STEP_GELU only.
template <int CH, int NSEG, bool RES = true>
__device__ __forceinline__ void row_block(const StepArgs& a, const StepOp& op, int m, int j, int wt,
                                       uint8_t* stage, int* flag, int wait_p) {
  static_assert(CH * NSEG <= 20, "partial staging exceeds the attention tiles");
  const int chunks = op.width >> 3;
  const bool hb = op.bias != nullptr;
  const bool res = RES && op.kind == STEP_RES;
  int seg[CH][NSEG];
  float b[CH][8], gt[RES ? CH : 1][8];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = (j * CH + i) * 128 + wt;
    if (c < chunks) {
      load_seg<NSEG>(op.segs, c * 8, seg[i]);
      if (hb) unpack8(__ldg(reinterpret_cast<const uint4*>(op.bias + c * 8)), b[i]);
      else
#pragma unroll
        for (int k = 0; k < 8; ++k) b[i][k] = 0.0f;
      if (RES && op.epi == EPI_GATED_RES) load8_f32(op.gate + c * 8, gt[RES ? i : 0]);
    }
  }
  if (wait_p >= 0 && !phase_wait(a, wait_p, wt, flag)) return;
  const uint32_t st_addr = smem_u32(stage);
  uint4 rr[RES ? CH : 1];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = (j * CH + i) * 128 + wt;
    if (c < chunks) {
      gather<NSEG>(a, st_addr, seg[i], m, c * 8, i, wt);
      if (res) rr[RES ? i : 0] = __ldcg(reinterpret_cast<const uint4*>(op.resid + static_cast<size_t>(m) * op.ldr + c * 8));
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = (j * CH + i) * 128 + wt;
    if (c < chunks) {
      float acc[8], r[8], v[8];
      reduce<NSEG>(stage, seg[i], i, wt, acc);
      if (res) unpack8(rr[RES ? i : 0], r);
      epilogue8(RES ? op.epi : EPI_BIAS_GELU, hb, acc, b[i], gt[RES ? i : 0], r, v);
      if (!res)
        *reinterpret_cast<uint4*>(a_tile_at(op.out_a, a.mr, m, c * 8)) = pack8_bf16(v);
      else
        *reinterpret_cast<uint4*>(op.resid + static_cast<size_t>(m) * op.ldr + c * 8) = pack8_bf16(v);
    }
  }
}

// Row-op variants: (chunks per thread, partial slots per tile) pairs the host
// plans (engine.cu step_ops); the host never plans a pair missing here. The
// batch-1 variants are inlined into the kernel; the wider ones (batch 2 and
// other widths) are called out of line so that their registers do not weigh
// on the kernel's allocation.
template <int CH, int NSEG>
__device__ __noinline__ void row_ln_call(const StepArgs& a, const StepOp& op, int m, int j, int wt,
                                         uint8_t* stage, float* red, int* flag, int wait_p) {
  row_ln<CH, NSEG>(a, op, m, j, wt, stage, red, flag, wait_p);
}
template <int CH, int NSEG>
__device__ __noinline__ void row_qkv_call(const StepArgs& a, const StepOp& op, int m, int part, int j,
                                          int wt, uint8_t* stage, float* red, int* flag, int wait_p) {
  row_qkv<CH, NSEG>(a, op, m, part, j, wt, stage, red, flag, wait_p);
}
template <int CH, int NSEG>
__device__ __noinline__ void row_block_call(const StepArgs& a, const StepOp& op, int m, int j, int wt,
                                            uint8_t* stage, int* flag, int wait_p) {
  row_block<CH, NSEG>(a, op, m, j, wt, stage, flag, wait_p);
}

__device__ __forceinline__ void run_row_ln(const StepArgs& a, const StepOp& op, int m, int j, int wt,
                                           uint8_t* stage, float* red, int* flag, int wait_p) {
  switch (op.ch * 16 + op.nseg) {
    case 1 * 16 + 8: row_ln<1, 8>(a, op, m, j, wt, stage, red, flag, wait_p); break;
    case 1 * 16 + 4: row_ln<1, 4>(a, op, m, j, wt, stage, red, flag, wait_p); break;
    case 2 * 16 + 4: row_ln_call<2, 4>(a, op, m, j, wt, stage, red, flag, wait_p); break;
    case 2 * 16 + 8: row_ln_call<2, 8>(a, op, m, j, wt, stage, red, flag, wait_p); break;
    case 3 * 16 + 4: row_ln_call<3, 4>(a, op, m, j, wt, stage, red, flag, wait_p); break;
    default: row_ln_call<4, 4>(a, op, m, j, wt, stage, red, flag, wait_p); break;
  }
}

__device__ __forceinline__ void run_row_qkv(const StepArgs& a, const StepOp& op, int m, int part,
                                            int j, int wt, uint8_t* stage, float* red, int* flag,
                                            int wait_p) {
  switch (op.ch * 16 + op.nseg) {
    case 3 * 16 + 4: row_qkv<3, 4>(a, op, m, part, j, wt, stage, red, flag, wait_p); break;
    case 1 * 16 + 8: row_qkv<1, 8>(a, op, m, part, j, wt, stage, red, flag, wait_p); break;
    case 1 * 16 + 4: row_qkv_call<1, 4>(a, op, m, part, j, wt, stage, red, flag, wait_p); break;
    case 2 * 16 + 4: row_qkv_call<2, 4>(a, op, m, part, j, wt, stage, red, flag, wait_p); break;
    case 2 * 16 + 8: row_qkv_call<2, 8>(a, op, m, part, j, wt, stage, red, flag, wait_p); break;
    default: row_qkv_call<4, 4>(a, op, m, part, j, wt, stage, red, flag, wait_p); break;
  }
}

__device__ __forceinline__ void run_row_block(const StepArgs& a, const StepOp& op, int m, int j,
                                              int wt, uint8_t* stage, int* flag, int wait_p) {
  switch (op.ch * 16 + op.nseg) {
    case 5 * 16 + 4: row_block<5, 4, false>(a, op, m, j, wt, stage, flag, wait_p); break;
    case 1 * 16 + 8: row_block<1, 8>(a, op, m, j, wt, stage, flag, wait_p); break;
    case 1 * 16 + 4: row_block_call<1, 4>(a, op, m, j, wt, stage, flag, wait_p); break;
    default: row_block_call<3, 4>(a, op, m, j, wt, stage, flag, wait_p); break;
  }
}

// ---------------------------------------------------------------- attention

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
    const bf16* src = g + (ok ? row : 0) * 128 + chunk * 8;
    cp_async_16(smem + swz(row, chunk), src, ok);
  }
}

struct AttnUnit {
  int seq, head, split, kb_begin, kb_end;
};

__device__ __forceinline__ AttnUnit attn_unit(const StepOp& op, int u) {
  AttnUnit r;
  r.split = u % op.splits;
  r.head = (u / op.splits) % op.heads;
  r.seq = u / (op.splits * op.heads);
  const int n_kb_all = (op.lk + 63) / 64;
  r.kb_begin = (r.split * n_kb_all) / op.splits;
  r.kb_end = ((r.split + 1) * n_kb_all) / op.splits;
  return r;
}

// Issues the first key block's K / V copies of unit u (group committed).
__device__ __forceinline__ void attn_load_kv(const StepOp& op, const AttnUnit& au, uint32_t sk,
                                             uint32_t sv, int kb, int wt) {
  const bf16* kg = op.att_k + au.seq * op.kv_seq_stride + au.head * op.kv_head_stride;
  const bf16* vg = op.att_v + au.seq * op.kv_seq_stride + au.head * op.kv_head_stride;
  load_tile(sk, kg + static_cast<long long>(kb) * 64 * 128, op.lk - kb * 64, wt);
  load_tile(sv, vg + static_cast<long long>(kb) * 64 * 128, op.lk - kb * 64, wt);
  cp_async_commit();
}

constexpr int kAttLd = 132;  // workspace row: 128 dims, max, sum, 2 pad (16-byte rows)

// One (sequence, head, key split) of softmax(scale Q K^T) V for <= 64 query
// rows on the 4 worker warps (attention.cu attention_kernel: F32 scores and
// online softmax, BF16 probabilities, F32 accumulation). With key splits every
// unit stages its unnormalised rows and (max, sum) in the workspace, waits
// until all splits of its (sequence, head) have (they run on distinct resident
// CTAs), and merges a 1/splits share of the rows in split order. Output goes to
// the token-tile layout of the O projection (k = head * 128 + d).
// kv0_issued: the first key block was loaded before the phase wait.
__device__ __noinline__ void attn_run(const StepArgs& a, const StepOp& op, int u, bool kv0_issued,
                                      uint8_t* att_smem, int* flag, int wt) {
  const AttnUnit au = attn_unit(op, u);
  const uint32_t s_q = smem_u32(att_smem);
  const uint32_t s_k[2] = {s_q + kAttTile, s_q + 3 * kAttTile};
  const uint32_t s_v[2] = {s_q + 2 * kAttTile, s_q + 4 * kAttTile};
  const int warp = wt >> 5, lane = wt & 31;
  const int n_kb = au.kb_end - au.kb_begin;
  const bf16* qg = op.att_q + au.seq * op.q_seq_stride + au.head * op.q_head_stride;
  const bf16* kg = op.att_k + au.seq * op.kv_seq_stride + au.head * op.kv_head_stride;
  const bf16* vg = op.att_v + au.seq * op.kv_seq_stride + au.head * op.kv_head_stride;
  load_tile(s_q, qg, op.lq, wt);
  cp_async_commit();
  if (!kv0_issued && n_kb > 0) attn_load_kv(op, au, s_k[0], s_v[0], au.kb_begin, wt);

  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  const float sl2 = op.scale * 1.4426950408889634f;

  if (n_kb == 0) cp_async_wait<0>();
  for (int it = 0; it < n_kb; ++it) {
    const int kb = au.kb_begin + it;
    const int buf = it & 1;
    if (it + 1 < n_kb) {
      const int nb = buf ^ 1;
      load_tile(s_k[nb], kg + static_cast<long long>(kb + 1) * 64 * 128, op.lk - (kb + 1) * 64, wt);
      load_tile(s_v[nb], vg + static_cast<long long>(kb + 1) * 64 * 128, op.lk - (kb + 1) * 64, wt);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    named_bar_sync(1, 128);
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int row = warp * 16 + (lane & 15);
        const int chunk = kk * 2 + (lane >> 4);
        ldmatrix_x4(s_q + swz(row, chunk), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    float s[8][4];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) s[jj][0] = s[jj][1] = s[jj][2] = s[jj][3] = 0.0f;
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
    const int kbase = kb * 64;
    if (kbase + 64 > op.lk) {
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int c = kbase + jj * 8 + (lane & 3) * 2;
        if (c >= op.lk) s[jj][0] = s[jj][2] = -INFINITY;
        if (c + 1 >= op.lk) s[jj][1] = s[jj][3] = -INFINITY;
      }
    }
    float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      mx[0] = fmaxf(mx[0], fmaxf(s[jj][0], s[jj][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[jj][2], s[jj][3]));
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
    for (int jj = 0; jj < 8; ++jj) {
      const float p0 = exp2f((s[jj][0] - mx[0]) * sl2);
      const float p1 = exp2f((s[jj][1] - mx[0]) * sl2);
      const float p2 = exp2f((s[jj][2] - mx[1]) * sl2);
      const float p3 = exp2f((s[jj][3] - mx[1]) * sl2);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int kk = jj >> 1;
      if ((jj & 1) == 0) {
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
    named_bar_sync(1, 128);
  }

  const int row_base = au.seq * a.rows_per_seq;
  if (op.splits == 1) {
    const float inv[2] = {1.0f / l_run[0], 1.0f / l_run[1]};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = warp * 16 + (lane >> 2) + r * 8;
      if (row >= op.lq) continue;
      const int mg = row_base + row;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int n = au.head * 128 + i * 8 + (lane & 3) * 2;
        bf16* dst = a_tile_at(op.out_a, a.mr, mg, n & ~7) + (n & 7);
        *reinterpret_cast<uint32_t*>(dst) = pack_bf16(o[i][2 * r] * inv[r], o[i][2 * r + 1] * inv[r]);
      }
    }
    return;
  }
  const size_t slot_floats = 64 * kAttLd;
  float* blk = a.attn_ws + static_cast<size_t>((au.seq * op.heads + au.head) * op.splits) * slot_floats;
  float* mine = blk + au.split * slot_floats;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = warp * 16 + (lane >> 2) + r * 8;
    if (row >= op.lq) continue;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      *reinterpret_cast<float2*>(mine + row * kAttLd + i * 8 + (lane & 3) * 2) =
          make_float2(o[i][2 * r], o[i][2 * r + 1]);
    if ((lane & 3) == 0) *reinterpret_cast<float2*>(mine + row * kAttLd + 128) = make_float2(m_run[r], l_run[r]);
  }
  named_bar_sync(1, 128);
  if (wt == 0) {
    unsigned* ctr = a.counters + a.num_ops + au.seq * op.heads + au.head;
    red_release_add(ctr, 1u);  // publishes this split's rows
    *flag = wait_counter(ctr, static_cast<unsigned>(op.sync_base + op.splits),
                         a.counters + a.num_ops + a.attn_counters + kRowCounters + 1, a.error)
                ? 1 : 0;
  }
  named_bar_sync(1, 128);
  if (*flag == 0) return;
  // This split merges rows [r0, r1): one (row, 8-dim group) item per thread
  // and pass, every split's values loaded before the sum.
  const int rps = (op.lq + op.splits - 1) / op.splits;
  const int r0 = au.split * rps, r1 = min(op.lq, r0 + rps);
  for (int idx = r0 * 16 + wt; idx < r1 * 16; idx += 128) {
    const int row = idx >> 4, d0 = (idx & 15) * 8;
    float2 ml[kMaxSplits];
    float4 x[kMaxSplits][2];
#pragma unroll
    for (int p = 0; p < kMaxSplits; ++p) {
      if (p < op.splits) {
        const float* src = blk + p * slot_floats + row * kAttLd;
        ml[p] = __ldcg(reinterpret_cast<const float2*>(src + 128));
        x[p][0] = __ldcg(reinterpret_cast<const float4*>(src + d0));
        x[p][1] = __ldcg(reinterpret_cast<const float4*>(src + d0) + 1);
      }
    }
    float mxv = -INFINITY;
#pragma unroll
    for (int p = 0; p < kMaxSplits; ++p)
      if (p < op.splits) mxv = fmaxf(mxv, ml[p].x);
    float den = 0.0f;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < kMaxSplits; ++p) {
      if (p < op.splits) {
        const float w = ml[p].x != -INFINITY ? exp2f((ml[p].x - mxv) * sl2) : 0.0f;
        den += w * ml[p].y;
        acc[0] = fmaf(w, x[p][0].x, acc[0]); acc[1] = fmaf(w, x[p][0].y, acc[1]);
        acc[2] = fmaf(w, x[p][0].z, acc[2]); acc[3] = fmaf(w, x[p][0].w, acc[3]);
        acc[4] = fmaf(w, x[p][1].x, acc[4]); acc[5] = fmaf(w, x[p][1].y, acc[5]);
        acc[6] = fmaf(w, x[p][1].z, acc[6]); acc[7] = fmaf(w, x[p][1].w, acc[7]);
      }
    }
    const float inv_den = 1.0f / den;
    float f[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = acc[k] * inv_den;
    *reinterpret_cast<uint4*>(a_tile_at(op.out_a, a.mr, row_base + row, au.head * 128 + d0)) =
        pack8_bf16(f);
  }
}

// ---------------------------------------------------------------- the kernel

// Shared memory: [token stages][weight stages][attention tiles][tail: barriers,
// flags, reduction scratch, two op descriptors][GEMM table].
constexpr int kDescOff = 1024;  // descriptors in the tail
constexpr int kQueueOff = 768;  // copy thread's pending token copies: kQ * (4 + 4 + 8) bytes
static_assert(kQueueOff + kQ * 16 <= kDescOff, "queue overlaps the descriptors");
static_assert(kDescOff + 2 * sizeof(StepOp) <= kTailBytes, "tail too small for two descriptors");

__host__ __device__ constexpr int fixed_smem(int num_gemms) {
  return kAttBytes + kTailBytes + num_gemms * static_cast<int>(sizeof(StepGemm)) + 1024;
}

__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = args.stages;
  const uint32_t a_bytes = static_cast<uint32_t>(args.mr) * 128;
  // Token stages first: a UMMA reads 128 token rows from its stage, so the rows
  // past mr land in shared memory that follows (never read back).
  uint8_t* s_a = smem;
  uint8_t* s_w = s_a + S * a_bytes;
  uint8_t* s_att = s_w + S * kWBytes;
  uint8_t* tail = s_att + kAttBytes;
  StepGemm* gt = reinterpret_cast<StepGemm*>(tail + kTailBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_full = empty + kMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint64_t* desc_bar = mma_done + 1;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(desc_bar + 2);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* last_cta = flag + 1;
  int* ready_op = last_cta + 1;  // last GEMM op whose token operand may be copied (poller)
  float* red = reinterpret_cast<float*>(tail + 512);
  StepOp* desc = reinterpret_cast<StepOp*>(tail + kDescOff);  // [2], op p in desc[p & 1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = gridDim.x, cta = blockIdx.x;
  unsigned* phase = args.counters;
  unsigned* exit_ctr = args.counters + args.num_ops + args.attn_counters + kRowCounters;
  unsigned* abort_flag = exit_ctr + 1;
  const int ng = args.num_gemms;

  // The GEMM table goes to shared memory (constant for the launch).
  for (int i = threadIdx.x; i < ng * static_cast<int>(sizeof(StepGemm) / 8); i += kThreads)
    reinterpret_cast<uint64_t*>(gt)[i] = __ldg(reinterpret_cast<const uint64_t*>(args.gemms) + i);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 1);
      mbar_init(&desc_bar[b], 1);
    }
    mbar_init(mma_done, 1);
    *ready_op = -1;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kWT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ copy producer
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      // Pending token copies (a ring in shared memory: dynamically indexed
      // arrays would live in local memory, whose L1 share is small here).
      int* q_slot = reinterpret_cast<int*>(tail + kQueueOff);
      int* q_op = q_slot + kQ;
      const bf16** q_src = reinterpret_cast<const bf16**>(q_op + kQ);
      int qh = 0, qt = 0;
      int fenced = -1;  // highest op whose readiness this thread has fenced for
      bool ok = true;
      int it = 0;
      // Issues the token copies of queued stages whose op the poller has
      // published as ready (all of them when `force`, on abort, so that every
      // issued stage completes). Never waits.
      auto service = [&](bool force) {
        while (qh != qt) {
          const int e = qh % kQ;
          const int p = q_op[e];
          if (!force && p > fenced) {
            if (ld_acquire_cta_shared(ready_op) < p) return;
            fence_proxy_async_global();  // generic-proxy writes of the op before -> bulk copies
            fenced = p;
          }
          bulk_load(s_a + q_slot[e] * a_bytes, q_src[e], a_bytes, &full[q_slot[e]], pol_a);
          ++qh;
        }
      };
      auto spin_check = [&](long long t0, int& n) -> bool {
        if ((++n & 63) == 0) {
          if (aborted(abort_flag)) return false;
          if (clock64() - t0 > kWaitLimitCycles) {
            raise_abort(abort_flag, args.error, kErrStepRingTimeout);
            return false;
          }
        }
        return true;
      };
      for (int gi = 0; gi < ng && ok; ++gi) {
        const StepGemm gm = gt[gi];
        const int n = gm.nk & 0xFFFF, k = gm.nk >> 16, ctas = gm.cop & 0xFFFF, p = gm.cop >> 16;
        const int nkb = k >> 6;
        const long long total = static_cast<long long>(n / kWT) * nkb;
        const long long i0 = cta < ctas ? sk_start(cta, total, ctas) : 0;
        const long long i1 = cta < ctas ? sk_start(cta + 1, total, ctas) : 0;
        for (long long i = i0; i < i1 && ok; ++i, ++it) {
          const int slot = it % S;
          if (it >= S) {
            const uint32_t par = ((it / S) - 1) & 1;
            const long long t0 = clock64();
            int cnt = 0;
            while (!mbar_try_wait(&empty[slot], par)) {
              service(false);
              if (!spin_check(t0, cnt)) {
                ok = false;
                break;
              }
            }
            if (!ok) break;
          }
          const int t = static_cast<int>(i / nkb), kb = static_cast<int>(i % nkb);
          mbar_arrive_expect_tx(&full[slot], a_bytes + kWBytes);
          // tile t = rows t * kWT.. of the re-tiled [n/256][k/64][256][64] layout
          const int r0 = t * kWT;
          const bf16* wsrc = gm.w + ((static_cast<size_t>(r0 >> 8) * nkb + kb) * 256 + (r0 & 255)) * kBK;
          bulk_load(s_w + slot * kWBytes, wsrc, kWBytes, &full[slot], pol_w);
          const int e = qt % kQ;
          q_slot[e] = slot;
          q_op[e] = p;
          q_src[e] = gm.a + static_cast<size_t>(kb) * args.mr * 64;
          ++qt;
          service(false);
        }
      }
      if (ok) {
        const long long t0 = clock64();
        int cnt = 0;
        while (qh != qt) {
          service(false);
          if (!spin_check(t0, cnt)) {
            ok = false;
            break;
          }
        }
      }
      if (!ok) {
        // Complete every issued stage (token copies of whatever is in the
        // buffers) so that no copy is in flight when the CTA exits.
        service(true);
        const int first = it > S ? it - S : 0;
        for (int j = first; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1);
      }
    }
  } else if (warp == 6) {
    if (lane == 0) {
      // ------------------------------------------------------------- poller
      // Follows the phase counters of the ops that write GEMM token operands
      // and publishes the last GEMM op whose operand is complete, so that the
      // copy thread never stalls on a global load.
      griddep_wait();  // phase counters are written only after the previous grid
      for (int gi = 0; gi < ng; ++gi) {
        const int p = gt[gi].cop >> 16;
        if (p > 0 &&
            !wait_counter(&phase[p - 1], static_cast<unsigned>(grid), abort_flag, args.error))
          break;
        st_release_cta_shared(ready_op, p);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16(128, kWT);
      int it = 0, sg = 0;
      bool ok = true;
      for (int gi = 0; gi < ng && ok; ++gi) {
        const StepGemm gm = gt[gi];
        const int n = gm.nk & 0xFFFF, k = gm.nk >> 16, ctas = gm.cop & 0xFFFF;
        const int nkb = k >> 6;
        const long long total = static_cast<long long>(n / kWT) * nkb;
        const long long i0 = cta < ctas ? sk_start(cta, total, ctas) : 0;
        const long long i1 = cta < ctas ? sk_start(cta + 1, total, ctas) : 0;
        long long i = i0;
        while (i < i1 && ok) {
          const long long t = i / nkb;
          const long long seg_end = (t + 1) * nkb < i1 ? (t + 1) * nkb : i1;
          const int b = sg & 1;
          if (sg >= 2 && !mbar_wait_ab(&acc_empty[b], ((sg >> 1) - 1) & 1, abort_flag, args.error,
                                       kErrMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t acc = tmem_base + static_cast<uint32_t>(b * kWT);
          for (long long j = i; j < seg_end; ++j, ++it) {
            const int slot = it % S;
            if (!mbar_wait_ab(&full[slot], (it / S) & 1, abort_flag, args.error, kErrMmaTimeout)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t da = sw128_kmajor_desc(smem_u32(s_a + slot * a_bytes));
            const uint64_t db = sw128_kmajor_desc(smem_u32(s_w + slot * kWBytes));
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_bf16_ss(acc, da + 2 * kk, db + 2 * kk, idesc, (j != i || kk != 0) ? 1u : 0u);
            umma_commit(&empty[slot]);
          }
          if (!ok) break;
          umma_commit(&acc_full[b]);
          ++sg;
          i = seg_end;
        }
      }
      // Every issued MMA completes before TMEM is released.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------- workers
    const int wt = threadIdx.x - 64;
    const int qd = warp & 3;  // TMEM lane quadrant of this warp
    const int trow = qd * 32 + lane;
    int sg = 0, gi = 0;
    bool ok = true, dep = false;
    // The CTA's writes of op p are published by one release add after a
    // named barrier (bar.sync orders the other workers' writes before it);
    // token tiles are read by bulk copies (async proxy), hence the proxy fence.
    auto signal = [&](int p, bool tiles) {
      if (tiles) fence_proxy_async_global();
      named_bar_sync(1, 128);
      if (wt == 0) red_release_add(&phase[p], 1u);
    };
    auto wait_phase = [&](int p) -> bool { return phase_wait(args, p, wt, flag); };
    // Op descriptors arrive one op ahead by bulk copy into desc[p & 1].
    auto fetch_desc = [&](int p) {
      fence_proxy_async_smem();  // the buffer's last generic reads precede the copy
      mbar_arrive_expect_tx(&desc_bar[p & 1], sizeof(StepOp));
      bulk_load(&desc[p & 1], args.ops + p, sizeof(StepOp), &desc_bar[p & 1], policy_evict_last());
    };
    int fetched = 0, consumed = -1;  // descriptor copies issued / waited for
    if (wt == 0) fetch_desc(0);
    for (int p = 0; p < args.num_ops && ok; ++p) {
      if (wt == 0) {
        *flag = mbar_wait_ab(&desc_bar[p & 1], (p >> 1) & 1, abort_flag, args.error,
                             kErrEpilogueTimeout) ? 1 : 0;
        consumed = p;
        if (*flag && p + 1 < args.num_ops) {
          fetch_desc(p + 1);
          fetched = p + 1;
        }
      }
      named_bar_sync(1, 128);
      if (*flag == 0) {
        ok = false;
        break;
      }
      const StepOp& op = desc[p & 1];
      if (op.kind == STEP_GEMM) {
        const StepGemm gm = gt[gi++];
        const int n = gm.nk & 0xFFFF, k = gm.nk >> 16, ctas = gm.cop & 0xFFFF;
        const int nkb = k >> 6;
        const long long total = static_cast<long long>(n / kWT) * nkb;
        const long long i0 = cta < ctas ? sk_start(cta, total, ctas) : 0;
        const long long i1 = cta < ctas ? sk_start(cta + 1, total, ctas) : 0;
        const long long t_first = i0 / nkb;
        long long i = i0;
        while (i < i1) {
          const long long t = i / nkb;
          const long long seg_end = (t + 1) * nkb < i1 ? (t + 1) * nkb : i1;
          const int b = sg & 1;
          // One thread waits and broadcasts, so that every worker takes the
          // same branch (a divergent timeout would strand the others at a
          // named barrier).
          if (wt == 0)
            *flag = mbar_wait_ab(&acc_full[b], (sg >> 1) & 1, abort_flag, args.error,
                                 kErrEpilogueTimeout) ? 1 : 0;
          named_bar_sync(1, 128);
          if (*flag == 0) {
            ok = false;
            break;
          }
          tc_fence_after();
          float* dst = args.ws + (static_cast<size_t>(cta) * 2 + static_cast<size_t>(t - t_first)) *
                                     args.mr * kWT;
          if (qd * 32 < args.mr) {
            const uint32_t taddr =
                tmem_base + static_cast<uint32_t>(b * kWT) + (static_cast<uint32_t>(qd * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < kWT; c += 32) {
              uint32_t r[32];
              tmem_ld_x32(taddr + c, r);
              tmem_ld_wait();
              if (trow < args.m) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  float4* d = reinterpret_cast<float4*>(
                      dst + (static_cast<size_t>(c / 16 + h) * args.mr + trow) * 16);
#pragma unroll
                  for (int j = 0; j < 4; ++j)
                    d[j] = make_float4(__uint_as_float(r[16 * h + 4 * j]), __uint_as_float(r[16 * h + 4 * j + 1]),
                                       __uint_as_float(r[16 * h + 4 * j + 2]),
                                       __uint_as_float(r[16 * h + 4 * j + 3]));
                }
              }
            }
          }
          tc_fence_before();
          named_bar_sync(1, 128);
          if (wt == 0) mbar_arrive(&acc_empty[b]);
          ++sg;
          i = seg_end;
        }
        if (!ok) break;
        signal(p, false);
        continue;
      }
      if (!dep) {
        griddep_wait();
        dep = true;
      }
      if (op.kind == STEP_ATTN) {
        // The first key block of this CTA's first unit is issued before the
        // phase wait when no key of it is written by the op before.
        const int units = op.batch * op.heads * op.splits;
        bool pre = false;
        if (cta < units) {
          const AttnUnit au = attn_unit(op, cta);
          const int key_end = au.kb_begin * 64 + 64 < op.lk ? au.kb_begin * 64 + 64 : op.lk;
          if (au.kb_end > au.kb_begin && key_end <= op.static_keys) {
            attn_load_kv(op, au, smem_u32(s_att) + kAttTile, smem_u32(s_att) + 2 * kAttTile,
                         au.kb_begin, wt);
            pre = true;
          }
        }
        if (p > 0 && !wait_phase(p - 1)) {
          cp_async_wait<0>();
          ok = false;
          break;
        }
        for (int u = cta; u < units; u += grid) attn_run(args, op, u, pre && u == cta, s_att, flag, wt);
      } else {
        // Units of row ops with a row join (nblk > 1) never exceed the grid
        // (the host plans nblk so), so every block of a row is resident. The
        // first unit of a CTA waits for op p - 1 itself, after loading its
        // constant operands.
        const int nb = op.nblk;
        const int parts = op.kind == STEP_QKV ? 3 : 1;
        const int units = args.m * parts * nb;
        if (cta >= units) {
          if (p > 0 && !wait_phase(p - 1)) {
            ok = false;
            break;
          }
        } else if (op.kind == STEP_LN) {
          for (int u = cta; u < units; u += grid)
            run_row_ln(args, op, u / nb, u % nb, wt, s_att, red, flag, u == cta ? p - 1 : -1);
        } else if (op.kind == STEP_QKV || op.kind == STEP_CQ) {
          for (int u = cta; u < units; u += grid)
            run_row_qkv(args, op, u / (parts * nb), (u / nb) % parts, u % nb, wt, s_att, red, flag,
                        u == cta ? p - 1 : -1);
        } else {  // STEP_GELU, STEP_RES
          for (int u = cta; u < units; u += grid)
            run_row_block(args, op, u / nb, u % nb, wt, s_att, flag, u == cta ? p - 1 : -1);
        }
      }
      if (aborted(abort_flag)) {
        ok = false;
        break;
      }
      signal(p, op.kind == STEP_LN || op.kind == STEP_GELU || op.kind == STEP_ATTN);
    }
    // A descriptor copy still in flight lands before the CTA exits.
    if (wt == 0 && fetched > consumed) mbar_wait(&desc_bar[fetched & 1], (fetched >> 1) & 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kWT);
  }
  // The last CTA to leave puts the phase counters back at rest for the next
  // launch (which reads them only after griddepcontrol.wait).
  if (threadIdx.x == 0) {
    __threadfence();
    *last_cta = atomicAdd(exit_ctr, 1u) == static_cast<unsigned>(grid - 1) ? 1 : 0;
  }
  __syncthreads();
  if (*last_cta) {
    __threadfence();
    for (int i = threadIdx.x; i < args.num_ops + args.attn_counters + kRowCounters; i += kThreads)
      args.counters[i] = 0u;
    __syncthreads();
    if (threadIdx.x == 0) {
      *abort_flag = 0u;
      __threadfence();
      *exit_ctr = 0u;
    }
  }
}

}  // namespace

int step_stages(int mr, int num_gemms) {
  const int stage = mr * 128 + kWBytes;
  int s = (kSmemLimit - fixed_smem(num_gemms)) / stage;
  return s > kMaxStages ? kMaxStages : s;
}

size_t step_smem_bytes(int mr, int num_gemms) {
  return static_cast<size_t>(step_stages(mr, num_gemms)) * (mr * 128 + kWBytes) + fixed_smem(num_gemms);
}

size_t step_ws_floats(int grid, int mr) { return static_cast<size_t>(grid) * 2 * mr * kWT; }

int step_tile_rows() { return kWT; }

cudaError_t step_init() {
  return cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
}

cudaError_t step_launch(const StepArgs& a, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = step_smem_bytes(a.mr, a.num_gemms);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel, a);
}

}  // namespace wamb
