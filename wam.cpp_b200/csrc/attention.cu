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

// Merge of one row slice of a split query tile: this thread's rows_per =
// 64 / SPL dims of query row row_l, over the SPL splits' partial O and
// (max, sum), from the L2 workspace (gx) or the peers' shared memory. Every
// load (16 float4 of O whatever SPL, plus the maxima and sums) is issued
// before any is used, and the sum runs in split order (deterministic).
template <int SPL>
__device__ __forceinline__ void merge_split_rows(const float* ws_blk, size_t slot_floats,
                                                 uint32_t o_base, uint32_t m_base,
                                                 uint32_t l_base, int kOld, int row_l, int dseg,
                                                 float sl2, bool gx, bf16* dst) {
  constexpr int kRowsPer = kBQ / SPL;
  constexpr int kC = kRowsPer / 4;  // float4 per split
  float mv[SPL], lv[SPL], wv[SPL];
  float4 vv[kC][SPL];
#pragma unroll
  for (int p = 0; p < SPL; ++p) {
    if (gx) {
      const float* st = ws_blk + p * slot_floats + row_l * kOld + kD;
      mv[p] = __ldcg(st);
      lv[p] = __ldcg(st + 1);
    } else {
      mv[p] = ld_shared_cluster_f32(mapa_shared(m_base + row_l * 4u, p));
      lv[p] = ld_shared_cluster_f32(mapa_shared(l_base + row_l * 4u, p));
    }
  }
#pragma unroll
  for (int ci = 0; ci < kC; ++ci)
#pragma unroll
    for (int p = 0; p < SPL; ++p) {
      const uint32_t off = (row_l * kOld + dseg + ci * 4) * 4u;
      vv[ci][p] = gx ? __ldcg(reinterpret_cast<const float4*>(ws_blk + p * slot_floats) + off / 16)
                     : ld_shared_cluster_f32x4(mapa_shared(o_base + off, p));
    }
  float mx = -INFINITY;
#pragma unroll
  for (int p = 0; p < SPL; ++p) mx = fmaxf(mx, mv[p]);
  float den = 0.0f;
#pragma unroll
  for (int p = 0; p < SPL; ++p) {
    wv[p] = mv[p] != -INFINITY ? exp2f((mv[p] - mx) * sl2) : 0.0f;
    den += wv[p] * lv[p];
  }
  const float inv_den = 1.0f / den;
  if (!dst) return;
#pragma unroll
  for (int ci = 0; ci < kC; ++ci) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < SPL; ++p) {
      acc.x = fmaf(wv[p], vv[ci][p].x, acc.x);
      acc.y = fmaf(wv[p], vv[ci][p].y, acc.y);
      acc.z = fmaf(wv[p], vv[ci][p].z, acc.z);
      acc.w = fmaf(wv[p], vv[ci][p].w, acc.w);
    }
    uint2 pk;
    pk.x = pack_bf16(acc.x * inv_den, acc.y * inv_den);
    pk.y = pack_bf16(acc.z * inv_den, acc.w * inv_den);
    *reinterpret_cast<uint2*>(dst + ci * 4) = pk;
  }
}

// SPLIT: the key range is divided among the `splits` CTAs of a cluster (CTA
// x = q_block * splits + split); each CTA stages its unnormalised output and
// running max / sum in shared memory and the cluster merges rows through
// distributed shared memory in fixed peer order.
template <bool SPLIT>
__global__ void __launch_bounds__(128) attention_kernel(const __grid_constant__ AttnArgs a, int splits) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t s_q = smem_u32(smem);
  const uint32_t s_k[2] = {s_q + kTileBytes, s_q + 3 * kTileBytes};
  const uint32_t s_v[2] = {s_q + 2 * kTileBytes, s_q + 4 * kTileBytes};

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int split = SPLIT ? static_cast<int>(blockIdx.x) % splits : 0;
  const int qblk = SPLIT ? static_cast<int>(blockIdx.x) / splits : static_cast<int>(blockIdx.x);
  const int q0 = a.q_begin + qblk * kBQ;
  const int q_end = a.q_end > 0 ? a.q_end : a.lq;
  const int head = blockIdx.y;
  const int seq = blockIdx.z;

  const bf16* qg = a.q + seq * a.q_seq_stride + head * a.q_head_stride + static_cast<long long>(q0) * kD;
  const bf16* kg = a.k + seq * a.kv_seq_stride + head * a.kv_head_stride;
  const bf16* vg = a.v + seq * a.kv_seq_stride + head * a.kv_head_stride;

  const int n_kb_all = (a.lk + kBKey - 1) / kBKey;
  const int kb_begin = SPLIT ? (split * n_kb_all) / splits : 0;
  const int kb_end = SPLIT ? ((split + 1) * n_kb_all) / splits : n_kb_all;
  const int n_kb = kb_end - kb_begin;
  // K/V that the preceding kernel does not write (cached prefix rows, prompt
  // K/V) start loading before waiting for it; Q always comes from it.
  const int key_end = kb_end * kBKey < a.lk ? kb_end * kBKey : a.lk;
  const bool kv_static = key_end <= a.static_keys;
  auto load_kv0 = [&]() {
    if (n_kb > 0) {
      load_tile(s_k[0], kg + static_cast<long long>(kb_begin) * kBKey * kD, a.lk - kb_begin * kBKey, tid);
      load_tile(s_v[0], vg + static_cast<long long>(kb_begin) * kBKey * kD, a.lk - kb_begin * kBKey, tid);
    }
    cp_async_commit();
  };
  if (kv_static) load_kv0();
  griddep_wait();
  griddep_launch_dependents();
  load_tile(s_q, qg, a.lq - q0, tid);
  cp_async_commit();
  if (!kv_static) load_kv0();

  // Q fragments for this warp's 16 rows, 8 k-steps of 16 dims.
  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  const float sl2 = a.scale * 1.4426950408889634f;

  if (n_kb == 0) cp_async_wait<0>();
  for (int it = 0; it < n_kb; ++it) {
    const int kb = kb_begin + it;
    const int buf = it & 1;
    if (it + 1 < n_kb) {
      const int nb = buf ^ 1;
      load_tile(s_k[nb], kg + static_cast<long long>(kb + 1) * kBKey * kD, a.lk - (kb + 1) * kBKey, tid);
      load_tile(s_v[nb], vg + static_cast<long long>(kb + 1) * kBKey * kD, a.lk - (kb + 1) * kBKey, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (it == 0) {
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
    for (int r = 0; r < 2; ++r) corr[r] = ex2_approx((m_run[r] - mx[r]) * sl2);
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = ex2_approx((s[j][0] - mx[0]) * sl2);
      const float p1 = ex2_approx((s[j][1] - mx[0]) * sl2);
      const float p2 = ex2_approx((s[j][2] - mx[1]) * sl2);
      const float p3 = ex2_approx((s[j][3] - mx[1]) * sl2);
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

  if constexpr (SPLIT) {
    // Stage unnormalised O [64][kOld] and (max, sum) per row, merge in the cluster.
    constexpr int kOld = kD + 4;  // padded row stride (floats)
    float* o_s = reinterpret_cast<float*>(smem);
    float* m_s = o_s + kBQ * kOld;
    float* l_s = m_s + kBQ;
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = warp * 16 + (lane >> 2) + r * 8;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        *reinterpret_cast<float2*>(o_s + row * kOld + i * 8 + (lane & 3) * 2) =
            make_float2(o[i][2 * r], o[i][2 * r + 1]);
      if ((lane & 3) == 0) {
        m_s[row] = m_run[r];
        l_s[row] = l_run[r];
      }
    }
    // With a workspace, this split's rows go to L2 ([row][kOld] floats with
    // max / sum in the last two columns) and the merge reads them from there.
    const bool gx = a.ws != nullptr;
    const size_t slot_floats = static_cast<size_t>(kBQ) * kOld;
    float* ws_blk = nullptr;
    if (gx) {
      const size_t blk = (static_cast<size_t>(seq) * gridDim.y + head) * (gridDim.x / splits) + qblk;
      ws_blk = a.ws + blk * splits * slot_floats;
      __syncthreads();
      float* mine = ws_blk + split * slot_floats;
      for (int i = tid; i < kBQ * (kD / 4); i += 128) {
        const int r = i / (kD / 4), c4 = i % (kD / 4);
        reinterpret_cast<float4*>(mine + r * kOld)[c4] =
            reinterpret_cast<const float4*>(o_s + r * kOld)[c4];
      }
      if (tid < kBQ) {
        mine[tid * kOld + kD] = m_s[tid];
        mine[tid * kOld + kD + 1] = l_s[tid];
      }
    }
    cluster_sync_all();
    // Each CTA merges kBQ / splits rows; a row's 128 dims are spread over
    // 128 / rows_per threads, each owning rows_per consecutive dims.
    const int rows_per = kBQ / splits;
    const int tpr = 128 / rows_per;
    const int row_l = split * rows_per + tid / tpr;
    const int dseg = (tid % tpr) * rows_per;
    const int row = q0 + row_l;
    const uint32_t o_base = smem_u32(o_s), m_base = smem_u32(m_s), l_base = smem_u32(l_s);
    bf16* dst = nullptr;
    if (row < q_end) {
      if (a.split_first) {
        dst = row == 0 ? a.out_first + static_cast<long long>(seq) * a.ldo_first
                       : a.out + (static_cast<long long>(seq) * (a.lq - 1) + row - 1) * a.ldo;
      } else {
        dst = a.out + (static_cast<long long>(seq) * a.lq + row) * a.ldo;
      }
      dst += head * kD + dseg;
    }
    if (splits == 8)
      merge_split_rows<8>(ws_blk, slot_floats, o_base, m_base, l_base, kOld, row_l, dseg, sl2, gx, dst);
    else if (splits == 4)
      merge_split_rows<4>(ws_blk, slot_floats, o_base, m_base, l_base, kOld, row_l, dseg, sl2, gx, dst);
    else
      merge_split_rows<2>(ws_blk, slot_floats, o_base, m_base, l_base, kOld, row_l, dseg, sl2, gx, dst);
    if (!gx) cluster_sync_all();  // peers may still read this CTA's shared memory
  } else {
    // Normalise and store BF16 rows.
    const float inv[2] = {1.0f / l_run[0], 1.0f / l_run[1]};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = q0 + warp * 16 + (lane >> 2) + r * 8;
      if (row >= q_end) continue;
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
}

}  // namespace

cudaError_t attention_init() {
  cudaError_t e = cudaFuncSetAttribute(attention_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  if ((e = attention_tc_init()) != cudaSuccess) return e;
  if ((e = attention_dec_tc_init()) != cudaSuccess) return e;
  return cudaFuncSetAttribute(attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSmem);
}

namespace {
// Query rows this launch computes.
int launch_rows(const AttnArgs& a) { return (a.q_end > 0 ? a.q_end : a.lq) - a.q_begin; }
}  // namespace

int attention_splits(const AttnArgs& a, int num_sms) {
  const int qblocks = (launch_rows(a) + kBQ - 1) / kBQ;
  const int ctas = qblocks * a.heads * a.batch;
  const int kblocks = (a.lk + kBKey - 1) / kBKey;
  const int slots = 2 * num_sms;  // 80 KB of shared memory per CTA
  if (ctas * 2 > slots) return 1;
  int best = 1;
  for (int s = 2; s <= 8; s *= 2)
    if (ctas * s <= slots && kblocks >= s) best = s;
  return best;
}

size_t attention_ws_floats(const AttnArgs& a) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int splits = attention_splits(a, sms);
  if (splits == 1) return 0;
  const size_t qblocks = (launch_rows(a) + kBQ - 1) / kBQ;
  return qblocks * a.heads * a.batch * splits * kBQ * (kD + 4);
}

namespace {

int num_sms_cached() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return sms;
}

// Rows of a tcgen05 launch that end in a ragged tile of <= 64 rows which alone
// would start a second wave of CTAs (e.g. 769 prefix queries x 24 heads: 144
// CTAs of full tiles + 24 of one row each): the full tiles run on the tcgen05
// kernel in one wave and the tail on the decode kernel (tcgen05 for <= 896
// keys, else mma.sync); else 0.
int tc_split_rows(const AttnArgs& a) {
  if (a.q_begin != 0 || a.q_end != 0) return 0;
  const int full = (a.lq / 128) * 128, rem = a.lq - full;
  const long long per_tile = static_cast<long long>(a.heads) * a.batch;
  const int sms = num_sms_cached();
  if (full == 0 || rem == 0 || rem > kBQ) return 0;
  if ((full / 128) * per_tile > sms || (full / 128 + 1) * per_tile <= sms) return 0;
  return full;
}

void launch_attention_decode(const AttnArgs& a_in, cudaStream_t s) {
  const int sms = num_sms_cached();
  AttnArgs a = a_in;
  const int splits = attention_splits(a, sms);
  const int qblocks = (launch_rows(a) + kBQ - 1) / kBQ;
  if (a.ws && static_cast<size_t>(qblocks) * a.heads * a.batch * splits * kBQ * (kD + 4) >
                  a.ws_floats)
    a.ws = nullptr;  // too small: merge through distributed shared memory
  if (splits == 1) {
    launch_pdl(attention_kernel<false>, dim3(qblocks, a.heads, a.batch), dim3(128), kSmem, s, a, 1);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(qblocks * splits, a.heads, a.batch);
  cfg.blockDim = dim3(128, 1, 1);
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
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, attention_kernel<true>, a, splits);
}

}  // namespace

int attention_launch_count(const AttnArgs& a) {
  return attention_tc_eligible(a) && tc_split_rows(a) > 0 ? 2 : 1;
}

void launch_attention(const AttnArgs& a, cudaStream_t s) {
  if (attention_tc_eligible(a)) {
    const int full = tc_split_rows(a);
    if (full > 0) {
      AttnArgs head = a;
      head.q_end = full;
      if (launch_attention_tc(head, s) == cudaSuccess) {
        AttnArgs tail = a;
        tail.q_begin = full;
        if (!attention_dec_tc_eligible(tail) || launch_attention_dec_tc(tail, s) != cudaSuccess)
          launch_attention_decode(tail, s);
        return;
      }
    } else if (launch_attention_tc(a, s) == cudaSuccess) {
      return;
    }
  }
  if (attention_dec_tc_eligible(a) && launch_attention_dec_tc(a, s) == cudaSuccess) return;
  launch_attention_decode(a, s);
}

}  // namespace wamb
