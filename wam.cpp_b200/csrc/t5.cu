// UMT5 encoder (the reference's run_t5, src/models/gwp05/engine/text_encoder.cpp:
// 112-204), per layer:
//   n = rms(h) * w_sa               (h: F32 residual stream, eps 1e-6)
//   q, k, v = n Wq, n Wk, n Wv      (no biases; BF16 operands, outputs BF16-exact)
//   a = softmax(q k^T + bias) v     (64-dim heads, NO 1/sqrt(d) scale, per-layer
//                                    relative position bias, F32 scores / softmax)
//   h += a Wo
//   n = rms(h) * w_ffn
//   h += (gelu_tanh(n Wi0) * (n Wi1)) Wo
// and out = rms(h) * w_final (F32). Rounding points of the reference's BF16
// weights: every matrix product takes its activations as BF16 and returns a
// BF16-exact value (cuBLAS through a BF16 temporary, the native-bf16 patch's
// ggml_cuda_mul_mat_batched_cublas); the residual stream, norms and softmax are
// F32. Deviations: the GELU output is rounded to BF16 before the product with the
// linear half, and the attention probabilities are rounded to BF16 for P V (the
// reference keeps both in F32); both stay inside the parity tolerance.
//
// The GEMMs are the engine's tcgen05 GEMMs (gemm.cu). The attention is a
// flash-style mma.sync kernel for 64-dim heads with the bias looked up in-kernel
// from a bucket table: it is ~2 % of the encoder's FLOPs.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "engine.h"
#include "gguf.h"
#include "mathops.cuh"
#include "ptx.cuh"
#include "t5.h"

namespace wamb {

int t5_relative_bucket(int relative, int buckets, int max_distance) {
  const int half = buckets / 2;
  const int base = relative > 0 ? half : 0;
  const int distance = relative < 0 ? -relative : relative;
  const int exact = half / 2;
  if (distance < exact) return base + distance;
  const float ratio = std::log(static_cast<float>(distance) / exact) /
                      std::log(static_cast<float>(max_distance) / exact);
  const int large = exact + static_cast<int>(ratio * (half - exact));
  return base + (large < half - 1 ? large : half - 1);
}

std::vector<std::pair<std::string, std::vector<int64_t>>> t5_tensor_specs(const T5Geometry& g) {
  std::vector<std::pair<std::string, std::vector<int64_t>>> s;
  const int64_t H = g.hidden, I = static_cast<int64_t>(g.heads) * g.head_dim, F = g.ffn;
  s.push_back({"t5.token_embd.weight", {g.vocab, H}});
  for (int l = 0; l < g.layers; ++l) {
    const std::string p = "t5.blk." + std::to_string(l);
    s.push_back({p + ".sa.q.weight", {I, H}});
    s.push_back({p + ".sa.k.weight", {I, H}});
    s.push_back({p + ".sa.v.weight", {I, H}});
    s.push_back({p + ".sa.o.weight", {H, I}});
    s.push_back({p + ".sa.rel.weight", {32, g.heads}});
    s.push_back({p + ".sa_norm.weight", {H}});
    s.push_back({p + ".ffn.wi0.weight", {F, H}});
    s.push_back({p + ".ffn.wi1.weight", {F, H}});
    s.push_back({p + ".ffn.wo.weight", {H, F}});
    s.push_back({p + ".ffn_norm.weight", {H}});
  }
  s.push_back({"t5.final_norm.weight", {H}});
  return s;
}

namespace {

constexpr float kT5Eps = 1e-6f;  // rms_norm(..., 1e-6f), text_encoder.cpp:169,183,196

__global__ void embed_kernel(const int32_t* __restrict__ ids, const bf16* __restrict__ table,
                             float* __restrict__ h, int n, int H) {
  const int row = blockIdx.x;
  if (row >= n) return;
  const bf16* src = table + static_cast<size_t>(ids[row]) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    h[static_cast<size_t>(row) * H + i] = __bfloat162float(src[i]);
}

// h += t (if given; F32 add of a BF16-exact branch output), then
// y = h * rsqrt(mean(h^2) + eps) * w: to n_out (BF16) or f_out (F32).
__global__ void __launch_bounds__(256) add_rms_kernel(float* __restrict__ h,
                                                      const bf16* __restrict__ t,
                                                      const bf16* __restrict__ w,
                                                      bf16* __restrict__ n_out,
                                                      float* __restrict__ f_out, int H) {
  __shared__ float red[8];
  const size_t base = static_cast<size_t>(blockIdx.x) * H;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < H; i += 256) {
    float v = h[base + i];
    if (t) {
      v += __bfloat162float(t[base + i]);
      h[base + i] = v;
    }
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) ss += red[k];
  const float inv = rsqrtf(ss / static_cast<float>(H) + kT5Eps);
  for (int i = threadIdx.x; i < H; i += 256) {
    const float y = h[base + i] * inv * __bfloat162float(w[i]);
    if (n_out) n_out[base + i] = __float2bfloat16_rn(y);
    if (f_out) f_out[base + i] = y;
  }
}

constexpr int kTQ = 64, kTK = 64, kTD = 64;
constexpr int kT5Tile = kTQ * kTD * 2;  // 8 KB

__device__ __forceinline__ uint32_t swz64(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// [64 rows][64 dims] BF16 tile from rows of stride ld (elements); rows past
// rows_valid read as zero.
__device__ __forceinline__ void load_tile64(uint32_t smem, const bf16* g, int ld, int rows_valid,
                                            int tid) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = tid + i * 128;
    const int row = idx >> 3, chunk = idx & 7;
    const bool ok = row < rows_valid;
    cp_async_16(smem + swz64(row, chunk), g + static_cast<size_t>(ok ? row : 0) * ld + chunk * 8, ok);
  }
}

// One CTA = 4 warps = 64 queries of one head. qkv: [T][3 * inner] (q | k | v,
// head h at columns h * 64), out: [T][inner]. bias(q, k) = rel[bucket(k - q)][h]
// with buckets[d + max_tokens - 1] the bucket of relative position d.
__global__ void __launch_bounds__(128) t5_attention_kernel(const bf16* __restrict__ qkv,
                                                           bf16* __restrict__ out,
                                                           const bf16* __restrict__ rel,
                                                           const int8_t* __restrict__ buckets,
                                                           int T, int heads, int max_tokens) {
  __shared__ __align__(128) uint8_t smem[5 * kT5Tile];
  const uint32_t s_q = smem_u32(smem);
  const uint32_t s_k[2] = {s_q + kT5Tile, s_q + 3 * kT5Tile};
  const uint32_t s_v[2] = {s_q + 2 * kT5Tile, s_q + 4 * kT5Tile};
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * kTQ, h = blockIdx.y;
  const int inner = heads * kTD, ld = 3 * inner;
  const bf16* qg = qkv + static_cast<size_t>(q0) * ld + h * kTD;
  const bf16* kg = qkv + inner + h * kTD;
  const bf16* vg = qkv + 2 * inner + h * kTD;
  const int n_kb = (T + kTK - 1) / kTK;
  const int lut_max = 2 * max_tokens - 2;

  load_tile64(s_q, qg, ld, T - q0, tid);
  load_tile64(s_k[0], kg, ld, T, tid);
  load_tile64(s_v[0], vg, ld, T, tid);
  cp_async_commit();

  uint32_t qf[4][4];
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
  const float kLog2e = 1.4426950408889634f;
  const int r0 = q0 + warp * 16 + (lane >> 2), r1 = r0 + 8;

  for (int it = 0; it < n_kb; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_kb) {
      const int nb = buf ^ 1;
      const size_t off = static_cast<size_t>(it + 1) * kTK * ld;
      load_tile64(s_k[nb], kg + off, ld, T - (it + 1) * kTK, tid);
      load_tile64(s_v[nb], vg + off, ld, T - (it + 1) * kTK, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        ldmatrix_x4(s_q + swz64(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), qf[kk][0],
                    qf[kk][1], qf[kk][2], qf[kk][3]);
    }
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        const int key = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(s_k[buf] + swz64(key, kk * 2 + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma_bf16_16816(s[2 * jp], qf[kk], b0, b1);
        mma_bf16_16816(s[2 * jp + 1], qf[kk], b2, b3);
      }
    }
    // Relative position bias; keys past T masked.
    const int kbase = it * kTK;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + j * 8 + (lane & 3) * 2 + (e & 1);
        const int qr = e < 2 ? r0 : r1;
        if (key >= T) {
          s[j][e] = -INFINITY;
        } else {
          int d = key - qr + max_tokens - 1;
          d = d < 0 ? 0 : (d > lut_max ? lut_max : d);
          s[j][e] += __bfloat162float(rel[static_cast<int>(buckets[d]) * heads + h]);
        }
      }
    }
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
    for (int r = 0; r < 2; ++r) corr[r] = ex2_approx((m_run[r] - mx[r]) * kLog2e);
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = ex2_approx((s[j][0] - mx[0]) * kLog2e);
      const float p1 = ex2_approx((s[j][1] - mx[0]) * kLog2e);
      const float p2 = ex2_approx((s[j][2] - mx[1]) * kLog2e);
      const float p3 = ex2_approx((s[j][3] - mx[1]) * kLog2e);
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
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(s_v[buf] + swz64(key, dp * 2 + (lane >> 4)), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * dp], pf[kk], b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();
  }
  const float inv0 = 1.0f / l_run[0], inv1 = 1.0f / l_run[1];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int col = h * kTD + i * 8 + (lane & 3) * 2;
    if (r0 < T)
      *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(r0) * inner + col) =
          pack_bf16(o[i][0] * inv0, o[i][1] * inv0);
    if (r1 < T)
      *reinterpret_cast<uint32_t*>(out + static_cast<size_t>(r1) * inner + col) =
          pack_bf16(o[i][2] * inv1, o[i][3] * inv1);
  }
}

}  // namespace

#define TK(call)                                                                     \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    if (e_ != cudaSuccess) {                                                         \
      *err = std::string(#call) + ": " + cudaGetErrorString(e_);                     \
      return false;                                                                  \
    }                                                                                \
  } while (0)

T5Encoder::~T5Encoder() {
  for (auto& kv : programs_)
    if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
  for (void* p : allocs_) cudaFree(p);
  if (stream_) cudaStreamDestroy(stream_);
}

double T5Encoder::flops(int n) const {
  const double H = g_.hidden, I = static_cast<double>(g_.heads) * g_.head_dim, F = g_.ffn;
  const double per_layer = 2.0 * n * (3 * I * H + I * H + 3 * F * H) + 4.0 * n * n * I;
  return per_layer * g_.layers;
}

int T5Encoder::launches(int n) {
  std::string err;
  Program* p = program(n, &err);
  return p ? static_cast<int>(p->ops.size()) : -1;
}

bool T5Encoder::init(const T5Options& opt, std::string* err) {
  opt_ = opt;
  g_ = opt.geometry;
  TK(cudaSetDevice(opt.device_index));
  TK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  if (gemm_init(opt.device_index) != cudaSuccess) {
    *err = "gemm_init failed";
    return false;
  }
  if (!load_weights(err)) return false;
  const T5Geometry& g = g_;
  if (g.head_dim != 64 || g.hidden % 64 || g.ffn % 64 || g.max_tokens < 1 || g.max_tokens > 4096 ||
      g.heads < 1 || g.vocab < 1 || g.layers < 1) {
    *err = "UMT5: head_dim must be 64, hidden and ffn multiples of 64, max_tokens in [1, 4096]";
    return false;
  }
  const int T = g.max_tokens, H = g.hidden, I = g.heads * g.head_dim, F = g.ffn;
  auto al = [&](void** p, size_t bytes) {
    if (cudaMalloc(p, bytes) != cudaSuccess) return false;
    allocs_.push_back(*p);
    return true;
  };
  if (!al(reinterpret_cast<void**>(&h_), sizeof(float) * T * H) ||
      !al(reinterpret_cast<void**>(&n_), 2ull * T * H) ||
      !al(reinterpret_cast<void**>(&qkv_), 2ull * T * 3 * I) ||
      !al(reinterpret_cast<void**>(&att_), 2ull * T * I) ||
      !al(reinterpret_cast<void**>(&tmp_), 2ull * T * H) ||
      !al(reinterpret_cast<void**>(&up_), 2ull * T * F) ||
      !al(reinterpret_cast<void**>(&out_), sizeof(float) * T * H) ||
      !al(reinterpret_cast<void**>(&ids_), sizeof(int32_t) * T) ||
      !al(reinterpret_cast<void**>(&buckets_), 2ull * T) ||
      !al(reinterpret_cast<void**>(&error_), sizeof(unsigned)) ||
      !al(reinterpret_cast<void**>(&counters_), 4096 * sizeof(unsigned))) {
    *err = "UMT5 activation allocation failed";
    return false;
  }
  TK(cudaMemset(error_, 0, sizeof(unsigned)));
  TK(cudaMemset(counters_, 0, 4096 * sizeof(unsigned)));
  // Bucket of every relative position key - query in [-(T - 1), T - 1].
  std::vector<int8_t> lut(2 * static_cast<size_t>(T) - 1);
  for (int d = -(T - 1); d <= T - 1; ++d)
    lut[static_cast<size_t>(d + T - 1)] = static_cast<int8_t>(t5_relative_bucket(d, 32, 128));
  TK(cudaMemcpy(buckets_, lut.data(), lut.size(), cudaMemcpyHostToDevice));
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, opt.device_index);
  // Split-K workspace: the largest plan over every token count (plans depend
  // on the count through its 16-row rounding).
  size_t ws = 1;
  const int shapes[4][3] = {{T, 3 * I, H}, {T, H, I}, {T, F, H}, {T, H, F}};
  for (const auto& s : shapes)
    for (int m = 16; m < T + 16; m += 16) {
      int tiles = 0;
      const size_t f = gemm_scratch_floats(m < T ? m : T, s[1], s[2], sms, 0, &tiles);
      if (f > ws) ws = f;
    }
  ws_floats_ = ws;
  if (!al(reinterpret_cast<void**>(&ws_), ws * sizeof(float))) {
    *err = "UMT5 GEMM workspace allocation failed";
    return false;
  }
  TK(cudaStreamSynchronize(stream_));
  return true;
}

bool T5Encoder::load_weights(std::string* err) {
  GgufFile file;
  const bool synthetic = opt_.artifact_path.empty();
  if (!synthetic) {
    if (!file.open(opt_.artifact_path, err)) return false;
    uint32_t u = 0;
    auto req = [&](const char* key, int* dst) {
      if (!file.get_u32(key, &u)) {
        *err = std::string("artifact lacks ") + key;
        return false;
      }
      *dst = static_cast<int>(u);
      return true;
    };
    if (!req("gwp05.t5_vocab_size", &g_.vocab) || !req("gwp05.t5_hidden", &g_.hidden) ||
        !req("gwp05.t5_ffn_dim", &g_.ffn) || !req("gwp05.t5_heads", &g_.heads) ||
        !req("gwp05.t5_head_dim", &g_.head_dim) || !req("gwp05.t5_layers", &g_.layers))
      return false;
  }
  const T5Geometry& g = g_;
  const auto specs = t5_tensor_specs(g);
  const int64_t H = g.hidden, I = static_cast<int64_t>(g.heads) * g.head_dim, F = g.ffn;
  auto al = [&](size_t bytes) -> bf16* {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    allocs_.push_back(p);
    return static_cast<bf16*>(p);
  };
  // q | k | v and wi_0 | wi_1 are packed per layer into one GEMM weight each.
  qkv_w_ = al(2ull * g.layers * 3 * I * H);
  up_w_ = al(2ull * g.layers * 2 * F * H);
  if (!qkv_w_ || !up_w_) {
    *err = "UMT5 weight allocation failed";
    return false;
  }
  std::vector<uint16_t> host;
  for (const auto& sp : specs) {
    int64_t n = 1;
    for (int64_t d : sp.second) n *= d;
    bf16* dst = nullptr;
    const std::string& name = sp.first;
    int layer = -1;
    if (name.rfind("t5.blk.", 0) == 0) layer = std::atoi(name.c_str() + 7);
    auto ends = [&](const char* suf) {
      const size_t k = std::strlen(suf);
      return name.size() >= k && name.compare(name.size() - k, k, suf) == 0;
    };
    if (layer >= 0 && (ends(".sa.q.weight") || ends(".sa.k.weight") || ends(".sa.v.weight"))) {
      const int part = ends(".sa.q.weight") ? 0 : (ends(".sa.k.weight") ? 1 : 2);
      dst = qkv_w_ + (static_cast<size_t>(layer) * 3 + part) * I * H;
    } else if (layer >= 0 && (ends(".ffn.wi0.weight") || ends(".ffn.wi1.weight"))) {
      const int part = ends(".ffn.wi0.weight") ? 0 : 1;
      dst = up_w_ + (static_cast<size_t>(layer) * 2 + part) * F * H;
    } else {
      dst = al(static_cast<size_t>(n) * 2);
      if (!dst) {
        *err = "UMT5 weight allocation failed";
        return false;
      }
    }
    w_[name] = dst;
    if (synthetic) {
      // Linear maps N(0, 1 / fan_in) (q additionally / sqrt(head_dim): T5 does
      // not scale its scores); embedding N(0, 1); position bias N(0, 0.5);
      // RMS gains 1 + N(0, 0.02).
      double scale = 0.02, center = 0.0;
      if (ends("norm.weight")) {
        center = 1.0;
      } else if (name == "t5.token_embd.weight") {
        scale = 1.0;
      } else if (ends(".rel.weight")) {
        scale = 0.5;
      } else {
        scale = 1.0 / std::sqrt(static_cast<double>(sp.second[1]));
        if (ends(".sa.q.weight")) scale /= std::sqrt(static_cast<double>(g.head_dim));
      }
      launch_synth_bf16(dst, n, tensor_seed(opt_.synthetic_seed, name), scale, center, stream_);
    } else {
      const GgufTensor* t = file.tensor(name);
      if (!t || t->type != GGML_BF16 || static_cast<int64_t>(t->elements()) != n) {
        *err = "UMT5 artifact: " + name + " missing, not BF16 or of the wrong size";
        return false;
      }
      const uint64_t chunk = 64ull << 20;
      host.resize(static_cast<size_t>(std::min<uint64_t>(chunk, t->bytes) / 2));
      for (uint64_t pos = 0; pos < t->bytes; pos += chunk) {
        const uint64_t len = std::min<uint64_t>(chunk, t->bytes - pos);
        if (!file.read(*t, pos, host.data(), len)) {
          *err = "UMT5 artifact: short read of " + name;
          return false;
        }
        TK(cudaMemcpy(reinterpret_cast<uint8_t*>(dst) + pos, host.data(), len,
                      cudaMemcpyHostToDevice));
      }
    }
  }
  TK(cudaGetLastError());
  TK(cudaStreamSynchronize(stream_));
  return true;
}

bool T5Encoder::gemm(Program* p, const bf16* x, int ldx, int m, const bf16* w, int n, int k,
                     int epi, const bf16* residual, int ldr, void* out, int ldo, std::string* err) {
  GemmScratch sc;
  sc.workspace = ws_;
  sc.workspace_floats = ws_floats_;
  sc.counters = counters_;
  sc.counter_slots = 4096;
  sc.error = error_;
  GemmOp op;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, opt_.device_index);
  const char* e = gemm_plan(&op, x, ldx, m, w, n, k, epi, nullptr, nullptr, residual, ldr, out,
                            ldo, sc, sms, 0);
  if (e) {
    *err = std::string("UMT5 GEMM: ") + e;
    return false;
  }
  p->ops.push_back([op](cudaStream_t s) { return gemm_launch(op, s) == cudaSuccess; });
  return true;
}

T5Encoder::Program* T5Encoder::program(int n, std::string* err) {
  auto it = programs_.find(n);
  if (it != programs_.end()) return it->second.get();
  auto prog = std::make_unique<Program>();
  Program* p = prog.get();
  const T5Geometry& g = g_;
  const int H = g.hidden, I = g.heads * g.head_dim, F = g.ffn, T = g.max_tokens;
  float* h = h_;
  const int32_t* ids = ids_;
  const bf16* emb = w_["t5.token_embd.weight"];
  p->ops.push_back([ids, emb, h, n, H](cudaStream_t s) {
    embed_kernel<<<n, 256, 0, s>>>(ids, emb, h, n, H);
    return cudaGetLastError() == cudaSuccess;
  });
  for (int l = 0; l < g.layers; ++l) {
    const std::string pre = "t5.blk." + std::to_string(l);
    const bf16* t = l == 0 ? nullptr : tmp_;
    const bf16* w_sa = w_[pre + ".sa_norm.weight"];
    const bf16* w_ffn = w_[pre + ".ffn_norm.weight"];
    bf16* nn = n_;
    bf16* tmp = tmp_;
    p->ops.push_back([h, t, w_sa, nn, n, H](cudaStream_t s) {
      add_rms_kernel<<<n, 256, 0, s>>>(h, t, w_sa, nn, nullptr, H);
      return cudaGetLastError() == cudaSuccess;
    });
    const bf16* wqkv = qkv_w_ + static_cast<size_t>(l) * 3 * I * H;
    if (!gemm(p, n_, H, n, wqkv, 3 * I, H, EPI_BIAS, nullptr, 0, qkv_, 3 * I, err)) return nullptr;
    const bf16* rel = w_[pre + ".sa.rel.weight"];
    const bf16* qkv = qkv_;
    bf16* att = att_;
    const int8_t* bk = buckets_;
    const int heads = g.heads;
    p->ops.push_back([qkv, att, rel, bk, n, heads, T](cudaStream_t s) {
      t5_attention_kernel<<<dim3((n + kTQ - 1) / kTQ, heads), 128, 0, s>>>(qkv, att, rel, bk, n,
                                                                          heads, T);
      return cudaGetLastError() == cudaSuccess;
    });
    if (!gemm(p, att_, I, n, w_[pre + ".sa.o.weight"], H, I, EPI_BIAS, nullptr, 0, tmp_, H, err))
      return nullptr;
    p->ops.push_back([h, tmp, w_ffn, nn, n, H](cudaStream_t s) {
      add_rms_kernel<<<n, 256, 0, s>>>(h, tmp, w_ffn, nn, nullptr, H);
      return cudaGetLastError() == cudaSuccess;
    });
    const bf16* wup = up_w_ + static_cast<size_t>(l) * 2 * F * H;
    if (!gemm(p, n_, H, n, wup, F, H, EPI_BIAS_GELU_R, nullptr, 0, up_, F, err) ||
        !gemm(p, n_, H, n, wup + static_cast<size_t>(F) * H, F, H, EPI_MUL, up_, F, up_, F, err) ||
        !gemm(p, up_, F, n, w_[pre + ".ffn.wo.weight"], H, F, EPI_BIAS, nullptr, 0, tmp_, H, err))
      return nullptr;
  }
  const bf16* w_fin = w_["t5.final_norm.weight"];
  bf16* tmp = tmp_;
  float* out = out_;
  p->ops.push_back([h, tmp, w_fin, out, n, H, T](cudaStream_t s) {
    add_rms_kernel<<<n, 256, 0, s>>>(h, tmp, w_fin, nullptr, out, H);
    if (n < T) cudaMemsetAsync(out + static_cast<size_t>(n) * H, 0, sizeof(float) * (T - n) * H, s);
    return cudaGetLastError() == cudaSuccess;
  });
  if (opt_.use_cuda_graph) {
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      *err = "UMT5 graph capture failed";
      return nullptr;
    }
    bool ok = true;
    for (auto& f : p->ops) ok = ok && f(stream_);
    const cudaError_t e = cudaStreamEndCapture(stream_, &graph);
    if (!ok || e != cudaSuccess || cudaGraphInstantiate(&p->graph, graph, 0) != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      *err = "UMT5 graph capture failed";
      return nullptr;
    }
    cudaGraphDestroy(graph);
  }
  programs_[n] = std::move(prog);
  return p;
}

bool T5Encoder::encode(const int32_t* tokens, int n, float* out, cudaStream_t stream,
                       std::string* err) {
  const T5Geometry& g = g_;
  if (!tokens || n < 1 || n > g.max_tokens) {
    *err = "UMT5: token count outside [1, n_lang]";
    return false;
  }
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= g.vocab) {
      *err = "UMT5: token " + std::to_string(tokens[i]) + " is outside the vocabulary";
      return false;
    }
  cudaSetDevice(opt_.device_index);
  Program* p = program(n, err);
  if (!p) return false;
  cudaStream_t s = stream;  // as given: NULL is the legacy default stream
  TK(cudaMemcpyAsync(ids_, tokens, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s));
  if (p->graph) {
    TK(cudaGraphLaunch(p->graph, s));
  } else {
    for (auto& f : p->ops)
      if (!f(s)) {
        *err = "UMT5 kernel launch failed";
        return false;
      }
  }
  if (out != out_)
    TK(cudaMemcpyAsync(out, out_, sizeof(float) * g.max_tokens * g.hidden, cudaMemcpyDeviceToDevice, s));
  return true;
}

}  // namespace wamb
