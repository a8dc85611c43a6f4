// Wan VAE encoder (single frame), the reference's run_vae graph
// (src/models/gwp05/engine/vae.cpp:136-388) on NHWC BF16 activations:
//   conv_in 3x3 (12 -> 160)
//   down 0: 2 resnets 160, downsampler 3x3/2 + 2x2 average shortcut
//   down 1: resnets 160 -> 320 (1x1 skip), downsampler + temporal average shortcut
//   down 2: resnets 320 -> 640, downsampler + temporal average shortcut
//   down 3: 2 resnets 640, block residual
//   mid: resnet, single-head self-attention over all pixels (C = 640), resnet
//   RMS + SiLU, conv_out 3x3 (640 -> 2z), quant_conv 1x1, latent (mode - mean) / std
// Resnet (vae_residual, :178-191): h = conv1(silu(rms(x) g1)); h = conv2(silu(rms(h) g2));
// out = h + (skip(x) or x). RMS over channels per pixel, eps 1e-12 (:162-176).
// Rounding points of the BF16 path: convolutions (cuDNN BF16 out) -> BF16, + bias -> BF16,
// + shortcut -> BF16; RMS / SiLU in F32, cast to BF16 for the next convolution;
// average pool in F32 -> BF16; attention scores F32, probabilities F32 -> BF16 for
// the value GEMM, output F32 -> BF16.
#include <cmath>
#include <cstring>

#include "engine.h"
#include "gguf.h"
#include "mathops.cuh"
#include "ptx.cuh"
#include "vae.h"

namespace wamb {
namespace {

constexpr float kVaeEps = 1e-12f;  // vae_rms (vae.cpp:169,173)

// Patchified F32 planes [12][H][W] -> NHWC BF16 [H][W][64] (channels 12..63 zero).
__global__ void to_nhwc64_kernel(const float* __restrict__ in, bf16* __restrict__ out, int hw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= hw) return;
  uint32_t w[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) w[c] = 0u;
#pragma unroll
  for (int c = 0; c < 6; ++c) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(in[static_cast<size_t>(2 * c) * hw + i],
                                                   in[static_cast<size_t>(2 * c + 1) * hw + i]);
    w[c] = *reinterpret_cast<const uint32_t*>(&h);
  }
  uint4* o = reinterpret_cast<uint4*>(out + static_cast<size_t>(i) * 64);
#pragma unroll
  for (int q = 0; q < 8; ++q) o[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

// Per-pixel RMS over C channels (ggml_rms_norm_bf16_f32: x * rsqrt(mean(x^2) + eps)
// * gamma in F32), optional SiLU, BF16 out. A 256-thread block covers
// P = 256 / (C / 8) whole pixels, one 16-byte chunk (8 channels) per thread, so
// every load of the block is issued at once and coalesced; a pixel's sum of
// squares is reduced in chunk order through shared memory (deterministic).
// C % 8 == 0, C <= 2048.
__global__ void __launch_bounds__(256) rms_act_kernel(const bf16* __restrict__ x,
                                                      const bf16* __restrict__ gamma,
                                                      bf16* __restrict__ out, int rows, int C,
                                                      int silu_on) {
  __shared__ float part[256];
  __shared__ float inv_s[256];
  const int chunks = C / 8, P = 256 / chunks;
  const int t = threadIdx.x, lp = t / chunks, ch = t - lp * chunks;
  const long long row = static_cast<long long>(blockIdx.x) * P + lp;
  const bool active = lp < P && row < rows;
  float v[8];
  float ss = 0.0f;
  if (active) {
    const uint4 u = reinterpret_cast<const uint4*>(x + row * C)[ch];
    const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] = __uint_as_float(wv[q] << 16);
      v[2 * q + 1] = __uint_as_float(wv[q] & 0xFFFF0000u);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) ss += v[q] * v[q];
  }
  part[t] = ss;
  __syncthreads();
  if (t < P) {
    float s = 0.0f;
    for (int k = 0; k < chunks; ++k) s += part[t * chunks + k];
    inv_s[t] = rsqrtf(s / static_cast<float>(C) + kVaeEps);
  }
  __syncthreads();
  if (!active) return;
  const float inv = inv_s[lp];
  const uint4 gu = reinterpret_cast<const uint4*>(gamma)[ch];
  const uint32_t gw[4] = {gu.x, gu.y, gu.z, gu.w};
  uint32_t ow[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float a = v[2 * q] * inv * __uint_as_float(gw[q] << 16);
    float b = v[2 * q + 1] * inv * __uint_as_float(gw[q] & 0xFFFF0000u);
    if (silu_on) {
      a = silu(a);
      b = silu(b);
    }
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    ow[q] = *reinterpret_cast<const uint32_t*>(&h);
  }
  reinterpret_cast<uint4*>(out + row * C)[ch] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

// 2x2 average pool of x [H][W][C] (F32 sum of the window in row order, x 1/4),
// to out [H/2][W/2][C] or, temporal, [H/2][W/2][2C] with channel 2c = 0 and
// 2c + 1 = the pooled channel c (vae_avg_shortcut, vae.cpp:193-213). One thread
// per output pixel and 8 input channels.
__global__ void avg_shortcut_kernel(const bf16* __restrict__ x, bf16* __restrict__ out, int H,
                                    int W, int C, int temporal) {
  const int groups = C / 8;
  const int oh = H / 2, ow = W / 2;
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<long long>(oh) * ow * groups) return;
  const int g = static_cast<int>(i % groups);
  const int p = static_cast<int>(i / groups);
  const int oy = p / ow, ox = p % ow;
  float s[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) s[q] = 0.0f;
#pragma unroll
  for (int dy = 0; dy < 2; ++dy)
#pragma unroll
    for (int dx = 0; dx < 2; ++dx) {
      const uint4 u = *reinterpret_cast<const uint4*>(
          x + (static_cast<size_t>(2 * oy + dy) * W + 2 * ox + dx) * C + g * 8);
      const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        s[2 * q] += __uint_as_float(wv[q] << 16);
        s[2 * q + 1] += __uint_as_float(wv[q] & 0xFFFF0000u);
      }
    }
  if (!temporal) {
    uint32_t ow4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(s[2 * q] * 0.25f, s[2 * q + 1] * 0.25f);
      ow4[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(p) * C + g * 8) =
        make_uint4(ow4[0], ow4[1], ow4[2], ow4[3]);
  } else {
    uint32_t ow8[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(0.0f, s[q] * 0.25f);
      ow8[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
    uint4* o = reinterpret_cast<uint4*>(out + static_cast<size_t>(p) * 2 * C + g * 16);
    o[0] = make_uint4(ow8[0], ow8[1], ow8[2], ow8[3]);
    o[1] = make_uint4(ow8[4], ow8[5], ow8[6], ow8[7]);
  }
}

// out = bf16(a + b), n % 8 == 0.
__global__ void add_bf16_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b,
                                bf16* __restrict__ out, long long n8) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= n8) return;
  const uint4 ua = reinterpret_cast<const uint4*>(a)[i];
  const uint4 ub = reinterpret_cast<const uint4*>(b)[i];
  const uint32_t wa[4] = {ua.x, ua.y, ua.z, ua.w}, wb[4] = {ub.x, ub.y, ub.z, ub.w};
  uint32_t wo[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(
        __uint_as_float(wa[q] << 16) + __uint_as_float(wb[q] << 16),
        __uint_as_float(wa[q] & 0xFFFF0000u) + __uint_as_float(wb[q] & 0xFFFF0000u));
    wo[q] = *reinterpret_cast<const uint32_t*>(&h);
  }
  reinterpret_cast<uint4*>(out)[i] = make_uint4(wo[0], wo[1], wo[2], wo[3]);
}

// Row softmax of s * scale (F32 [rows][cols], ggml_soft_max_ext) to BF16
// probabilities. One 256-thread block per row; the row is staged in shared memory.
__global__ void __launch_bounds__(256) softmax_rows_kernel(const float* __restrict__ s,
                                                           bf16* __restrict__ p, int cols,
                                                           float scale) {
  extern __shared__ float row[];
  __shared__ float red[8];
  const float* sr = s + static_cast<size_t>(blockIdx.x) * cols;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < cols; i += 256) {
    const float v = sr[i] * scale;
    row[i] = v;
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.0f;
  for (int i = threadIdx.x; i < cols; i += 256) {
    const float e = expf(row[i] - mx);
    row[i] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) sum += red[w];
  const float inv = 1.0f / sum;
  bf16* pr = p + static_cast<size_t>(blockIdx.x) * cols;
  for (int i = threadIdx.x; i < cols; i += 256) pr[i] = __float2bfloat16_rn(row[i] * inv);
}

// out [C][T] = transpose of in [T][C] (row stride ld), 32 x 32 tiles.
__global__ void transpose_kernel(const bf16* __restrict__ in, int ld, bf16* __restrict__ out,
                                 int T, int C) {
  __shared__ bf16 tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int t = t0 + r, c = c0 + threadIdx.x;
    if (t < T && c < C) tile[r][threadIdx.x] = in[static_cast<size_t>(t) * ld + c];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int c = c0 + r, t = t0 + threadIdx.x;
    if (t < T && c < C) out[static_cast<size_t>(c) * T + t] = tile[threadIdx.x][r];
  }
}

// latent [z][hw] = (moments[hw][c] - mean[c]) / std[c] for the first z channels
// (vae.cpp:376-386; the graph output is cast to F32 first).
__global__ void latent_out_kernel(const bf16* __restrict__ m, int cm, const float* __restrict__ stats,
                                  float* __restrict__ out, int hw, int z) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= hw * z) return;
  const int c = i / hw, p = i % hw;
  out[i] = (__bfloat162float(m[static_cast<size_t>(p) * cm + c]) - stats[c]) / stats[z + c];
}

}  // namespace

std::vector<std::pair<std::string, std::vector<int64_t>>> vae_tensor_specs(int z_dim) {
  std::vector<std::pair<std::string, std::vector<int64_t>>> s;
  auto conv = [&](const std::string& p, int64_t co, int64_t ci, int64_t k) {
    s.push_back({p + ".weight", {co, ci, k, k}});
    s.push_back({p + ".bias", {co}});
  };
  auto res = [&](const std::string& p, int64_t ci, int64_t co) {
    s.push_back({p + ".n1", {ci}});
    conv(p + ".c1", co, ci, 3);
    s.push_back({p + ".n2", {co}});
    conv(p + ".c2", co, co, 3);
    if (ci != co) conv(p + ".skip", co, ci, 1);
  };
  conv("vae.enc.in", 160, 12, 3);
  const int64_t cin[4] = {160, 160, 320, 640}, cout[4] = {160, 320, 640, 640};
  for (int b = 0; b < 4; ++b) {
    const std::string p = "vae.enc.down." + std::to_string(b);
    res(p + ".res.0", cin[b], cout[b]);
    res(p + ".res.1", cout[b], cout[b]);
    if (b < 3) conv(p + ".ds", cout[b], cout[b], 3);
  }
  res("vae.enc.mid.res.0", 640, 640);
  s.push_back({"vae.enc.mid.attn.norm", {640}});
  conv("vae.enc.mid.attn.qkv", 1920, 640, 1);
  conv("vae.enc.mid.attn.proj", 640, 640, 1);
  res("vae.enc.mid.res.1", 640, 640);
  s.push_back({"vae.enc.out_norm", {640}});
  conv("vae.enc.out", 2 * z_dim, 640, 3);
  conv("vae.quant", 2 * z_dim, 2 * z_dim, 1);
  return s;
}

namespace {

int64_t numel(const std::vector<int64_t>& shape) {
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  return n;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = std::strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

}  // namespace

VaeEncoder::~VaeEncoder() {
  if (graph_) cudaGraphExecDestroy(graph_);
  for (void* p : view_buf_) cudaFree(p);
  for (void* p : allocs_) cudaFree(p);
  if (stream_) cudaStreamDestroy(stream_);
}

#define VK(call)                                                                     \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    if (e_ != cudaSuccess) {                                                         \
      *err = std::string(#call) + ": " + cudaGetErrorString(e_);                     \
      return false;                                                                  \
    }                                                                                \
  } while (0)

VaeEncoder::Act VaeEncoder::act(int h, int w, int c, std::string* err) {
  Act a;
  a.h = h;
  a.w = w;
  a.c = c;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(h) * w * c * 2) != cudaSuccess) {
    *err = "VAE activation allocation failed";
    return a;
  }
  allocs_.push_back(p);
  a.p = static_cast<bf16*>(p);
  return a;
}

bool VaeEncoder::init(const VaeOptions& opt, std::string* err) {
  opt_ = opt;
  if (opt_.image_width <= 0 || opt_.image_height <= 0 || opt_.image_width % 32 ||
      opt_.image_height % 32) {
    *err = "VAE: image width and height must be positive multiples of 32";
    return false;
  }
  if (opt_.z_dim <= 0 || (2 * opt_.z_dim) % 16) {
    *err = "VAE: 2 * z_dim must be a multiple of 16";
    return false;
  }
  VK(cudaSetDevice(opt_.device_index));
  VK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  VK(cudaMalloc(&error_, sizeof(unsigned)));
  allocs_.push_back(error_);
  VK(cudaMemset(error_, 0, sizeof(unsigned)));
  if (gemm_init(opt_.device_index) != cudaSuccess) {
    *err = "gemm_init failed";
    return false;
  }
  if (!load_weights(err) || !build(err)) return false;
  if (opt_.use_cuda_graph) {
    cudaGraph_t g = nullptr;
    VK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    bool ok = true;
    for (auto& f : program_) ok = ok && f(stream_);
    cudaError_t e = cudaStreamEndCapture(stream_, &g);
    if (!ok || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      *err = "VAE graph capture failed";
      return false;
    }
    e = cudaGraphInstantiate(&graph_, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      *err = std::string("VAE graph instantiate: ") + cudaGetErrorString(e);
      return false;
    }
  }
  VK(cudaStreamSynchronize(stream_));
  return true;
}

bool VaeEncoder::load_weights(std::string* err) {
  const auto specs = vae_tensor_specs(opt_.z_dim);
  GgufFile file;
  const bool synthetic = opt_.artifact_path.empty();
  if (!synthetic && !file.open(opt_.artifact_path, err)) return false;
  std::vector<uint16_t> host;
  for (const auto& sp : specs) {
    const int64_t n = numel(sp.second);
    void* p = nullptr;
    VK(cudaMalloc(&p, static_cast<size_t>(n) * 2));
    allocs_.push_back(p);
    bf16* d = static_cast<bf16*>(p);
    w_[sp.first] = d;
    if (synthetic) {
      // Convolutions: N(0, 1 / fan_in); biases N(0, 0.02); RMS gains 1 + N(0, 0.02).
      double scale = 0.02, center = 0.0;
      const bool gain = !ends_with(sp.first, ".weight") && !ends_with(sp.first, ".bias");
      if (gain) center = 1.0;
      if (ends_with(sp.first, ".weight"))
        scale = 1.0 / std::sqrt(static_cast<double>(sp.second[1] * sp.second[2] * sp.second[3]));
      launch_synth_bf16(d, n, tensor_seed(opt_.synthetic_seed, sp.first), scale, center,
                        stream_);
    } else {
      const GgufTensor* t = file.tensor(sp.first);
      if (!t || t->type != GGML_BF16 || static_cast<int64_t>(t->elements()) != n) {
        *err = "VAE artifact: " + sp.first + " missing, not BF16 or of the wrong size";
        return false;
      }
      host.resize(static_cast<size_t>(n));
      if (!file.read(*t, 0, host.data(), static_cast<uint64_t>(n) * 2)) {
        *err = "VAE artifact: short read of " + sp.first;
        return false;
      }
      VK(cudaMemcpy(d, host.data(), static_cast<size_t>(n) * 2, cudaMemcpyHostToDevice));
    }
    if (sp.second.size() == 4 && sp.first != "vae.enc.mid.attn.qkv.weight" &&
        sp.first != "vae.enc.mid.attn.proj.weight") {
      const int co = static_cast<int>(sp.second[0]), ci = static_cast<int>(sp.second[1]);
      const int taps = static_cast<int>(sp.second[2] * sp.second[3]);
      void* q = nullptr;
      const size_t laid = static_cast<size_t>(conv_cout_pad(co)) * taps * conv_cin_pad(ci);
      VK(cudaMalloc(&q, laid * 2));
      allocs_.push_back(q);
      launch_conv_weight_layout(d, static_cast<bf16*>(q), co, ci, taps, stream_);
      wconv_[sp.first] = static_cast<bf16*>(q);
    }
  }
  const int z = opt_.z_dim;
  mean_.assign(z, 0.0f);
  std_.assign(z, 1.0f);
  if (synthetic) {
    for (int c = 0; c < z; ++c) {
      mean_[c] = 0.05f * std::sin(static_cast<float>(c));
      std_[c] = 0.5f + 0.01f * static_cast<float>(c);
    }
  } else if (!file.get_f32_array("gwp05.vae_latents_mean", &mean_) ||
             !file.get_f32_array("gwp05.vae_latents_std", &std_) ||
             static_cast<int>(mean_.size()) != z || static_cast<int>(std_.size()) != z) {
    *err = "VAE artifact lacks gwp05.vae_latents_mean / vae_latents_std of z_dim values";
    return false;
  }
  for (float s : std_)
    if (!(s > 0.0f) || !std::isfinite(s)) {
      *err = "VAE latent std must be positive and finite";
      return false;
    }
  VK(cudaMalloc(&stats_dev_, sizeof(float) * 2 * z));
  allocs_.push_back(stats_dev_);
  VK(cudaMemcpy(stats_dev_, mean_.data(), sizeof(float) * z, cudaMemcpyHostToDevice));
  VK(cudaMemcpy(stats_dev_ + z, std_.data(), sizeof(float) * z, cudaMemcpyHostToDevice));
  VK(cudaGetLastError());
  VK(cudaStreamSynchronize(stream_));
  return true;
}

bool VaeEncoder::conv(const Act& x, const std::string& wname, int mode, Act* out,
                      const Act* residual, std::string* err, const std::string& bias_name) {
  const auto it = wconv_.find(wname + ".weight");
  if (it == wconv_.end()) {
    *err = "VAE: no convolution " + wname;
    return false;
  }
  const int cout = static_cast<int>(out->c);
  ConvOp op;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, opt_.device_index);
  const char* e = conv_plan(&op, x.p, x.w, x.h, x.c, mode, it->second, cout,
                            residual ? EPI_RES : EPI_BIAS,
                            w_[bias_name.empty() ? wname + ".bias" : bias_name],
                            residual ? residual->p : nullptr, out->p, sms);
  if (e) {
    *err = std::string("VAE ") + wname + ": " + e;
    return false;
  }
  const int taps = mode == 2 ? 1 : 9;
  flops_ += 2.0 * out->h * out->w * cout * static_cast<double>(x.c) * taps;
  unsigned* errw = error_;
  program_.push_back([op, errw](cudaStream_t s) { return conv_launch(op, errw, s, false); });
  return true;
}

void VaeEncoder::rms(const Act& x, const std::string& gamma, bool silu_on, Act* out) {
  const bf16* g = w_[gamma];
  const Act in = x, o = *out;
  program_.push_back([in, o, g, silu_on](cudaStream_t s) {
    const int rows = in.h * in.w;
    const int per_block = 256 / (in.c / 8);
    rms_act_kernel<<<(rows + per_block - 1) / per_block, 256, 0, s>>>(in.p, g, o.p, rows, in.c,
                                                                       silu_on ? 1 : 0);
    return cudaGetLastError() == cudaSuccess;
  });
}

bool VaeEncoder::gemm(const bf16* x, int ldx, int m, const bf16* w, int n, int k, int epi,
                      const bf16* bias, const bf16* residual, void* out, std::string* err,
                      bool weights_from_prev) {
  GemmScratch sc;
  sc.workspace = gemm_ws_;
  sc.workspace_floats = gemm_ws_floats_;
  sc.counters = gemm_counters_;
  sc.counter_slots = 4096;
  sc.error = error_;
  GemmOp op;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, opt_.device_index);
  const char* e = gemm_plan(&op, x, ldx, m, w, n, k, epi, bias, nullptr, residual, n, out, n, sc,
                            sms, 0);
  if (e) {
    *err = std::string("VAE attention GEMM: ") + e;
    return false;
  }
  op.weights_from_prev = weights_from_prev;
  flops_ += 2.0 * m * n * static_cast<double>(k);
  program_.push_back([op](cudaStream_t s) { return gemm_launch(op, s) == cudaSuccess; });
  return true;
}

bool VaeEncoder::resnet(const std::string& p, const Act& x, int cout, Act* out, std::string* err) {
  Act a1 = act(x.h, x.w, x.c, err);
  Act h1 = act(x.h, x.w, cout, err);
  Act a2 = act(x.h, x.w, cout, err);
  *out = act(x.h, x.w, cout, err);
  if (!a1.p || !h1.p || !a2.p || !out->p) return false;
  Act sc = x;
  if (x.c != cout) {
    sc = act(x.h, x.w, cout, err);
    if (!sc.p || !conv(x, p + ".skip", 2, &sc, nullptr, err)) return false;
  }
  rms(x, p + ".n1", true, &a1);
  if (!conv(a1, p + ".c1", 0, &h1, nullptr, err)) return false;
  rms(h1, p + ".n2", true, &a2);
  return conv(a2, p + ".c2", 0, out, &sc, err);
}

bool VaeEncoder::down_block(int index, const Act& x, bool downsample, bool temporal, int cout,
                            Act* out, std::string* err) {
  const std::string p = "vae.enc.down." + std::to_string(index);
  Act r0, r1;
  if (!resnet(p + ".res.0", x, cout, &r0, err) || !resnet(p + ".res.1", r0, cout, &r1, err))
    return false;
  if (!downsample) {
    *out = act(x.h, x.w, cout, err);
    if (!out->p) return false;
    const Act a = r1, b = x, o = *out;
    program_.push_back([a, b, o](cudaStream_t s) {
      const long long n8 = static_cast<long long>(o.h) * o.w * o.c / 8;
      add_bf16_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(a.p, b.p, o.p, n8);
      return cudaGetLastError() == cudaSuccess;
    });
    return true;
  }
  if ((temporal ? 2 * x.c : x.c) != cout) {
    *err = "VAE: average shortcut channel mismatch";
    return false;
  }
  Act sc = act(x.h / 2, x.w / 2, cout, err);
  *out = act(x.h / 2, x.w / 2, cout, err);
  if (!sc.p || !out->p) return false;
  const Act in = x, so = sc;
  program_.push_back([in, so, temporal](cudaStream_t s) {
    const long long n = static_cast<long long>(in.h / 2) * (in.w / 2) * (in.c / 8);
    avg_shortcut_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
        in.p, so.p, in.h, in.w, in.c, temporal ? 1 : 0);
    return cudaGetLastError() == cudaSuccess;
  });
  return conv(r1, p + ".ds", 1, out, &sc, err);
}

bool VaeEncoder::mid_attention(const Act& x, Act* out, std::string* err) {
  const int T = x.h * x.w, C = x.c;
  if (T % 64 != 0) {
    *err = "VAE: the mid attention needs H/16 * W/16 to be a multiple of 64";
    return false;
  }
  Act n = act(x.h, x.w, C, err);
  if (!n.p) return false;
  rms(x, "vae.enc.mid.attn.norm", false, &n);
  void* buf = nullptr;
  const size_t qkv = static_cast<size_t>(T) * C;
  VK(cudaMalloc(&buf, qkv * 2 * 5 + static_cast<size_t>(T) * T * 6));
  allocs_.push_back(buf);
  bf16* q = static_cast<bf16*>(buf);
  bf16* k = q + qkv;
  bf16* v = k + qkv;
  bf16* vt = v + qkv;
  bf16* o = vt + qkv;
  float* scores = reinterpret_cast<float*>(o + qkv);
  bf16* probs = reinterpret_cast<bf16*>(scores + static_cast<size_t>(T) * T);
  const bf16* wq = w_["vae.enc.mid.attn.qkv.weight"];
  const bf16* bq = w_["vae.enc.mid.attn.qkv.bias"];
  // to_qkv is one [3C][C] projection; q, k, v are its row blocks (vae.cpp:239-256).
  if (!gemm(n.p, C, T, wq, C, C, EPI_BIAS, bq, nullptr, q, err) ||
      !gemm(n.p, C, T, wq + static_cast<size_t>(C) * C, C, C, EPI_BIAS, bq + C, nullptr, k, err) ||
      !gemm(n.p, C, T, wq + 2 * static_cast<size_t>(C) * C, C, C, EPI_BIAS, bq + 2 * C, nullptr,
            v, err))
    return false;
  // scores = q k^T (F32, GGML_PREC_F32), softmax(scores / sqrt(C)) (vae.cpp:262-265).
  if (!gemm(q, C, T, k, T, C, EPI_F32_OUT, nullptr, nullptr, scores, err, true)) return false;
  const float scale = 1.0f / std::sqrt(static_cast<float>(C));
  const int cols = T;
  program_.push_back([scores, probs, cols, scale](cudaStream_t s) {
    softmax_rows_kernel<<<cols, 256, cols * sizeof(float), s>>>(scores, probs, cols, scale);
    return cudaGetLastError() == cudaSuccess;
  });
  const int TT = T, CC = C;
  program_.push_back([v, vt, TT, CC](cudaStream_t s) {
    transpose_kernel<<<dim3((TT + 31) / 32, (CC + 31) / 32), dim3(32, 8), 0, s>>>(v, CC, vt, TT, CC);
    return cudaGetLastError() == cudaSuccess;
  });
  // attended = probs v (F32 out, cast to BF16 for the projection).
  if (!gemm(probs, T, T, vt, C, T, EPI_BIAS, nullptr, nullptr, o, err, true)) return false;
  *out = act(x.h, x.w, C, err);
  if (!out->p) return false;
  // proj + residual (vae.cpp:268-276).
  return gemm(o, C, T, w_["vae.enc.mid.attn.proj.weight"], C, C, EPI_RES,
              w_["vae.enc.mid.attn.proj.bias"], x.p, out->p, err);
}

bool VaeEncoder::build(std::string* err) {
  const int H2 = opt_.image_height / 2, W2 = opt_.image_width / 2;
  // Split-K workspace for the attention GEMMs (largest plan at this size).
  const int T = (H2 / 8) * (W2 / 8);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, opt_.device_index);
  size_t ws = 0;
  const int shapes[3][3] = {{T, 640, 640}, {T, T, 640}, {T, 640, T}};
  for (const auto& sh : shapes) {
    int tiles = 0;
    const size_t f = gemm_scratch_floats(sh[0], sh[1], sh[2], sms, 0, &tiles);
    if (f > ws) ws = f;
  }
  gemm_ws_floats_ = ws > 0 ? ws : 1;
  VK(cudaMalloc(&gemm_ws_, gemm_ws_floats_ * sizeof(float)));
  allocs_.push_back(gemm_ws_);
  VK(cudaMalloc(&gemm_counters_, 4096 * sizeof(unsigned)));
  allocs_.push_back(gemm_counters_);
  VK(cudaMemset(gemm_counters_, 0, 4096 * sizeof(unsigned)));

  VK(cudaMalloc(&pixels_slot_, sizeof(float) * 12 * H2 * W2));
  allocs_.push_back(pixels_slot_);
  VK(cudaMalloc(&latent_slot_, sizeof(float) * latent_count()));
  allocs_.push_back(latent_slot_);
  Act px = act(H2, W2, 64, err);
  if (!px.p) return false;
  const float* pin = pixels_slot_;
  program_.push_back([pin, px](cudaStream_t s) {
    const int hw = px.h * px.w;
    to_nhwc64_kernel<<<(hw + 255) / 256, 256, 0, s>>>(pin, px.p, hw);
    return cudaGetLastError() == cudaSuccess;
  });
  // conv_in: the 12 real channels of the 64-channel input (weights zero past 12).
  Act x = act(H2, W2, 160, err);
  if (!x.p) return false;
  {
    const auto it = wconv_.find("vae.enc.in.weight");
    ConvOp op;
    const char* e = conv_plan(&op, px.p, px.w, px.h, 64, 0, it->second, 160, EPI_BIAS,
                              w_["vae.enc.in.bias"], nullptr, x.p, sms);
    if (e) {
      *err = std::string("VAE conv_in: ") + e;
      return false;
    }
    flops_ += 2.0 * H2 * W2 * 160 * 12.0 * 9;
    unsigned* errw = error_;
    program_.push_back([op, errw](cudaStream_t s) { return conv_launch(op, errw, s, false); });
  }
  stages_["conv_in"] = x;
  const int couts[4] = {160, 320, 640, 640};
  for (int b = 0; b < 4; ++b) {
    Act y;
    if (!down_block(b, x, b < 3, b == 1 || b == 2, couts[b], &y, err)) return false;
    stages_["down" + std::to_string(b)] = y;
    x = y;
  }
  Act m0, ma, m1;
  if (!resnet("vae.enc.mid.res.0", x, 640, &m0, err) || !mid_attention(m0, &ma, err) ||
      !resnet("vae.enc.mid.res.1", ma, 640, &m1, err))
    return false;
  stages_["mid"] = m1;
  // conv_out emits 2z channels; below 64 they are padded with zero channels
  // (zero weight rows, zero bias) so that quant_conv reads a whole channel block.
  const int zc = 2 * opt_.z_dim, zc_pad = zc < 64 ? 64 : zc;
  Act a = act(m1.h, m1.w, 640, err);
  Act co = act(m1.h, m1.w, zc_pad, err);
  Act mo = act(m1.h, m1.w, zc, err);
  if (!a.p || !co.p || !mo.p) return false;
  rms(m1, "vae.enc.out_norm", true, &a);
  if (zc_pad != zc) {
    void* b = nullptr;
    VK(cudaMalloc(&b, zc_pad * 2));
    allocs_.push_back(b);
    VK(cudaMemset(b, 0, zc_pad * 2));
    VK(cudaMemcpy(b, w_["vae.enc.out.bias"], zc * 2, cudaMemcpyDeviceToDevice));
    w_["vae.enc.out.bias_padded"] = static_cast<bf16*>(b);
  }
  if (!conv(a, "vae.enc.out", 0, &co, nullptr, err, zc_pad != zc ? "vae.enc.out.bias_padded" : "") ||
      !conv(co, "vae.quant", 2, &mo, nullptr, err))
    return false;
  stages_["moments"] = mo;
  float* lat = latent_slot_;
  const float* st = stats_dev_;
  const int z = opt_.z_dim;
  program_.push_back([mo, st, lat, z](cudaStream_t s) {
    const int hw = mo.h * mo.w;
    latent_out_kernel<<<(hw * z + 255) / 256, 256, 0, s>>>(mo.p, mo.c, st, lat, hw, z);
    return cudaGetLastError() == cudaSuccess;
  });
  return true;
}

bool VaeEncoder::encode(const float* pixels, float* latent, cudaStream_t stream, std::string* err) {
  cudaSetDevice(opt_.device_index);
  const size_t pbytes = sizeof(float) * 12 * (opt_.image_height / 2) * (opt_.image_width / 2);
  cudaStream_t s = stream;  // as given: NULL is the legacy default stream
  if (pixels != pixels_slot_) VK(cudaMemcpyAsync(pixels_slot_, pixels, pbytes, cudaMemcpyDeviceToDevice, s));
  if (graph_) {
    VK(cudaGraphLaunch(graph_, s));
  } else {
    for (auto& f : program_)
      if (!f(s)) {
        *err = "VAE kernel launch failed";
        return false;
      }
  }
  if (latent != latent_slot_)
    VK(cudaMemcpyAsync(latent, latent_slot_, sizeof(float) * latent_count(), cudaMemcpyDeviceToDevice, s));
  return true;
}

bool VaeEncoder::encode_images(const PreprocessView* views, int n_views, float* latent,
                               cudaStream_t stream, std::string* err) {
  if (!views || n_views != 3) {
    *err = "exactly three input images are required";
    return false;
  }
  cudaSetDevice(opt_.device_index);
  cudaStream_t s = stream;  // as given: NULL is the legacy default stream
  PreprocessView dev[3];
  for (int i = 0; i < 3; ++i) {
    const PreprocessView& v = views[i];
    if (!v.data || v.w <= 0 || v.h <= 0 || (v.format != 0 && v.format != 1) ||
        static_cast<long long>(v.w) * v.h > (1ll << 30)) {
      *err = "invalid image " + std::to_string(i);
      return false;
    }
    const size_t bytes = static_cast<size_t>(v.w) * v.h * 3 * (v.format == 0 ? 1 : 4);
    if (bytes > view_cap_[i]) {
      // The stream may still read the old buffer (a previous encode).
      VK(cudaStreamSynchronize(s));
      cudaFree(view_buf_[i]);
      view_buf_[i] = nullptr;
      view_cap_[i] = 0;
      VK(cudaMalloc(&view_buf_[i], bytes));
      view_cap_[i] = bytes;
    }
    VK(cudaMemcpyAsync(view_buf_[i], v.data, bytes, cudaMemcpyHostToDevice, s));
    dev[i] = PreprocessView{view_buf_[i], v.w, v.h, v.format};
  }
  if (!launch_preprocess(dev, opt_.image_width, opt_.image_height, pixels_slot_, s)) {
    *err = "preprocess kernel launch failed";
    return false;
  }
  return encode(pixels_slot_, latent, s, err);
}

bool VaeEncoder::read_stage(const std::string& name, std::vector<float>* out, int* h, int* w, int* c) {
  const auto it = stages_.find(name);
  if (it == stages_.end()) return false;
  const Act& a = it->second;
  std::vector<uint16_t> raw(static_cast<size_t>(a.h) * a.w * a.c);
  if (cudaMemcpy(raw.data(), a.p, raw.size() * 2, cudaMemcpyDeviceToHost) != cudaSuccess) return false;
  out->resize(raw.size());
  for (size_t i = 0; i < raw.size(); ++i) {
    const uint32_t u = static_cast<uint32_t>(raw[i]) << 16;
    std::memcpy(&(*out)[i], &u, 4);
  }
  *h = a.h;
  *w = a.w;
  *c = a.c;
  return true;
}

}  // namespace wamb
