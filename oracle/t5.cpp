// CPU oracle (TEST INFRASTRUCTURE ONLY) of the UMT5 text encoder: a
// restatement of the reference's run_t5 (src/models/gwp05/engine/
// text_encoder.cpp:112-204) in F32 with the rounding points of its BF16
// weights: every matrix product takes BF16 activations and returns a BF16
// value (ggml's cuBLAS route through a BF16 temporary); the residual stream,
// RMS norms (eps 1e-6), softmax (no 1/sqrt(d) scale, relative position bias)
// and the GELU(tanh) x linear product stay F32; the final norm is F32.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "oracle.h"

namespace {

float bfr(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  u &= 0xFFFF0000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

float b2f(uint16_t b) {
  const uint32_t u = static_cast<uint32_t>(b) << 16;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

// relative_position_bucket (text_encoder.cpp:14-24).
int bucket(int relative, int buckets, int max_distance) {
  const int half = buckets / 2;
  int b = relative > 0 ? half : 0;
  const int d = std::abs(relative);
  const int exact = half / 2;
  if (d < exact) return b + d;
  const float ratio = std::log(static_cast<float>(d) / exact) /
                      std::log(static_cast<float>(max_distance) / exact);
  return b + std::min(half - 1, exact + static_cast<int>(ratio * (half - exact)));
}

std::vector<float> rms(const std::vector<float>& h, int n, int H, const uint16_t* w) {
  std::vector<float> y(static_cast<size_t>(n) * H);
  for (int i = 0; i < n; ++i) {
    const float* r = &h[static_cast<size_t>(i) * H];
    float ss = 0.0f;
    for (int c = 0; c < H; ++c) ss += r[c] * r[c];
    const float inv = 1.0f / std::sqrt(ss / static_cast<float>(H) + 1e-6f);
    for (int c = 0; c < H; ++c) y[static_cast<size_t>(i) * H + c] = r[c] * inv * b2f(w[c]);
  }
  return y;
}

// y [n][N] = bf(bf(x) w^T), w [N][K] BF16.
std::vector<float> mm(const std::vector<float>& x, int n, int K, const uint16_t* w, int N) {
  std::vector<float> xb(x.size());
  for (size_t i = 0; i < x.size(); ++i) xb[i] = bfr(x[i]);
  std::vector<float> y(static_cast<size_t>(n) * N);
#pragma omp parallel for schedule(static)
  for (int j = 0; j < N; ++j) {
    std::vector<float> wr(K);
    for (int k = 0; k < K; ++k) wr[k] = b2f(w[static_cast<size_t>(j) * K + k]);
    for (int i = 0; i < n; ++i) {
      float acc = 0.0f;
      const float* xr = &xb[static_cast<size_t>(i) * K];
      for (int k = 0; k < K; ++k) acc += xr[k] * wr[k];
      y[static_cast<size_t>(i) * N + j] = bfr(acc);
    }
  }
  return y;
}

float gelu_tanh(float x) {
  return 0.5f * x * (1.0f + std::tanh(0.7978845608028654f * x * (1.0f + 0.044715f * x * x)));
}

}  // namespace

extern "C" int oracle_t5_encode(const char* const* names, const uint16_t* const* tensors,
                                int n_tensors, int hidden, int heads, int head_dim, int ffn,
                                int layers, int vocab, const int32_t* tokens, int n,
                                int max_tokens, float* out) {
  std::map<std::string, const uint16_t*> W;
  for (int i = 0; i < n_tensors; ++i) W[names[i]] = tensors[i];
  const int H = hidden, I = heads * head_dim, F = ffn;
  if (n < 1 || n > max_tokens) return 1;
  try {
    std::vector<float> h(static_cast<size_t>(n) * H);
    const uint16_t* emb = W.at("t5.token_embd.weight");
    for (int i = 0; i < n; ++i) {
      if (tokens[i] < 0 || tokens[i] >= vocab) return 1;
      for (int c = 0; c < H; ++c) h[static_cast<size_t>(i) * H + c] = b2f(emb[static_cast<size_t>(tokens[i]) * H + c]);
    }
    for (int l = 0; l < layers; ++l) {
      const std::string p = "t5.blk." + std::to_string(l);
      const std::vector<float> x = rms(h, n, H, W.at(p + ".sa_norm.weight"));
      const std::vector<float> q = mm(x, n, H, W.at(p + ".sa.q.weight"), I);
      const std::vector<float> k = mm(x, n, H, W.at(p + ".sa.k.weight"), I);
      const std::vector<float> v = mm(x, n, H, W.at(p + ".sa.v.weight"), I);
      const uint16_t* rel = W.at(p + ".sa.rel.weight");
      std::vector<float> att(static_cast<size_t>(n) * I, 0.0f);
#pragma omp parallel for schedule(static)
      for (int hd = 0; hd < heads; ++hd) {
        std::vector<float> s(n);
        for (int i = 0; i < n; ++i) {
          float mx = -INFINITY;
          for (int j = 0; j < n; ++j) {
            float acc = 0.0f;
            for (int d = 0; d < head_dim; ++d)
              acc += q[static_cast<size_t>(i) * I + hd * head_dim + d] *
                     k[static_cast<size_t>(j) * I + hd * head_dim + d];
            s[j] = acc + b2f(rel[bucket(j - i, 32, 128) * heads + hd]);
            mx = std::max(mx, s[j]);
          }
          float sum = 0.0f;
          for (int j = 0; j < n; ++j) {
            s[j] = std::exp(s[j] - mx);
            sum += s[j];
          }
          for (int d = 0; d < head_dim; ++d) {
            float acc = 0.0f;
            for (int j = 0; j < n; ++j) acc += s[j] * v[static_cast<size_t>(j) * I + hd * head_dim + d];
            att[static_cast<size_t>(i) * I + hd * head_dim + d] = acc / sum;
          }
        }
      }
      const std::vector<float> o = mm(att, n, I, W.at(p + ".sa.o.weight"), H);
      for (size_t i = 0; i < h.size(); ++i) h[i] += o[i];
      const std::vector<float> x2 = rms(h, n, H, W.at(p + ".ffn_norm.weight"));
      const std::vector<float> g = mm(x2, n, H, W.at(p + ".ffn.wi0.weight"), F);
      const std::vector<float> lin = mm(x2, n, H, W.at(p + ".ffn.wi1.weight"), F);
      std::vector<float> prod(g.size());
      for (size_t i = 0; i < g.size(); ++i) prod[i] = gelu_tanh(g[i]) * lin[i];
      const std::vector<float> f = mm(prod, n, F, W.at(p + ".ffn.wo.weight"), H);
      for (size_t i = 0; i < h.size(); ++i) h[i] += f[i];
    }
    const std::vector<float> y = rms(h, n, H, W.at("t5.final_norm.weight"));
    std::memset(out, 0, sizeof(float) * static_cast<size_t>(max_tokens) * H);
    std::memcpy(out, y.data(), sizeof(float) * y.size());
  } catch (const std::out_of_range&) {
    return 2;
  }
  return 0;
}
