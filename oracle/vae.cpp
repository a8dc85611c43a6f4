// CPU oracle (TEST INFRASTRUCTURE ONLY) of the Wan VAE encoder, single frame:
// a restatement of the reference's run_vae graph (src/models/gwp05/engine/
// vae.cpp:136-388) in F32 with the BF16 rounding points of its native-BF16
// path (policy mot-vae-bf16*):
//   vae_conv (:141-160): BF16 input, BF16 weight, F32 accumulation, the
//     convolution rounded to BF16 (cuDNN BF16 output), + bias rounded to BF16;
//   vae_rms (:162-176): x * rsqrt(mean(x^2) + 1e-12) * gamma in F32
//     (ggml_rms_norm_bf16_f32), SiLU in F32, cast to BF16 by the next conv;
//   vae_residual (:178-191): conv2 + shortcut rounded to BF16;
//   vae_avg_shortcut (:193-213): 2x2 average in F32 -> BF16, temporal form
//     interleaving zero channels (2c = 0, 2c + 1 = pooled c);
//   vae_down_block (:215-232): downsampler = zero pad right / bottom, 3x3
//     stride 2; no downsample: + block input;
//   vae_mid_attention (:234-277): RMS (no SiLU) -> BF16, to_qkv linear (BF16
//     out + bias -> BF16), scores F32, softmax(scores / sqrt(C)) F32, rounded
//     to BF16 for the value product, output F32 -> BF16, proj + bias -> BF16,
//     + input -> BF16;
//   latent (:376-386): (moments[c] - mean[c]) / std[c] for c < z.
// Activations are NHWC. Weights are BF16 bit patterns addressed by the
// reference's compact tensor names.
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

float bf(float x) {  // round to nearest even BF16 (finite inputs)
  uint32_t u;
  std::memcpy(&u, &x, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  u &= 0xFFFF0000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

float bits(uint16_t b) {
  const uint32_t u = static_cast<uint32_t>(b) << 16;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

struct T {  // NHWC activation
  int h = 0, w = 0, c = 0;
  std::vector<float> v;
  T() = default;
  T(int h_, int w_, int c_) : h(h_), w(w_), c(c_), v(static_cast<size_t>(h_) * w_ * c_, 0.0f) {}
  float& at(int y, int x, int ch) { return v[(static_cast<size_t>(y) * w + x) * c + ch]; }
  float at(int y, int x, int ch) const { return v[(static_cast<size_t>(y) * w + x) * c + ch]; }
};

struct Weights {
  std::map<std::string, const uint16_t*> m;
  std::vector<float> get(const std::string& n, size_t count) const {
    std::vector<float> r(count);
    const uint16_t* p = m.at(n);
    for (size_t i = 0; i < count; ++i) r[i] = bits(p[i]);
    return r;
  }
};

// y = bf(bf(conv(x)) + b) [+ residual, bf]; mode 0: 3x3 pad 1, 1: 3x3 stride 2
// with the zero pad at the end, 2: 1x1. x holds BF16-exact values.
T conv(const Weights& W, const std::string& name, const T& x, int cout, int mode,
       const T* residual) {
  const int k = mode == 2 ? 1 : 3;
  const std::vector<float> w = W.get(name + ".weight", static_cast<size_t>(cout) * x.c * k * k);
  const std::vector<float> b = W.get(name + ".bias", cout);
  const int oh = mode == 1 ? x.h / 2 : x.h, ow = mode == 1 ? x.w / 2 : x.w;
  T y(oh, ow, cout);
  // Weight as [tap][cin][cout] for a contiguous inner loop over cout.
  std::vector<float> wt(static_cast<size_t>(k) * k * x.c * cout);
  for (int o = 0; o < cout; ++o)
    for (int ci = 0; ci < x.c; ++ci)
      for (int t = 0; t < k * k; ++t)
        wt[(static_cast<size_t>(t) * x.c + ci) * cout + o] =
            w[(static_cast<size_t>(o) * x.c + ci) * k * k + t];
#pragma omp parallel for schedule(static)
  for (int p = 0; p < oh * ow; ++p) {
    const int oy = p / ow, ox = p % ow;
    std::vector<float> acc(cout, 0.0f);
    for (int t = 0; t < k * k; ++t) {
      const int dy = t / k, dx = t % k;
      int iy, ix;
      if (mode == 0) {
        iy = oy + dy - 1;
        ix = ox + dx - 1;
      } else if (mode == 1) {
        iy = 2 * oy + dy;
        ix = 2 * ox + dx;
      } else {
        iy = oy;
        ix = ox;
      }
      if (iy < 0 || ix < 0 || iy >= x.h || ix >= x.w) continue;
      const float* xp = &x.v[(static_cast<size_t>(iy) * x.w + ix) * x.c];
      const float* wp = &wt[static_cast<size_t>(t) * x.c * cout];
      for (int ci = 0; ci < x.c; ++ci) {
        const float xv = xp[ci];
        const float* wr = wp + static_cast<size_t>(ci) * cout;
        for (int o = 0; o < cout; ++o) acc[o] += xv * wr[o];
      }
    }
    float* yp = &y.v[static_cast<size_t>(p) * cout];
    for (int o = 0; o < cout; ++o) {
      float r = bf(bf(acc[o]) + b[o]);
      if (residual) r = bf(r + residual->v[static_cast<size_t>(p) * cout + o]);
      yp[o] = r;
    }
  }
  return y;
}

T rms(const Weights& W, const std::string& gamma, const T& x, bool silu) {
  const std::vector<float> g = W.get(gamma, x.c);
  T y(x.h, x.w, x.c);
#pragma omp parallel for schedule(static)
  for (int p = 0; p < x.h * x.w; ++p) {
    const float* xp = &x.v[static_cast<size_t>(p) * x.c];
    float ss = 0.0f;
    for (int c = 0; c < x.c; ++c) ss += xp[c] * xp[c];
    const float inv = 1.0f / std::sqrt(ss / static_cast<float>(x.c) + 1e-12f);
    for (int c = 0; c < x.c; ++c) {
      float v = xp[c] * inv * g[c];
      if (silu) v = v / (1.0f + std::exp(-v));
      y.v[static_cast<size_t>(p) * x.c + c] = bf(v);
    }
  }
  return y;
}

T resnet(const Weights& W, const std::string& p, const T& x, int cout) {
  T sc = x.c != cout ? conv(W, p + ".skip", x, cout, 2, nullptr) : x;
  T h = conv(W, p + ".c1", rms(W, p + ".n1", x, true), cout, 0, nullptr);
  return conv(W, p + ".c2", rms(W, p + ".n2", h, true), cout, 0, &sc);
}

T avg_shortcut(const T& x, int cout, bool temporal) {
  T y(x.h / 2, x.w / 2, cout);
  for (int oy = 0; oy < y.h; ++oy)
    for (int ox = 0; ox < y.w; ++ox)
      for (int c = 0; c < x.c; ++c) {
        const float s = x.at(2 * oy, 2 * ox, c) + x.at(2 * oy, 2 * ox + 1, c) +
                        x.at(2 * oy + 1, 2 * ox, c) + x.at(2 * oy + 1, 2 * ox + 1, c);
        const float a = bf(s * 0.25f);
        if (temporal) {
          y.at(oy, ox, 2 * c) = 0.0f;
          y.at(oy, ox, 2 * c + 1) = a;
        } else {
          y.at(oy, ox, c) = a;
        }
      }
  return y;
}

T down_block(const Weights& W, int b, const T& x, bool down, bool temporal, int cout) {
  const std::string p = "vae.enc.down." + std::to_string(b);
  T h = resnet(W, p + ".res.1", resnet(W, p + ".res.0", x, cout), cout);
  if (!down) {
    for (size_t i = 0; i < h.v.size(); ++i) h.v[i] = bf(h.v[i] + x.v[i]);
    return h;
  }
  const T sc = avg_shortcut(x, cout, temporal);
  return conv(W, p + ".ds", h, cout, 1, &sc);
}

// y [T][n] = bf(bf(x w^T) + b) for a [n][k] weight (w offset by rows).
std::vector<float> linear(const std::vector<float>& x, int t, int k, const std::vector<float>& w,
                          const std::vector<float>& b, int n, int row0) {
  std::vector<float> y(static_cast<size_t>(t) * n);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < t; ++i)
    for (int j = 0; j < n; ++j) {
      float acc = 0.0f;
      const float* xr = &x[static_cast<size_t>(i) * k];
      const float* wr = &w[static_cast<size_t>(row0 + j) * k];
      for (int q = 0; q < k; ++q) acc += xr[q] * wr[q];
      y[static_cast<size_t>(i) * n + j] = bf(bf(acc) + b[row0 + j]);
    }
  return y;
}

T mid_attention(const Weights& W, const T& x) {
  const int t = x.h * x.w, c = x.c;
  const T n = rms(W, "vae.enc.mid.attn.norm", x, false);
  const std::vector<float> wq = W.get("vae.enc.mid.attn.qkv.weight", static_cast<size_t>(3) * c * c);
  const std::vector<float> bq = W.get("vae.enc.mid.attn.qkv.bias", 3 * c);
  const std::vector<float> q = linear(n.v, t, c, wq, bq, c, 0);
  const std::vector<float> k = linear(n.v, t, c, wq, bq, c, c);
  const std::vector<float> v = linear(n.v, t, c, wq, bq, c, 2 * c);
  const float scale = 1.0f / std::sqrt(static_cast<float>(c));
  std::vector<float> o(static_cast<size_t>(t) * c);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < t; ++i) {
    std::vector<float> s(t);
    float mx = -INFINITY;
    for (int j = 0; j < t; ++j) {
      float acc = 0.0f;
      for (int q2 = 0; q2 < c; ++q2) acc += q[static_cast<size_t>(i) * c + q2] * k[static_cast<size_t>(j) * c + q2];
      s[j] = acc * scale;
      mx = std::max(mx, s[j]);
    }
    float sum = 0.0f;
    for (int j = 0; j < t; ++j) {
      s[j] = std::exp(s[j] - mx);
      sum += s[j];
    }
    const float inv = 1.0f / sum;
    for (int j = 0; j < t; ++j) s[j] = bf(s[j] * inv);
    for (int q2 = 0; q2 < c; ++q2) {
      float acc = 0.0f;
      for (int j = 0; j < t; ++j) acc += s[j] * v[static_cast<size_t>(j) * c + q2];
      o[static_cast<size_t>(i) * c + q2] = bf(acc);
    }
  }
  const std::vector<float> wp = W.get("vae.enc.mid.attn.proj.weight", static_cast<size_t>(c) * c);
  const std::vector<float> bp = W.get("vae.enc.mid.attn.proj.bias", c);
  const std::vector<float> pr = linear(o, t, c, wp, bp, c, 0);
  T y(x.h, x.w, c);
  for (size_t i = 0; i < y.v.size(); ++i) y.v[i] = bf(x.v[i] + pr[i]);
  return y;
}

void put_stage(const T& a, const char* want, const char* name, float* out, int* dims) {
  if (!want || !out || std::strcmp(want, name) != 0) return;
  std::memcpy(out, a.v.data(), a.v.size() * sizeof(float));
  if (dims) {
    dims[0] = a.h;
    dims[1] = a.w;
    dims[2] = a.c;
  }
}

}  // namespace

extern "C" int oracle_vae_encode(const char* const* names, const uint16_t* const* tensors,
                                 int n_tensors, const float* mean, const float* stdv, int z,
                                 const float* pixels, int width, int height, float* latent,
                                 const char* stage, float* stage_out, int* stage_dims) {
  if (width % 32 || height % 32 || z <= 0) return 1;
  Weights W;
  for (int i = 0; i < n_tensors; ++i) W.m[names[i]] = tensors[i];
  const int h2 = height / 2, w2 = width / 2;
  T x(h2, w2, 12);
  for (int c = 0; c < 12; ++c)
    for (int p = 0; p < h2 * w2; ++p)
      x.v[static_cast<size_t>(p) * 12 + c] = bf(pixels[static_cast<size_t>(c) * h2 * w2 + p]);
  try {
    x = conv(W, "vae.enc.in", x, 160, 0, nullptr);
    put_stage(x, stage, "conv_in", stage_out, stage_dims);
    const int couts[4] = {160, 320, 640, 640};
    for (int b = 0; b < 4; ++b) {
      x = down_block(W, b, x, b < 3, b == 1 || b == 2, couts[b]);
      put_stage(x, stage, ("down" + std::to_string(b)).c_str(), stage_out, stage_dims);
    }
    x = resnet(W, "vae.enc.mid.res.0", x, 640);
    x = mid_attention(W, x);
    x = resnet(W, "vae.enc.mid.res.1", x, 640);
    put_stage(x, stage, "mid", stage_out, stage_dims);
    x = conv(W, "vae.enc.out", rms(W, "vae.enc.out_norm", x, true), 2 * z, 0, nullptr);
    x = conv(W, "vae.quant", x, 2 * z, 2, nullptr);
    put_stage(x, stage, "moments", stage_out, stage_dims);
  } catch (const std::out_of_range&) {
    return 2;  // a tensor is missing
  }
  const int hw = x.h * x.w;
  for (int c = 0; c < z; ++c)
    for (int p = 0; p < hw; ++p)
      latent[static_cast<size_t>(c) * hw + p] = (x.v[static_cast<size_t>(p) * x.c + c] - mean[c]) / stdv[c];
  return 0;
}
