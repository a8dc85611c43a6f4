// CPU oracle for the GWP-0.5 MoT forward pass — TEST INFRASTRUCTURE ONLY.
// See oracle.h for scope and parity status. Each function cites the reference
// file:line it restates (paths relative to the GigaAI-research/wam.cpp tree).
//
// Precision: F32 arithmetic over BF16 weights, with the BF16 rounding points of
// the reference's bf16_latency dispatch (engine.cpp:52-78: native_bf16,
// bf16_output_gemm, bf16_hidden_and_kv, f32_accumulation):
//   * every linear: y = bf16(bf16(x·W) + b)               weights.cpp:819-831
//   * hidden stream, K/V caches, GEMM inputs: BF16
//   * AdaLN parameters, norms' statistics, scores, softmax: F32
//   * q/k RMSNorm output and RoPE in F32, then cast to BF16  mot.cpp:245-265
//   * Euler step in F32, state stored as BF16               weights.cpp:885-902
#include "oracle.h"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

using Vec = std::vector<float>;

inline float bf2f(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// Round to the nearest BF16, ties to even (ggml_fp32_to_bf16 semantics for
// finite values).
inline float bfr(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return x;
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline void bfr_inplace(Vec& v) {
  for (float& x : v) x = bfr(x);
}

// ggml CUDA op definitions, restated from their formulas.
inline float gelu_tanh(float x) {
  return 0.5f * x * (1.0f + std::tanh(0.79788456080286535588f * x * (1.0f + 0.044715f * x * x)));
}
inline float gelu_erf(float x) { return 0.5f * x * (1.0f + std::erf(x * 0.70710678118654752440f)); }
inline float silu(float x) { return x / (1.0f + std::exp(-x)); }

// F32 -> IEEE fp16 (round to nearest even, subnormals kept) -> F32.
inline float f16_round(float x) {
  if (x == 0.0f || !std::isfinite(x)) return x;
  int e;
  std::frexp(x, &e);  // |x| = m * 2^e, m in [0.5, 1)
  // fp16 keeps 11 significant bits for normals (e >= -13), fewer below.
  const int bits = e >= -13 ? 11 : 11 - (-13 - e);
  if (bits <= 0) return std::copysign(0.0f, x);
  const float q = std::ldexp(1.0f, e - bits);  // spacing of representable values
  const float r = std::nearbyint(x / q) * q;   // current rounding mode: to nearest even
  return std::fabs(r) > 65504.0f ? std::copysign(INFINITY, x) : r;
}

// Row length of a linear layer's weight as the Q8_0 policy sees it (0: not a
// linear weight); the same rule as the engine's linear_inner().
int64_t linear_inner(const std::string& n, const oracle_geometry& g) {
  auto ends = [&](const char* suf) {
    const size_t k = std::strlen(suf);
    return n.size() >= k && n.compare(n.size() - k, k, suf) == 0;
  };
  auto starts = [&](const char* pre) { return n.rfind(pre, 0) == 0; };
  if (!ends(".weight") || ends(".qn.weight") || ends(".kn.weight") || ends("ca_norm.weight"))
    return 0;
  const int64_t E = g.action_hidden, H = g.hidden;
  if (n == "gwp.patch.weight") return static_cast<int64_t>(g.vae_z) * 4;
  if (ends(".in.weight") && (starts("gwp.state") || starts("gwp.action"))) return 128;
  if (ends(".mid.weight") || n == "gwp.state.out.weight" || n == "gwp.action.out.weight") return 128;
  if (n == "gwp.decode.in.weight") return E;
  if (n == "gwp.decode.out.weight") return g.action_dim;
  if (ends(".time.0.weight")) return 256;
  if (ends(".text.0.weight")) return g.text_dim;
  if (starts("gwp.acond")) return E;
  if (starts("gwp.cond")) return H;
  const bool act = n.find(".a.") != std::string::npos;
  const int64_t W = act ? E : H, F = act ? g.action_ffn : g.ffn;
  if (ends(".sa.o.weight") || ends(".ca.o.weight")) return H;
  if (ends(".ffn.out.weight")) return F;
  return W;
}

struct Tensor {
  std::vector<uint16_t> data;
  std::vector<float> f32;  // Q8_0 mode: exact F32 dequantised values q * d (data unused)
  int64_t numel = 0;
};

struct Model {
  oracle_geometry g{};
  std::unordered_map<std::string, Tensor> t;
  Vec sq01, sq99, aq01, aq99;
  bool uncached = false;  // recompute the prefix every step (the reference's CPU mode)
  // Block variants (config 1 as BASELINE states it): ffn_kind 0 = GELU(tanh)
  // FFN (the reference), 1 = SiLU-gated FFN with ffn.in = [gate rows | up rows];
  // norm_kind 0 = LayerNorm inside AdaLN (the reference), 1 = RMSNorm.
  int ffn_kind = 0, norm_kind = 0;

  // F32 weights of a tensor the Q8_0 policy quantised (nullptr otherwise).
  const float* wf(const std::string& name) const {
    auto it = t.find(name);
    return it == t.end() || it->second.f32.empty() ? nullptr : it->second.f32.data();
  }

  const uint16_t* w(const std::string& name, int64_t expect) const {
    auto it = t.find(name);
    if (it == t.end()) {
      std::fprintf(stderr, "oracle: missing tensor %s\n", name.c_str());
      return nullptr;
    }
    if (expect >= 0 && it->second.numel != expect) {
      std::fprintf(stderr, "oracle: tensor %s has %lld elements, expected %lld\n", name.c_str(),
                   static_cast<long long>(it->second.numel), static_cast<long long>(expect));
      return nullptr;
    }
    return it->second.data.data();
  }
};

// ---------------------------------------------------------------- GEMM
// acc[m][n] = sum_k x[m][k] * W[n][k], F32. W is BF16 [N][K] row-major (GGUF
// ne = {K, N}); ggml_mul_mat(W, x) (weights.cpp:788, 826).
// Wf (when given) holds F32 weights of the same layout, used instead of W.
void gemm_acc(const float* x, int M, int K, const uint16_t* W, int N, float* acc,
              const float* Wf = nullptr) {
#pragma omp parallel
  {
    std::vector<float> wb(static_cast<size_t>(4) * K);
#pragma omp for schedule(dynamic, 1)
    for (int nb = 0; nb < (N + 3) / 4; ++nb) {
      const int n0 = nb * 4;
      const int nn = std::min(4, N - n0);
      for (int j = 0; j < 4; ++j) {
        float* dst = wb.data() + static_cast<size_t>(j) * K;
        if (j < nn && Wf) {
          std::memcpy(dst, Wf + static_cast<size_t>(n0 + j) * K, sizeof(float) * K);
        } else if (j < nn) {
          const uint16_t* src = W + static_cast<size_t>(n0 + j) * K;
          for (int k = 0; k < K; ++k) dst[k] = bf2f(src[k]);
        } else {
          std::fill(dst, dst + K, 0.0f);
        }
      }
      const float* w0 = wb.data();
      const float* w1 = w0 + K;
      const float* w2 = w1 + K;
      const float* w3 = w2 + K;
      int m = 0;
      for (; m + 1 < M; m += 2) {
        const float* x0 = x + static_cast<size_t>(m) * K;
        const float* x1 = x0 + K;
        float s00 = 0, s01 = 0, s02 = 0, s03 = 0, s10 = 0, s11 = 0, s12 = 0, s13 = 0;
#pragma omp simd reduction(+ : s00, s01, s02, s03, s10, s11, s12, s13)
        for (int k = 0; k < K; ++k) {
          const float a0 = x0[k], a1 = x1[k];
          s00 += a0 * w0[k];
          s01 += a0 * w1[k];
          s02 += a0 * w2[k];
          s03 += a0 * w3[k];
          s10 += a1 * w0[k];
          s11 += a1 * w1[k];
          s12 += a1 * w2[k];
          s13 += a1 * w3[k];
        }
        const float r0[4] = {s00, s01, s02, s03};
        const float r1[4] = {s10, s11, s12, s13};
        for (int j = 0; j < nn; ++j) {
          acc[static_cast<size_t>(m) * N + n0 + j] = r0[j];
          acc[static_cast<size_t>(m + 1) * N + n0 + j] = r1[j];
        }
      }
      for (; m < M; ++m) {
        const float* x0 = x + static_cast<size_t>(m) * K;
        float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma omp simd reduction(+ : s0, s1, s2, s3)
        for (int k = 0; k < K; ++k) {
          s0 += x0[k] * w0[k];
          s1 += x0[k] * w1[k];
          s2 += x0[k] * w2[k];
          s3 += x0[k] * w3[k];
        }
        const float r0[4] = {s0, s1, s2, s3};
        for (int j = 0; j < nn; ++j) acc[static_cast<size_t>(m) * N + n0 + j] = r0[j];
      }
    }
  }
}

// linear_with_activation with BF16 output (weights.cpp:819-831):
// y = bf16(bf16(x·W) + b); the input is cast to BF16 first. With gelu set, the
// linear_gelu_with_activation form (weights.cpp:833-849, bias_gelu_bf16_kernel):
// y = bf16(gelu_tanh(bf16(x·W) + b)).
// Rows [row0, row0 + N) of a weight with `total` rows (total = N: the whole
// weight). act 1: GELU(tanh) as above; act 2: SiLU of the BF16 linear output
// (ggml_silu on a BF16 tensor): y = bf16(silu(bf16(bf16(x·W) + b))).
Vec linear_rows(const Model& md, const Vec& x, int M, int K, const std::string& name, int row0,
                int N, int total, int act) {
  Vec xb(x);
  bfr_inplace(xb);
  const uint16_t* W = md.w(name + ".weight", static_cast<int64_t>(total) * K);
  const uint16_t* b = md.w(name + ".bias", total);
  Vec y(static_cast<size_t>(M) * N);
  if (!W || !b) return Vec();
  const float* Wf = md.wf(name + ".weight");
  gemm_acc(xb.data(), M, K, W + static_cast<size_t>(row0) * K, N, y.data(),
           Wf ? Wf + static_cast<size_t>(row0) * K : nullptr);
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      float& v = y[static_cast<size_t>(m) * N + n];
      const float bb = bf2f(b[row0 + n]);
      v = act == 1 ? bfr(gelu_tanh(bfr(v) + bb)) : act == 2 ? bfr(silu(bfr(bfr(v) + bb)))
                                                            : bfr(bfr(v) + bb);
    }
  return y;
}

Vec linear(const Model& md, const Vec& x, int M, int K, const std::string& name, int N,
           bool gelu = false) {
  return linear_rows(md, x, M, K, name, 0, N, N, gelu ? 1 : 0);
}

// Embodiment-sliced projection (mot.cpp:1-14): torch weight [emb][in][out],
// bias [emb][out]; y = bf16(bf16(x·W_e) + b_e).
Vec embodiment_linear(const Model& md, const Vec& x, int M, int in, int out,
                      const std::string& name) {
  const int emb = md.g.embodiment_id;
  const uint16_t* W = md.w(name + ".weight", static_cast<int64_t>(md.g.num_embodiments) * in * out);
  const uint16_t* b = md.w(name + ".bias", static_cast<int64_t>(md.g.num_embodiments) * out);
  const uint16_t* We = W + static_cast<size_t>(emb) * in * out;
  const float* Wf = md.wf(name + ".weight");
  const float* Wfe = Wf ? Wf + static_cast<size_t>(emb) * in * out : nullptr;
  Vec y(static_cast<size_t>(M) * out);
  for (int m = 0; m < M; ++m)
    for (int o = 0; o < out; ++o) {
      float s = 0.0f;
      for (int i = 0; i < in; ++i) {
        const size_t wi = static_cast<size_t>(i) * out + o;
        s += bfr(x[static_cast<size_t>(m) * in + i]) * (Wfe ? Wfe[wi] : bf2f(We[wi]));
      }
      y[static_cast<size_t>(m) * out + o] = bfr(bfr(s) + bf2f(b[static_cast<size_t>(emb) * out + o]));
    }
  return y;
}

// action_encoder / action_decoder (mot.cpp:16-55): 3 linears, exact-erf GELU.
Vec action_encoder(const Model& md, const std::string& comp, const Vec& x, int M) {
  const oracle_geometry& g = md.g;
  Vec h = embodiment_linear(md, x, M, g.action_dim, 128, "gwp." + comp + ".in");
  for (float& v : h) v = bfr(gelu_erf(v));
  h = linear(md, h, M, 128, "gwp." + comp + ".mid", 128);
  for (float& v : h) v = bfr(gelu_erf(v));
  return linear(md, h, M, 128, "gwp." + comp + ".out", g.action_hidden);
}

Vec action_decoder(const Model& md, const Vec& x, int M) {
  const oracle_geometry& g = md.g;
  Vec h = linear(md, x, M, g.action_hidden, "gwp.decode.in", 128);
  for (float& v : h) v = bfr(gelu_erf(v));
  h = linear(md, h, M, 128, "gwp.decode.mid", 128);
  for (float& v : h) v = bfr(gelu_erf(v));
  return embodiment_linear(md, h, M, 128, g.action_dim, "gwp.decode.out");
}

// LayerNorm statistics as norm_bf16_fused (native-bf16.patch:368-409):
// two-pass mean, centred variance, inv_std = 1/sqrt(var + eps).
void ln_stats(const float* x, int n, float eps, float* mean, float* inv_std) {
  float s = 0.0f;
  for (int i = 0; i < n; ++i) s += x[i];
  const float mu = s / n;
  float v = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float c = x[i] - mu;
    v += c * c;
  }
  *mean = mu;
  *inv_std = 1.0f / std::sqrt(v / n + eps);
}

// modulated_norm (mot.cpp:147-159): bf16(LN(x) * (1 + scale) + shift).
// rms: the config-1 RMSNorm variant, n = x * rsqrt(mean(x^2) + eps) (no mean
// subtraction), then the same AdaLN modulation.
Vec modulated_norm(const Vec& x, int M, int n, const float* scale, const float* shift, float eps,
                   bool rms = false) {
  Vec y(x.size());
  for (int m = 0; m < M; ++m) {
    const float* r = x.data() + static_cast<size_t>(m) * n;
    float mu, is;
    if (rms) {
      float ss = 0.0f;
      for (int i = 0; i < n; ++i) ss += r[i] * r[i];
      mu = 0.0f;
      is = 1.0f / std::sqrt(ss / n + eps);
    } else {
      ln_stats(r, n, eps, &mu, &is);
    }
    for (int i = 0; i < n; ++i)
      y[static_cast<size_t>(m) * n + i] = bfr(std::fma((r[i] - mu) * is, 1.0f + scale[i], shift[i]));
  }
  return y;
}

// layer_norm with BF16 affine (weights.cpp:919-930): bf16(LN(x) * w + b).
Vec layer_norm_affine(const Model& md, const Vec& x, int M, int n, const std::string& name,
                      float eps) {
  const uint16_t* w = md.w(name + ".weight", n);
  const uint16_t* b = md.w(name + ".bias", n);
  Vec y(x.size());
  for (int m = 0; m < M; ++m) {
    const float* r = x.data() + static_cast<size_t>(m) * n;
    float mu, is;
    ln_stats(r, n, eps, &mu, &is);
    for (int i = 0; i < n; ++i)
      y[static_cast<size_t>(m) * n + i] = bfr(std::fma((r[i] - mu) * is, bf2f(w[i]), bf2f(b[i])));
  }
  return y;
}

// rms_norm (weights.cpp:904-917, rms_norm_bf16_f32): F32 x * rsqrt(mean(x^2) + eps) * w
// over a strided sub-row of width n.
void rms_norm_rows(Vec& x, int M, int ld, int off, int n, const uint16_t* w, float eps) {
  for (int m = 0; m < M; ++m) {
    float* r = x.data() + static_cast<size_t>(m) * ld + off;
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s += r[i] * r[i];
    const float inv = 1.0f / std::sqrt(s / n + eps);
    for (int i = 0; i < n; ++i) r[i] = r[i] * inv * bf2f(w[i]);
  }
}

// RoPE NORMAL mode over n_dims of one head slice (mot.cpp:175-202, ggml_rope_ext
// with ext_factor 0, freq_scale 1, attn_factor 1): pairs (2i, 2i+1),
// theta_i = pos * base^(-2i/n_dims).
void rope_slice(float* v, int n_dims, int pos) {
  const float theta_scale = std::pow(10000.0f, -2.0f / static_cast<float>(n_dims));
  for (int i = 0; i < n_dims / 2; ++i) {
    const float theta = static_cast<float>(pos) * std::pow(theta_scale, static_cast<float>(i));
    const float c = std::cos(theta), s = std::sin(theta);
    const float x0 = v[2 * i], x1 = v[2 * i + 1];
    v[2 * i] = x0 * c - x1 * s;
    v[2 * i + 1] = x0 * s + x1 * c;
  }
}

// Attention for one head: out[i] = softmax(scale * q_i·K^T) V, F32 scores and
// softmax (GGML_PREC_F32, ggml_soft_max_ext), F32 accumulation.
// q: [Lq][ldq] at column offset; k, v likewise. out: [Lq][ldo].
void attend_head(const float* q, int ldq, int lq, const float* k, const float* v, int ldkv,
                 int lk, float scale, float* out, int ldo) {
  std::vector<float> s(lk);
  for (int i = 0; i < lq; ++i) {
    const float* qi = q + static_cast<size_t>(i) * ldq;
    float mx = -INFINITY;
    for (int j = 0; j < lk; ++j) {
      const float* kj = k + static_cast<size_t>(j) * ldkv;
      float d = 0.0f;
      for (int e = 0; e < 128; ++e) d += qi[e] * kj[e];
      s[j] = d * scale;
      mx = std::max(mx, s[j]);
    }
    float sum = 0.0f;
    for (int j = 0; j < lk; ++j) {
      s[j] = std::exp(s[j] - mx);
      sum += s[j];
    }
    const float inv = 1.0f / sum;
    float* o = out + static_cast<size_t>(i) * ldo;
    for (int e = 0; e < 128; ++e) o[e] = 0.0f;
    for (int j = 0; j < lk; ++j) {
      const float p = s[j] * inv;
      const float* vj = v + static_cast<size_t>(j) * ldkv;
      for (int e = 0; e < 128; ++e) o[e] += p * vj[e];
    }
  }
}

// Multi-head attention over token-major q [lq][H], k/v [lk][H]; returns
// BF16-rounded [lq][H] (the O projection casts its input to BF16).
Vec attention(const Vec& q, int lq, const Vec& k, const Vec& v, int lk, int heads) {
  const int H = heads * 128;
  Vec out(static_cast<size_t>(lq) * H);
  const float scale = 1.0f / std::sqrt(128.0f);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int h = 0; h < heads; ++h)
    for (int i0 = 0; i0 < lq; i0 += 16) {
      const int n = std::min(16, lq - i0);
      attend_head(q.data() + static_cast<size_t>(i0) * H + h * 128, H, n, k.data() + h * 128,
                  v.data() + h * 128, H, lk, scale, out.data() + static_cast<size_t>(i0) * H + h * 128, H);
    }
  bfr_inplace(out);
  return out;
}

// timestep_embedding (text_encoder.cpp:1-12): [cos(t f_i) | sin(t f_i)],
// f_i = exp(-ln(1e4) i / half).
Vec timestep_embedding(float t, int dim) {
  const int half = dim / 2;
  Vec out(dim, 0.0f);
  for (int i = 0; i < half; ++i) {
    const float f = std::exp(-std::log(10000.0f) * static_cast<float>(i) / static_cast<float>(half));
    const float v = t * f;
    out[i] = std::cos(v);
    out[i + half] = std::sin(v);
  }
  return out;
}

struct Condition {
  Vec temb;  // [W] BF16 values
  Vec mod;   // [6W] BF16 values
};

// build_condition time branch (mot.cpp:63-82).
Condition condition(const Model& md, const std::string& comp, float t, int W) {
  Vec f = timestep_embedding(t, 256);
  Vec h = linear(md, f, 1, 256, "gwp." + comp + ".time.0", W);
  for (float& v : h) v = bfr(silu(v));
  Condition c;
  c.temb = linear(md, h, 1, W, "gwp." + comp + ".time.1", W);
  Vec s(c.temb);
  for (float& v : s) v = bfr(silu(v));
  c.mod = linear(md, s, 1, W, "gwp." + comp + ".time.out", 6 * W);
  return c;
}

// build_condition text branch (mot.cpp:84-92): W2 gelu_tanh(W1 x + b1) + b2.
Vec text_embed(const Model& md, const std::string& comp, const Vec& prompt, int W) {
  const oracle_geometry& g = md.g;
  Vec h = linear(md, prompt, g.prompt_tokens, g.text_dim, "gwp." + comp + ".text.0", W);
  for (float& v : h) v = bfr(gelu_tanh(v));
  return linear(md, h, g.prompt_tokens, W, "gwp." + comp + ".text.1", W);
}

// modulation_add (mot.cpp:137-145) with f32_accumulation: F32(mod) + F32(table).
Vec combined_mod(const Model& md, const Vec& mod, const std::string& table, int W) {
  const uint16_t* tb = md.w(table, 6LL * W);
  Vec c(6 * W);
  for (int i = 0; i < 6 * W; ++i) c[i] = mod[i] + bf2f(tb[i]);
  return c;
}

struct ExpertQkv {
  Vec q, k, v;  // token-major [rows][H], q/k after RMSNorm+RoPE and BF16 cast
};

// expert_qkv (mot.cpp:210-267) with packed QKV (artifact policy mot-vae-bf16-qkv-v1).
ExpertQkv expert_qkv(const Model& md, const std::string& pfx, const Vec& hidden, int rows, int W,
                     const float* shift, const float* scale, bool visual, int pos_base,
                     const int32_t* pt, const int32_t* ph, const int32_t* pw) {
  const oracle_geometry& g = md.g;
  const int H = g.hidden;
  Vec n = modulated_norm(hidden, rows, W, scale, shift, g.norm_eps, md.norm_kind == 1);
  Vec qkv = linear(md, n, rows, W, pfx + ".sa.qkv", 3 * H);
  rms_norm_rows(qkv, rows, 3 * H, 0, H, md.w(pfx + ".sa.qn.weight", H), g.norm_eps);
  rms_norm_rows(qkv, rows, 3 * H, H, H, md.w(pfx + ".sa.kn.weight", H), g.norm_eps);
  ExpertQkv o;
  o.q.resize(static_cast<size_t>(rows) * H);
  o.k.resize(static_cast<size_t>(rows) * H);
  o.v.resize(static_cast<size_t>(rows) * H);
  for (int r = 0; r < rows; ++r) {
    std::memcpy(&o.q[static_cast<size_t>(r) * H], &qkv[static_cast<size_t>(r) * 3 * H], H * 4);
    std::memcpy(&o.k[static_cast<size_t>(r) * H], &qkv[static_cast<size_t>(r) * 3 * H + H], H * 4);
    std::memcpy(&o.v[static_cast<size_t>(r) * H], &qkv[static_cast<size_t>(r) * 3 * H + 2 * H], H * 4);
    for (int h = 0; h < g.heads; ++h) {
      for (Vec* t : {&o.q, &o.k}) {
        float* s = t->data() + static_cast<size_t>(r) * H + h * 128;
        if (visual) {
          // apply_visual_rope: sections 44/42/42 at positions (t, h, w).
          rope_slice(s, 44, pt[r]);
          rope_slice(s + 44, 42, ph[r]);
          rope_slice(s + 86, 42, pw[r]);
        } else {
          rope_slice(s, 128, pos_base + r);
        }
      }
    }
  }
  bfr_inplace(o.q);
  bfr_inplace(o.k);
  return o;
}


// Cross attention + FFN of one expert (mot.cpp:284-347). With cached prompt
// K/V (pk/pv given, BF16, token-major [N_t][H]) the query is RMS-normalised and
// cast to BF16 (cached branch, :299-325). Without them (visual expert in the
// prefix) K/V are projected from `text` through build_attention
// (text_encoder.cpp:26-73), where q and k stay F32.
Vec cross_ffn(const Model& md, const std::string& pfx, const Vec& hidden, int rows, int W, int F,
              const Vec* pk, const Vec* pv, const Vec* text, int text_w, const float* cshift,
              const float* cscale, const float* cgate) {
  const oracle_geometry& g = md.g;
  const int H = g.hidden;
  Vec n = layer_norm_affine(md, hidden, rows, W, pfx + ".ca_norm", g.norm_eps);
  Vec q = linear(md, n, rows, W, pfx + ".ca.q", H);
  rms_norm_rows(q, rows, H, 0, H, md.w(pfx + ".ca.qn.weight", H), g.norm_eps);
  Vec att;
  if (pk && pv) {
    bfr_inplace(q);
    att = attention(q, rows, *pk, *pv, g.prompt_tokens, g.heads);
  } else {
    Vec k = linear(md, *text, g.prompt_tokens, text_w, pfx + ".ca.k", H);
    Vec v = linear(md, *text, g.prompt_tokens, text_w, pfx + ".ca.vproj", H);
    rms_norm_rows(k, g.prompt_tokens, H, 0, H, md.w(pfx + ".ca.kn.weight", H), g.norm_eps);
    att = attention(q, rows, k, v, g.prompt_tokens, g.heads);
  }
  Vec o = linear(md, att, rows, H, pfx + ".ca.o", W);
  Vec h(hidden.size());
  for (size_t i = 0; i < h.size(); ++i) h[i] = bfr(hidden[i] + o[i]);  // ggml_add, :338
  Vec m = modulated_norm(h, rows, W, cscale, cshift, g.norm_eps, md.norm_kind == 1);
  Vec f;
  if (md.ffn_kind == 1) {
    // SiLU-gated FFN: silu(gate) * up, each a BF16 linear output, product in BF16
    f = linear_rows(md, m, rows, W, pfx + ".ffn.in", 0, F, 2 * F, 2);
    Vec u = linear_rows(md, m, rows, W, pfx + ".ffn.in", F, F, 2 * F, 0);
    for (size_t i = 0; i < f.size(); ++i) f[i] = bfr(f[i] * u[i]);
  } else {
    f = linear(md, m, rows, W, pfx + ".ffn.in", F, true);
  }
  Vec d = linear(md, f, rows, F, pfx + ".ffn.out", W);
  for (size_t i = 0; i < h.size(); ++i)  // gated_residual (mot.cpp:161-173)
    h[i] = bfr(std::fma(d[i], cgate[i % W], h[i]));
  return h;
}

// Gated residual of an attention output (mot.cpp:451; cache.cpp:301-302).
void gated_add(Vec& h, const Vec& branch, const float* gate, int W) {
  for (size_t i = 0; i < h.size(); ++i) h[i] = bfr(std::fma(branch[i], gate[i % W], h[i]));
}

// Euler schedule (scheduler.cpp:26-55).
void schedule(int steps, float shift, float* ts, float* sig) {
  const float training_sigma = 1.0f / 1000.0f;
  const float smin = shift * training_sigma / (1.0f + (shift - 1.0f) * training_sigma);
  const double tmin = static_cast<double>(smin) * 1000.0;
  for (int s = 0; s < steps; ++s) {
    const double u = steps == 1 ? 1000.0 : 1000.0 + (tmin - 1000.0) * s / (steps - 1);
    const double sigma = u / 1000.0;
    const double shifted = static_cast<double>(shift) * sigma / (1.0 + (static_cast<double>(shift) - 1.0) * sigma);
    sig[s] = static_cast<float>(shifted);
    ts[s] = sig[s] * 1000.0f;
  }
  sig[steps] = 0.0f;
}

struct PrefixOut {
  std::vector<Vec> k, v;    // per layer, token-major [P][H] (P = 1 + V), BF16 values
  std::vector<Vec> pk, pv;  // per layer prompt K/V [N_t][H]
};

// build_prefix_cache (cache.cpp:139-485) + update_projected_prompt_cache
// (cache.cpp:53-137): state token through the action expert, visual tokens
// through the visual expert, joint self-attention over the P prefix tokens.
PrefixOut prefix(const Model& md, const Vec& state_norm, const float* latent, const Vec& prompt) {
  const oracle_geometry& g = md.g;
  const int H = g.hidden, E = g.action_hidden, V = g.grid_h * g.grid_w, P = 1 + V;
  PrefixOut out;
  // Projected action prompt + per-layer prompt K/V (build_cross_kv, mot.cpp:101-128).
  Vec text_a = text_embed(md, "acond", prompt, E);
  for (int l = 0; l < g.layers; ++l) {
    const std::string p = "gwp.blk." + std::to_string(l) + ".a";
    Vec k = linear(md, text_a, g.prompt_tokens, E, p + ".ca.k", H);
    Vec v = linear(md, text_a, g.prompt_tokens, E, p + ".ca.vproj", H);
    rms_norm_rows(k, g.prompt_tokens, H, 0, H, md.w(p + ".ca.kn.weight", H), g.norm_eps);
    bfr_inplace(k);
    out.pk.push_back(std::move(k));
    out.pv.push_back(std::move(v));
  }
  // state encoder (cache.cpp:201-202)
  Vec hs = action_encoder(md, "state", state_norm, 1);
  // patch embedding conv2d k2 s2 (cache.cpp:203-218): BF16 im2col, F32 GEMM,
  // + F32 bias, cast to BF16.
  const int C = g.vae_z, gw = g.grid_w, lw = 2 * g.grid_w, lh = 2 * g.grid_h;
  Vec cols(static_cast<size_t>(V) * C * 4);
  for (int y = 0; y < g.grid_h; ++y)
    for (int x = 0; x < gw; ++x)
      for (int c = 0; c < C; ++c)
        for (int dy = 0; dy < 2; ++dy)
          for (int dx = 0; dx < 2; ++dx)
            cols[(static_cast<size_t>(y) * gw + x) * C * 4 + c * 4 + dy * 2 + dx] =
                bfr(latent[(static_cast<size_t>(c) * lh + 2 * y + dy) * lw + 2 * x + dx]);
  Vec hv(static_cast<size_t>(V) * H);
  gemm_acc(cols.data(), V, C * 4, md.w("gwp.patch.weight", static_cast<int64_t>(H) * C * 4), H,
           hv.data(), md.wf("gwp.patch.weight"));
  const uint16_t* pb = md.w("gwp.patch.bias", H);
  for (int t = 0; t < V; ++t)
    for (int n = 0; n < H; ++n) hv[static_cast<size_t>(t) * H + n] = bfr(hv[static_cast<size_t>(t) * H + n] + bf2f(pb[n]));
  // conditions at t = 0 (cache.cpp:227-240, 419-422)
  Condition ca = condition(md, "acond", 0.0f, E);
  Condition cv = condition(md, "cond", 0.0f, H);
  Vec text_v = text_embed(md, "cond", prompt, H);
  std::vector<int32_t> pt(V), ph(V), pw(V);
  oracle_visual_positions(g.grid_h, g.grid_w, pt.data(), ph.data(), pw.data());
  for (int l = 0; l < g.layers; ++l) {
    const std::string ap = "gwp.blk." + std::to_string(l) + ".a";
    const std::string vp = "gwp.blk." + std::to_string(l) + ".v";
    Vec am = combined_mod(md, ca.mod, ap + ".mod", E);
    Vec vm = combined_mod(md, cv.mod, vp + ".mod", H);
    ExpertQkv s = expert_qkv(md, ap, hs, 1, E, &am[0], &am[E], false, 0, nullptr, nullptr, nullptr);
    ExpertQkv v = expert_qkv(md, vp, hv, V, H, &vm[0], &vm[H], true, 0, pt.data(), ph.data(), pw.data());
    Vec q(static_cast<size_t>(P) * H), k(static_cast<size_t>(P) * H), vv(static_cast<size_t>(P) * H);
    std::memcpy(q.data(), s.q.data(), H * 4);
    std::memcpy(k.data(), s.k.data(), H * 4);
    std::memcpy(vv.data(), s.v.data(), H * 4);
    std::memcpy(q.data() + H, v.q.data(), static_cast<size_t>(V) * H * 4);
    std::memcpy(k.data() + H, v.k.data(), static_cast<size_t>(V) * H * 4);
    std::memcpy(vv.data() + H, v.v.data(), static_cast<size_t>(V) * H * 4);
    out.k.push_back(k);
    out.v.push_back(vv);
    if (l + 1 == g.layers) break;  // the last layer's outputs feed no cached K/V
    Vec att = attention(q, P, k, vv, P, g.heads);
    Vec att_s(att.begin(), att.begin() + H);
    Vec att_v(att.begin() + H, att.end());
    Vec os = linear(md, att_s, 1, H, ap + ".sa.o", E);
    Vec ov = linear(md, att_v, V, H, vp + ".sa.o", H);
    gated_add(hs, os, &am[2 * E], E);
    gated_add(hv, ov, &vm[2 * H], H);
    hs = cross_ffn(md, ap, hs, 1, E, g.action_ffn, &out.pk[l], &out.pv[l], nullptr, 0, &am[3 * E],
                   &am[4 * E], &am[5 * E]);
    hv = cross_ffn(md, vp, hv, V, H, g.ffn, nullptr, nullptr, &text_v, H, &vm[3 * H], &vm[4 * H],
                   &vm[5 * H]);
  }
  return out;
}

// One cached action-expert step (build_cached_action_body, mot.cpp:358-496):
// returns the BF16 velocity [T][A].
Vec action_step(const Model& md, const PrefixOut& pre, const Vec& action, float t) {
  const oracle_geometry& g = md.g;
  const int H = g.hidden, E = g.action_hidden, T = g.action_chunk, V = g.grid_h * g.grid_w;
  const int P = 1 + V, J = P + T;
  Vec h = action_encoder(md, "action", action, T);
  Condition c = condition(md, "acond", t, E);
  for (int l = 0; l < g.layers; ++l) {
    const std::string ap = "gwp.blk." + std::to_string(l) + ".a";
    Vec m = combined_mod(md, c.mod, ap + ".mod", E);
    ExpertQkv a = expert_qkv(md, ap, h, T, E, &m[0], &m[E], false, 1, nullptr, nullptr, nullptr);
    // joint K/V in the [state, action, visual] order (mot.cpp:402-431)
    Vec k(static_cast<size_t>(J) * H), v(static_cast<size_t>(J) * H);
    std::memcpy(k.data(), pre.k[l].data(), H * 4);
    std::memcpy(v.data(), pre.v[l].data(), H * 4);
    std::memcpy(k.data() + H, a.k.data(), static_cast<size_t>(T) * H * 4);
    std::memcpy(v.data() + H, a.v.data(), static_cast<size_t>(T) * H * 4);
    std::memcpy(k.data() + static_cast<size_t>(1 + T) * H, pre.k[l].data() + H, static_cast<size_t>(V) * H * 4);
    std::memcpy(v.data() + static_cast<size_t>(1 + T) * H, pre.v[l].data() + H, static_cast<size_t>(V) * H * 4);
    Vec att = attention(a.q, T, k, v, J, g.heads);
    Vec o = linear(md, att, T, H, ap + ".sa.o", E);
    gated_add(h, o, &m[2 * E], E);
    h = cross_ffn(md, ap, h, T, E, g.action_ffn, &pre.pk[l], &pre.pv[l], nullptr, 0, &m[3 * E],
                  &m[4 * E], &m[5 * E]);
  }
  // final AdaLN from action_scale_shift_table + temb (mot.cpp:468-488)
  const uint16_t* tb = md.w("gwp.action_mod", 2LL * E);
  Vec shift(E), scale(E);
  for (int i = 0; i < E; ++i) {
    shift[i] = bf2f(tb[i]) + c.temb[i];
    scale[i] = bf2f(tb[E + i]) + c.temb[i];
  }
  Vec n = modulated_norm(h, T, E, scale.data(), shift.data(), g.norm_eps);
  return action_decoder(md, n, T);
}

// One MoT layer (layer 0) of the reference's un-cached forward (run_mot_step,
// src/models/gwp05/engine/mot.cpp:870-1100, layer body :1008-1067): the action
// stream [state; actions] through the action expert with the state row at
// timestep 0 and the action rows at t (action_timesteps with the clean state,
// semantics.cpp:224-233), the visual tokens through the visual expert at
// t = 0, one joint self-attention in which state and visual queries see only
// state and visual keys and action queries see every key (the mask built at
// mot.cpp:1147-1158), then each expert's cross attention over its text hidden
// states (projected by the layer: build_attention, text_encoder.cpp:26-73, F32
// q/k) and its FFN. xv [V][H], xa [1 + T][E], tv [Nt][H], ta [Nt][E] (F32,
// rounded to BF16 as the hidden stream is); outputs likewise.
void block_forward(const Model& md, float t, const float* xv, const float* xa, const float* tv,
                   const float* ta, float* ov, float* oa) {
  const oracle_geometry& g = md.g;
  const int H = g.hidden, E = g.action_hidden, T = g.action_chunk, V = g.grid_h * g.grid_w;
  const int P = 1 + V, J = P + T, Nt = g.prompt_tokens;
  const std::string ap = "gwp.blk.0.a", vp = "gwp.blk.0.v";
  Vec hv(xv, xv + static_cast<size_t>(V) * H), hs(xa, xa + E);
  Vec ha(xa + E, xa + static_cast<size_t>(1 + T) * E);
  Vec text_v(tv, tv + static_cast<size_t>(Nt) * H), text_a(ta, ta + static_cast<size_t>(Nt) * E);
  for (Vec* v : {&hv, &hs, &ha, &text_v, &text_a}) bfr_inplace(*v);
  Condition c0a = condition(md, "acond", 0.0f, E);
  Condition cta = condition(md, "acond", t, E);
  Condition c0v = condition(md, "cond", 0.0f, H);
  Vec am0 = combined_mod(md, c0a.mod, ap + ".mod", E);
  Vec amt = combined_mod(md, cta.mod, ap + ".mod", E);
  Vec vm = combined_mod(md, c0v.mod, vp + ".mod", H);
  std::vector<int32_t> pt(V), ph(V), pw(V);
  oracle_visual_positions(g.grid_h, g.grid_w, pt.data(), ph.data(), pw.data());
  ExpertQkv s = expert_qkv(md, ap, hs, 1, E, &am0[0], &am0[E], false, 0, nullptr, nullptr, nullptr);
  ExpertQkv a = expert_qkv(md, ap, ha, T, E, &amt[0], &amt[E], false, 1, nullptr, nullptr, nullptr);
  ExpertQkv v = expert_qkv(md, vp, hv, V, H, &vm[0], &vm[H], true, 0, pt.data(), ph.data(), pw.data());
  auto cat = [&](std::initializer_list<const Vec*> parts, size_t rows) {
    Vec out;
    out.reserve(rows * H);
    for (const Vec* p : parts) out.insert(out.end(), p->begin(), p->end());
    return out;
  };
  Vec qp = cat({&s.q, &v.q}, P), kp = cat({&s.k, &v.k}, P), vv = cat({&s.v, &v.v}, P);
  Vec kj = cat({&s.k, &a.k, &v.k}, J), vj = cat({&s.v, &a.v, &v.v}, J);
  Vec att_p = attention(qp, P, kp, vv, P, g.heads);
  Vec att_a = attention(a.q, T, kj, vj, J, g.heads);
  Vec att_s(att_p.begin(), att_p.begin() + H), att_v(att_p.begin() + H, att_p.end());
  gated_add(hs, linear(md, att_s, 1, H, ap + ".sa.o", E), &am0[2 * E], E);
  gated_add(ha, linear(md, att_a, T, H, ap + ".sa.o", E), &amt[2 * E], E);
  gated_add(hv, linear(md, att_v, V, H, vp + ".sa.o", H), &vm[2 * H], H);
  hs = cross_ffn(md, ap, hs, 1, E, g.action_ffn, nullptr, nullptr, &text_a, E, &am0[3 * E],
                 &am0[4 * E], &am0[5 * E]);
  ha = cross_ffn(md, ap, ha, T, E, g.action_ffn, nullptr, nullptr, &text_a, E, &amt[3 * E],
                 &amt[4 * E], &amt[5 * E]);
  hv = cross_ffn(md, vp, hv, V, H, g.ffn, nullptr, nullptr, &text_v, H, &vm[3 * H], &vm[4 * H],
                 &vm[5 * H]);
  std::memcpy(ov, hv.data(), sizeof(float) * hv.size());
  std::memcpy(oa, hs.data(), sizeof(float) * E);
  std::memcpy(oa + E, ha.data(), sizeof(float) * ha.size());
}

}  // namespace

extern "C" {

void oracle_schedule(int steps, float shift, float* ts, float* sig) { schedule(steps, shift, ts, sig); }

void oracle_timestep_embedding(float t, int dim, float* out) {
  Vec e = timestep_embedding(t, dim);
  std::memcpy(out, e.data(), sizeof(float) * dim);
}

// visual_positions (semantics.cpp:235-257): t = 0, h = y, w = x, row-major.
void oracle_visual_positions(int gh, int gw, int32_t* t, int32_t* h, int32_t* w) {
  for (int y = 0; y < gh; ++y)
    for (int x = 0; x < gw; ++x) {
      t[y * gw + x] = 0;
      h[y * gw + x] = y;
      w[y * gw + x] = x;
    }
}

int oracle_threads(void) { return omp_get_max_threads(); }

void* oracle_create(const oracle_geometry* g, int n, const char** names, const uint16_t** data,
                    const int64_t* numel, const float* sq01, const float* sq99, const float* aq01,
                    const float* aq99, char* err, int errlen) {
  auto fail = [&](const std::string& m) -> void* {
    if (err && errlen > 0) std::snprintf(err, errlen, "%s", m.c_str());
    return nullptr;
  };
  if (!g || g->heads * 128 != g->hidden) return fail("hidden must equal heads * 128");
  if (g->action_chunk <= 0 || g->steps <= 0 || g->layers <= 0) return fail("bad counts");
  Model* md = new Model();
  md->g = *g;
  for (int i = 0; i < n; ++i) {
    Tensor t;
    t.numel = numel[i];
    t.data.assign(data[i], data[i] + numel[i]);
    md->t.emplace(names[i], std::move(t));
  }
  const int A = g->action_dim;
  md->sq01.assign(sq01, sq01 + A);
  md->sq99.assign(sq99, sq99 + A);
  md->aq01.assign(aq01, aq01 + A);
  md->aq99.assign(aq99, aq99 + A);
  return md;
}

// Builds a model over the deterministic synthetic weights (the generator of
// oracle/synth.py, restated here so full-width CPU baselines do not have to
// materialise weights in Python): same names, shapes and bits.
void* oracle_create_synthetic(const oracle_geometry* g, uint64_t seed, double bias_scale,
                              char* err, int errlen) {
  return oracle_create_synthetic_ex(g, seed, bias_scale, 0, err, errlen);
}

void* oracle_create_synthetic_ex(const oracle_geometry* g, uint64_t seed, double bias_scale,
                                 int ffn_kind, char* err, int errlen) {
  auto fail = [&](const std::string& m) -> void* {
    if (err && errlen > 0) std::snprintf(err, errlen, "%s", m.c_str());
    return nullptr;
  };
  if (!g || g->heads * 128 != g->hidden) return fail("hidden must equal heads * 128");
  Model* md = new Model();
  md->g = *g;
  md->ffn_kind = ffn_kind;
  const int64_t fin = ffn_kind == 1 ? 2 : 1;  // SiLU-gated: ffn.in holds gate and up rows
  const int64_t E = g->action_hidden, H = g->hidden, A = g->action_dim, D = g->text_dim;
  const int64_t emb = g->num_embodiments;
  std::vector<std::pair<std::string, int64_t>> s;
  s.push_back({"gwp.patch.weight", H * g->vae_z * 4});
  s.push_back({"gwp.patch.bias", H});
  for (const char* c : {"state", "action"}) {
    const std::string p = std::string("gwp.") + c;
    s.push_back({p + ".in.weight", emb * A * 128});
    s.push_back({p + ".in.bias", emb * 128});
    s.push_back({p + ".mid.weight", 128 * 128});
    s.push_back({p + ".mid.bias", 128});
    s.push_back({p + ".out.weight", E * 128});
    s.push_back({p + ".out.bias", E});
  }
  s.push_back({"gwp.decode.in.weight", 128 * E});
  s.push_back({"gwp.decode.in.bias", 128});
  s.push_back({"gwp.decode.mid.weight", 128 * 128});
  s.push_back({"gwp.decode.mid.bias", 128});
  s.push_back({"gwp.decode.out.weight", emb * 128 * A});
  s.push_back({"gwp.decode.out.bias", emb * A});
  s.push_back({"gwp.action_mod", 2 * E});
  for (int x = 0; x < 2; ++x) {
    const std::string p = x == 0 ? "gwp.acond" : "gwp.cond";
    const int64_t W = x == 0 ? E : H;
    for (auto& kv : std::vector<std::pair<std::string, int64_t>>{
             {".time.0.weight", W * 256}, {".time.0.bias", W}, {".time.1.weight", W * W},
             {".time.1.bias", W}, {".time.out.weight", 6 * W * W}, {".time.out.bias", 6 * W},
             {".text.0.weight", W * D}, {".text.0.bias", W}, {".text.1.weight", W * W},
             {".text.1.bias", W}})
      s.push_back({p + kv.first, kv.second});
  }
  for (int l = 0; l < g->layers; ++l)
    for (int x = 0; x < 2; ++x) {
      const int64_t W = x == 0 ? E : H, F = x == 0 ? g->action_ffn : g->ffn;
      const std::string p = "gwp.blk." + std::to_string(l) + (x == 0 ? ".a" : ".v");
      for (auto& kv : std::vector<std::pair<std::string, int64_t>>{
               {".sa.qkv.weight", 3 * H * W}, {".sa.qkv.bias", 3 * H}, {".sa.qn.weight", H},
               {".sa.kn.weight", H}, {".sa.o.weight", W * H}, {".sa.o.bias", W},
               {".ca.q.weight", H * W}, {".ca.q.bias", H}, {".ca.k.weight", H * W},
               {".ca.k.bias", H}, {".ca.vproj.weight", H * W}, {".ca.vproj.bias", H},
               {".ca.o.weight", W * H}, {".ca.o.bias", W}, {".ca.qn.weight", H},
               {".ca.kn.weight", H}, {".ca_norm.weight", W}, {".ca_norm.bias", W},
               {".ffn.in.weight", fin * F * W}, {".ffn.in.bias", fin * F}, {".ffn.out.weight", W * F},
               {".ffn.out.bias", W}, {".mod", 6 * W}})
        s.push_back({p + kv.first, kv.second});
    }
  const double ih4 = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  auto ends = [](const std::string& a, const char* b) {
    const size_t n = std::strlen(b);
    return a.size() >= n && a.compare(a.size() - n, n, b) == 0;
  };
  auto fnv = [](const std::string& x) {
    uint64_t h = 0xCBF29CE484222325ull;
    for (unsigned char c : x) {
      h ^= c;
      h *= 0x100000001B3ull;
    }
    return h;
  };
  auto mix = [](uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  };
  for (const auto& kv : s) {
    double scale = 0.02, center = 0.0;
    if (ends(kv.first, ".bias")) scale = bias_scale;
    else if (ends(kv.first, ".qn.weight") || ends(kv.first, ".kn.weight") || ends(kv.first, ".ca_norm.weight")) center = 1.0;
    const uint64_t ts = mix((seed ^ fnv(kv.first)) + 0x9E3779B97F4A7C15ull);
    const float k = static_cast<float>(scale / ih4), c = static_cast<float>(center);
    Tensor t;
    t.numel = kv.second;
    t.data.resize(kv.second);
    uint16_t* d = t.data.data();
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < kv.second; ++i) {
      const uint64_t h = mix(ts + static_cast<uint64_t>(i + 1) * 0x9E3779B97F4A7C15ull);
      const int z = static_cast<int>((h & 0xFFFFull) + ((h >> 16) & 0xFFFFull) + ((h >> 32) & 0xFFFFull) + (h >> 48)) - 131070;
      volatile float prod = static_cast<float>(z) * k;  // two separately rounded F32 ops
      const float v = prod + c;
      uint32_t u;
      std::memcpy(&u, &v, 4);
      u += 0x7fffu + ((u >> 16) & 1u);
      d[i] = static_cast<uint16_t>(u >> 16);
    }
    md->t.emplace(kv.first, std::move(t));
  }
  for (int i = 0; i < A; ++i) {
    md->sq01.push_back(-1.0f - 0.01f * static_cast<float>(i));
    md->sq99.push_back(1.0f + 0.02f * static_cast<float>(i));
  }
  md->aq01 = md->sq01;
  md->aq99 = md->sq99;
  return md;
}

// GGML Q8_0 round trip of 32-value blocks, restating the gguf-py codec
// (gguf.quants Q8_0, gguf 0.19.0; the wam.cpp reference has no Q8_0): d =
// max|x| / 127 in F32, q = x * (1/d) rounded half away from zero, d stored as
// fp16; dequantised value = fp16(d) * q in F32 (dequantize_row_q8_0).
void oracle_q8_roundtrip(const uint16_t* bf16, int64_t n, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n / 32; ++b) {
    float x[32], amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      x[j] = bf2f(bf16[b * 32 + j]);
      amax = std::max(amax, std::fabs(x[j]));
    }
    const float d = amax / 127.0f;
    const float id = d == 0.0f ? 0.0f : 1.0f / d;
    const float d16 = f16_round(d);
    for (int j = 0; j < 32; ++j) {
      const float v = x[j] * id;
      const float a = std::fabs(v);
      const float fl = std::floor(a);
      // stored as int8, so a negative value that rounds to 0 is +0
      const int q = static_cast<int>(std::copysign(fl + std::floor(2.0f * (a - fl)), v));
      out[b * 32 + j] = d16 * static_cast<float>(q);
    }
  }
}

// Config-5 policy: every linear weight whose rows are whole 32-value blocks
// (linear_inner) is replaced by its exact F32 Q8_0 dequantisation.
int oracle_quantize_q8(void* model) {
  Model& md = *static_cast<Model*>(model);
  for (auto& kv : md.t) {
    const int64_t inner = linear_inner(kv.first, md.g);
    if (inner <= 0 || inner % 32 != 0 || kv.second.numel % 32 != 0) continue;
    kv.second.f32.resize(kv.second.numel);
    oracle_q8_roundtrip(kv.second.data.data(), kv.second.numel, kv.second.f32.data());
  }
  return 0;
}

int oracle_block(void* model, int norm_kind, float t, const float* xv, const float* xa,
                 const float* tv, const float* ta, float* ov, float* oa) {
  Model& md = *static_cast<Model*>(model);
  md.norm_kind = norm_kind;
  block_forward(md, t, xv, xa, tv, ta, ov, oa);
  md.norm_kind = 0;
  return 0;
}

void oracle_set_uncached(void* model, int uncached) {
  static_cast<Model*>(model)->uncached = uncached != 0;
}

void oracle_destroy(void* m) { delete static_cast<Model*>(m); }

int oracle_predict(void* model, const float* state, const float* latent, const float* prompt,
                   const float* noise, float* action_out, float* prefix_k, float* prefix_v,
                   float* prompt_k, float* prompt_v, float* velocity, float* actions) {
  const Model& md = *static_cast<Model*>(model);
  const oracle_geometry& g = md.g;
  const int A = g.action_dim, T = g.action_chunk, H = g.hidden;
  const int V = g.grid_h * g.grid_w, P = 1 + V;
  // state normalisation (engine.cpp:249-253)
  Vec sn(A, 0.0f);
  for (int i = 0; i < g.real_state_dim; ++i) {
    const float range = std::max(md.sq99[i] - md.sq01[i], 1e-8f);
    sn[i] = ((state[i] - md.sq01[i]) / range) * 2.0f - 1.0f;
  }
  Vec pr(prompt, prompt + static_cast<size_t>(g.prompt_tokens) * g.text_dim);
  PrefixOut pre = prefix(md, sn, latent, pr);
  auto dump_heads = [&](const Vec& src, int rows, float* dst) {
    for (int hd = 0; hd < g.heads; ++hd)
      for (int r = 0; r < rows; ++r)
        std::memcpy(dst + (static_cast<size_t>(hd) * rows + r) * 128,
                    src.data() + static_cast<size_t>(r) * H + hd * 128, 128 * 4);
  };
  for (int l = 0; l < g.layers; ++l) {
    const size_t lp = static_cast<size_t>(l) * g.heads * P * 128;
    const size_t lt = static_cast<size_t>(l) * g.heads * g.prompt_tokens * 128;
    if (prefix_k) dump_heads(pre.k[l], P, prefix_k + lp);
    if (prefix_v) dump_heads(pre.v[l], P, prefix_v + lp);
    if (prompt_k) dump_heads(pre.pk[l], g.prompt_tokens, prompt_k + lt);
    if (prompt_v) dump_heads(pre.pv[l], g.prompt_tokens, prompt_v + lt);
  }
  std::vector<float> ts(g.steps), sig(g.steps + 1);
  schedule(g.steps, g.flow_shift, ts.data(), sig.data());
  // action state is BF16 on the device (set_f32_tensor, weights.cpp:858-869)
  Vec a(noise, noise + static_cast<size_t>(T) * A);
  bfr_inplace(a);
  for (int s = 0; s < g.steps; ++s) {
    // The reference's CPU mode runs the whole MoT every step (engine.cpp:334-337,
    // run_mot_step): the prefix half is recomputed from the same inputs.
    if (md.uncached && s > 0) pre = prefix(md, sn, latent, pr);
    Vec vel = action_step(md, pre, a, ts[s]);
    const float dt = sig[s + 1] - sig[s];
    for (size_t i = 0; i < a.size(); ++i) {
      const float prod = vel[i] * dt;  // ggml_mul then ggml_add (weights.cpp:897-901)
      a[i] = bfr(a[i] + prod);
    }
    if (velocity) std::memcpy(velocity + static_cast<size_t>(s) * T * A, vel.data(), sizeof(float) * T * A);
    if (actions) std::memcpy(actions + static_cast<size_t>(s) * T * A, a.data(), sizeof(float) * T * A);
  }
  // de-normalisation + delta action (engine.cpp:436-445)
  for (int t = 0; t < T; ++t)
    for (int d = 0; d < g.real_action_dim; ++d) {
      const float range = std::max(md.aq99[d] - md.aq01[d], 1e-8f);
      float v = ((a[static_cast<size_t>(t) * A + d] + 1.0f) * 0.5f) * range + md.aq01[d];
      if ((d >= 0 && d < 6) || (d >= 7 && d < 13)) v += state[d];
      action_out[static_cast<size_t>(t) * g.real_action_dim + d] = v;
    }
  return 0;
}

}  // extern "C"
