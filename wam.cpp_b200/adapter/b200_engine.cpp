// B200Engine: the reference's Engine interface over the wam_b200 C ABI
// (see b200_engine.h). Plus a small C harness (wam_b200_adapter_*) through
// which tests drive an Engine* polymorphically: every predict/reset there is a
// virtual call on the reference's Engine type.
#include "b200_engine.h"

#include <cstddef>

#include <cmath>
#include <cstdio>
#include <cstring>

namespace wam::internal::gwp05::engine {

namespace {

void log_status(const char* what, wam_b200_status* st) {
  std::fprintf(stderr, "wam(b200): %s failed: %s\n", what, st->message ? st->message : "");
  wam_b200_status_free(st);
}

}  // namespace

B200Engine::B200Engine(wam_b200_engine* handle, bool text_encoder) : h_(handle) {
  wam_b200_geometry_of(h_, &g_);
  // Config (engine.h:40-80) as the reference's loader fills it for this geometry.
  cfg.n_img = static_cast<std::int64_t>(g_.grid_h) * g_.grid_w;
  cfg.n_lang = g_.prompt_tokens;
  cfg.n_state = 1;
  cfg.n_prefix = cfg.n_state + cfg.n_img;
  cfg.n_suffix = g_.action_chunk;
  cfg.n_full = cfg.n_prefix + cfg.n_suffix;
  cfg.hidden = g_.hidden;
  cfg.expert_h = g_.action_hidden;
  cfg.intermediate = g_.ffn;
  cfg.expert_inter = g_.action_ffn;
  cfg.n_q_heads = g_.heads;
  cfg.n_kv_heads = g_.heads;
  cfg.head_dim = 128;
  cfg.q_full_dim = static_cast<std::int64_t>(g_.heads) * 128;
  cfg.kv_full_dim = cfg.q_full_dim;
  cfg.n_layers = g_.layers;
  cfg.max_state_dim = g_.action_dim;
  cfg.max_action_dim = g_.action_dim;
  cfg.real_state_dim = g_.real_state_dim;
  cfg.real_action_dim = g_.real_action_dim;
  cfg.norm_eps = g_.norm_eps;
  cfg.num_steps = g_.steps;
  cfg.action_chunk = g_.action_chunk;
  cfg.rms_eps = g_.norm_eps;
  cfg.rope_n_dims = 128;
  cfg.rope_freq_base = 10000.0f;
  cfg.image_height = static_cast<std::int64_t>(g_.grid_h) * 32;  // latent = image / 16, tokens = latent / 2
  cfg.image_width = static_cast<std::int64_t>(g_.grid_w) * 32;
  cfg.t5_hidden = g_.text_dim;
  cfg.vae_z_dim = g_.vae_z;
  cfg.num_embodiments = g_.num_embodiments;
  cfg.embodiment_id = g_.embodiment_id;
  cfg.flow_shift = g_.flow_shift;
  language_encoder_policy =
      text_encoder ? LanguageEncoderPolicy::resident : LanguageEncoderPolicy::external_embedding;
  text_encoder_resident = text_encoder;  // resident_device_bytes: reported by every predict
}

B200Engine::~B200Engine() {
  if (h_) wam_b200_destroy(h_);
}

std::vector<float> B200Engine::predict(const EngineInputsView& in) {
  stats = {};
  if (!in.state) {
    std::fprintf(stderr, "wam(b200): state is required\n");
    return {};
  }
  // Raw camera views go through the engine's vision front-end (compose + VAE
  // on the device), the reference's run_vae path (engine.cpp:260-270).
  wam_b200_image views[3] = {};
  const bool from_images = !in.precomputed_ref_latent;
  if (from_images) {
    if (!in.images || in.n_images != 3) {
      std::fprintf(stderr, "wam(b200): exactly three input images are required\n");
      return {};
    }
    for (int i = 0; i < 3; ++i)
      views[i] = wam_b200_image{in.images[i].data, in.images[i].w, in.images[i].h,
                                in.images[i].format == PixelFormat::U8 ? WAM_B200_PIXEL_U8
                                                                       : WAM_B200_PIXEL_F32_RGB_01};
  }
  // Without a precomputed prompt embedding the token ids go to the engine's
  // resident UMT5 encoder (run_t5, text_encoder.cpp:112-204).
  if (!in.precomputed_prompt_emb && !in.lang_tokens) {
    std::fprintf(stderr, "wam(b200): a precomputed prompt embedding or prompt token ids are "
                         "required\n");
    return {};
  }
  wam_b200_request r{};
  r.state = in.state;
  r.state_n = g_.real_state_dim;
  r.noise = in.noise;
  r.ref_latent = in.precomputed_ref_latent;
  r.ref_latent_n = in.precomputed_ref_latent_n;
  r.prompt_emb = in.precomputed_prompt_emb;
  r.prompt_tokens = in.precomputed_prompt_tokens;
  if (from_images) {
    r.images = views;
    r.n_images = 3;
  }
  if (!in.precomputed_prompt_emb) {
    r.lang_tokens = in.lang_tokens;
    r.n_lang = in.n_lang;
    r.attention_mask = in.attention_mask;
    r.attention_mask_n = in.attention_mask_n;
  }
  std::vector<float> out(static_cast<size_t>(g_.action_chunk) * g_.real_action_dim);
  wam_b200_stats s{};
  wam_b200_status st{};
  if (wam_b200_predict(h_, &r, out.data(), out.size(), &s, &st) != WAM_B200_OK) {
    log_status("predict", &st);
    return {};
  }
  wam_b200_status_free(&st);
  float prompt_ms = 0.0f, prefix_ms = 0.0f, denoise_ms = 0.0f;
  wam_b200_phase_ms(h_, &prompt_ms, &prefix_ms, &denoise_ms);
  stats.ms_total = s.ms_total;
  stats.ms_inference = s.ms_device;
  stats.ms_prompt_projection = prompt_ms;
  stats.ms_prefix_cache = prefix_ms;
  stats.ms_prefill = prompt_ms + prefix_ms;
  stats.ms_denoise = denoise_ms;
  stats.ms_denoise_steps.assign(static_cast<size_t>(g_.steps), denoise_ms / g_.steps);
  stats.projected_prompt_cache_hit = s.prompt_cache_hit != 0;
  resident_device_bytes = s.resident_device_bytes;
  peak_component_device_bytes = s.resident_device_bytes;
  return out;
}

void B200Engine::reset() { wam_b200_reset(h_); }

std::unique_ptr<Engine> create_b200_synthetic(const wam_b200_options& options) {
  wam_b200_engine* h = nullptr;
  wam_b200_status st{};
  if (wam_b200_create(&options, &h, &st) != WAM_B200_OK) {
    log_status("create", &st);
    return nullptr;
  }
  wam_b200_status_free(&st);
  return std::make_unique<B200Engine>(
      h, options.struct_size >= offsetof(wam_b200_options, t5) + sizeof(int) && options.t5 != 0);
}

std::unique_ptr<Engine> create_b200(const ArtifactContract& artifact, const EngineOptions& options,
                                    const std::string& artifact_path) {
  wam_b200_options o{};
  o.struct_size = sizeof(o);
  o.artifact_path = artifact_path.c_str();
  o.device_index = options.device_index;
  o.max_batch = 1;
  o.use_cuda_graphs = 1;
  o.prompt_cache = options.prompt_cache_capacity > 0 ? 1 : 0;
  o.vae = 1;  // the artifact contract carries the VAE (artifact.cpp:159), so images work
  o.t5 = 1;   // ... and UMT5 (resident language-encoder policy: token ids work)
  auto e = create_b200_synthetic(o);
  if (!e) return nullptr;
  const Geometry& a = artifact.geometry;
  const Config& c = e->cfg;
  if ((a.hidden && a.hidden != c.hidden) || (a.layers && a.layers != c.n_layers) ||
      (a.heads && a.heads != c.n_q_heads) || (a.action_hidden && a.action_hidden != c.expert_h) ||
      (a.action_chunk && a.action_chunk != c.action_chunk)) {
    std::fprintf(stderr, "wam(b200): artifact %s does not match the contract's geometry\n",
                 artifact_path.c_str());
    return nullptr;
  }
  return e;
}

}  // namespace wam::internal::gwp05::engine

using wam::internal::gwp05::engine::Engine;

// ------------------------------------------------------------ test harness
// Opaque Engine* handles for ctypes: every call below goes through the
// reference's Engine vtable.
extern "C" {

__attribute__((visibility("default"))) void* wam_b200_adapter_create(const wam_b200_options* o) {
  if (!o) return nullptr;
  return wam::internal::gwp05::engine::create_b200_synthetic(*o).release();
}

__attribute__((visibility("default"))) void wam_b200_adapter_destroy(void* e) {
  delete static_cast<Engine*>(e);
}

// Engine::predict through the base class. Returns the number of values
// written to out (action_chunk * real_action_dim), 0 if predict returned {}
// (the reference's failure convention), or -1 if out is too small.
__attribute__((visibility("default"))) long long wam_b200_adapter_predict(
    void* e, const float* state, const float* latent, int latent_n, const float* prompt,
    int prompt_tokens, const float* noise, float* out, long long out_n) {
  wam::internal::gwp05::engine::EngineInputsView in{};
  in.state = state;
  in.precomputed_ref_latent = latent;
  in.precomputed_ref_latent_n = latent_n;
  in.precomputed_prompt_emb = prompt;
  in.precomputed_prompt_tokens = prompt_tokens;
  in.noise = noise;
  std::vector<float> r = static_cast<Engine*>(e)->predict(in);
  if (static_cast<long long>(r.size()) > out_n) return -1;
  std::memcpy(out, r.data(), r.size() * sizeof(float));
  return static_cast<long long>(r.size());
}

// Engine::predict from three camera views (uint8 RGB, w x h each) instead of a
// latent: the vision front-end path.
__attribute__((visibility("default"))) long long wam_b200_adapter_predict_images(
    void* e, const float* state, const unsigned char* const* views, const int* w, const int* h,
    const float* prompt, int prompt_tokens, const float* noise, float* out, long long out_n) {
  wam::internal::gwp05::engine::ImageView im[3];
  for (int i = 0; i < 3; ++i) {
    im[i].data = views[i];
    im[i].w = w[i];
    im[i].h = h[i];
    im[i].format = wam::internal::gwp05::engine::PixelFormat::U8;
  }
  wam::internal::gwp05::engine::EngineInputsView in{};
  in.state = state;
  in.images = im;
  in.n_images = 3;
  in.precomputed_prompt_emb = prompt;
  in.precomputed_prompt_tokens = prompt_tokens;
  in.noise = noise;
  std::vector<float> r = static_cast<Engine*>(e)->predict(in);
  if (static_cast<long long>(r.size()) > out_n) return -1;
  std::memcpy(out, r.data(), r.size() * sizeof(float));
  return static_cast<long long>(r.size());
}

// Engine::predict with prompt token ids (and an optional mask) instead of a
// prompt embedding: the resident UMT5 path.
__attribute__((visibility("default"))) long long wam_b200_adapter_predict_tokens(
    void* e, const float* state, const float* latent, int latent_n, const int32_t* tokens,
    int n_lang, const int32_t* mask, int mask_n, const float* noise, float* out, long long out_n) {
  wam::internal::gwp05::engine::EngineInputsView in{};
  in.state = state;
  in.precomputed_ref_latent = latent;
  in.precomputed_ref_latent_n = latent_n;
  in.lang_tokens = tokens;
  in.n_lang = n_lang;
  in.attention_mask = mask;
  in.attention_mask_n = mask_n;
  in.noise = noise;
  std::vector<float> r = static_cast<Engine*>(e)->predict(in);
  if (static_cast<long long>(r.size()) > out_n) return -1;
  std::memcpy(out, r.data(), r.size() * sizeof(float));
  return static_cast<long long>(r.size());
}

__attribute__((visibility("default"))) void wam_b200_adapter_reset(void* e) {
  static_cast<Engine*>(e)->reset();
}

// Engine::cfg fields by name ("real_state_dim", "n_full", ...); -1 if unknown.
__attribute__((visibility("default"))) long long wam_b200_adapter_cfg(void* e, const char* name) {
  const auto& c = static_cast<Engine*>(e)->cfg;
  const struct {
    const char* n;
    long long v;
  } f[] = {{"n_img", c.n_img}, {"n_lang", c.n_lang}, {"n_state", c.n_state},
           {"n_prefix", c.n_prefix}, {"n_suffix", c.n_suffix}, {"n_full", c.n_full},
           {"hidden", c.hidden}, {"expert_h", c.expert_h}, {"intermediate", c.intermediate},
           {"expert_inter", c.expert_inter}, {"n_q_heads", c.n_q_heads}, {"head_dim", c.head_dim},
           {"n_layers", c.n_layers}, {"max_state_dim", c.max_state_dim},
           {"max_action_dim", c.max_action_dim}, {"real_state_dim", c.real_state_dim},
           {"real_action_dim", c.real_action_dim}, {"num_steps", c.num_steps},
           {"action_chunk", c.action_chunk}, {"vae_z_dim", c.vae_z_dim},
           {"t5_hidden", c.t5_hidden}, {"image_height", c.image_height},
           {"image_width", c.image_width}};
  for (const auto& x : f)
    if (std::strcmp(x.n, name) == 0) return x.v;
  return -1;
}

// Engine::stats after the last predict: ms_total, ms_inference, ms_denoise.
__attribute__((visibility("default"))) void wam_b200_adapter_stats(void* e, float* out3) {
  const auto& s = static_cast<Engine*>(e)->stats;
  out3[0] = s.ms_total;
  out3[1] = s.ms_inference;
  out3[2] = s.ms_denoise;
}

}  // extern "C"
