// Engine-level C ABI (include/wam_b200.h): wraps MotEngine with the reference
// C ABI's conventions (int return codes, malloc'd status messages,
// src/serving/c_api.cpp:18-55) and translates its structs.
#include <cstdlib>
#include <cstddef>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "c_api_util.h"
#include "engine.h"
#include "wam_b200.h"

struct wam_b200_engine {
  std::unique_ptr<wamb::MotEngine> impl;
};

namespace {

int fail(wam_b200_status* st, int code, const std::string& msg) {
  wamb::set_last_error(msg);
  if (st) {
    st->code = code;
    st->message = static_cast<char*>(std::malloc(msg.size() + 1));
    if (st->message) std::memcpy(st->message, msg.c_str(), msg.size() + 1);
  }
  return code;
}

int ok(wam_b200_status* st) {
  if (st) {
    st->code = WAM_B200_OK;
    st->message = nullptr;
  }
  return WAM_B200_OK;
}

wamb::Geometry to_geometry(const wam_b200_geometry& g) {
  wamb::Geometry o;
  o.hidden = g.hidden;
  o.layers = g.layers;
  o.heads = g.heads;
  o.ffn = g.ffn;
  o.action_hidden = g.action_hidden;
  o.action_ffn = g.action_ffn;
  o.action_dim = g.action_dim;
  o.real_state_dim = g.real_state_dim;
  o.real_action_dim = g.real_action_dim;
  o.num_embodiments = g.num_embodiments;
  o.embodiment_id = g.embodiment_id;
  o.grid_h = g.grid_h;
  o.grid_w = g.grid_w;
  o.vae_z = g.vae_z;
  o.action_chunk = g.action_chunk;
  o.steps = g.steps;
  o.prompt_tokens = g.prompt_tokens;
  o.text_dim = g.text_dim;
  o.norm_eps = g.norm_eps;
  o.flow_shift = g.flow_shift;
  return o;
}

std::vector<wamb::RequestView> views(const wam_b200_request* r, int n) {
  std::vector<wamb::RequestView> v(n > 0 ? n : 0);
  for (int i = 0; i < n; ++i) {
    v[i].state = r[i].state;
    v[i].state_n = r[i].state_n;
    v[i].noise = r[i].noise;
    v[i].latent = r[i].ref_latent;
    v[i].latent_n = r[i].ref_latent_n;
    v[i].prompt = r[i].prompt_emb;
    v[i].prompt_tokens = r[i].prompt_tokens;
    v[i].n_images = r[i].images ? r[i].n_images : 0;
    v[i].tokens = r[i].lang_tokens;
    v[i].n_tokens = r[i].n_lang;
    v[i].mask = r[i].attention_mask;
    v[i].mask_n = r[i].attention_mask_n;
    for (int j = 0; j < 3 && j < v[i].n_images; ++j)
      v[i].images[j] = wamb::PreprocessView{r[i].images[j].data, r[i].images[j].w,
                                            r[i].images[j].h, r[i].images[j].format};
  }
  return v;
}

int code_of(const std::string& err) {
  if (err.find("timed out") != std::string::npos) return WAM_B200_DEVICE_TIMEOUT;
  if (err.find("cuda") != std::string::npos || err.find("graph") != std::string::npos)
    return WAM_B200_CUDA_ERROR;
  return WAM_B200_INFERENCE_FAILED;
}

}  // namespace

extern "C" {

WAM_B200_API void wam_b200_status_free(wam_b200_status* st) {
  if (st && st->message) {
    std::free(st->message);
    st->message = nullptr;
  }
}

WAM_B200_API int wam_b200_create(const wam_b200_options* o, wam_b200_engine** out,
                                 wam_b200_status* st) {
  if (!o || !out) return fail(st, WAM_B200_INVALID_ARGUMENT, "options and engine pointer are required");
  // struct_size versioning: the first layout ends at weight_format.
  if (o->struct_size < offsetof(wam_b200_options, weight_format))
    return fail(st, WAM_B200_INVALID_ARGUMENT, "wam_b200_options.struct_size is too small");
  const bool has_format = o->struct_size >= offsetof(wam_b200_options, weight_format) + sizeof(int);
  *out = nullptr;
  wamb::EngineOptions eo;
  if (o->artifact_path) eo.artifact_path = o->artifact_path;
  eo.synthetic = to_geometry(o->synthetic_geometry);
  eo.seed = o->synthetic_seed;
  eo.bias_scale = o->synthetic_bias_scale;
  eo.device = o->device_index;
  eo.max_batch = o->max_batch;
  eo.graphs = o->use_cuda_graphs != 0;
  eo.prompt_cache = o->prompt_cache != 0;
  eo.weight_format = has_format ? o->weight_format : 0;
  if (eo.weight_format != 0 && eo.weight_format != 1)
    return fail(st, WAM_B200_INVALID_ARGUMENT, "weight_format must be 0 (BF16) or 1 (Q8_0)");
  if (o->struct_size >= offsetof(wam_b200_options, block_mode) + sizeof(int)) {
    eo.synthetic.ffn_kind = o->ffn_kind;
    eo.synthetic.norm_kind = o->norm_kind;
    eo.block = o->block_mode != 0;
    if ((o->ffn_kind || o->norm_kind || eo.block) && o->artifact_path)
      return fail(st, WAM_B200_INVALID_ARGUMENT,
                  "ffn_kind / norm_kind / block_mode apply to synthetic weights only");
  }
  if (o->struct_size >= offsetof(wam_b200_options, vae) + sizeof(int)) eo.vae = o->vae != 0;
  if (o->struct_size >= offsetof(wam_b200_options, t5_layers) + sizeof(int)) {
    eo.t5 = o->t5 != 0;
    if (o->t5_vocab > 0) eo.t5_vocab = o->t5_vocab;
    if (o->t5_ffn > 0) eo.t5_ffn = o->t5_ffn;
    if (o->t5_layers > 0) eo.t5_layers = o->t5_layers;
  }
  std::string err;
  auto e = wamb::MotEngine::create(eo, &err);
  if (!e) {
    const int code = err.find("artifact") != std::string::npos || err.find("GGUF") != std::string::npos
                         ? WAM_B200_ARTIFACT_ERROR
                         : (err.find("sm_100") != std::string::npos ? WAM_B200_UNSUPPORTED
                                                                    : WAM_B200_INVALID_ARGUMENT);
    return fail(st, code, err);
  }
  *out = new wam_b200_engine{std::move(e)};
  return ok(st);
}

WAM_B200_API void wam_b200_destroy(wam_b200_engine* e) { delete e; }

WAM_B200_API int wam_b200_reset(wam_b200_engine* e) {
  if (!e) return WAM_B200_INVALID_ARGUMENT;
  e->impl->reset();
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_geometry_of(const wam_b200_engine* e, wam_b200_geometry* out) {
  if (!e || !out) return WAM_B200_INVALID_ARGUMENT;
  const wamb::Geometry& g = e->impl->geometry();
  *out = wam_b200_geometry{g.hidden, g.layers, g.heads, g.ffn, g.action_hidden, g.action_ffn,
                           g.action_dim, g.real_state_dim, g.real_action_dim, g.num_embodiments,
                           g.embodiment_id, g.grid_h, g.grid_w, g.vae_z, g.action_chunk, g.steps,
                           g.prompt_tokens, g.text_dim, g.norm_eps, g.flow_shift};
  return WAM_B200_OK;
}

WAM_B200_API int wam_b200_predict_batch(wam_b200_engine* e, const wam_b200_request* r, int batch,
                                        float* out, size_t n, wam_b200_stats* stats,
                                        wam_b200_status* st) {
  if (!e || !r || !out) return fail(st, WAM_B200_INVALID_ARGUMENT, "engine, requests and output are required");
  const wamb::Geometry& g = e->impl->geometry();
  if (n < static_cast<size_t>(batch) * g.action_chunk * g.real_action_dim)
    return fail(st, WAM_B200_INVALID_ARGUMENT, "action output buffer is too small");
  cudaSetDevice(e->impl->device());  // callers may be on another thread (the batcher's)
  auto v = views(r, batch);
  wamb::EngineStats es;
  std::string err;
  if (!e->impl->predict(v.data(), batch, out, &es, &err)) return fail(st, code_of(err), err);
  if (stats) {
    stats->ms_total = es.ms_total;
    stats->ms_device = es.ms_prompt + es.ms_prefix + es.ms_denoise;
    stats->prompt_cache_hit = es.prompt_cache_hit;
    stats->kernel_launches = e->impl->kernels_per_chunk(batch, !es.prompt_cache_hit);
    stats->resident_device_bytes = e->impl->resident_bytes();
  }
  return ok(st);
}

WAM_B200_API int wam_b200_max_batch(const wam_b200_engine* e) {
  return e ? e->impl->max_batch() : 0;
}

WAM_B200_API int wam_b200_predict(wam_b200_engine* e, const wam_b200_request* r, float* out,
                                  size_t n, wam_b200_stats* stats, wam_b200_status* st) {
  return wam_b200_predict_batch(e, r, 1, out, n, stats, st);
}

WAM_B200_API int wam_b200_stage(wam_b200_engine* e, const wam_b200_request* r, int batch,
                                wam_b200_status* st) {
  if (!e || !r) return fail(st, WAM_B200_INVALID_ARGUMENT, "engine and requests are required");
  cudaSetDevice(e->impl->device());
  auto v = views(r, batch);
  std::string err;
  if (!e->impl->stage(v.data(), batch, &err)) return fail(st, WAM_B200_INVALID_ARGUMENT, err);
  return ok(st);
}

WAM_B200_API int wam_b200_run(wam_b200_engine* e, int batch, wam_b200_status* st) {
  if (!e) return fail(st, WAM_B200_INVALID_ARGUMENT, "engine is required");
  cudaSetDevice(e->impl->device());
  std::string err;
  if (!e->impl->run(batch, &err)) return fail(st, code_of(err), err);
  return ok(st);
}

WAM_B200_API int wam_b200_fetch(wam_b200_engine* e, const wam_b200_request* r, int batch,
                                float* out, size_t n, wam_b200_status* st) {
  if (!e || !r || !out) return fail(st, WAM_B200_INVALID_ARGUMENT, "engine, requests and output are required");
  const wamb::Geometry& g = e->impl->geometry();
  if (n < static_cast<size_t>(batch) * g.action_chunk * g.real_action_dim)
    return fail(st, WAM_B200_INVALID_ARGUMENT, "action output buffer is too small");
  auto v = views(r, batch);
  std::string err;
  if (!e->impl->fetch(v.data(), batch, out, &err)) return fail(st, code_of(err), err);
  return ok(st);
}

WAM_B200_API void* wam_b200_stream(wam_b200_engine* e) {
  return e ? static_cast<void*>(e->impl->stream()) : nullptr;
}

WAM_B200_API int wam_b200_kernel_launches(wam_b200_engine* e, int batch, int with_prompt) {
  return e ? e->impl->kernels_per_chunk(batch, with_prompt != 0) : -1;
}

WAM_B200_API int wam_b200_phase_ms(wam_b200_engine* e, float* prompt, float* prefix,
                                   float* denoise) {
  if (!e || !prompt || !prefix || !denoise) return WAM_B200_INVALID_ARGUMENT;
  return e->impl->last_phase_ms(prompt, prefix, denoise) ? WAM_B200_OK : WAM_B200_CUDA_ERROR;
}

WAM_B200_API int wam_b200_profile(wam_b200_engine* e, int batch, wam_b200_op_profile* out,
                                  int max_ops, wam_b200_status* st) {
  if (!e || !out) return -fail(st, WAM_B200_INVALID_ARGUMENT, "engine and output are required");
  std::vector<wamb::OpProfile> prof;
  std::string err;
  if (!e->impl->profile(batch, &prof, &err)) return -fail(st, code_of(err), err);
  const int n = static_cast<int>(prof.size()) < max_ops ? static_cast<int>(prof.size()) : max_ops;
  for (int i = 0; i < n; ++i)
    out[i] = wam_b200_op_profile{prof[i].phase, prof[i].kind, prof[i].launches, prof[i].ms,
                                 prof[i].bytes, prof[i].flops,
                                 {prof[i].shape[0], prof[i].shape[1], prof[i].shape[2],
                                  prof[i].shape[3]}};
  ok(st);
  return n;
}

WAM_B200_API int wam_b200_profile_graph(wam_b200_engine* e, int batch, int phase, int kind,
                                        int reps, wam_b200_graph_profile* out,
                                        wam_b200_status* st) {
  return wam_b200_profile_graph_lane(e, batch, phase, kind, -1, reps, out, st);
}

WAM_B200_API int wam_b200_profile_graph_lane(wam_b200_engine* e, int batch, int phase, int kind,
                                             int lane, int reps, wam_b200_graph_profile* out,
                                             wam_b200_status* st) {
  if (!e || !out) return fail(st, WAM_B200_INVALID_ARGUMENT, "engine and output are required");
  if (lane < -1 || lane > 1) return fail(st, WAM_B200_INVALID_ARGUMENT, "lane is -1, 0 or 1");
  std::string err;
  float ms = 0.0f;
  double bytes = 0.0, flops = 0.0;
  int launches = 0;
  if (!e->impl->profile_graph(batch, phase, kind, lane, reps, &ms, &bytes, &flops, &launches,
                              &err))
    return fail(st, code_of(err), err);
  out->ms = ms;
  out->bytes = bytes;
  out->flops = flops;
  out->launches = launches;
  return ok(st);
}

WAM_B200_API int wam_b200_block_forward(wam_b200_engine* e, const wam_b200_block_inputs* in,
                                        float* visual_out, size_t visual_out_n, float* action_out,
                                        size_t action_out_n, float* device_ms,
                                        wam_b200_status* st) {
  if (!e || !in) return fail(st, WAM_B200_INVALID_ARGUMENT, "engine and inputs are required");
  const wamb::Geometry& g = e->impl->geometry();
  const size_t nv = static_cast<size_t>(g.visual()) * g.hidden;
  const size_t na = static_cast<size_t>(1 + g.action_chunk) * g.action_hidden;
  if (visual_out_n < nv || action_out_n < na)
    return fail(st, WAM_B200_INVALID_ARGUMENT,
                "block outputs need [V][H] and [1 + T][E] floats (" + std::to_string(nv) + ", " +
                    std::to_string(na) + ")");
  std::string err;
  if (!e->impl->block_forward(in->visual, in->action, in->text_visual, in->text_action,
                              in->timestep, visual_out, action_out, device_ms, &err))
    return fail(st, code_of(err), err);
  return ok(st);
}

WAM_B200_API int wam_b200_read_tensor(wam_b200_engine* e, const char* name, int slot, int layer,
                                      float* out, size_t n, wam_b200_status* st) {
  if (!e || !name || !out) return fail(st, WAM_B200_INVALID_ARGUMENT, "engine, name and output are required");
  std::string err;
  if (!e->impl->read_tensor(name, slot, layer, out, n, &err))
    return fail(st, WAM_B200_INVALID_ARGUMENT, err);
  return ok(st);
}

}  // extern "C"
