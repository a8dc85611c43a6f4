// MotEngine: device weights, caches and the launch programs of one GWP-0.5
// action chunk (prompt projection, prefix cache, flow-matching denoise).
//
// Reference call stacks this follows (GigaAI-research/wam.cpp):
//   Gwp05ModelArch::predict                     src/models/gwp05/engine/engine.cpp:230-449
//   update_projected_prompt_cache / build_cross_kv  engine/cache.cpp:53-137, mot.cpp:101-128
//   build_prefix_cache                          engine/cache.cpp:139-485
//   build_cached_action_body (x num_steps)      engine/mot.cpp:358-496
//   run_unrolled_action_denoise                 engine/mot.cpp:498-594
// Differences in structure, not in arithmetic: the prefix K/V and the action
// K/V of a layer share one head-major buffer [P + T][128] per head (the joint
// order of keys does not change the softmax); the conditioning MLPs of all
// denoise steps run as one M = 1 + S GEMM; the visual expert's text K/V are
// projected with the prompt (they depend only on the prompt and weights).
#include "engine.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "gguf.h"
#include "host_math.h"
#include "t5.h"
#include "vae.h"

namespace wamb {

namespace {

uint64_t fnv1a64(const std::string& s) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 0x100000001B3ull;
  }
  return h;
}

uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = std::strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

#define CK(expr)                                                                  \
  do {                                                                            \
    cudaError_t e_ = (expr);                                                      \
    if (e_ != cudaSuccess) {                                                      \
      *err = std::string(#expr) + ": " + cudaGetErrorString(e_);                  \
      return false;                                                               \
    }                                                                             \
  } while (0)

}  // namespace

uint64_t tensor_seed(uint64_t seed, const std::string& name) {
  return mix64((seed ^ fnv1a64(name)) + 0x9E3779B97F4A7C15ull);
}

void synth_rule(const std::string& name, double bias_scale, double* scale, double* center) {
  if (ends_with(name, ".bias")) {
    *scale = bias_scale;
    *center = 0.0;
  } else if (ends_with(name, ".qn.weight") || ends_with(name, ".kn.weight") ||
             ends_with(name, ".ca_norm.weight")) {
    *scale = 0.02;
    *center = 1.0;
  } else {
    *scale = 0.02;
    *center = 0.0;
  }
}

// Compact GGUF names (src/models/gwp05/engine/weights.cpp:116-167) and element
// counts of every tensor the action-chunk path reads.
int64_t linear_inner(const std::string& name, const Geometry& g) {
  auto ends = [&](const char* suf) {
    const size_t n = std::strlen(suf);
    return name.size() >= n && name.compare(name.size() - n, n, suf) == 0;
  };
  if (!ends(".weight") || ends(".qn.weight") || ends(".kn.weight") || ends("ca_norm.weight"))
    return 0;
  const int64_t E = g.action_hidden, H = g.hidden;
  if (name == "gwp.patch.weight") return g.vae_z * 4;
  if (ends(".in.weight") && (name.rfind("gwp.state", 0) == 0 || name.rfind("gwp.action", 0) == 0))
    return 128;  // [emb][A][128], torch layout
  if (ends(".mid.weight") || name == "gwp.state.out.weight" || name == "gwp.action.out.weight")
    return 128;
  if (name == "gwp.decode.in.weight") return E;
  if (name == "gwp.decode.out.weight") return g.action_dim;  // [emb][128][A]
  if (ends(".time.0.weight")) return 256;
  if (ends(".text.0.weight")) return g.text_dim;
  if (name.rfind("gwp.acond", 0) == 0) return E;  // time.1 / time.out / text.1
  if (name.rfind("gwp.cond", 0) == 0) return H;
  const bool act = name.find(".a.") != std::string::npos;
  const int64_t W = act ? E : H, F = act ? g.action_ffn : g.ffn;
  if (ends(".sa.o.weight") || ends(".ca.o.weight")) return H;
  if (ends(".ffn.out.weight")) return F;
  return W;  // sa.qkv, ca.q, ca.k, ca.vproj, ffn.in
}

std::vector<std::pair<std::string, int64_t>> tensor_specs(const Geometry& g) {
  const int64_t E = g.action_hidden, H = g.hidden, A = g.action_dim, D = g.text_dim;
  const int64_t emb = g.num_embodiments;
  std::vector<std::pair<std::string, int64_t>> s;
  s.push_back({"gwp.patch.weight", H * g.vae_z * 4});
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
    s.push_back({p + ".time.0.weight", W * 256});
    s.push_back({p + ".time.0.bias", W});
    s.push_back({p + ".time.1.weight", W * W});
    s.push_back({p + ".time.1.bias", W});
    s.push_back({p + ".time.out.weight", 6 * W * W});
    s.push_back({p + ".time.out.bias", 6 * W});
    s.push_back({p + ".text.0.weight", W * D});
    s.push_back({p + ".text.0.bias", W});
    s.push_back({p + ".text.1.weight", W * W});
    s.push_back({p + ".text.1.bias", W});
  }
  for (int l = 0; l < g.layers; ++l) {
    for (int x = 0; x < 2; ++x) {
      const int64_t W = x == 0 ? E : H;
      const int64_t F = x == 0 ? g.action_ffn : g.ffn;
      const std::string p = "gwp.blk." + std::to_string(l) + (x == 0 ? ".a" : ".v");
      s.push_back({p + ".sa.qkv.weight", 3 * H * W});
      s.push_back({p + ".sa.qkv.bias", 3 * H});
      s.push_back({p + ".sa.qn.weight", H});
      s.push_back({p + ".sa.kn.weight", H});
      s.push_back({p + ".sa.o.weight", W * H});
      s.push_back({p + ".sa.o.bias", W});
      s.push_back({p + ".ca.q.weight", H * W});
      s.push_back({p + ".ca.q.bias", H});
      s.push_back({p + ".ca.k.weight", H * W});
      s.push_back({p + ".ca.k.bias", H});
      s.push_back({p + ".ca.vproj.weight", H * W});
      s.push_back({p + ".ca.vproj.bias", H});
      s.push_back({p + ".ca.o.weight", W * H});
      s.push_back({p + ".ca.o.bias", W});
      s.push_back({p + ".ca.qn.weight", H});
      s.push_back({p + ".ca.kn.weight", H});
      s.push_back({p + ".ca_norm.weight", W});
      s.push_back({p + ".ca_norm.bias", W});
      const int64_t fin = g.ffn_kind == 1 ? 2 : 1;  // SiLU-gated: [gate; up] rows
      s.push_back({p + ".ffn.in.weight", fin * F * W});
      s.push_back({p + ".ffn.in.bias", fin * F});
      s.push_back({p + ".ffn.out.weight", W * F});
      s.push_back({p + ".ffn.out.bias", W});
      s.push_back({p + ".mod", 6 * W});
    }
  }
  return s;
}

template <class T>
T* MotEngine::dalloc(size_t n, std::string* err) {
  void* p = nullptr;
  const size_t bytes = std::max<size_t>(n, 1) * sizeof(T);
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    *err = "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e);
    return nullptr;
  }
  cudaMemsetAsync(p, 0, bytes, stream_);
  allocs_.push_back(p);
  resident_bytes_ += bytes;
  return static_cast<T*>(p);
}

std::unique_ptr<MotEngine> MotEngine::create(const EngineOptions& opt, std::string* err) {
  std::unique_ptr<MotEngine> e(new MotEngine());
  if (!e->init(opt, err)) return nullptr;
  return e;
}

MotEngine::~MotEngine() {
  if (side_) cudaStreamSynchronize(side_);
  if (stream_) cudaStreamSynchronize(stream_);
  vae_.reset();
  t5_.reset();
  drop_plans();
  for (auto& e : phase_ev_)
    if (e) cudaEventDestroy(e);
  if (h2d_ev_) cudaEventDestroy(h2d_ev_);
  for (void* p : allocs_) cudaFree(p);
  if (h_state_) cudaFreeHost(h_state_);
  if (h_latent_) cudaFreeHost(h_latent_);
  if (h_prompt_) cudaFreeHost(h_prompt_);
  if (h_noise_) cudaFreeHost(h_noise_);
  if (h_out_) cudaFreeHost(h_out_);
  if (warena_) cudaFree(warena_);
  if (retile_tmp_) cudaFree(retile_tmp_);
  if (ev_fork_) cudaEventDestroy(ev_fork_);
  if (ev_join_) cudaEventDestroy(ev_join_);
  if (side_) cudaStreamDestroy(side_);
  if (stream_) cudaStreamDestroy(stream_);
}

bool MotEngine::init(const EngineOptions& opt, std::string* err) {
  opt_ = opt;
  if (opt.max_batch < 1 || opt.max_batch > 1024) {
    *err = "max_batch must be in [1, 1024]";
    return false;
  }
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (opt.device < 0 || opt.device >= ndev) {
    *err = "device index out of range";
    return false;
  }
  CK(cudaSetDevice(opt.device));
  int major = 0, minor = 0;
  CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, opt.device));
  CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, opt.device));
  if (major != 10 || minor != 0) {
    *err = "the wam_b200 engine runs on sm_100 (B200) only";
    return false;
  }
  CK(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, opt.device));
  CK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  CK(cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking));
  CK(cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming));
  CK(cudaEventCreateWithFlags(&ev_join_, cudaEventDisableTiming));
  // Diagnostic switch: keep GEMM weights in GGUF's row-major layout.
  const char* rm = std::getenv("WAM_B200_ROWMAJOR_WEIGHTS");
  rowmajor_weights_ = rm && rm[0] && rm[0] != '0';
  CK(gemm_init(opt.device));
  CK(attention_init());
  if (!load_weights(err)) return false;
  const Geometry& g = g_;
  if (g.heads * 128 != g.hidden || g.hidden % 128 || g.action_hidden % 128 || g.ffn % 128 ||
      g.action_ffn % 128 || g.text_dim % 64 || (g.vae_z * 4) % 64 || g.action_dim % 8 ||
      g.action_dim > 128 || g.action_chunk < 1 || g.steps < 1 || g.layers < 1 ||
      g.prompt_tokens < 1 || g.grid_h < 1 || g.grid_w < 1 || g.real_action_dim > g.action_dim ||
      g.real_state_dim > g.action_dim || g.embodiment_id >= g.num_embodiments) {
    *err = "unsupported geometry: widths must be multiples of 128 (text_dim, 4*vae_z of 64), "
           "head_dim 128, action_dim a multiple of 8 <= 128";
    return false;
  }
  if (opt.block && (g.layers != 1 || g.steps != 1 || opt.max_batch != 1 || opt.prompt_cache)) {
    *err = "block engines need layers == 1, steps == 1, max_batch == 1 and no prompt cache";
    return false;
  }
  if ((g.ffn_kind != 0 && g.ffn_kind != 1) || (g.norm_kind != 0 && g.norm_kind != 1)) {
    *err = "ffn_kind and norm_kind must be 0 or 1";
    return false;
  }
  flow_schedule(g.steps, g.flow_shift, &timesteps_, &sigmas_);
  if (!alloc_buffers(err)) return false;
  if (opt.vae) {
    if (opt.block) {
      *err = "block engines take hidden states, not images (vae must be 0)";
      return false;
    }
    VaeOptions vo;
    vo.artifact_path = opt.artifact_path;
    vo.synthetic_seed = opt.seed;
    vo.image_width = g.grid_w * 32;
    vo.image_height = g.grid_h * 32;
    vo.z_dim = g.vae_z;
    vo.device_index = opt.device;
    vo.use_cuda_graph = opt.graphs;
    vae_.reset(new VaeEncoder());
    std::string verr;
    if (!vae_->init(vo, &verr)) {
      *err = "VAE encoder: " + verr;
      return false;
    }
  }
  if (opt.t5) {
    if (opt.block) {
      *err = "block engines take hidden states, not prompt tokens (t5 must be 0)";
      return false;
    }
    T5Options to;
    to.artifact_path = opt.artifact_path;
    to.synthetic_seed = opt.seed;
    to.geometry.vocab = opt.t5_vocab;
    to.geometry.hidden = g.text_dim;
    to.geometry.ffn = opt.t5_ffn;
    to.geometry.heads = g.text_dim / 64;
    to.geometry.head_dim = 64;
    to.geometry.layers = opt.t5_layers;
    to.geometry.max_tokens = g.prompt_tokens;
    to.device_index = opt.device;
    to.use_cuda_graph = opt.graphs;
    t5_.reset(new T5Encoder());
    std::string terr;
    if (!t5_->init(to, &terr)) {
      *err = "UMT5 encoder: " + terr;
      return false;
    }
    if (t5_->geometry().hidden != g.text_dim) {
      *err = "UMT5 encoder: t5_hidden differs from the prompt width (text_dim)";
      return false;
    }
  }
  CK(cudaStreamSynchronize(stream_));
  prompt_key_.assign(opt.max_batch, {});
  in_prompt_key_.assign(opt.max_batch, {});
  h_prompt_ver_.assign(opt.max_batch, 0);
  h_prompt_rows_.assign(opt.max_batch, 0);
  prompt_copy_.assign(opt.max_batch, 0);
  ok_ = true;
  return true;
}

const bf16* MotEngine::W(const std::string& name, int64_t numel) {
  auto it = w_.find(name);
  if (it == w_.end()) return nullptr;
  if (numel >= 0 && wn_[name] != numel) return nullptr;
  return it->second;
}

// Q8_0 policy (weight_format 1): every linear weight whose rows are whole
// 32-value blocks and that the artifact did not already hold as Q8_0 is
// quantised on the device; its BF16 slot is overwritten with q * d (rounded to
// BF16), which is what every consumer of the weight then computes with.
bool MotEngine::quantize_linear_weights(const std::vector<std::pair<std::string, int64_t>>& specs,
                                        std::string* err) {
  for (const auto& s : specs) {
    const int64_t inner = linear_inner(s.first, g_);
    if (inner <= 0 || inner % 32 != 0 || q8_blocks_.count(s.first)) continue;
    uint8_t* blocks = dalloc<uint8_t>(static_cast<size_t>(s.second / 32) * 34, err);
    if (!blocks) return false;
    launch_q8_quantize(w_[s.first], s.second, blocks, stream_);
    launch_q8_dequantize(blocks, s.second, w_[s.first], stream_);
    q8_blocks_[s.first] = blocks;
  }
  CK(cudaGetLastError());
  return true;
}

bool MotEngine::load_weights(std::string* err) {
  GgufFile file;
  const bool synthetic = opt_.artifact_path.empty();
  if (synthetic) {
    g_ = opt_.synthetic;
    loader_ = "synthetic";
  } else {
    if (!file.open(opt_.artifact_path, err)) return false;
    std::string arch;
    if (!file.get_str("gwp05.architecture", &arch) || arch != "gwp05") {
      *err = "artifact is not a gwp05 GGUF (gwp05.architecture)";
      return false;
    }
    uint32_t u = 0;
    auto req = [&](const char* key, int* dst) {
      if (!file.get_u32(key, &u)) {
        *err = std::string("artifact lacks ") + key;
        return false;
      }
      *dst = static_cast<int>(u);
      return true;
    };
    int img_h = 0, img_w = 0, head_dim = 0;
    if (!req("gwp05.hidden", &g_.hidden) || !req("gwp05.n_layers", &g_.layers) ||
        !req("gwp05.n_heads", &g_.heads) || !req("gwp05.head_dim", &head_dim) ||
        !req("gwp05.ffn_dim", &g_.ffn) || !req("gwp05.action_hidden", &g_.action_hidden) ||
        !req("gwp05.action_ffn_dim", &g_.action_ffn) || !req("gwp05.action_dim", &g_.action_dim) ||
        !req("gwp05.real_state_dim", &g_.real_state_dim) ||
        !req("gwp05.real_action_dim", &g_.real_action_dim) ||
        !req("gwp05.num_embodiments", &g_.num_embodiments) ||
        !req("gwp05.embodiment_id", &g_.embodiment_id) || !req("gwp05.image_height", &img_h) ||
        !req("gwp05.image_width", &img_w) || !req("gwp05.action_chunk", &g_.action_chunk) ||
        !req("gwp05.inference_steps", &g_.steps) || !req("gwp05.t5_hidden", &g_.text_dim) ||
        !req("gwp05.vae_z_dim", &g_.vae_z))
      return false;
    if (head_dim != 128 || img_h % 32 || img_w % 32) {
      *err = "artifact geometry: head_dim must be 128 and image dims multiples of 32";
      return false;
    }
    g_.grid_h = img_h / 32;
    g_.grid_w = img_w / 32;
    g_.prompt_tokens = 64;  // semantics.h:11 kPromptTokens
    if (file.get_u32("gwp05.prompt_tokens", &u)) g_.prompt_tokens = static_cast<int>(u);
    if (!file.get_f32("gwp05.norm_eps", &g_.norm_eps) ||
        !file.get_f32("gwp05.flow_shift", &g_.flow_shift)) {
      *err = "artifact lacks gwp05.norm_eps / gwp05.flow_shift";
      return false;
    }
    // Weight policy (scripts/inspect/inspect_gguf.py:60-75 _policy): an
    // artifact that names one must be the packed-QKV BF16 policy the engine
    // reads (mot-vae-bf16-qkv-v1) or its Q8_0 variant (mot-q8_0-v1, written by
    // wam_b200.artifact), and conversion_policy must agree. Artifacts without
    // the key (test fixtures) are read as their tensor types say.
    std::string policy, conversion;
    if (file.get_str("gwp05.weight_policy", &policy)) {
      if (file.get_str("gwp05.conversion_policy", &conversion) && conversion != policy) {
        *err = "artifact gwp05.weight_policy differs from gwp05.conversion_policy";
        return false;
      }
      if (policy == "mot-q8_0-v1") {
        policy_ = 2;
        opt_.weight_format = 1;  // what the file does not hold as Q8_0 is quantised at load
      } else if (policy == "mot-vae-bf16-qkv-v1") {
        policy_ = 1;
      } else {
        *err = "unsupported weight policy " + policy +
               " (this engine reads mot-vae-bf16-qkv-v1 and mot-q8_0-v1 artifacts)";
        return false;
      }
    }
    loader_ = "gguf";
  }
  const auto specs = tensor_specs(g_);
  size_t total = 0;
  for (const auto& s : specs) total += (static_cast<size_t>(s.second) * 2 + 255) / 256 * 256;
  cudaError_t e = cudaMalloc(&warena_, total);
  if (e != cudaSuccess) {
    *err = "weight arena cudaMalloc(" + std::to_string(total) + "): " + cudaGetErrorString(e);
    return false;
  }
  warena_bytes_ = total;
  resident_bytes_ += total;
  uint8_t* base = static_cast<uint8_t*>(warena_);
  size_t off = 0;
  // Arena order: each expert's prompt projections (ca.k and ca.vproj of every
  // layer, weights then biases) come first and back to back, so that their
  // re-tiled weights form one [layers * 2H][K] matrix (256-row tiles are the
  // outermost dimension of the re-tiled layout) and the prompt projection of
  // an expert runs as one GEMM; every other tensor follows in spec order.
  std::unordered_map<std::string, int64_t> numel;
  for (const auto& s : specs) numel[s.first] = s.second;
  std::vector<std::string> order;
  for (const char* x : {".a", ".v"})
    for (const char* part : {".weight", ".bias"})
      for (int l = 0; l < g_.layers; ++l)
        for (const char* proj : {".ca.k", ".ca.vproj"})
          order.push_back("gwp.blk." + std::to_string(l) + x + proj + part);
  {
    std::unordered_map<std::string, bool> first;
    for (const auto& n : order) first[n] = true;
    for (const auto& s : specs)
      if (!first.count(s.first)) order.push_back(s.first);
  }
  for (const auto& name : order) {
    w_[name] = reinterpret_cast<bf16*>(base + off);
    wn_[name] = numel[name];
    off += (static_cast<size_t>(numel[name]) * 2 + 255) / 256 * 256;
  }
  const int A = g_.action_dim;
  sq01_.resize(A);
  sq99_.resize(A);
  aq01_.resize(A);
  aq99_.resize(A);
  if (synthetic) {
    for (const auto& s : specs) {
      double scale, center;
      synth_rule(s.first, opt_.bias_scale, &scale, &center);
      launch_synth_bf16(w_[s.first], s.second, tensor_seed(opt_.seed, s.first), scale, center,
                        stream_);
    }
    for (int i = 0; i < A; ++i) {
      sq01_[i] = aq01_[i] = -1.0f - 0.01f * static_cast<float>(i);
      sq99_[i] = aq99_[i] = 1.0f + 0.02f * static_cast<float>(i);
    }
    CK(cudaGetLastError());
    if (opt_.weight_format == 1 && !quantize_linear_weights(specs, err)) return false;
    CK(cudaStreamSynchronize(stream_));
    return true;
  }
  // GGUF: stream each tensor through a pinned staging buffer.
  const size_t chunk = 64ull << 20;
  void* staging[2] = {nullptr, nullptr};
  cudaEvent_t done[2];
  CK(cudaHostAlloc(&staging[0], chunk, cudaHostAllocDefault));
  CK(cudaHostAlloc(&staging[1], chunk, cudaHostAllocDefault));
  CK(cudaEventCreate(&done[0]));
  CK(cudaEventCreate(&done[1]));
  bool ok = true;
  int slot = 0;
  for (const auto& s : specs) {
    const GgufTensor* t = file.tensor(s.first);
    if (!t) {
      *err = "artifact lacks tensor " + s.first;
      ok = false;
      break;
    }
    const int64_t inner = linear_inner(s.first, g_);
    const bool q8 = t->type == GGML_Q8_0 && inner > 0 && inner % 32 == 0;
    if ((t->type != GGML_BF16 && !q8) || static_cast<int64_t>(t->elements()) != s.second) {
      *err = "artifact tensor " + s.first + " must be BF16 (or Q8_0 for a linear weight) with " +
             std::to_string(s.second) + " elements";
      ok = false;
      break;
    }
    // mot-q8_0-v1 stores every linear weight whose GGUF rows are whole
    // 32-value blocks as Q8_0; the BF16 policy stores none.
    const bool q8_row = inner > 0 && inner % 32 == 0 && !t->ne.empty() && t->ne[0] % 32 == 0;
    if ((policy_ == 2 && q8_row && !q8) || (policy_ == 1 && q8)) {
      *err = "artifact tensor " + s.first + " is " + (q8 ? "Q8_0" : "BF16") + ", which policy " +
             (policy_ == 2 ? "mot-q8_0-v1" : "mot-vae-bf16-qkv-v1") + " does not allow";
      ok = false;
      break;
    }
    uint8_t* dst = reinterpret_cast<uint8_t*>(w_[s.first]);
    if (q8) {
      // Q8_0 blocks go to their own buffer; the BF16 slot gets q * d below.
      if (t->bytes != static_cast<uint64_t>(s.second / 32) * 34) {
        *err = "artifact tensor " + s.first + ": Q8_0 size mismatch";
        ok = false;
        break;
      }
      if (!(dst = dalloc<uint8_t>(t->bytes, err))) {
        ok = false;
        break;
      }
      q8_blocks_[s.first] = dst;
    }
    for (uint64_t pos = 0; pos < t->bytes; pos += chunk) {
      const uint64_t n = std::min<uint64_t>(chunk, t->bytes - pos);
      cudaEventSynchronize(done[slot]);
      if (!file.read(*t, pos, staging[slot], n)) {
        *err = "short read of " + s.first;
        ok = false;
        break;
      }
      cudaMemcpyAsync(dst + pos, staging[slot], n, cudaMemcpyHostToDevice, stream_);
      cudaEventRecord(done[slot], stream_);
      slot ^= 1;
    }
    if (!ok) break;
  }
  cudaStreamSynchronize(stream_);
  for (const auto& kv : q8_blocks_)
    launch_q8_dequantize(kv.second, wn_[kv.first], w_[kv.first], stream_);
  if (ok && opt_.weight_format == 1 && !quantize_linear_weights(specs, err)) ok = false;
  if (ok) {
    const char* names[4] = {"state_q01", "state_q99", "action_q01", "action_q99"};
    std::vector<float>* dsts[4] = {&sq01_, &sq99_, &aq01_, &aq99_};
    for (int i = 0; i < 4 && ok; ++i) {
      const GgufTensor* t = file.tensor(names[i]);
      if (!t || t->type != GGML_F32 || t->elements() != static_cast<uint64_t>(A) ||
          !file.read(*t, 0, dsts[i]->data(), static_cast<uint64_t>(A) * 4)) {
        *err = std::string("artifact lacks F32 statistic ") + names[i];
        ok = false;
      }
    }
  }
  cudaEventDestroy(done[0]);
  cudaEventDestroy(done[1]);
  cudaFreeHost(staging[0]);
  cudaFreeHost(staging[1]);
  if (ok) {
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) {
      *err = std::string("weight upload: ") + cudaGetErrorString(ce);
      ok = false;
    }
  }
  return ok;
}

bool MotEngine::alloc_buffers(std::string* err) {
  const Geometry& g = g_;
  const size_t B = opt_.max_batch, T = g.action_chunk, V = g.visual(), P = g.prefix();
  const size_t Nt = g.prompt_tokens, D = g.text_dim, H = g.hidden, E = g.action_hidden;
  const size_t F = std::max(g.ffn, g.action_ffn), A = g.action_dim, L = g.layers;
  const size_t S = g.steps, C = g.vae_z, heads = g.heads;
  const size_t VT = std::max(V, T), HE = std::max(H, E);
  const size_t lat = C * 4 * V;
#define AL(ptr, T_, n)                      \
  if (!((ptr) = dalloc<T_>((n), err))) return false;
  AL(in_state_, float, B * A);
  AL(in_latent_, float, B * lat);
  AL(in_prompt_, float, B * Nt * D);
  AL(in_noise_, float, B * T * A);
  AL(d_out_, float, B * T * A);
  CK(cudaHostAlloc(reinterpret_cast<void**>(&h_state_), B * A * 4, cudaHostAllocDefault));
  CK(cudaHostAlloc(reinterpret_cast<void**>(&h_latent_), B * lat * 4, cudaHostAllocDefault));
  CK(cudaHostAlloc(reinterpret_cast<void**>(&h_prompt_), B * Nt * D * 4, cudaHostAllocDefault));
  CK(cudaHostAlloc(reinterpret_cast<void**>(&h_noise_), B * T * A * 4, cudaHostAllocDefault));
  CK(cudaHostAlloc(reinterpret_cast<void**>(&h_out_), B * T * A * 4, cudaHostAllocDefault));
  AL(prompt_bf_, bf16, B * Nt * D);
  AL(state_bf_, bf16, B * A);
  AL(action_bf_, bf16, B * T * A);
  AL(text_tmp_, bf16, B * Nt * HE);
  AL(text_a_, bf16, B * Nt * E);
  AL(text_v_, bf16, B * Nt * H);
  AL(ckv_, bf16, B * Nt * 2 * H);
  AL(cols_, bf16, B * V * C * 4);
  AL(hv_, bf16, B * V * H);
  AL(hs_, bf16, B * E);
  AL(ha_, bf16, B * T * E);
  AL(nrm_, bf16, B * VT * HE);
  AL(nrm_s_, bf16, B * E);
  AL(qkv_, bf16, B * VT * 3 * H);
  AL(qkv_s_, bf16, B * 3 * H);
  AL(qbuf_, bf16, B * heads * std::max(P, T) * 128);
  AL(att_, bf16, B * VT * H);
  AL(att_s_, bf16, B * H);
  AL(cq_, bf16, B * VT * H);
  AL(cq_s_, bf16, B * H);
  AL(qc_, bf16, B * heads * VT * 128);
  AL(qc_s_, bf16, B * heads * 128);
  AL(catt_, bf16, B * VT * H);
  AL(catt_s_, bf16, B * H);
  AL(ffn_, bf16, B * VT * F);
  AL(ffn_s_, bf16, B * F);
  AL(s1_, bf16, B * 128);
  AL(s2_, bf16, B * 128);
  AL(e1_, bf16, B * T * 128);
  AL(e2_, bf16, B * T * 128);
  AL(d1_, bf16, B * T * 128);
  AL(d2_, bf16, B * T * 128);
  AL(vel_, bf16, S * B * T * A);
  AL(freq_bf_, bf16, (1 + S) * 256);
  AL(ct1_, bf16, (1 + S) * E);
  AL(temb_a_, bf16, (1 + S) * E);
  AL(ct2_, bf16, (1 + S) * E);
  AL(mod_a_, bf16, (1 + S) * 6 * E);
  AL(cv1_, bf16, H);
  AL(temb_v_, bf16, H);
  AL(cv2_, bf16, H);
  AL(mod_v_, bf16, 6 * H);
  AL(comb_a0_, float, L * 6 * E);
  AL(comb_v_, float, L * 6 * H);
  AL(comb_steps_, float, S * L * 6 * E);
  AL(comb_final_, float, S * 2 * E);
  AL(dt_, float, S);
  AL(inv_freq1_, float, 64);
  AL(inv_freq3_, float, 64);
  AL(pos_thw_, int, V * 3);
  AL(tables_a_, const bf16*, L);
  AL(tables_v_, const bf16*, L);
  AL(tables_final_, const bf16*, 1);
  AL(k_self_, bf16, B * L * heads * (P + T) * 128);
  AL(v_self_, bf16, B * L * heads * (P + T) * 128);
  AL(k_prompt_, bf16, B * L * heads * Nt * 128);
  AL(v_prompt_, bf16, B * L * heads * Nt * 128);
  AL(k_vis_, bf16, B * L * heads * Nt * 128);
  AL(v_vis_, bf16, B * L * heads * Nt * 128);
  {
    // Prompt-projection output of up to 4 GB worth of layers at a time.
    const size_t per_layer = B * Nt * 2 * H * sizeof(bf16);
    pkv_layers_ = static_cast<int>(std::min<size_t>(L, std::max<size_t>(1, (4ull << 30) / per_layer)));
    AL(pkv_, bf16, B * Nt * static_cast<size_t>(pkv_layers_) * 2 * H);
    AL(knorm_tab_, const bf16*, 2 * static_cast<size_t>(L));
  }
  AL(err_word_, unsigned, 1);
  // A split GEMM holds at most one wave of CTAs, each with a partial tile of
  // <= 128 tokens x 256 features: sms x 128 x 256 floats bound every plan.
  gemm_ws_floats_ = static_cast<size_t>(sms_) * 128 * 256;
  AL(gemm_ws_[0], float, gemm_ws_floats_);
  AL(gemm_ws_[1], float, gemm_ws_floats_);
  if (opt_.block) {
    AL(blk_in_, float, V * H + (1 + T) * E + Nt * H + Nt * E);
    AL(blk_out_, float, V * H + (1 + T) * E);
  }
#undef AL
  // constants: timestep frequencies (row 0: t = 0 for the prefix, rows 1..S the
  // schedule), dt, RoPE inverse frequencies, visual positions, table pointers.
  std::vector<float> freq((1 + S) * 256);
  timestep_embedding(0.0f, 256, freq.data());
  for (size_t s = 0; s < S; ++s) timestep_embedding(timesteps_[s], 256, freq.data() + (1 + s) * 256);
  if (!(freq_f32_ = dalloc<float>(freq.size(), err))) return false;
  CK(cudaMemcpyAsync(freq_f32_, freq.data(), freq.size() * 4, cudaMemcpyHostToDevice, stream_));
  launch_f32_to_bf16(freq_f32_, freq_bf_, static_cast<long long>(freq.size()), stream_);
  std::vector<float> dt(S);
  for (size_t s = 0; s < S; ++s) dt[s] = sigmas_[s + 1] - sigmas_[s];
  CK(cudaMemcpyAsync(dt_, dt.data(), S * 4, cudaMemcpyHostToDevice, stream_));
  // RoPE inverse frequencies: one table for the 1-D action rope and one for
  // the three visual sections.
  std::vector<float> f1(64), f3(64);
  rope_inv_freq(1, f1.data());
  rope_inv_freq(2, f3.data());
  CK(cudaMemcpyAsync(inv_freq1_, f1.data(), 256, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(inv_freq3_, f3.data(), 256, cudaMemcpyHostToDevice, stream_));
  // visual_positions (semantics.cpp:235-257): t = 0, h = y, w = x.
  std::vector<int> pos(V * 3);
  visual_positions(g.grid_h, g.grid_w, pos.data());
  CK(cudaMemcpyAsync(pos_thw_, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice, stream_));
  std::vector<const bf16*> ta(L), tv(L);
  for (size_t l = 0; l < L; ++l) {
    ta[l] = W("gwp.blk." + std::to_string(l) + ".a.mod", 6 * E);
    tv[l] = W("gwp.blk." + std::to_string(l) + ".v.mod", 6 * H);
  }
  const bf16* tf = W("gwp.action_mod", 2 * E);
  CK(cudaMemcpyAsync(tables_a_, ta.data(), L * sizeof(void*), cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(tables_v_, tv.data(), L * sizeof(void*), cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(tables_final_, &tf, sizeof(void*), cudaMemcpyHostToDevice, stream_));
  CK(cudaStreamSynchronize(stream_));  // host vectors above go out of scope
  return true;
}

bool MotEngine::ensure_tiled(const std::string& wname, int n, int k, std::string* err) {
  if (tiled_[wname]) return true;
  if (n % gemm_weight_tile_rows() != 0 || k % 64 != 0 || !W(wname + ".weight", static_cast<int64_t>(n) * k)) {
    *err = "cannot re-tile weight " + wname;
    return false;
  }
  const size_t elems = static_cast<size_t>(n) * k;
  if (elems > retile_tmp_elems_) {
    if (retile_tmp_) {
      CK(cudaStreamSynchronize(stream_));
      cudaFree(retile_tmp_);
      retile_tmp_ = nullptr;
    }
    cudaError_t ae = cudaMalloc(&retile_tmp_, elems * sizeof(bf16));
    if (ae != cudaSuccess) {
      retile_tmp_elems_ = 0;
      *err = std::string("re-tiling staging buffer: ") + cudaGetErrorString(ae);
      return false;
    }
    retile_tmp_elems_ = elems;
  }
  bf16* wm = w_[wname + ".weight"];
  CK(cudaMemcpyAsync(retile_tmp_, wm, elems * sizeof(bf16), cudaMemcpyDeviceToDevice, stream_));
  launch_retile_weights(retile_tmp_, wm, n, k, stream_);
  CK(cudaGetLastError());
  tiled_[wname] = true;
  return true;
}

bool MotEngine::gemm(Program& p, const bf16* x, int ldx, int m, const std::string& wname, int n,
                     int k, int epi, bool bias, const float* gate, const bf16* resid, int ldr,
                     void* out, int ldo, std::string* err, int total_n, int row0) {
  // Rows [row0, row0 + n) of a weight with total_n rows (default: all n rows).
  if (total_n < 0) total_n = n;
  if (row0 < 0 || row0 + n > total_n ||
      (row0 % gemm_weight_tile_rows() != 0 && total_n % gemm_weight_tile_rows() == 0)) {
    *err = "bad weight row range of " + wname;
    return false;
  }
  const bf16* w_all = W(wname + ".weight", static_cast<int64_t>(total_n) * k);
  const bf16* b_all = bias ? W(wname + ".bias", total_n) : nullptr;
  if (!w_all || (bias && !b_all)) {
    *err = "missing or mis-shaped weight " + wname;
    return false;
  }
  // Row-major and re-tiled layouts both keep rows in order (whole 256-row
  // tiles outermost), so a row range starting on a tile starts at row0 * k.
  const bf16* w = w_all + static_cast<size_t>(row0) * k;
  const bf16* b = b_all ? b_all + row0 : nullptr;
  // Q8_0 linear weights with whole 256-row tiles stream as Q8_0 GEMM tiles
  // (made from the blocks the first time a plan uses them).
  const auto qb = q8_blocks_.find(wname + ".weight");
  // Only the weight-streaming GEMMs (few tokens) take the Q8_0 tiles; the
  // tensor-bound ones (prefix, batched) read the dequantised BF16 copy, which
  // gives the same results (the Q8_0 GEMM is bit-identical to the BF16 GEMM on
  // q * d) without converting every tile on the CUDA cores.
  const bool q8 = qb != q8_blocks_.end() && m <= 64 && total_n % gemm_weight_tile_rows() == 0 &&
                  n % gemm_weight_tile_rows() == 0 && k % 64 == 0;
  if (q8 && !q8_tiles_.count(wname)) {
    uint8_t* tiles =
        dalloc<uint8_t>(static_cast<size_t>(total_n / 256) * (k / 64) * kQ8TileBytes, err);
    if (!tiles) return false;
    launch_q8_retile(qb->second, tiles, total_n, k, stream_);
    CK(cudaGetLastError());
    q8_tiles_[wname] = tiles;
  }
  // Every other weight with whole 256-row tiles is re-tiled in place, the
  // first time a plan uses it, into contiguous 32 KB UMMA tiles (one bulk copy
  // per stage).
  const bool tiled = !q8 && !rowmajor_weights_ && total_n % gemm_weight_tile_rows() == 0 &&
                     n % gemm_weight_tile_rows() == 0 && k % 64 == 0;
  if (tiled && !ensure_tiled(wname, total_n, k, err)) return false;
  const bf16* wsrc =
      q8 ? reinterpret_cast<const bf16*>(q8_tiles_[wname] +
                                         static_cast<size_t>(row0 / 256) * (k / 64) * kQ8TileBytes)
         : w;
  return add_gemm(p, x, ldx, m, wsrc, n, k, epi, b, gate, resid, ldr, out, ldo, tiled, q8, wname, err);
}

bool MotEngine::add_gemm(Program& p, const bf16* x, int ldx, int m, const bf16* wsrc, int n, int k,
                         int epi, const bf16* b, const float* gate, const bf16* resid, int ldr,
                         void* out, int ldo, bool tiled, bool q8, const std::string& label,
                         std::string* err) {
  // Split-K partials go through this lane's workspace inside a cluster.
  GemmScratch sc;
  sc.workspace = gemm_ws_[p.lane];
  sc.workspace_floats = gemm_ws_floats_;
  sc.error = err_word_;
  GemmOp op;
  const char* e =
      gemm_plan(&op, x, ldx, m, wsrc, n, k, epi, b, gate, resid, ldr, out, ldo, sc, sms_, 0, tiled, q8);
  if (e) {
    *err = std::string(e) + " (" + label + ")";
    return false;
  }
  const double extra = (epi == EPI_GATED_RES || epi == EPI_RES) ? 2.0 * m * n : 0.0;
  p.add([op](cudaStream_t s) { return gemm_launch(op, s); }, OP_GEMM, 1,
        2.0 * (static_cast<double>(n) * k + static_cast<double>(m) * k + static_cast<double>(m) * n) +
            2.0 * extra,
        2.0 * m * n * static_cast<double>(k));
  Op& rec = p.ops.back();
  rec.shape[0] = m;
  rec.shape[1] = n;
  rec.shape[2] = k;
  rec.shape[3] = op.pair ? -op.args.splits : op.args.splits;  // negative: CTA-pair kernel
  return true;
}

bool MotEngine::build(int b, std::string* err) {
  for (int attempt = 0; attempt < 16; ++attempt) {
    auto plan = std::make_unique<Plan>();
    const Geometry& g = g_;
    const int T = g.action_chunk, V = g.visual(), P = g.prefix(), Nt = g.prompt_tokens;
    const int D = g.text_dim, H = g.hidden, E = g.action_hidden, A = g.action_dim;
    const int L = g.layers, S = g.steps, heads = g.heads, C = g.vae_z;
    const int Fv = g.ffn, Fa = g.action_ffn, emb = g.embodiment_id;
    const long long selfL = static_cast<long long>(heads) * (P + T) * 128;  // per layer
    const long long selfB = selfL * L;                                       // per request
    const long long prL = static_cast<long long>(heads) * Nt * 128;
    const long long prB = prL * L;
    const float eps = g.norm_eps;
    const bool rms = g.norm_kind == 1;   // config-1 variant: RMSNorm inside AdaLN
    const bool block = opt_.block;       // config 1: one layer over given hidden states
    bool ok = true;
    std::string e2;
    auto G = [&](Program& p, const bf16* x, int ldx, int m, const std::string& wn, int n, int k,
                 int epi, bool bias, const float* gate, const bf16* resid, int ldr, void* out,
                 int ldo) {
      if (ok && !gemm(p, x, ldx, m, wn, n, k, epi, bias, gate, resid, ldr, out, ldo, &e2)) ok = false;
    };
    auto K = [](Program& p, Launch f) { p.add(std::move(f), OP_ELEMENTWISE); };
    // FFN up projection: GELU(tanh) (the reference), or the config-1 SiLU-gated
    // form silu(x Wg + bg) * (x Wu + bu) over ffn.in's [gate; up] rows.
    auto ffn_in = [&](Program& p, const bf16* x, int ldx, int m, const std::string& pfx, int F,
                      int W, bf16* out) {
      if (g.ffn_kind == 0) {
        G(p, x, ldx, m, pfx + ".ffn.in", F, W, EPI_BIAS_GELU, true, nullptr, nullptr, 0, out, F);
        return;
      }
      if (ok && !gemm(p, x, ldx, m, pfx + ".ffn.in", F, W, EPI_BIAS_SILU, true, nullptr, nullptr,
                      0, out, F, &e2, 2 * F, 0))
        ok = false;
      if (ok && !gemm(p, x, ldx, m, pfx + ".ffn.in", F, W, EPI_MUL, true, nullptr, out, F, out, F,
                      &e2, 2 * F, F))
        ok = false;
    };
    // Lane hand-offs: the side stream waits for everything the main stream has
    // issued so far (fork), or the main stream for the side stream (join).
    auto fork_side = [&](Program& p) {
      const int lane = p.lane;
      p.lane = 0;
      p.add([this](cudaStream_t) {
        cudaError_t e = cudaEventRecord(ev_fork_, stream_);
        return e == cudaSuccess ? cudaStreamWaitEvent(side_, ev_fork_, 0) : e;
      }, OP_SYNC, 0);
      p.lane = lane;
    };
    auto join_side = [&](Program& p) {
      const int lane = p.lane;
      p.lane = 0;
      p.add([this](cudaStream_t) {
        cudaError_t e = cudaEventRecord(ev_join_, side_);
        return e == cudaSuccess ? cudaStreamWaitEvent(stream_, ev_join_, 0) : e;
      }, OP_SYNC, 0);
      p.lane = lane;
    };
    auto scatter = [&](Program& p, const QkvScatter& q) {
      const double parts = (q.q_col >= 0) + (q.k_col >= 0) + (q.v_col >= 0);
      p.add([q](cudaStream_t s) {
        launch_qkv_scatter(q, s);
        return cudaGetLastError();
      }, OP_QKV, 1, 4.0 * parts * q.rows * q.hidden * q.layers);
    };
    auto attend = [&](Program& p, const AttnArgs& a_in) {
      // Key splits merge through the lane's workspace (dead between GEMMs).
      AttnArgs a = a_in;
      a.ws = gemm_ws_[p.lane];
      a.ws_floats = gemm_ws_floats_;
      a.error = err_word_;
      const double bq = 2.0 * a.batch * a.heads * a.lq * 128.0;
      const double bkv = 4.0 * a.batch * a.heads * a.lk * 128.0;
      p.add([a](cudaStream_t s) {
        launch_attention(a, s);
        return cudaGetLastError();
      }, OP_ATTENTION, attention_launch_count(a), 2.0 * bq + bkv, 4.0 * a.batch * a.heads * double(a.lq) * a.lk * 128.0);
    };
    auto ln_mod = [&](Program& p, const bf16* x, int rows, int cols, const float* scale,
                      const float* shift, bf16* y) {
      p.add([=](cudaStream_t s) {
        if (rms)
          launch_rms_modulate(x, cols, rows, cols, scale, shift, eps, y, cols, s);
        else
          launch_ln_modulate(x, cols, rows, cols, scale, shift, eps, y, cols, s);
        return cudaGetLastError();
      }, OP_LAYERNORM, 1, 4.0 * rows * double(cols) + 8.0 * cols);
    };
    auto p_ln_final = [&](Program& p, const bf16* x, int rows, int cols, const float* scale,
                          const float* shift, bf16* y) {
      p.add([=](cudaStream_t s) {
        launch_ln_modulate(x, cols, rows, cols, scale, shift, eps, y, cols, s);
        return cudaGetLastError();
      }, OP_LAYERNORM, 1, 4.0 * rows * double(cols) + 8.0 * cols);
    };
    auto ln_aff = [&](Program& p, const bf16* x, int rows, int cols, const std::string& wn, bf16* y) {
      const bf16* w = W(wn + ".weight", cols);
      const bf16* bb = W(wn + ".bias", cols);
      if (!w || !bb) {
        ok = false;
        e2 = "missing " + wn;
        return;
      }
      p.add([=](cudaStream_t s) {
        launch_ln_affine(x, cols, rows, cols, w, bb, eps, y, cols, s);
        return cudaGetLastError();
      }, OP_LAYERNORM, 1, 4.0 * rows * double(cols) + 4.0 * cols);
    };
    auto small = [&](Program& p, const bf16* x, int m, int k, const bf16* w, long long sn,
                     long long sk, const bf16* bias, int n, int act, bf16* y) {
      if (!w || !bias) {
        ok = false;
        e2 = "missing encoder/decoder weight";
        return;
      }
      p.add([=](cudaStream_t s) {
        launch_small_linear(x, k, m, k, w, sn, sk, bias, n, act, y, n, s);
        return cudaGetLastError();
      }, OP_SMALL, 1, 2.0 * (double(n) * k + double(m) * k + double(m) * n), 2.0 * m * n * double(k));
    };
    auto cross_q = [&](Program& p, const bf16* src, int rows, int rows_per_seq,
                       const std::string& pfx, bf16* qout) {
      QkvScatter q{};
      q.src = src;
      q.ld_src = H;
      q.rows = rows;
      q.rows_per_seq = rows_per_seq;
      q.hidden = H;
      q.heads = heads;
      q.q_col = 0;
      q.k_col = -1;
      q.v_col = -1;
      q.q_norm = W(pfx + ".ca.qn.weight", H);
      q.eps = eps;
      q.q_out = qout;
      q.q_seq_stride = static_cast<long long>(heads) * rows_per_seq * 128;
      q.q_head_stride = static_cast<long long>(rows_per_seq) * 128;
      if (!q.q_norm) {
        ok = false;
        e2 = "missing " + pfx + ".ca.qn";
      }
      scatter(p, q);
    };
    auto prompt_kv = [&](Program& p, const bf16* text, int tw, const std::string& pfx, bf16* kdst,
                         bf16* vdst) {
      G(p, text, tw, b * Nt, pfx + ".ca.k", H, tw, EPI_BIAS, true, nullptr, nullptr, 0, ckv_, 2 * H);
      G(p, text, tw, b * Nt, pfx + ".ca.vproj", H, tw, EPI_BIAS, true, nullptr, nullptr, 0, ckv_ + H, 2 * H);
      QkvScatter q{};
      q.src = ckv_;
      q.ld_src = 2 * H;
      q.rows = b * Nt;
      q.rows_per_seq = Nt;
      q.hidden = H;
      q.heads = heads;
      q.q_col = -1;
      q.k_col = 0;
      q.v_col = H;
      q.k_norm = W(pfx + ".ca.kn.weight", H);
      q.eps = eps;
      q.k_out = kdst;
      q.v_out = vdst;
      q.kv_seq_stride = prB;
      q.kv_head_stride = static_cast<long long>(Nt) * 128;
      if (!q.k_norm) {
        ok = false;
        e2 = "missing " + pfx + ".ca.kn";
      }
      scatter(p, q);
    };

    // ---------------- prompt projection (cache.cpp:53-137 + build_condition text)
    Program& pp = plan->prog[0];
    // Block engines: [xv | xa | tv | ta] F32 in blk_in_.
    const float* blk_xv = blk_in_;
    const float* blk_xa = blk_in_ ? blk_in_ + static_cast<size_t>(V) * H : nullptr;
    const float* blk_tv = blk_xa ? blk_xa + static_cast<size_t>(1 + T) * E : nullptr;
    const float* blk_ta = blk_tv ? blk_tv + static_cast<size_t>(Nt) * H : nullptr;
    if (block) {
      // the experts' text hidden states are the inputs (no text embedders)
      K(pp, [=](cudaStream_t s) {
        launch_f32_to_bf16(blk_tv, text_v_, static_cast<long long>(Nt) * H, s);
        launch_f32_to_bf16(blk_ta, text_a_, static_cast<long long>(Nt) * E, s);
        return cudaGetLastError();
      });
      pp.ops.back().launches = 2;
      pp.kernels += 1;
    } else {
      K(pp, [=](cudaStream_t s) {
        launch_f32_to_bf16(in_prompt_, prompt_bf_, static_cast<long long>(b) * Nt * D, s);
        return cudaGetLastError();
      });
      G(pp, prompt_bf_, D, b * Nt, "gwp.acond.text.0", E, D, EPI_BIAS_GELU_R, true, nullptr, nullptr, 0, text_tmp_, E);
      G(pp, text_tmp_, E, b * Nt, "gwp.acond.text.1", E, E, EPI_BIAS, true, nullptr, nullptr, 0, text_a_, E);
      G(pp, prompt_bf_, D, b * Nt, "gwp.cond.text.0", H, D, EPI_BIAS_GELU_R, true, nullptr, nullptr, 0, text_tmp_, H);
      G(pp, text_tmp_, H, b * Nt, "gwp.cond.text.1", H, H, EPI_BIAS, true, nullptr, nullptr, 0, text_v_, H);
    }
    // An expert's ca.k / ca.vproj weights of all layers are one re-tiled
    // [L * 2H][tw] matrix (arena order, load_weights): the projection of the
    // prompt into every layer's K | V runs as one GEMM per chunk of
    // pkv_layers_ layers, then a norm / scatter per layer.
    auto pkv_block = [&](const char* xs, int tw, const bf16** wb, const bf16** bb) {
      const std::string p0 = std::string("gwp.blk.0") + xs;
      const bf16* w0 = W(p0 + ".ca.k.weight", static_cast<int64_t>(H) * tw);
      const bf16* b0 = W(p0 + ".ca.k.bias", H);
      if (!w0 || !b0) return false;
      for (int l = 0; l < L; ++l)
        for (int j = 0; j < 2; ++j) {
          const std::string nm = "gwp.blk." + std::to_string(l) + xs + (j ? ".ca.vproj" : ".ca.k");
          const size_t idx = static_cast<size_t>(2 * l + j);
          if (W(nm + ".weight", static_cast<int64_t>(H) * tw) != w0 + idx * H * tw ||
              W(nm + ".bias", H) != b0 + idx * H)
            return false;
        }
      *wb = w0;
      *bb = b0;
      return true;
    };
    const bf16 *pw[2] = {nullptr, nullptr}, *pb[2] = {nullptr, nullptr};
    const bool pkv_ok = pkv_ && !rowmajor_weights_ && H % 256 == 0 && E % 64 == 0 &&
                        pkv_block(".a", E, &pw[0], &pb[0]) && pkv_block(".v", H, &pw[1], &pb[1]);
    if (pkv_ok) {
      // Every layer's prompt k-norm weight, in a device table for the scatter.
      std::vector<const bf16*> knorms(2 * static_cast<size_t>(L), nullptr);
      for (int x = 0; x < 2; ++x)
        for (int l = 0; l < L; ++l) {
          const std::string pfx = "gwp.blk." + std::to_string(l) + (x ? ".v" : ".a");
          knorms[static_cast<size_t>(x) * L + l] = W(pfx + ".ca.kn.weight", H);
          if (!knorms[static_cast<size_t>(x) * L + l]) {
            ok = false;
            e2 = "missing " + pfx + ".ca.kn";
          }
        }
      if (ok && cudaMemcpy(knorm_tab_, knorms.data(), knorms.size() * sizeof(const bf16*),
                           cudaMemcpyHostToDevice) != cudaSuccess) {
        ok = false;
        e2 = "prompt k-norm table upload failed";
      }
      for (int x = 0; x < 2 && ok; ++x) {
        const bf16* text = x ? text_v_ : text_a_;
        const int tw = x ? H : E;
        const char* xs = x ? ".v" : ".a";
        for (int l0 = 0; l0 < L && ok; l0 += pkv_layers_) {
          const int l1 = std::min(L, l0 + pkv_layers_), nl = l1 - l0;
          for (int l = l0; l < l1 && ok; ++l)
            for (const char* proj : {".ca.k", ".ca.vproj"})
              if (!ensure_tiled("gwp.blk." + std::to_string(l) + xs + proj, H, tw, &e2)) ok = false;
          if (ok && !add_gemm(pp, text, tw, b * Nt, pw[x] + static_cast<size_t>(l0) * 2 * H * tw,
                              nl * 2 * H, tw, EPI_BIAS, pb[x] + static_cast<size_t>(l0) * 2 * H,
                              nullptr, nullptr, 0, pkv_, nl * 2 * H, true, false,
                              std::string("prompt projection") + xs, &e2))
            ok = false;
          if (ok) {
            // K-norm + head-major scatter of the chunk's layers in one launch.
            QkvScatter q{};
            q.src = pkv_;
            q.ld_src = nl * 2 * H;
            q.rows = b * Nt;
            q.rows_per_seq = Nt;
            q.hidden = H;
            q.heads = heads;
            q.q_col = -1;
            q.k_col = 0;
            q.v_col = H;
            q.k_norm = knorms[static_cast<size_t>(x) * L + l0];
            q.k_norms = knorm_tab_ + static_cast<size_t>(x) * L + l0;
            q.eps = eps;
            q.k_out = (x ? k_vis_ : k_prompt_) + l0 * prL;
            q.v_out = (x ? v_vis_ : v_prompt_) + l0 * prL;
            q.kv_seq_stride = prB;
            q.kv_head_stride = static_cast<long long>(Nt) * 128;
            q.layers = nl;
            q.src_layer_stride = 2 * static_cast<long long>(H);
            q.out_layer_stride = prL;
            scatter(pp, q);
          }
        }
      }
    } else {
      for (int l = 0; l < L && ok; ++l) {
        const std::string ap = "gwp.blk." + std::to_string(l) + ".a";
        const std::string vp = "gwp.blk." + std::to_string(l) + ".v";
        prompt_kv(pp, text_a_, E, ap, k_prompt_ + l * prL, v_prompt_ + l * prL);
        prompt_kv(pp, text_v_, H, vp, k_vis_ + l * prL, v_vis_ + l * prL);
      }
    }

    // ---------------- prefix (cache.cpp:139-485)
    Program& mp = plan->prog[1];
    if (block) {
      // state token (row 0 of xa), action tokens (rows 1..T) and visual tokens
      K(mp, [=](cudaStream_t s) {
        launch_f32_to_bf16(blk_xa, hs_, static_cast<long long>(E), s);
        launch_f32_to_bf16(blk_xa + E, ha_, static_cast<long long>(T) * E, s);
        launch_f32_to_bf16(blk_xv, hv_, static_cast<long long>(V) * H, s);
        return cudaGetLastError();
      });
      mp.ops.back().launches = 3;
      mp.kernels += 2;
    } else {
    K(mp, [=](cudaStream_t s) {
      launch_f32_to_bf16(in_state_, state_bf_, static_cast<long long>(b) * A, s);
      launch_f32_to_bf16(in_noise_, action_bf_, static_cast<long long>(b) * T * A, s);
      return cudaGetLastError();
    });
    mp.ops.back().launches = 2;
    mp.kernels += 1;
    {
      const bf16* w_in = W("gwp.state.in.weight", static_cast<int64_t>(g.num_embodiments) * A * 128);
      const bf16* b_in = W("gwp.state.in.bias", static_cast<int64_t>(g.num_embodiments) * 128);
      small(mp, state_bf_, b, A, w_in ? w_in + static_cast<size_t>(emb) * A * 128 : nullptr, 1, 128,
            b_in ? b_in + emb * 128 : nullptr, 128, ACT_GELU_ERF, s1_);
      small(mp, s1_, b, 128, W("gwp.state.mid.weight", 128 * 128), 128, 1,
            W("gwp.state.mid.bias", 128), 128, ACT_GELU_ERF, s2_);
      G(mp, s2_, 128, b, "gwp.state.out", E, 128, EPI_BIAS, true, nullptr, nullptr, 0, hs_, E);
    }
    K(mp, [=](cudaStream_t s) {
      launch_patchify(in_latent_, b, C, g.grid_h, g.grid_w, cols_, s);
      return cudaGetLastError();
    });
    G(mp, cols_, 4 * C, b * V, "gwp.patch", H, 4 * C, EPI_F32_BIAS, true, nullptr, nullptr, 0, hv_, H);
    }  // not block
    // conditioning MLPs: acond at t = 0 and every schedule timestep, cond at t = 0.
    G(mp, freq_bf_, 256, 1 + S, "gwp.acond.time.0", E, 256, EPI_BIAS_SILU, true, nullptr, nullptr, 0, ct1_, E);
    G(mp, ct1_, E, 1 + S, "gwp.acond.time.1", E, E, EPI_BIAS, true, nullptr, nullptr, 0, temb_a_, E);
    K(mp, [=](cudaStream_t s) {
      launch_silu(temb_a_, ct2_, (1 + S) * E, s);
      return cudaGetLastError();
    });
    G(mp, ct2_, E, 1 + S, "gwp.acond.time.out", 6 * E, E, EPI_BIAS, true, nullptr, nullptr, 0, mod_a_, 6 * E);
    G(mp, freq_bf_, 256, 1, "gwp.cond.time.0", H, 256, EPI_BIAS_SILU, true, nullptr, nullptr, 0, cv1_, H);
    G(mp, cv1_, H, 1, "gwp.cond.time.1", H, H, EPI_BIAS, true, nullptr, nullptr, 0, temb_v_, H);
    K(mp, [=](cudaStream_t s) {
      launch_silu(temb_v_, cv2_, H, s);
      return cudaGetLastError();
    });
    G(mp, cv2_, H, 1, "gwp.cond.time.out", 6 * H, H, EPI_BIAS, true, nullptr, nullptr, 0, mod_v_, 6 * H);
    K(mp, [=](cudaStream_t s) {
      launch_modulation_add(mod_a_, 6 * E, 6 * E, 1, tables_a_, L, 6 * E, comb_a0_, s);
      launch_modulation_add(mod_v_, 6 * H, 6 * H, 1, tables_v_, L, 6 * H, comb_v_, s);
      launch_modulation_add(mod_a_ + 6 * E, 6 * E, 6 * E, S, tables_a_, L, 6 * E, comb_steps_, s);
      launch_modulation_add(temb_a_ + E, E, E, S, tables_final_, 1, 2 * E, comb_final_, s);
      return cudaGetLastError();
    });
    mp.ops.back().launches = 4;
    mp.kernels += 3;
    fork_side(mp);  // the state lane starts from hs_ and the modulation tables
    for (int l = 0; l < L && ok; ++l) {
      const std::string ap = "gwp.blk." + std::to_string(l) + ".a";
      const std::string vp = "gwp.blk." + std::to_string(l) + ".v";
      const float* ca = comb_a0_ + static_cast<size_t>(l) * 6 * E;
      const float* cv = comb_v_ + static_cast<size_t>(l) * 6 * H;
      // Two lanes: the visual expert (768 tokens, tensor bound) stays on the main
      // stream, the state token's action-expert work (one token, weight
      // streaming) runs beside it on the side stream; they meet at the joint
      // self-attention, which needs both halves of the layer's K/V.
      auto scatter_part = [&](int x) {
        QkvScatter q{};
        const bool vis = x == 1;
        const std::string& pf = vis ? vp : ap;
        q.src = vis ? qkv_ : qkv_s_;
        q.ld_src = 3 * H;
        q.rows = vis ? b * V : b;
        q.rows_per_seq = vis ? V : 1;
        q.hidden = H;
        q.heads = heads;
        q.q_col = 0;
        q.k_col = H;
        q.v_col = 2 * H;
        q.q_norm = W(pf + ".sa.qn.weight", H);
        q.k_norm = W(pf + ".sa.kn.weight", H);
        q.eps = eps;
        q.rope_mode = vis ? 2 : 1;
        q.pos_base = 0;
        q.pos_thw = pos_thw_;
        q.inv_freq = vis ? inv_freq3_ : inv_freq1_;
        q.q_out = qbuf_;
        q.q_seq_stride = static_cast<long long>(heads) * P * 128;
        q.q_head_stride = static_cast<long long>(P) * 128;
        q.q_row_offset = vis ? 1 : 0;
        q.k_out = k_self_ + l * selfL;
        q.v_out = v_self_ + l * selfL;
        q.kv_seq_stride = selfB;
        q.kv_head_stride = static_cast<long long>(P + T) * 128;
        q.kv_row_offset = vis ? 1 : 0;
        if (!q.q_norm || !q.k_norm) {
          ok = false;
          e2 = "missing q/k norm of " + pf;
        }
        scatter(mp, q);
      };
      mp.lane = 1;
      ln_mod(mp, hs_, b, E, ca + E, ca, nrm_s_);
      G(mp, nrm_s_, E, b, ap + ".sa.qkv", 3 * H, E, EPI_BIAS, true, nullptr, nullptr, 0, qkv_s_, 3 * H);
      scatter_part(0);
      mp.lane = 0;
      ln_mod(mp, hv_, b * V, H, cv + H, cv, nrm_);
      G(mp, nrm_, H, b * V, vp + ".sa.qkv", 3 * H, H, EPI_BIAS, true, nullptr, nullptr, 0, qkv_, 3 * H);
      scatter_part(1);
      join_side(mp);
      if (l + 1 == L && !block) break;  // the last layer's outputs feed no cached K/V
      AttnArgs at{};
      at.q = qbuf_;
      at.q_seq_stride = static_cast<long long>(heads) * P * 128;
      at.q_head_stride = static_cast<long long>(P) * 128;
      at.k = k_self_ + l * selfL;
      at.v = v_self_ + l * selfL;
      at.kv_seq_stride = selfB;
      at.kv_head_stride = static_cast<long long>(P + T) * 128;
      at.lq = P;
      at.lk = P;
      at.heads = heads;
      at.batch = b;
      at.scale = 1.0f / std::sqrt(128.0f);
      at.out = att_;
      at.ldo = H;
      at.out_first = att_s_;
      at.ldo_first = H;
      at.split_first = 1;
      attend(mp, at);
      fork_side(mp);
      G(mp, att_, H, b * V, vp + ".sa.o", H, H, EPI_GATED_RES, true, cv + 2 * H, hv_, H, hv_, H);
      // visual expert: cross attention over its text K/V, FFN
      ln_aff(mp, hv_, b * V, H, vp + ".ca_norm", nrm_);
      G(mp, nrm_, H, b * V, vp + ".ca.q", H, H, EPI_BIAS, true, nullptr, nullptr, 0, cq_, H);
      cross_q(mp, cq_, b * V, V, vp, qc_);
      AttnArgs cx{};
      cx.q = qc_;
      cx.q_seq_stride = static_cast<long long>(heads) * V * 128;
      cx.q_head_stride = static_cast<long long>(V) * 128;
      cx.k = k_vis_ + l * prL;
      cx.v = v_vis_ + l * prL;
      cx.kv_seq_stride = prB;
      cx.kv_head_stride = static_cast<long long>(Nt) * 128;
      cx.lq = V;
      cx.lk = Nt;
      cx.static_keys = Nt;  // prompt K/V, projected before the prefix
      cx.heads = heads;
      cx.batch = b;
      cx.scale = 1.0f / std::sqrt(128.0f);
      cx.out = catt_;
      cx.ldo = H;
      attend(mp, cx);
      G(mp, catt_, H, b * V, vp + ".ca.o", H, H, EPI_RES, true, nullptr, hv_, H, hv_, H);
      ln_mod(mp, hv_, b * V, H, cv + 4 * H, cv + 3 * H, nrm_);
      ffn_in(mp, nrm_, H, b * V, vp, Fv, H, ffn_);
      G(mp, ffn_, Fv, b * V, vp + ".ffn.out", H, Fv, EPI_GATED_RES, true, cv + 5 * H, hv_, H, hv_, H);
      mp.lane = 1;
      G(mp, att_s_, H, b, ap + ".sa.o", E, H, EPI_GATED_RES, true, ca + 2 * E, hs_, E, hs_, E);
      // state token (action expert): cross attention over the prompt K/V, FFN
      ln_aff(mp, hs_, b, E, ap + ".ca_norm", nrm_s_);
      G(mp, nrm_s_, E, b, ap + ".ca.q", H, E, EPI_BIAS, true, nullptr, nullptr, 0, cq_s_, H);
      cross_q(mp, cq_s_, b, 1, ap, qc_s_);
      AttnArgs cs = cx;
      cs.q = qc_s_;
      cs.q_seq_stride = static_cast<long long>(heads) * 128;
      cs.q_head_stride = 128;
      cs.k = k_prompt_ + l * prL;
      cs.v = v_prompt_ + l * prL;
      cs.lq = 1;
      cs.out = catt_s_;
      attend(mp, cs);
      G(mp, catt_s_, H, b, ap + ".ca.o", E, H, EPI_RES, true, nullptr, hs_, E, hs_, E);
      ln_mod(mp, hs_, b, E, ca + 4 * E, ca + 3 * E, nrm_s_);
      ffn_in(mp, nrm_s_, E, b, ap, Fa, E, ffn_s_);
      G(mp, ffn_s_, Fa, b, ap + ".ffn.out", E, Fa, EPI_GATED_RES, true, ca + 5 * E, hs_, E, hs_, E);
      mp.lane = 0;
    }
    if (block) join_side(mp);  // the state token's last layer ran on the side lane
    // ---------------- denoise (mot.cpp:358-496, unrolled over the schedule)
    Program& dp = plan->prog[2];
    const bf16* ain_w = W("gwp.action.in.weight", static_cast<int64_t>(g.num_embodiments) * A * 128);
    const bf16* ain_b = W("gwp.action.in.bias", static_cast<int64_t>(g.num_embodiments) * 128);
    const bf16* dout_w = W("gwp.decode.out.weight", static_cast<int64_t>(g.num_embodiments) * 128 * A);
    const bf16* dout_b = W("gwp.decode.out.bias", static_cast<int64_t>(g.num_embodiments) * A);
    for (int s = 0; s < S && ok; ++s) {
      const int M = b * T;
      if (!block) {  // block engines take the action tokens' hidden states as input
        small(dp, action_bf_, M, A, ain_w ? ain_w + static_cast<size_t>(emb) * A * 128 : nullptr, 1,
              128, ain_b ? ain_b + emb * 128 : nullptr, 128, ACT_GELU_ERF, e1_);
        small(dp, e1_, M, 128, W("gwp.action.mid.weight", 128 * 128), 128, 1,
              W("gwp.action.mid.bias", 128), 128, ACT_GELU_ERF, e2_);
        G(dp, e2_, 128, M, "gwp.action.out", E, 128, EPI_BIAS, true, nullptr, nullptr, 0, ha_, E);
      }
      for (int l = 0; l < L && ok; ++l) {
        const std::string ap = "gwp.blk." + std::to_string(l) + ".a";
        const float* c = comb_steps_ + (static_cast<size_t>(s) * L + l) * 6 * E;
        ln_mod(dp, ha_, M, E, c + E, c, nrm_);
        G(dp, nrm_, E, M, ap + ".sa.qkv", 3 * H, E, EPI_BIAS, true, nullptr, nullptr, 0, qkv_, 3 * H);
        QkvScatter q{};
        q.src = qkv_;
        q.ld_src = 3 * H;
        q.rows = M;
        q.rows_per_seq = T;
        q.hidden = H;
        q.heads = heads;
        q.q_col = 0;
        q.k_col = H;
        q.v_col = 2 * H;
        q.q_norm = W(ap + ".sa.qn.weight", H);
        q.k_norm = W(ap + ".sa.kn.weight", H);
        q.eps = eps;
        q.rope_mode = 1;
        q.pos_base = 1;  // action_positions(tokens, false) = 1..T (semantics.cpp:210-222)
        q.inv_freq = inv_freq1_;
        q.q_out = qbuf_;
        q.q_seq_stride = static_cast<long long>(heads) * T * 128;
        q.q_head_stride = static_cast<long long>(T) * 128;
        q.k_out = k_self_ + l * selfL;
        q.v_out = v_self_ + l * selfL;
        q.kv_seq_stride = selfB;
        q.kv_head_stride = static_cast<long long>(P + T) * 128;
        q.kv_row_offset = P;
        scatter(dp, q);
        AttnArgs at{};
        at.q = qbuf_;
        at.q_seq_stride = q.q_seq_stride;
        at.q_head_stride = q.q_head_stride;
        at.k = k_self_ + l * selfL;
        at.v = v_self_ + l * selfL;
        at.kv_seq_stride = selfB;
        at.kv_head_stride = q.kv_head_stride;
        at.lq = T;
        at.lk = P + T;
        at.static_keys = P;  // prefix rows; this layer's scatter writes rows P..P+T
        at.heads = heads;
        at.batch = b;
        at.scale = 1.0f / std::sqrt(128.0f);
        at.out = att_;
        at.ldo = H;
        attend(dp, at);
        G(dp, att_, H, M, ap + ".sa.o", E, H, EPI_GATED_RES, true, c + 2 * E, ha_, E, ha_, E);
        ln_aff(dp, ha_, M, E, ap + ".ca_norm", nrm_);
        G(dp, nrm_, E, M, ap + ".ca.q", H, E, EPI_BIAS, true, nullptr, nullptr, 0, cq_, H);
        cross_q(dp, cq_, M, T, ap, qc_);
        AttnArgs cx{};
        cx.q = qc_;
        cx.q_seq_stride = static_cast<long long>(heads) * T * 128;
        cx.q_head_stride = static_cast<long long>(T) * 128;
        cx.k = k_prompt_ + l * prL;
        cx.v = v_prompt_ + l * prL;
        cx.kv_seq_stride = prB;
        cx.kv_head_stride = static_cast<long long>(Nt) * 128;
        cx.lq = T;
        cx.lk = Nt;
        cx.static_keys = Nt;  // prompt K/V, projected before the prefix
        cx.heads = heads;
        cx.batch = b;
        cx.scale = at.scale;
        cx.out = catt_;
        cx.ldo = H;
        attend(dp, cx);
        G(dp, catt_, H, M, ap + ".ca.o", E, H, EPI_RES, true, nullptr, ha_, E, ha_, E);
        ln_mod(dp, ha_, M, E, c + 4 * E, c + 3 * E, nrm_);
        ffn_in(dp, nrm_, E, M, ap, Fa, E, ffn_);
        G(dp, ffn_, Fa, M, ap + ".ffn.out", E, Fa, EPI_GATED_RES, true, c + 5 * E, ha_, E, ha_, E);
      }
      if (block) break;  // one layer, no decoder / Euler step
      const float* cf = comb_final_ + static_cast<size_t>(s) * 2 * E;
      // the final head's modulated norm is the reference's LayerNorm in every variant
      p_ln_final(dp, ha_, M, E, cf + E, cf, nrm_);
      G(dp, nrm_, E, M, "gwp.decode.in", 128, E, EPI_BIAS_GELU_ERF, true, nullptr, nullptr, 0, d1_, 128);
      small(dp, d1_, M, 128, W("gwp.decode.mid.weight", 128 * 128), 128, 1,
            W("gwp.decode.mid.bias", 128), 128, ACT_GELU_ERF, d2_);
      bf16* vel = vel_ + static_cast<size_t>(s) * opt_.max_batch * T * A;
      small(dp, d2_, M, 128, dout_w ? dout_w + static_cast<size_t>(emb) * 128 * A : nullptr, 1, A,
            dout_b ? dout_b + emb * A : nullptr, A, ACT_NONE, vel);
      const float* dts = dt_ + s;
      K(dp, [=](cudaStream_t st) {
        launch_euler(action_bf_, vel, M * A, dts, st);
        return cudaGetLastError();
      });
    }
    if (block) {
      float* ov = blk_out_;
      float* oa = blk_out_ ? blk_out_ + static_cast<size_t>(V) * H : nullptr;
      K(dp, [=](cudaStream_t s) {
        launch_bf16_to_f32(hv_, ov, static_cast<long long>(V) * H, s);
        launch_bf16_to_f32(hs_, oa, static_cast<long long>(E), s);
        launch_bf16_to_f32(ha_, oa + E, static_cast<long long>(T) * E, s);
        return cudaGetLastError();
      });
      dp.ops.back().launches = 3;
      dp.kernels += 2;
    } else {
      K(dp, [=](cudaStream_t s) {
        launch_bf16_to_f32(action_bf_, d_out_, static_cast<long long>(b) * T * A, s);
        return cudaGetLastError();
      });
    }
    if (!ok) {
      if (e2 == "__rebuild__") continue;  // scratch grew: rebuild with the new pointers
      *err = e2;
      return false;
    }
    plan->scratch_gen = scratch_gen_;
    // Plans built against an older split-K scratch hold freed pointers.
    for (auto it = plans_.begin(); it != plans_.end();) {
      if (it->second->scratch_gen != scratch_gen_) {
        for (auto& gx : it->second->graph)
          if (gx) cudaGraphExecDestroy(gx);
        it = plans_.erase(it);
      } else {
        ++it;
      }
    }
    if (retile_tmp_) {  // weights re-tiled while planning; the staging copy is no longer needed
      CK(cudaStreamSynchronize(stream_));
      cudaFree(retile_tmp_);
      retile_tmp_ = nullptr;
      retile_tmp_elems_ = 0;
    }
    if (opt_.graphs) {
      for (int which = 0; which < 3; ++which) {
        Program& p = plan->prog[which];
        cudaGraph_t graph = nullptr;
        CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        cudaError_t le = cudaSuccess;
        for (auto& op : p.ops) {
          le = op.fn(op.lane ? side_ : stream_);
          if (le != cudaSuccess) break;
        }
        cudaError_t ce = cudaStreamEndCapture(stream_, &graph);
        if (le != cudaSuccess || ce != cudaSuccess) {
          if (graph) cudaGraphDestroy(graph);
          *err = std::string("graph capture: ") + cudaGetErrorString(le != cudaSuccess ? le : ce);
          return false;
        }
        cudaGraphExec_t exec = nullptr;
        cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) {
          *err = std::string("graph instantiate: ") + cudaGetErrorString(ie);
          return false;
        }
        plan->graph[which] = exec;
      }
    }
    plans_[b] = std::move(plan);
    return true;
  }
  *err = "could not size the split-K scratch";
  return false;
}

void MotEngine::drop_plans() {
  for (auto& kv : plans_)
    for (auto& gx : kv.second->graph)
      if (gx) cudaGraphExecDestroy(gx);
  plans_.clear();
}

int MotEngine::kernels_per_chunk(int batch, bool with_prompt) {
  std::string err;
  auto it = plans_.find(batch);
  if (it == plans_.end() || it->second->scratch_gen != scratch_gen_) {
    if (!build(batch, &err)) return -1;
    it = plans_.find(batch);
  }
  return it->second->prog[1].kernels + it->second->prog[2].kernels +
         (with_prompt ? it->second->prog[0].kernels : 0);
}

bool MotEngine::stage(const RequestView* reqs, int batch, std::string* err) {
  if (opt_.block) {
    *err = "a block engine runs wam_b200_block_forward only (no action-chunk requests)";
    return false;
  }
  const Geometry& g = g_;
  if (!ok_) {
    *err = "engine is not initialised";
    return false;
  }
  if (batch < 1 || batch > opt_.max_batch) {
    *err = "batch must be in [1, max_batch]";
    return false;
  }
  const int A = g.action_dim, T = g.action_chunk, Nt = g.prompt_tokens, D = g.text_dim;
  const long long lat = static_cast<long long>(g.vae_z) * 4 * g.visual();
  // The previous batch's copies out of the pinned buffers have completed.
  if (h2d_ev_) CK(cudaEventSynchronize(h2d_ev_));
  staged_keys_.assign(batch, {});
  for (int i = 0; i < batch; ++i) {
    const RequestView& r = reqs[i];
    if (!r.state || r.state_n < g.real_state_dim) {
      *err = "state is required (real_state_dim values)";
      return false;
    }
    for (int d = 0; d < g.real_state_dim; ++d)
      if (!std::isfinite(r.state[d])) {
        *err = "state contains NaN/Inf";
        return false;
      }
    const bool from_images = !r.latent && r.n_images > 0;
    if (from_images) {
      if (!vae_) {
        *err = "camera images need an engine created with the VAE encoder (options.vae = 1)";
        return false;
      }
      if (r.n_images != 3) {
        *err = "exactly three input images are required";
        return false;
      }
    } else if (!r.latent || r.latent_n != lat) {
      *err = "reference latent must have vae_z * (2 grid_h) * (2 grid_w) values";
      return false;
    }
    std::vector<uint8_t>& key = staged_keys_[i];
    if (!r.prompt && r.tokens) {
      if (!t5_) {
        *err = "prompt token ids need an engine created with the UMT5 encoder (options.t5 = 1)";
        return false;
      }
      std::string why;
      const int valid = t5_valid_tokens(r.n_tokens, r.mask, r.mask_n, Nt, &why);
      if (valid < 0) {
        *err = why;
        return false;
      }
      for (int j = 0; j < valid; ++j)
        if (r.tokens[j] < 0 || r.tokens[j] >= t5_->geometry().vocab) {
          *err = "token " + std::to_string(r.tokens[j]) + " is outside T5 vocabulary";
          return false;
        }
      key.assign(1, 'T');
      const uint8_t* tb = reinterpret_cast<const uint8_t*>(r.tokens);
      key.insert(key.end(), tb, tb + static_cast<size_t>(valid) * 4);
    } else if (!r.prompt || r.prompt_tokens < 1 || r.prompt_tokens > Nt) {
      *err = "prompt embedding must have 1..prompt_tokens rows";
      return false;
    }
    normalize_state(r.state, g.real_state_dim, A, sq01_.data(), sq99_.data(),
                    h_state_ + static_cast<size_t>(i) * A);
    if (!from_images) {
      std::memcpy(h_latent_ + i * lat, r.latent, lat * 4);
      for (long long j = 0; j < lat; ++j)
        if (!std::isfinite(h_latent_[i * lat + j])) {
          *err = "reference latent contains NaN/Inf";
          return false;
        }
    }
    if (r.prompt) {
      // The slot's pinned buffer keeps the last prompt staged through it. With
      // the projected-prompt cache, an unchanged prompt (compared byte for
      // byte) keeps the slot's version, which is its cache key; any other
      // prompt is copied in under a new version. (The device copy below runs
      // for every request either way.)
      // The host copy itself runs below, in pieces overlapped with their
      // device copies.
      float* pr = h_prompt_ + static_cast<size_t>(i) * Nt * D;
      const size_t nb = static_cast<size_t>(r.prompt_tokens) * D * 4;
      const bool same = opt_.prompt_cache && h_prompt_ver_[i] != 0 &&
                        h_prompt_rows_[i] == r.prompt_tokens && std::memcmp(pr, r.prompt, nb) == 0;
      prompt_copy_[i] = !same;
      if (!same) {
        h_prompt_ver_[i] = prompt_ver_next_++;
        h_prompt_rows_[i] = r.prompt_tokens;
      }
      key.assign(1, 'E');
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(&h_prompt_ver_[i]);
      key.insert(key.end(), vb, vb + sizeof(uint64_t));
    }
    float* nz = h_noise_ + static_cast<size_t>(i) * T * A;
    if (r.noise) {
      std::memcpy(nz, r.noise, static_cast<size_t>(T) * A * 4);
      for (int j = 0; j < T * A; ++j)
        if (!std::isfinite(nz[j])) {
          *err = "action noise contains NaN/Inf";
          return false;
        }
    } else {
      std::normal_distribution<float> normal(0.0f, 1.0f);
      for (int j = 0; j < T * A; ++j) nz[j] = normal(rng_);
    }
  }
  CK(cudaMemcpyAsync(in_state_, h_state_, static_cast<size_t>(batch) * A * 4, cudaMemcpyHostToDevice, stream_));
  // Latents: copied from the host, or made on the device from the views
  // (stage 1 + the captured VAE encoder, writing the request's latent slot).
  for (int i = 0; i < batch; ++i) {
    float* dst = in_latent_ + static_cast<size_t>(i) * lat;
    if (reqs[i].latent) {
      CK(cudaMemcpyAsync(dst, h_latent_ + static_cast<size_t>(i) * lat, lat * 4,
                         cudaMemcpyHostToDevice, stream_));
    } else {
      std::string verr;
      if (!vae_->encode_images(reqs[i].images, 3, dst, stream_, &verr)) {
        *err = "VAE encoder: " + verr;
        return false;
      }
    }
  }
  // Prompt embeddings: copied from the host, or (token ids) made by UMT5 on the
  // device, skipped when the slot already holds that prompt's embedding.
  for (int i = 0; i < batch; ++i) {
    const size_t pn = static_cast<size_t>(Nt) * D;
    if (reqs[i].prompt) {
      float* pr = h_prompt_ + i * pn;
      if (prompt_copy_[i]) {
        // 1 MB pieces: each piece's DMA runs while the next one is copied
        // into the pinned slot (no earlier copy reads the slot any more:
        // h2d_ev_ was waited for above).
        const size_t rows_b = static_cast<size_t>(reqs[i].prompt_tokens) * D * 4;
        const size_t piece = size_t(1) << 20;
        for (size_t off = 0; off < pn * 4; off += piece) {
          const size_t len = pn * 4 - off < piece ? pn * 4 - off : piece;
          uint8_t* dst = reinterpret_cast<uint8_t*>(pr) + off;
          if (off + len <= rows_b) {
            std::memcpy(dst, reinterpret_cast<const uint8_t*>(reqs[i].prompt) + off, len);
          } else if (off >= rows_b) {
            std::memset(dst, 0, len);
          } else {
            std::memcpy(dst, reinterpret_cast<const uint8_t*>(reqs[i].prompt) + off, rows_b - off);
            std::memset(dst + (rows_b - off), 0, off + len - rows_b);
          }
          CK(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(in_prompt_ + i * pn) + off, dst, len,
                             cudaMemcpyHostToDevice, stream_));
        }
      } else {
        CK(cudaMemcpyAsync(in_prompt_ + i * pn, pr, pn * 4, cudaMemcpyHostToDevice, stream_));
      }
      in_prompt_key_[i].clear();
    } else if (in_prompt_key_[i] != staged_keys_[i]) {
      std::string terr;
      const int valid = static_cast<int>((staged_keys_[i].size() - 1) / 4);
      if (!t5_->encode(reinterpret_cast<const int32_t*>(staged_keys_[i].data() + 1), valid,
                       in_prompt_ + i * pn, stream_, &terr)) {
        *err = "UMT5 encoder: " + terr;
        in_prompt_key_[i].clear();
        return false;
      }
      in_prompt_key_[i] = staged_keys_[i];
    }
  }
  CK(cudaMemcpyAsync(in_noise_, h_noise_, static_cast<size_t>(batch) * T * A * 4, cudaMemcpyHostToDevice, stream_));
  if (!h2d_ev_) CK(cudaEventCreateWithFlags(&h2d_ev_, cudaEventDisableTiming));
  CK(cudaEventRecord(h2d_ev_, stream_));
  staged_batch_ = batch;
  return true;
}

bool MotEngine::run(int batch, std::string* err, EngineStats* stats) {
  if (batch != staged_batch_) {
    *err = "run() batch differs from the staged batch";
    return false;
  }
  auto it = plans_.find(batch);
  if (it == plans_.end() || it->second->scratch_gen != scratch_gen_) {
    if (!build(batch, err)) return false;
    it = plans_.find(batch);
  }
  Plan& plan = *it->second;
  // Projected-prompt cache (cache.cpp:53-68): skip the projection when every
  // slot's prompt equals the one projected last time.
  bool hit = opt_.prompt_cache && prompt_valid_;
  const size_t pn = static_cast<size_t>(g_.prompt_tokens) * g_.text_dim;
  for (int i = 0; i < batch && hit; ++i) hit = prompt_key_[i] == staged_keys_[i];
  (void)pn;
  auto exec = [&](int which) -> bool {
    if (plan.graph[which]) {
      CK(cudaGraphLaunch(plan.graph[which], stream_));
      return true;
    }
    for (auto& op : plan.prog[which].ops) CK(op.fn(op.lane ? side_ : stream_));
    return true;
  };
  if (!phase_ev_[0])
    for (auto& e : phase_ev_) CK(cudaEventCreate(&e));
  CK(cudaEventRecord(phase_ev_[0], stream_));
  phase_prompt_ran_ = !hit;
  if (!hit) {
    if (!exec(0)) return false;
    if (opt_.prompt_cache) {
      for (int i = 0; i < batch; ++i) prompt_key_[i] = staged_keys_[i];
      for (int i = batch; i < opt_.max_batch; ++i) prompt_key_[i].clear();
      prompt_valid_ = true;
    }
  }
  if (stats) stats->prompt_cache_hit = hit ? 1 : 0;
  CK(cudaEventRecord(phase_ev_[1], stream_));
  if (!exec(1)) return false;
  CK(cudaEventRecord(phase_ev_[2], stream_));
  if (!exec(2)) return false;
  CK(cudaEventRecord(phase_ev_[3], stream_));
  return true;
}

bool MotEngine::last_phase_ms(float* prompt, float* prefix, float* denoise) {
  if (!phase_ev_[0] || cudaEventSynchronize(phase_ev_[3]) != cudaSuccess) return false;
  cudaEventElapsedTime(prompt, phase_ev_[0], phase_ev_[1]);
  cudaEventElapsedTime(prefix, phase_ev_[1], phase_ev_[2]);
  cudaEventElapsedTime(denoise, phase_ev_[2], phase_ev_[3]);
  return true;
}

bool MotEngine::profile(int batch, std::vector<OpProfile>* out, std::string* err) {
  if (batch != staged_batch_) {
    *err = "profile() batch differs from the staged batch";
    return false;
  }
  auto it = plans_.find(batch);
  if (it == plans_.end() || it->second->scratch_gen != scratch_gen_) {
    if (!build(batch, err)) return false;
    it = plans_.find(batch);
  }
  Plan& plan = *it->second;
  // Every op runs alone on the main stream, timed by a pair of events; the
  // lane hand-offs are skipped.
  size_t n = 0;
  for (auto& p : plan.prog)
    for (auto& op : p.ops) n += op.kind != OP_SYNC;
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto& e : ev) CK(cudaEventCreate(&e));
  size_t i = 0;
  CK(cudaEventRecord(ev[0], stream_));
  for (auto& p : plan.prog)
    for (auto& op : p.ops) {
      if (op.kind == OP_SYNC) continue;
      CK(op.fn(stream_));
      CK(cudaEventRecord(ev[++i], stream_));
    }
  CK(cudaStreamSynchronize(stream_));
  out->clear();
  i = 0;
  for (int ph = 0; ph < 3; ++ph)
    for (auto& op : plan.prog[ph].ops) {
      if (op.kind == OP_SYNC) continue;
      OpProfile r{ph, op.kind, op.launches, 0.0f, op.bytes, op.flops,
                  {op.shape[0], op.shape[1], op.shape[2], op.shape[3]}};
      cudaEventElapsedTime(&r.ms, ev[i], ev[i + 1]);
      out->push_back(r);
      ++i;
    }
  for (auto& e : ev) cudaEventDestroy(e);
  return true;
}

bool MotEngine::profile_graph(int batch, int phase, int kind, int lane, int reps, float* ms,
                              double* bytes,
                              double* flops, int* launches, std::string* err) {
  if (batch != staged_batch_) {
    *err = "profile_graph() batch differs from the staged batch";
    return false;
  }
  if (phase < 0 || phase > 2 || reps < 1) {
    *err = "profile_graph(): phase 0..2 and reps >= 1";
    return false;
  }
  auto it = plans_.find(batch);
  if (it == plans_.end() || it->second->scratch_gen != scratch_gen_) {
    if (!build(batch, err)) return false;
    it = plans_.find(batch);
  }
  Program& p = it->second->prog[phase];
  *bytes = 0.0;
  *flops = 0.0;
  *launches = 0;
  cudaGraph_t graph = nullptr;
  CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
  cudaError_t le = cudaSuccess;
  for (auto& op : p.ops) {
    if (op.kind != kind || (lane >= 0 && op.lane != lane)) continue;
    le = op.fn(stream_);  // every lane on the main stream: one chain of launches
    if (le != cudaSuccess) break;
    *bytes += op.bytes;
    *flops += op.flops;
    *launches += op.launches;
  }
  cudaError_t ce = cudaStreamEndCapture(stream_, &graph);
  if (le != cudaSuccess || ce != cudaSuccess || !graph) {
    if (graph) cudaGraphDestroy(graph);
    *err = std::string("profile_graph capture: ") + cudaGetErrorString(le != cudaSuccess ? le : ce);
    return false;
  }
  cudaGraphExec_t exec = nullptr;
  ce = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ce != cudaSuccess) {
    *err = std::string("profile_graph instantiate: ") + cudaGetErrorString(ce);
    return false;
  }
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  ce = cudaEventCreate(&e0);
  if (ce == cudaSuccess) ce = cudaEventCreate(&e1);
  if (ce == cudaSuccess) ce = cudaGraphLaunch(exec, stream_);  // warm-up replay
  if (ce == cudaSuccess) ce = cudaEventRecord(e0, stream_);
  for (int r = 0; r < reps && ce == cudaSuccess; ++r) ce = cudaGraphLaunch(exec, stream_);
  if (ce == cudaSuccess) ce = cudaEventRecord(e1, stream_);
  if (ce == cudaSuccess) ce = cudaEventSynchronize(e1);
  float total = 0.0f;
  if (ce == cudaSuccess) ce = cudaEventElapsedTime(&total, e0, e1);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaGraphExecDestroy(exec);
  if (ce != cudaSuccess) {
    *err = std::string("profile_graph replay: ") + cudaGetErrorString(ce);
    return false;
  }
  *ms = total / reps;
  return true;
}

bool MotEngine::fetch(const RequestView* reqs, int batch, float* out, std::string* err) {
  const Geometry& g = g_;
  const int A = g.action_dim, T = g.action_chunk, R = g.real_action_dim;
  CK(cudaMemcpyAsync(h_out_, d_out_, static_cast<size_t>(batch) * T * A * 4, cudaMemcpyDeviceToHost, stream_));
  unsigned code = 0;
  CK(cudaMemcpyAsync(&code, err_word_, 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  if (code != 0) {
    cudaMemsetAsync(err_word_, 0, 4, stream_);
    cudaStreamSynchronize(stream_);
    *err = "device pipeline wait timed out (code " + std::to_string(code) + ")";
    return false;
  }
  for (size_t j = 0; j < static_cast<size_t>(batch) * T * A; ++j)
    if (!std::isfinite(h_out_[j])) {
      *err = "non-finite action output";
      return false;
    }
  for (int i = 0; i < batch; ++i)
    postprocess_action(h_out_ + static_cast<size_t>(i) * T * A, T, A, R, aq01_.data(), aq99_.data(),
                       reqs[i].state, out + static_cast<size_t>(i) * T * R);
  return true;
}

bool MotEngine::block_forward(const float* xv, const float* xa, const float* tv, const float* ta,
                              float t, float* ov, float* oa, float* device_ms, std::string* err) {
  if (!opt_.block || !blk_in_) {
    *err = "block_forward needs an engine created for block runs";
    return false;
  }
  if (!xv || !xa || !tv || !ta || !ov || !oa || !std::isfinite(t) || t < 0.0f) {
    *err = "block_forward: inputs, outputs and a finite timestep >= 0 are required";
    return false;
  }
  const Geometry& g = g_;
  const size_t V = g.visual(), H = g.hidden, E = g.action_hidden, T = g.action_chunk;
  const size_t Nt = g.prompt_tokens;
  const size_t nxv = V * H, nxa = (1 + T) * E, ntv = Nt * H, nta = Nt * E;
  CK(cudaMemcpyAsync(blk_in_, xv, nxv * 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(blk_in_ + nxv, xa, nxa * 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(blk_in_ + nxv + nxa, tv, ntv * 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(blk_in_ + nxv + nxa + ntv, ta, nta * 4, cudaMemcpyHostToDevice, stream_));
  // Row 1 of the timestep frequencies conditions the action tokens (row 0,
  // t = 0, the state and visual tokens).
  std::vector<float> f(256);
  timestep_embedding(t, 256, f.data());
  CK(cudaMemcpyAsync(freq_f32_ + 256, f.data(), 256 * 4, cudaMemcpyHostToDevice, stream_));
  launch_f32_to_bf16(freq_f32_ + 256, freq_bf_ + 256, 256, stream_);
  CK(cudaGetLastError());
  staged_batch_ = 1;
  if (!run(1, err)) return false;
  CK(cudaMemcpyAsync(ov, blk_out_, nxv * 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaMemcpyAsync(oa, blk_out_ + nxv, nxa * 4, cudaMemcpyDeviceToHost, stream_));
  unsigned code = 0;
  CK(cudaMemcpyAsync(&code, err_word_, 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  if (code != 0) {
    cudaMemsetAsync(err_word_, 0, 4, stream_);
    cudaStreamSynchronize(stream_);
    *err = "device pipeline wait timed out (code " + std::to_string(code) + ")";
    return false;
  }
  if (device_ms) {
    float a = 0.0f, b = 0.0f, c = 0.0f;
    last_phase_ms(&a, &b, &c);
    *device_ms = a + b + c;
  }
  return true;
}

bool MotEngine::predict(const RequestView* reqs, int batch, float* out, EngineStats* stats,
                        std::string* err) {
  using clk = std::chrono::steady_clock;
  const auto t0 = clk::now();
  bool ok = stage(reqs, batch, err);
  if (ok) ok = run(batch, err, stats);
  if (ok) ok = fetch(reqs, batch, out, err);
  if (ok && stats) {
    last_phase_ms(&stats->ms_prompt, &stats->ms_prefix, &stats->ms_denoise);
    stats->ms_total = std::chrono::duration<float, std::milli>(clk::now() - t0).count();
  }
  return ok;
}

void MotEngine::reset() {
  // Session reset (Gwp05ModelArch::reset, engine.cpp:89-97): forget the
  // projected prompt so the next request re-projects it.
  prompt_valid_ = false;
  for (auto& s : prompt_key_) s.clear();
}

bool MotEngine::read_tensor(const std::string& name, int slot, int layer, float* out, size_t n,
                            std::string* err) {
  const Geometry& g = g_;
  const int heads = g.heads, P = g.prefix(), T = g.action_chunk, Nt = g.prompt_tokens, L = g.layers;
  const int A = g.action_dim, S = g.steps;
  if (slot < 0 || slot >= opt_.max_batch || layer < 0 || layer >= L) {
    *err = "slot or layer out of range";
    return false;
  }
  std::vector<bf16> tmp;
  auto gather = [&](const bf16* base, long long slot_stride, long long layer_stride,
                    long long head_stride, int rows) -> bool {
    const size_t need = static_cast<size_t>(heads) * rows * 128;
    if (n < need) {
      *err = "output buffer too small";
      return false;
    }
    tmp.resize(need);
    for (int h = 0; h < heads; ++h) {
      const bf16* src = base + slot * slot_stride + layer * layer_stride + h * head_stride;
      CK(cudaMemcpyAsync(tmp.data() + static_cast<size_t>(h) * rows * 128, src,
                         static_cast<size_t>(rows) * 128 * 2, cudaMemcpyDeviceToHost, stream_));
    }
    CK(cudaStreamSynchronize(stream_));
    for (size_t i = 0; i < need; ++i) out[i] = __bfloat162float(tmp[i]);
    return true;
  };
  const long long selfL = static_cast<long long>(heads) * (P + T) * 128, prL = static_cast<long long>(heads) * Nt * 128;
  if (name == "prefix_k") return gather(k_self_, selfL * L, selfL, (P + T) * 128LL, P);
  if (name == "prefix_v") return gather(v_self_, selfL * L, selfL, (P + T) * 128LL, P);
  if (name == "prompt_k") return gather(k_prompt_, prL * L, prL, Nt * 128LL, Nt);
  if (name == "prompt_v") return gather(v_prompt_, prL * L, prL, Nt * 128LL, Nt);
  if (name == "velocity") {
    const size_t need = static_cast<size_t>(S) * T * A;
    if (n < need) {
      *err = "output buffer too small";
      return false;
    }
    tmp.resize(need);
    for (int s = 0; s < S; ++s)
      CK(cudaMemcpyAsync(tmp.data() + static_cast<size_t>(s) * T * A,
                         vel_ + (static_cast<size_t>(s) * opt_.max_batch + slot) * T * A,
                         static_cast<size_t>(T) * A * 2, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    for (size_t i = 0; i < need; ++i) out[i] = __bfloat162float(tmp[i]);
    return true;
  }
  *err = "unknown tensor " + name;
  return false;
}

}  // namespace wamb
