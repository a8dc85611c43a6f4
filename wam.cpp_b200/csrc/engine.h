// B200 MoT engine: the C++ object behind the wam_b200_* C ABI. It plays the
// role of the reference's Gwp05ModelArch (src/models/gwp05/engine/weights.cpp:339-462,
// engine.cpp:99-449): owns the device weights, the prefix and prompt K/V caches,
// and runs prefix + flow-matching denoise for a batch of requests.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <random>
#include <string>
#include <unordered_map>
#include <vector>

#include "kernels.h"

namespace wamb {

struct Geometry {
  int hidden = 3072, layers = 30, heads = 24, ffn = 14336;
  int action_hidden = 3072, action_ffn = 14336, action_dim = 32;
  int real_state_dim = 14, real_action_dim = 14, num_embodiments = 1, embodiment_id = 0;
  int grid_h = 32, grid_w = 24, vae_z = 48;
  int action_chunk = 48, steps = 10, prompt_tokens = 64, text_dim = 4096;
  float norm_eps = 1e-6f, flow_shift = 5.0f;
  // Config-1 block variants (BASELINE's literal statement; the reference's
  // MoT uses 0 / 0): ffn_kind 1 = SiLU-gated FFN (ffn.in holds [gate; up]
  // rows, 2F x W), norm_kind 1 = RMSNorm inside the AdaLN modulated norms.
  int ffn_kind = 0, norm_kind = 0;
  int visual() const { return grid_h * grid_w; }
  int prefix() const { return 1 + visual(); }
};

struct EngineOptions {
  std::string artifact_path;  // empty: synthetic weights from (geometry, seed)
  Geometry synthetic;
  uint64_t seed = 0;
  double bias_scale = 0.0;
  int device = 0;
  int max_batch = 1;
  bool graphs = true;
  bool prompt_cache = true;
  int weight_format = 0;  // 0 BF16, 1 Q8_0 linear weights
  // Config 1: the engine runs one MoT layer over given hidden states
  // (block_forward) instead of action chunks; needs layers == 1, max_batch == 1.
  bool block = false;
  // Vision front-end: load the Wan VAE encoder so that requests may carry the
  // three camera views instead of a precomputed latent.
  bool vae = false;
  // Resident language encoder: load UMT5 so that requests may carry prompt
  // token ids instead of a precomputed prompt embedding (synthetic geometry:
  // hidden = text_dim, 64-dim heads, max tokens = prompt_tokens, these sizes).
  bool t5 = false;
  int t5_vocab = 256384, t5_ffn = 10240, t5_layers = 24;
};

struct RequestView {
  const float* state = nullptr;
  int state_n = 0;
  const float* noise = nullptr;  // [T * A] or null
  const float* latent = nullptr;
  long long latent_n = 0;
  const float* prompt = nullptr;  // [prompt_tokens_in * text_dim]
  int prompt_tokens = 0;
  // Camera views (host pixels) used when latent is null: stage 1 + the VAE
  // encoder write the latent on the device.
  PreprocessView images[3] = {};
  int n_images = 0;
  // Prompt token ids used when prompt is null (UMT5 on the device).
  const int32_t* tokens = nullptr;
  int n_tokens = 0;
  const int32_t* mask = nullptr;
  int mask_n = 0;
};

struct EngineStats {
  float ms_total = 0, ms_prompt = 0, ms_prefix = 0, ms_denoise = 0;
  int prompt_cache_hit = 0;
};

using Launch = std::function<cudaError_t(cudaStream_t)>;

// Kernel families, for the per-kernel profile (wam_b200_profile).
enum OpKind : int { OP_GEMM = 0, OP_ATTENTION = 1, OP_LAYERNORM = 2, OP_QKV = 3, OP_SMALL = 4,
                    OP_ELEMENTWISE = 5, OP_SYNC = 6 /* lane hand-off, no kernel */ };

struct Op {
  Launch fn;
  int kind = OP_ELEMENTWISE;
  int launches = 1;     // kernels this op launches
  double bytes = 0.0;   // algorithmic HBM bytes (operands read + results written)
  double flops = 0.0;   // algorithmic FLOPs
  int shape[4] = {0, 0, 0, 0};  // GEMM: m, n, k, split-K factor (negative: CTA-pair kernel)
  int lane = 0;                 // 0: main stream, 1: side stream
};

// Ops in issue order. Each op runs on the stream of its lane; OP_SYNC ops
// hand work between the lanes with events (captured as graph edges).
struct Program {
  std::vector<Op> ops;
  int kernels = 0;
  int lane = 0;  // lane of the ops added next
  void add(Launch f, int kind, int launches = 1, double bytes = 0.0, double flops = 0.0) {
    ops.push_back(Op{std::move(f), kind, launches, bytes, flops});
    ops.back().lane = lane;
    kernels += launches;
  }
};

// One profiled op: phase 0 = prompt projection, 1 = prefix, 2 = denoise.
struct OpProfile {
  int phase, kind, launches;
  float ms;
  double bytes, flops;
  int shape[4];
};

// Synthetic tensor distribution rule (scale, center); mirrors init_rule() of
// the test fixtures' generator.
void synth_rule(const std::string& name, double bias_scale, double* scale, double* center);
// (name, element count) of every BF16 tensor the MoT path reads.
std::vector<std::pair<std::string, int64_t>> tensor_specs(const Geometry& g);
// Innermost (contiguous) length of a linear layer's weight, 0 for tensors that
// are not linear weights (norm gains, modulation tables, biases). Q8_0 applies
// to linear weights whose rows are whole 32-value blocks.
int64_t linear_inner(const std::string& name, const Geometry& g);
uint64_t tensor_seed(uint64_t seed, const std::string& name);

class VaeEncoder;
class T5Encoder;

class MotEngine {
 public:
  static std::unique_ptr<MotEngine> create(const EngineOptions& opt, std::string* err);
  ~MotEngine();

  const Geometry& geometry() const { return g_; }
  int device() const { return opt_.device; }
  int max_batch() const { return opt_.max_batch; }
  cudaStream_t stream() const { return stream_; }
  uint64_t resident_bytes() const { return resident_bytes_; }

  // H2D of a batch's inputs (normalises state on the host, pads the prompt).
  bool stage(const RequestView* reqs, int batch, std::string* err);
  // Enqueues prompt projection (unless cached), prefix and denoise.
  bool run(int batch, std::string* err, EngineStats* stats = nullptr);
  // Waits, reads the device error word, copies actions back and
  // de-normalises them: out [batch][T][real_action_dim].
  bool fetch(const RequestView* reqs, int batch, float* out, std::string* err);
  bool predict(const RequestView* reqs, int batch, float* out, EngineStats* stats, std::string* err);
  // Config 1 (block engines): one MoT layer, the reference's un-cached layer
  // (run_mot_step, mot.cpp:1008-1067) over given hidden states: xv [V][H]
  // visual tokens, xa [1 + T][E] state token then action tokens, tv [Nt][H] /
  // ta [Nt][E] the experts' text hidden states, t the action tokens' timestep
  // (state and visual tokens at 0). Outputs ov [V][H], oa [1 + T][E] (F32).
  bool block_forward(const float* xv, const float* xa, const float* tv, const float* ta, float t,
                     float* ov, float* oa, float* device_ms, std::string* err);
  void reset();
  int kernels_per_chunk(int batch, bool with_prompt);
  // Runs one chunk eagerly with CUDA events around every op (staged inputs).
  bool profile(int batch, std::vector<OpProfile>* out, std::string* err);
  // Device time of the ops of one (phase, kind) of the staged batch's plan,
  // captured alone into a CUDA graph (same launches, same buffers, PDL between
  // them) and replayed `reps` times between events: ms per replay, plus their
  // algorithmic bytes / FLOPs and kernel launches per replay.
  // lane: -1 = every lane, else only the ops of that lane (0 main, 1 side).
  bool profile_graph(int batch, int phase, int kind, int lane, int reps, float* ms, double* bytes,
                     double* flops, int* launches, std::string* err);
  // Device times of the phases of the last run() (ms): prompt, prefix, denoise.
  bool last_phase_ms(float* prompt, float* prefix, float* denoise);
  // Debug view of device state as F32 (names: prefix_k, prefix_v, prompt_k,
  // prompt_v, velocity, actions).
  bool read_tensor(const std::string& name, int slot, int layer, float* out, size_t n,
                   std::string* err);

 private:
  MotEngine() = default;
  bool init(const EngineOptions& opt, std::string* err);
  bool load_weights(std::string* err);
  bool quantize_linear_weights(const std::vector<std::pair<std::string, int64_t>>& specs,
                               std::string* err);
  bool alloc_buffers(std::string* err);
  const bf16* W(const std::string& name, int64_t numel);
  bool build(int batch, std::string* err);
  bool gemm(Program& p, const bf16* x, int ldx, int m, const std::string& wname, int n, int k,
            int epi, bool bias, const float* gate, const bf16* resid, int ldr, void* out, int ldo,
            std::string* err, int total_n = -1, int row0 = 0);
  // Plans one GEMM on prepared weights (re-tiled, Q8_0 tiles or row-major).
  bool add_gemm(Program& p, const bf16* x, int ldx, int m, const bf16* wsrc, int n, int k, int epi,
                const bf16* bias, const float* gate, const bf16* resid, int ldr, void* out, int ldo,
                bool tiled, bool q8, const std::string& label, std::string* err);
  // Re-tiles a GEMM weight in place into 32 KB UMMA tiles (once).
  bool ensure_tiled(const std::string& wname, int n, int k, std::string* err);
  // Whether the denoise step of `batch` requests runs as the persistent step
  // kernel (step.cu): <= 128 tokens, BF16 re-tiled weights, widths that are
  // multiples of 256 (<= 4096) and no GEMM with more 128-row tiles than SMs.

  struct Plan {
    Program prog[3];                      // prompt projection, prefix, denoise
    cudaGraphExec_t graph[3] = {nullptr, nullptr, nullptr};
    int scratch_gen = 0;  // split-K scratch generation the launches point into
  };
  cudaEvent_t phase_ev_[4] = {nullptr, nullptr, nullptr, nullptr};
  // Recorded after a batch's host-to-device copies: the next stage() waits
  // for it before it rewrites the pinned host buffers those copies read.
  cudaEvent_t h2d_ev_ = nullptr;
  bool phase_prompt_ran_ = false;
  void drop_plans();
  int scratch_gen_ = 0;

  EngineOptions opt_;
  Geometry g_;
  int sms_ = 148;
  cudaStream_t stream_ = nullptr;
  cudaStream_t side_ = nullptr;  // second lane of the prefix program
  cudaEvent_t ev_fork_ = nullptr, ev_join_ = nullptr;
  bool ok_ = false;
  std::string loader_;
  int policy_ = 0;  // artifact weight policy: 0 none named, 1 mot-vae-bf16-qkv-v1, 2 mot-q8_0-v1

  // weights
  void* warena_ = nullptr;
  size_t warena_bytes_ = 0;
  std::unordered_map<std::string, bf16*> w_;
  std::unordered_map<std::string, int64_t> wn_;
  // Q8_0 mode: GGML blocks of every linear weight (its BF16 slot holds the
  // dequantised values) and the GEMM tiles made from them.
  std::unordered_map<std::string, uint8_t*> q8_blocks_;
  std::unordered_map<std::string, uint8_t*> q8_tiles_;
  // GEMM weights already re-tiled in place into 16 KB UMMA tiles.
  std::unordered_map<std::string, bool> tiled_;
  bf16* retile_tmp_ = nullptr;  // staging copy for in-place re-tiling (build only)
  size_t retile_tmp_elems_ = 0;
  bool rowmajor_weights_ = false;
  std::vector<float> sq01_, sq99_, aq01_, aq99_;
  uint64_t resident_bytes_ = 0;

  // device buffers (sized for max_batch)
  std::vector<void*> allocs_;
  template <class T>
  T* dalloc(size_t n, std::string* err);

  float *in_state_ = nullptr, *in_latent_ = nullptr, *in_prompt_ = nullptr, *in_noise_ = nullptr;
  float *h_state_ = nullptr, *h_latent_ = nullptr, *h_prompt_ = nullptr, *h_noise_ = nullptr;
  float *h_out_ = nullptr, *d_out_ = nullptr;
  // block engines: F32 inputs [xv | xa | tv | ta] and outputs [ov | oa], the
  // F32 timestep-frequency rows (row 1 is rewritten per block call)
  float *blk_in_ = nullptr, *blk_out_ = nullptr, *freq_f32_ = nullptr;
  bf16 *prompt_bf_ = nullptr, *state_bf_ = nullptr, *action_bf_ = nullptr;
  bf16 *text_tmp_ = nullptr, *text_a_ = nullptr, *text_v_ = nullptr, *ckv_ = nullptr;
  bf16 *cols_ = nullptr, *hv_ = nullptr, *hs_ = nullptr, *ha_ = nullptr;
  bf16 *nrm_ = nullptr, *nrm_s_ = nullptr, *qkv_ = nullptr, *qkv_s_ = nullptr;
  bf16 *qbuf_ = nullptr, *att_ = nullptr, *att_s_ = nullptr, *cq_ = nullptr, *cq_s_ = nullptr;
  bf16 *qc_ = nullptr, *qc_s_ = nullptr, *catt_ = nullptr, *catt_s_ = nullptr;
  bf16 *ffn_ = nullptr, *ffn_s_ = nullptr, *s1_ = nullptr, *s2_ = nullptr;
  bf16 *e1_ = nullptr, *e2_ = nullptr, *d1_ = nullptr, *d2_ = nullptr, *vel_ = nullptr;
  bf16 *freq_bf_ = nullptr, *ct1_ = nullptr, *temb_a_ = nullptr, *ct2_ = nullptr, *mod_a_ = nullptr;
  bf16 *cv1_ = nullptr, *temb_v_ = nullptr, *cv2_ = nullptr, *mod_v_ = nullptr;
  float *comb_a0_ = nullptr, *comb_v_ = nullptr, *comb_steps_ = nullptr, *comb_final_ = nullptr;
  float *dt_ = nullptr, *inv_freq1_ = nullptr, *inv_freq3_ = nullptr;
  int* pos_thw_ = nullptr;
  const bf16** tables_a_ = nullptr;
  const bf16** tables_v_ = nullptr;
  const bf16** tables_final_ = nullptr;
  bf16 *k_self_ = nullptr, *v_self_ = nullptr;      // [B][L][heads][P+T][128]
  bf16 *k_prompt_ = nullptr, *v_prompt_ = nullptr;  // [B][L][heads][Nt][128] (action expert)
  bf16 *k_vis_ = nullptr, *v_vis_ = nullptr;        // [B][L][heads][Nt][128] (visual expert)
  // Prompt projection of a chunk of layers, [B * Nt][pkv_layers * 2H] (K | V of
  // each layer), when an expert's ca.k / ca.vproj weights form one matrix.
  bf16* pkv_ = nullptr;
  int pkv_layers_ = 0;
  // Split-K exchange workspace, one per lane (the lanes' GEMMs may overlap).
  float* gemm_ws_[2] = {nullptr, nullptr};
  // Device table of the prompt k-norm weights, [expert][layer] (one prompt
  // K / V scatter launch covers the layers of a projection chunk).
  const bf16** knorm_tab_ = nullptr;
  size_t gemm_ws_floats_ = 0;
  unsigned* err_word_ = nullptr;

  std::vector<float> timesteps_, sigmas_;
  std::map<int, std::unique_ptr<Plan>> plans_;
  std::unique_ptr<VaeEncoder> vae_;  // vision front-end (options.vae)
  std::unique_ptr<T5Encoder> t5_;    // resident language encoder (options.t5)
  // Prompt cache keys per batch slot: 'E' + embedding bytes, or 'T' + the
  // valid token ids; staged_keys_ are those of the staged batch.
  std::vector<std::vector<uint8_t>> prompt_key_, staged_keys_;
  std::vector<std::vector<uint8_t>> in_prompt_key_;  // token prompt held in in_prompt_ per slot
  // Version of the embedding prompt in each slot of h_prompt_ (0: none yet) and
  // its row count: the key of an embedding prompt is its slot's version, which
  // changes only when a different prompt is staged through the slot.
  std::vector<uint64_t> h_prompt_ver_;
  std::vector<int> h_prompt_rows_;
  std::vector<char> prompt_copy_;  // staged batch: slot's prompt is copied into h_prompt_
  uint64_t prompt_ver_next_ = 1;
  bool prompt_valid_ = false;
  int staged_batch_ = 0;
  std::mt19937 rng_{0x5eed};
};

}  // namespace wamb
