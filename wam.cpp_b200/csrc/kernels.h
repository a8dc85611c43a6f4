// Host-side interface to the engine's CUDA kernels (sm_100a). Every launcher
// takes device pointers and a stream; nothing here allocates.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace wamb {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ GEMM
// y[m, n] = epilogue( sum_k x[m, k] * w[n, k] ), x: [M, K] (row stride ldx),
// w: [N, K] row-major (GGUF ne = {K, N}). The epilogues restate the rounding
// points of the reference's BF16 path (src/models/gwp05/engine/weights.cpp:819-849,
// patches/llama-b9866-native-bf16.patch:79-91,507-514):
enum GemmEpilogue : int {
  EPI_BIAS = 0,       // y = bf16(bf16(acc) + b)                    linear_with_activation
  EPI_BIAS_GELU = 1,  // y = bf16(gelu_tanh(bf16(acc) + b))         linear_gelu_with_activation
  EPI_BIAS_SILU = 2,  // y = bf16(silu(bf16(bf16(acc) + b)))        linear + ggml_silu
  EPI_GATED_RES = 3,  // y = bf16(r + bf16(bf16(acc) + b) * gate)   linear + gated_residual
  EPI_RES = 4,        // y = bf16(r + bf16(bf16(acc) + b))          linear + ggml_add(hidden, .)
  EPI_F32_BIAS = 5,   // y = bf16(acc + b)                          conv_2d (F32 out) + bias, cast
  EPI_F32_OUT = 6,    // y_f32 = acc                                 raw accumulator (tests)
  EPI_BIAS_GELU_R = 7,  // y = bf16(gelu_tanh(bf16(bf16(acc) + b)))   linear + ggml_gelu (text MLP)
  EPI_BIAS_GELU_ERF = 8,  // y = bf16(gelu_erf(bf16(bf16(acc) + b)))  linear + ggml_gelu_erf (decoder)
  EPI_MUL = 9,        // y = bf16(r * bf16(bf16(acc) + b))          linear + ggml_mul (SiLU-gated FFN up)
};

// Split-K reduction. SPLIT_CLUSTER: the splits of a tile form a thread-block
// cluster and reduce their F32 partial tiles through distributed shared memory
// (no global scratch). SPLIT_CLUSTER_GLOBAL: the same cluster exchanges the
// partial tiles through a caller-provided global workspace (L2). SPLIT_WORKSPACE
// (more than 8 splits): partial tiles in the workspace, the last CTA of a tile
// to arrive (tile counters) reduces them.
enum SplitMode : int { SPLIT_CLUSTER = 0, SPLIT_WORKSPACE = 1, SPLIT_CLUSTER_GLOBAL = 2 };

struct GemmArgs {
  int m, n, k;
  int num_kb;  // k / 64
  int splits;
  int split_mode;
  int a_rows;  // token rows loaded per tile (<= 128)
  int stages;  // pipeline stages (one weight + one token k-block each)
  int pre_w;   // stages whose weight copies start before the grid-dependency wait
  int nt;      // stream kernel: output features per CTA (32, 64 or 128)
  int kb;      // stream kernel: k-blocks of 64 per pipeline stage
  const bf16* w_tiled;  // weights re-tiled by launch_retile_weights, or null (tensor map)
  const uint8_t* w_q8;  // Q8_0 weight tiles (launch_q8_retile), or null
  int tiles_m, tiles_n;
  int group_m;  // persistent / pair kernels: token tiles per group of the tile order (tile_coords)
  int epilogue;
  const bf16* bias;      // [n] or null
  const float* gate;     // [n] (EPI_GATED_RES)
  const bf16* residual;  // [m, ldr] (EPI_GATED_RES / EPI_RES); may alias out
  int ldr;
  void* out;  // bf16 [m, ldo] (float for EPI_F32_OUT)
  int ldo;
  float* workspace;    // SPLIT_WORKSPACE: partial tiles [tile][split][a_rows][256]
  unsigned* counters;  // SPLIT_WORKSPACE: arrival counters, one per tile, zero at rest
  unsigned* error;     // device error word
};

struct GemmScratch {
  float* workspace = nullptr;
  size_t workspace_floats = 0;
  unsigned* counters = nullptr;
  int counter_slots = 0;
  unsigned* error = nullptr;
};

struct GemmOp {
  CUtensorMap tm_w;
  CUtensorMap tm_x;
  GemmArgs args;
  int grid = 0;
  bool persistent = false;  // gemm_tc_persistent_kernel (tiles > SMs, no split-K)
  bool pair = false;        // gemm_tc_pair_kernel (>= 256 tokens, CTA pairs, cta_group::2)
  bool stream = false;      // gemm_stream_kernel (<= 64 tokens, full K per CTA, no split-K)
  int cluster = 1;          // pair kernel: cluster size (2 x splits)
  int smem_bytes = 0;
  // The "weights" (B operand) are activations written by earlier kernels of the
  // stream (attention products as GEMMs): the launch then waits for the
  // preceding kernel to finish (no programmatic early start), because the GEMM
  // kernels fetch weight stages before their grid-dependency wait.
  bool weights_from_prev = false;
};

// Plans one GEMM: picks the token tile and split-K factor, encodes the TMA
// descriptors. With w_tiled the weights are in the layout written by
// launch_retile_weights. pair asks for the CTA-pair (cta_group::2) kernel when
// m >= 256 (BF16 weights, automatic split count; WAM_B200_GEMM_PAIR=1 asks for
// it everywhere). Returns nullptr on success or a static error message.
const char* gemm_plan(GemmOp* op, const bf16* x, int ldx, int m, const bf16* w, int n, int k,
                      int epilogue, const bf16* bias, const float* gate, const bf16* residual,
                      int ldr, void* out, int ldo, const GemmScratch& scratch, int num_sms,
                      int force_splits, bool w_tiled = false, bool w_q8 = false,
                      bool pair = false);
// Re-tiles a row-major [n][k] BF16 weight (n % 256 == 0, k % 64 == 0) into
// contiguous 32 KB tiles [n/256][k/64][256][64] with the 128-byte swizzle of
// the UMMA operand pre-applied, so one bulk copy fetches a pipeline stage.
void launch_retile_weights(const bf16* src, bf16* dst, int n, int k, cudaStream_t s);
// Weight rows per re-tiled tile (256).
int gemm_weight_tile_rows();

// Q8_0 weights (q8.cu). Bytes of one GEMM weight tile (256 rows x 64 of K):
// int8 [256][64] then fp16 scales [256][2].
constexpr int kQ8TileBytes = 256 * 64 + 256 * 2 * 2;
// BF16 weights (n_elems % 32 == 0) -> GGML Q8_0 blocks (34 bytes per 32).
void launch_q8_quantize(const bf16* w, long long n_elems, uint8_t* out, cudaStream_t s);
// Q8_0 blocks -> BF16 (q * d rounded to BF16), n_elems values.
void launch_q8_dequantize(const uint8_t* blocks, long long n_elems, bf16* w, cudaStream_t s);
// Row-major Q8_0 blocks of an [n][k] weight (n % 256 == 0, k % 64 == 0) ->
// GEMM tiles [n/256][k/64][kQ8TileBytes].
void launch_q8_retile(const uint8_t* src, uint8_t* dst, int n, int k, cudaStream_t s);
cudaError_t gemm_launch(const GemmOp& op, cudaStream_t stream);
// Sets per-kernel launch attributes on the current device (call once per
// device before the first launch or graph capture).
cudaError_t gemm_init(int device);
// Split-K scratch a GEMM of this shape would use (floats), and its tile count.
size_t gemm_scratch_floats(int m, int n, int k, int num_sms, int force_splits, int* tiles_out);

// ------------------------------------------------------------ elementwise
// LayerNorm (two-pass mean / centred variance, no affine) then AdaLN
// modulation: y = bf16(n * (1 + scale[c]) + shift[c]); scale/shift F32 [cols]
// shared by all rows (norm_bf16_fused<affine=false>, native-bf16.patch:368-409).
void launch_ln_modulate(const bf16* x, int ldx, int rows, int cols, const float* scale,
                        const float* shift, float eps, bf16* y, int ldy, cudaStream_t s);
// RMSNorm (n = x * rsqrt(mean(x^2) + eps)) then the same AdaLN modulation: the
// config-1 "RMSNorm + AdaLN" block variant (no reference counterpart).
void launch_rms_modulate(const bf16* x, int ldx, int rows, int cols, const float* scale,
                         const float* shift, float eps, bf16* y, int ldy, cudaStream_t s);
// Affine LayerNorm: y = bf16(n * w[c] + b[c]), w/b BF16 (norm_bf16_fused<affine=true>).
void launch_ln_affine(const bf16* x, int ldx, int rows, int cols, const bf16* w, const bf16* b,
                      float eps, bf16* y, int ldy, cudaStream_t s);

// Per-token RMSNorm of q and k over the full attention width, RoPE, BF16 cast
// and scatter into head-major attention buffers (expert_qkv, mot.cpp:210-267;
// build_cross_kv, mot.cpp:101-128). Source row r holds q / k / v at column
// offsets q_col / k_col / v_col (-1 = absent). Destination element
// (seq, head, row, d) of q is q_out[seq * q_seq_stride + head * q_head_stride +
// (q_row_offset + row) * 128 + d]; k and v likewise with kv_* strides.
struct QkvScatter {
  const bf16* src;
  int ld_src;
  int rows;          // tokens in this launch
  int rows_per_seq;  // tokens of one request in this launch
  int hidden;        // H = heads * 128
  int heads;
  int q_col, k_col, v_col;
  const bf16* q_norm;  // [H] RMSNorm weight, or null for no norm
  const bf16* k_norm;
  float eps;
  // rope: 0 = none, 1 = 1-D over 128 dims at position pos_base + row_in_seq,
  // 2 = 3-D sections 44/42/42 at (t, h, w) = pos_thw[row_in_seq * 3 + {0,1,2}]
  int rope_mode;
  int pos_base;
  const int* pos_thw;
  const float* inv_freq;  // 1-D: [64]; 3-D: [22 | 21 | 21]
  bf16* q_out;
  long long q_seq_stride, q_head_stride;
  int q_row_offset;
  bf16* k_out;
  bf16* v_out;
  long long kv_seq_stride, kv_head_stride;
  int kv_row_offset;
  // Several layers in one launch (grid y = layer): layer l reads its rows at
  // src + l * src_layer_stride, takes its k norm from k_norms[l] (a device
  // array) when k_norms is set, and writes q_out / k_out / v_out +
  // l * out_layer_stride.
  int layers = 1;
  long long src_layer_stride = 0, out_layer_stride = 0;
  const bf16* const* k_norms = nullptr;
};
// Blocks carry only the parts a launch writes (k and v when q_col < 0).
void launch_qkv_scatter(const QkvScatter& a, cudaStream_t s);

// Flash attention over head-major Q/K/V with softmax(scale * QK^T) V,
// F32 scores, BF16 probabilities, F32 accumulation. Output row r of sequence b
// goes to out[(b * out_seq_rows + r) * ldo + head * 128 + d]; if split_first,
// row 0 of each sequence goes to out_first[b * ldo_first + ...] instead and
// rows 1.. to out[(b * (lq - 1) + r - 1) * ldo ...].
struct AttnArgs {
  const bf16* q;
  long long q_seq_stride, q_head_stride;
  const bf16* k;
  const bf16* v;
  long long kv_seq_stride, kv_head_stride;
  int lq, lk, heads, batch;
  float scale;
  bf16* out;
  int ldo;
  bf16* out_first;
  int ldo_first;
  int split_first;
  // Keys [0, static_keys) are not written by the preceding kernel: a CTA whose
  // whole key range lies there loads its K/V before waiting for it.
  int static_keys = 0;
  // Split-KV merge workspace (attention_ws_floats floats) or null: with it the
  // key splits of a query block exchange their partial rows through L2,
  // without it through distributed shared memory.
  float* ws = nullptr;
  size_t ws_floats = 0;
  unsigned* error = nullptr;  // device error word for a wait that gave up (tcgen05 kernel)
  // Query rows [q_begin, q_end) of each sequence are computed by this launch
  // (q_end 0: lq); lq stays the sequence's query count (output addressing).
  int q_begin = 0, q_end = 0;
};
// Picks the kernel: 128-query tcgen05 tiles (attention_tc.cu) for >= 128
// queries; for <= 64 queries over <= 896 keys tcgen05 with every key's score
// in TMEM, one CTA or a key-split cluster of 2 / 4 per (sequence, head)
// (attention_dec_tc.cu); the mma.sync kernel (attention.cu) otherwise.
void launch_attention(const AttnArgs& a, cudaStream_t s);
// Kernels launch_attention(a) issues (2 when a ragged tail of < 64 query rows
// runs on the mma.sync kernel so that the 128-row tiles fit one wave).
int attention_launch_count(const AttnArgs& a);
cudaError_t attention_tc_init();
bool attention_tc_eligible(const AttnArgs& a);
cudaError_t launch_attention_tc(const AttnArgs& a, cudaStream_t s);
// tcgen05 attention for <= 64 queries over <= 896 keys per (sequence, head)
// (attention_dec_tc.cu).
cudaError_t attention_dec_tc_init();
bool attention_dec_tc_eligible(const AttnArgs& a);
cudaError_t launch_attention_dec_tc(const AttnArgs& a, cudaStream_t s);
// TMA map of [batch][heads][rows][128] BF16 (element strides), boxes of
// box_rows rows x 64 dims, 128-byte swizzle, rows past `rows` zero-filled.
bool attn_encode_rows(CUtensorMap* m, const void* base, int rows, int heads, int batch,
                      long long head_stride, long long seq_stride, int box_rows);

// Workspace the split-KV merge of `a` needs (0 when it does not split).
size_t attention_ws_floats(const AttnArgs& a);
cudaError_t attention_init();

// y[m, n] = act(bf16(bf16(sum_k x[m, k] * w(n, k)) + b[n])) for the small
// action/state encoder and decoder projections, with w(n, k) =
// w[n * w_sn + k * w_sk] (handles the transposed embodiment slices).
enum SmallAct : int { ACT_NONE = 0, ACT_GELU_ERF = 1 };
void launch_small_linear(const bf16* x, int ldx, int m, int k, const bf16* w, long long w_sn,
                         long long w_sk, const bf16* b, int n, int act, bf16* y, int ldy,
                         cudaStream_t s);

// combined[s][l][j] = f32(mod[s * ld_mod + j % period]) + f32(table_l[j]) for
// steps s, layers l, j < width (modulation_add with f32_accumulation,
// mot.cpp:137-145; the final head uses period = E to add temb to both halves,
// mot.cpp:468-486). tables: device array of `layers` BF16 pointers.
void launch_modulation_add(const bf16* mod, int ld_mod, int period, int steps,
                           const bf16* const* tables, int layers, int width, float* combined,
                           cudaStream_t s);
// y = bf16(silu(x)), elementwise.
void launch_silu(const bf16* x, bf16* y, int n, cudaStream_t s);
// F32 -> BF16 round to nearest even.
void launch_f32_to_bf16(const float* x, bf16* y, long long n, cudaStream_t s);
// im2col of a [C, 2gh, 2gw] F32 latent for the 2x2 stride-2 patch conv:
// cols[b][y*gw + x][c*4 + dy*2 + dx] = bf16(latent[b][c][2y+dy][2x+dx]).
void launch_patchify(const float* latent, int batch, int channels, int gh, int gw, bf16* cols,
                     cudaStream_t s);
// Euler step a = bf16(f32(a) + f32(v) * dt), with v read from a [rows, ldv] buffer.
void launch_euler(bf16* action, const bf16* velocity, int n, const float* dt, cudaStream_t s);
// BF16 -> F32.
void launch_bf16_to_f32(const bf16* x, float* y, long long n, cudaStream_t s);
// Deterministic synthetic weights: w[i] = bf16(center + scale * g(seed, i)),
// g an integer-hash approximation of N(0,1) (sum of four uniform 16-bit draws).
void launch_synth_bf16(bf16* w, long long n, unsigned long long seed, double scale, double center,
                       cudaStream_t s);

// Vision front-end: three camera views composed, resized (cover + centre crop,
// triangle filter), patchified 2x2 into [12][out_h/2][out_w/2] F32 in [-1, 1]
// (vision.cu). A view is the reference's ImageView
// (src/models/gwp05/engine/engine.h:82-89) with its pixels on the device.
struct PreprocessView {
  const void* data;
  int w, h, format;  // format 0: U8 RGB (3 bytes per pixel), 1: F32 RGB in [0, 1]
};
bool launch_preprocess(const PreprocessView* views, int out_w, int out_h, float* out,
                       cudaStream_t stream);

// Implicit-GEMM convolution (conv.cu) over NHWC BF16 activations of one
// image: mode 0 = 3x3 stride 1 padding 1, 1 = 3x3 stride 2 after a one-pixel
// zero pad at the right / bottom, 2 = 1x1. Weights in the layout of
// launch_conv_weight_layout: [conv_cout_pad(cout)][taps][conv_cin_pad(cin)]
// (zero padded); cin >= 64 (pad narrower inputs).
struct ConvParams {
  int mode, taps, cblocks;
  int out_w, out_h;
  int tiles_x, tiles_y, tiles_n;
};
struct ConvOp {
  CUtensorMap tm_w;
  CUtensorMap tm_x;
  ConvParams params;
  GemmArgs args;
  int grid = 0;
  int wn = 256;  // N tile: 160 when Cout is a multiple of 160, else 256
};
int conv_cin_pad(int cin);
int conv_cout_pad(int cout);
// src: the GGUF / torch layout [cout][cin][kh][kw] (taps = kh * kw).
void launch_conv_weight_layout(const bf16* src, bf16* dst, int cout, int cin, int taps,
                               cudaStream_t stream);
// Epilogue EPI_BIAS (out = bf16(bf16(conv) + b)) or EPI_RES (out = bf16(residual
// + bf16(bf16(conv) + b))). Returns nullptr or a static error message.
const char* conv_plan(ConvOp* op, const bf16* x, int in_w, int in_h, int cin, int mode,
                      const bf16* w_laid, int cout, int epilogue, const bf16* bias,
                      const bf16* residual, bf16* out, int num_sms);
bool conv_launch(const ConvOp& op, unsigned* error, cudaStream_t stream, bool pdl);

}  // namespace wamb
