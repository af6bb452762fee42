// Host-side model/session objects of the device path.
#pragma once
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "../kernels/kernels.h"
#include "common.h"
#include "tokenizer.h"

namespace yl {

// One repacked weight matrix in HBM: quants [rows][row_bytes] and (for
// quantized formats) scales [rows][scale_row_bytes], rows 16-byte aligned.
struct DevWeight {
  int fmt = YL_Q8_0;  // yl_weight_format
  bool sf16 = true;   // scale element type
  uint32_t rows = 0, cols = 0;
  uint32_t row_bytes = 0, scale_row_bytes = 0;
  uint8_t* q = nullptr;
  uint8_t* s = nullptr;
  bool no_inf_scales = true;  // no f16 scale is +-inf (the tcgen05 GEMM's fused fold needs that)
};

struct Layer {
  DevWeight wqkv;  // rows: q (att_dim) | k (kv_dim) | v (kv_dim)
  DevWeight wo;
  DevWeight w13;   // rows interleaved: gate j at 2j, up j at 2j+1
  DevWeight w2;
  float* rms_att = nullptr;
  float* rms_ffn = nullptr;
};

struct Model {
  yl_shape shape{};
  std::string name = "TransformerLlamaGguf";
  std::string path;
  int device = 0;
  int num_sms = 148;
  uint32_t bos = 0, eos = 0;
  float attn_scale = 0.f;
  DevWeight emb;
  DevWeight lm;  // aliases emb when tied
  std::vector<Layer> layers;
  float* rms_final = nullptr;
  float2* rope_cs = nullptr;  // [ctx_len][head_size/2] (cos, sin)
  std::vector<void*> allocs;
  uint64_t device_bytes = 0;
  // tensor parallelism (Megatron split over tp_size ranks): this rank's
  // query heads, KV heads, ffn rows and vocabulary rows (all of them at 1)
  int tp_rank = 0, tp_size = 1;
  uint32_t l_heads = 0, l_kv = 0, l_ffn = 0, l_vocab = 0, vocab0 = 0;
  // Transformer::tokenizer(): loaded from `path` at the first request
  mutable std::mutex tok_mu;
  mutable std::unique_ptr<yl_tokenizer> tok;
  ~Model();
};

struct Session {
  const Model* m = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  float* kcache = nullptr;
  float* vcache = nullptr;
  uint64_t kv_elems = 0;  // per cache
  uint32_t pos = 0;
  // workspace sized for `cap` tokens
  uint32_t cap = 0;
  float* x = nullptr;     // residual stream [cap][dim]
  float* xf = nullptr;    // f32 activations [cap][max(dim,att,ffn)] (F16 format) / final norm
  int8_t* xq = nullptr;   // [cap][max(dim,att,ffn)]
  float* xs = nullptr;    // [cap][max/32]
  float* qkv = nullptr;   // [cap][att + 2 kv]
  float* q = nullptr;     // [cap][att]
  float* h = nullptr;     // [cap][ffn]
  int8_t* hq = nullptr;   // [cap][ffn] quantized h (SwiGLU epilogue)
  float* hs = nullptr;    // [cap][ffn/32]
  unsigned int* hcount = nullptr;  // [cap][ffn/32] arrival counters (zero between launches)
  unsigned int* work = nullptr;    // [n_layers + 1][2] dynamic row-set counters (decode gate/up, lm_head)
  void* f16ws = nullptr;  // F16 models: the f16 GEMM's split rows for cap tokens (single-GPU models)
  uint32_t* tok = nullptr;  // [cap]
  float* logits = nullptr;  // [vocab]
  float* part = nullptr;    // decode attention scores / weights [local heads][part_stride]
  uint32_t part_stride = 0;
  float* ascr = nullptr;    // multi-token attention scores / weights (grown on demand)
  uint64_t ascr_floats = 0;
  float* am_val = nullptr;            // lm_head per-CTA winners
  uint32_t* am_idx = nullptr;
  unsigned int* am_count = nullptr;
  uint32_t* hist = nullptr; // [ctx_len] greedy ids of device steps
  k::StepState* state = nullptr;
  int* err = nullptr;
  // pinned host staging
  float* logits_h = nullptr;
  uint32_t* hist_h = nullptr;
  uint32_t n_splits = 1;
  std::vector<cudaEvent_t>* prof = nullptr;  // profiling: events recorded after each launch
  uint64_t* trace = nullptr;  // timeline tracing: [launch][TRACE_STRIDE] stamps
  bool trace_on = false;
  cudaGraphExec_t graph = nullptr;
  cudaGraphExec_t graph_lg = nullptr;  // tensor-parallel decode step that also gathers logits
  uint32_t graph_launches = 0;     // kernel nodes of `graph` (one decode step)
  uint32_t graph_launches_lg = 0;  // kernel nodes of `graph_lg`
  // tensor parallelism: this rank's exchange region (shared with the peers
  // through CUDA IPC) and every rank's region as mapped here
  uint8_t* tp_region = nullptr;
  uint64_t tp_bytes = 0, tp_flags_off = 0, tp_part_off[2] = {0, 0}, tp_lm_off = 0, tp_logit_off = 0;
  uint32_t tp_cap = 0;  // tokens per forward the partial buffers hold
  uint8_t* tp_base[8] = {};
  std::vector<void*> tp_opened;
  bool tp_ready = false;
  uint32_t* tp_epoch = nullptr;  // completed steps (device)
  uint32_t* tp_pepoch = nullptr; // completed single-token steps (device): the push exchanges' epoch
  uint64_t tp_inbox_off[2] = {0, 0};  // push inboxes [2][world][dim] of {f32, flag} entries
  float* x2 = nullptr;           // second residual row (single-token tensor-parallel steps alternate)
  std::vector<void*> allocs;
  ~Session();
};

int model_load_gguf(const char* path, uint32_t max_ctx_len, int fmt_override, int tp_rank, int tp_size, Model** out);
// safetensors + config.json beside it (MLX affine 8-bit requantized to Q8
// with f32 scales, or F16), and lm.rs files (Q8 with f32 scales); one rank.
int model_load_st(const char* path, uint32_t max_ctx_len, int fmt_override, Model** out);
int model_load_lmrs(const char* path, uint32_t max_ctx_len, int fmt_override, Model** out);
// Tensor-parallel sessions: export this rank's exchange-region handle (64
// bytes, cudaIpcMemHandle_t), then map all ranks' regions (handles[rank]).
int session_tp_handle(Session* s, void* handle_out);
int session_tp_connect(Session* s, const void* handles);
int session_create(const Model* m, Session** out);
// with_kv = false: a workspace session without a KV cache (batched decode)
int session_create_ex(const Model* m, bool with_kv, Session** out);
int session_reset(Session* s);
// General forward over n tokens (prefill or decode); last-token logits stay in
// s->logits (device), greedy id in s->hist[0].
int forward(Session* s, const uint32_t* tokens_host, uint32_t n, uint32_t start_pos, bool want_logits = true);
// One batch-1 step launched kernel by kernel (no graph, no PDL) with events
// between launches; writes per-launch device times in microseconds.
int profile_step(Session* s, uint32_t token, uint32_t pos, float* us, uint32_t cap, uint32_t* n_out);
// The captured batch-1 decode step (state set on device before a launch):
// s->graph, or with logits (tensor-parallel) s->graph_lg, which also gathers
// the full logits.
int ensure_decode_graph(Session* s, bool logits = false);
int capture_decode_graph(Session* s, bool gather);  // into s->graph
// One batch-1 step captured exactly like the decode graph (PDL, state on the
// device) with every matvec / attention CTA stamping globaltimer at fixed
// points: out[launch * TRACE_STRIDE + cta * 8 + i].
constexpr uint32_t TRACE_STRIDE = 8 * 1024;
int trace_step(Session* s, uint32_t token, uint32_t pos, uint64_t* out, uint64_t cap, uint32_t* n_launches);
// Tunables read once from the environment (YL_MV_KC_BYTES, YL_MV_SMEM, YL_PDL,
// YL_MV_GRID_MULT, YL_LM_LIMBS; YL_MV_KC_BYTES=0 streams whole rows).
struct Tunables {
  uint32_t kc_bytes = 4096;  // weight bytes per row per bulk copy
  uint32_t smem = 100 * 1024;  // per CTA: two matvec CTAs fit on one SM
  bool pdl = true;
  uint32_t grid_mult = 2;    // matvec CTAs per SM
  bool limbs = true;         // Q8_0 lm_head on three-limb int8 activations
  bool gemm = true;          // multi-token passes on the int8 tensor-core GEMM
  // from this many tokens: measured on B200, 8-token passes run 2.1x faster on
  // the GEMM than on the 8-token matvec, 4-token passes 9 % slower
  uint32_t gemm_min = 5;
  // Q8_0 GEMMs on the tcgen05 tensor-memory kernel (YL_GEMM_TC=1), from
  // gemm_tc_min tokens (its tiles are 128 tokens wide). Off by default: it is
  // bit-identical to the mma.sync kernel but measured no faster (both are
  // bound by the exact per-block fold on the FP32 pipe, not by the tensor core).
  bool gemm_tc = false;
  uint32_t gemm_tc_min = 96;
  // F16 passes of this many tokens on the f16 tensor-core GEMM (YL_GEMM_F16_MIN;
  // 0 turns it off; the matvec below)
  uint32_t gemm_f16_min = 16;
  bool tp_fused = true;      // tensor-parallel decode: exchange fused into the projections (else exchange kernels)
  // decode: L2 prefetch of the next matrix's first bytes per launch (YL_PF_MB).
  // Off: measured slower at every size tried (16, 32, 48 MB).
  uint64_t pf_bytes = 0;
};
// Batched decode of independent sessions (one token each per step): the
// projections run once over the stacked rows, the attention is one launch
// over every session's own cache and position. Holds the workspace.
struct Batch {
  const Model* m = nullptr;
  Session* ws = nullptr;     // workspace: activations of up to `cap` rows, no KV cache
  uint32_t cap = 0;
  float* sc = nullptr;       // decode attention scores [cap][local heads][part_stride]
  float* logits = nullptr;   // [cap][vocab]
  uint32_t* ids = nullptr;   // [cap] greedy ids
  uint32_t* tok_h = nullptr; // page-locked staging: tokens in, ids and the error word out
  ~Batch();
};
int batch_create(const Model* m, uint32_t cap, Batch** out);
// One decode step for n sessions: token i at position pos[i] of session ss[i]
// (distinct sessions of b's model). Logits and ids stay in b->logits / b->ids;
// the caller synchronizes b->ws->stream.
int forward_batch(Batch* b, Session* const* ss, uint32_t n, const uint32_t* tokens, const uint32_t* pos);

const Tunables& tunables();
// Runtime override of a tunable (yl_config_set): gemm, gemm_tc, gemm_tc_min, gemm_f16_min.
int set_tunable(const std::string& key, int64_t value);
// Launches the matvec for `ntok` tokens (groups of 8) with activations x*.
int run_matvec(const DevWeight& w, bool f32act, const int8_t* xq, const float* xs, const float* xf,
               uint64_t x_stride, uint64_t xs_stride, uint32_t ntok, float* out, uint64_t out_stride, int epi,
               uint32_t quirk_cols, int* err, cudaStream_t st, bool pdl, int num_sms);
// Optional prologue / epilogue operands of run_matvec_ex.
struct MvExtra {
  int pro = 0;                 // k::PRO_*
  const float* xres = nullptr; // PRO_NORM: residual rows (stride x_stride)
  int8_t* gq = nullptr;        // PRO_NORM through the multi-token GEMM: the
  float* gs = nullptr;         // normalized, quantized rows [ntok][K] / [ntok][K/32]
  const float* norm_w = nullptr;
  float eps = 0.f;
  int8_t* hq = nullptr;        // EPI_SWIGLU_Q8 outputs and block counters
  float* hs = nullptr;
  unsigned int* hcount = nullptr;
  float* am_val = nullptr;     // EPI_ARGMAX scratch / outputs
  uint32_t* am_idx = nullptr;
  unsigned int* am_count = nullptr;
  uint32_t* am_out = nullptr;
  k::StepState* state = nullptr;
  uint64_t* trace = nullptr;   // timeline stamps of this launch (nullable)
  unsigned int* work = nullptr;  // dynamic row-set counters of this launch site (nullable)
  float* am_shard = nullptr;     // EPI_ARGMAX over a vocabulary shard: published winner
  uint32_t am_base = 0;          // first vocabulary row of the shard
  // tensor parallel, single token: 1 push epilogue, 2 all-reduce prologue
  int tp_mode = 0;
  const k::TpArgs* tp = nullptr;     // ranks' exchange regions (base, rank, world)
  const uint32_t* tp_epoch = nullptr;
  uint64_t tp_inbox_off = 0;
  uint32_t tp_site = 0, tp_nsites = 0;
  float* tp_xout = nullptr;
  k::L2Prefetch pf;              // the next weight-streaming launch's first rows (decode)
  // F16 multi-token passes: workspace of the f16 tensor-core GEMM, at least
  // gemm_f16_workspace_bytes(ntok, K) (nullable: the matvec runs instead)
  void* f16ws = nullptr;
};
int run_matvec_ex(const DevWeight& w, bool f32act, const int8_t* xq, const float* xs, const float* xf,
                  uint64_t x_stride, uint64_t xs_stride, uint32_t ntok, float* out, uint64_t out_stride, int epi,
                  uint32_t quirk_cols, int* err, cudaStream_t st, bool pdl, int num_sms, const MvExtra& ex,
                  uint32_t* launches);

}  // namespace yl
