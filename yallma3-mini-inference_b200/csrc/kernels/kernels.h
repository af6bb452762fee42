// Host-visible interface of the device kernels (launch wrappers + argument
// structs). Every wrapper enqueues on lc.stream and returns the launch error;
// with lc.pdl set the launch carries the programmatic-stream-serialization
// attribute so the kernel may start while its predecessor drains (each kernel
// calls griddepcontrol.wait before touching data the predecessor produced).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

// Diagnostics build switch (timeline stamps inside the decode kernels).
#ifndef YL_WITH_TRACE
#define YL_WITH_TRACE 0
#endif

namespace yl {
namespace k {

// Sessions one batched decode step can carry (yl_batch_forward).
constexpr uint32_t YL_MAX_BATCH = 16;

// FMT_Q8X: Q8_0 weights against f32 activations held as three int8 limbs per
// 32-block, y = s * (a + b/254 + c/254^2) (|error| <= s/2/254^2, about 6e-8 of
// the block's absmax), so the f32-activation lm_head runs on dp4a.
enum Fmt : int { FMT_Q8 = 0, FMT_Q4 = 1, FMT_F16 = 2, FMT_Q8F = 3, FMT_Q4F = 4, FMT_Q8X = 5 };
// EPI_SWIGLU_Q8: SwiGLU on (gate, up) row pairs, f32 h stored and h quantized
// to Q8_0 blocks (for the next matvec); a block straddling two CTAs is
// quantized by whichever finishes it last (per-block arrival counters).
// EPI_ARGMAX: store + greedy id over all rows (last CTA to finish reduces the
// per-CTA winners).
enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_QUIRK = 2, EPI_SWIGLU = 3, EPI_SWIGLU_Q8 = 4, EPI_ARGMAX = 5 };
// Activation prologue: PRO_LOAD reads prepared activations; PRO_NORM computes
// RMSNorm of the f32 residual rows (util.rs:389-426) and quantizes them
// (quantization.rs:29-52) into shared memory (f32 for f32-activation formats).
// PRO_QUANT quantizes f32 rows (xres) without a norm (the SwiGLU output h
// feeding the down projection).
enum Pro : int { PRO_LOAD = 0, PRO_NORM = 1, PRO_QUANT = 2 };

struct StepState;

struct LaunchCfg {
  cudaStream_t stream = nullptr;
  bool pdl = false;
  uint32_t grid = 0;              // 0 = kernel default (number of SMs)
  uint32_t smem_budget = 100 * 1024;
};

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, uint32_t smem, const LaunchCfg& lc,
                                 Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = lc.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ---- L2 prefetch of the next kernel's weights ------------------------------
// Batch-1 decode streams every weight once per token, and HBM idles while a
// kernel drains, while the next one starts and during attention. A kernel
// given this descriptor asks the TMA unit to prefetch into L2 the rows the
// NEXT weight-streaming kernel reads first, so those gaps carry useful bytes.
// Slots c = 0..slots-1 are spread over the prefetching kernel's CTAs:
//  * static split (dyn = 0): slot c is next-kernel CTA c's contiguous row
//    range (units = rows/unit split evenly over `slots` CTAs), of which the
//    first rows_each rows are fetched;
//  * dynamic row sets (dyn = 1): slot c is rows [c*rows_each, (c+1)*rows_each).
struct L2Prefetch {
  const uint8_t* q = nullptr;  // quants of the next matrix (null: nothing to prefetch)
  const uint8_t* s = nullptr;  // its scales (nullable)
  uint32_t rows = 0, row_bytes = 0, srow_bytes = 0;
  uint32_t unit = 1;
  uint32_t slots = 0;
  uint32_t rows_each = 0;
  uint32_t dyn = 0;
};

// ---- matvec -------------------------------------------------------------
struct MvArgs {
  const uint8_t* wq;        // weight quants (row-major, row_bytes per row)
  const uint8_t* ws;        // weight scales (row stride scale_row_bytes), null for F16
  uint32_t rows, K;
  uint32_t row_bytes, scale_row_bytes;
  uint32_t kc;              // K-chunk per stage (elements, multiple of 256)
  int stages;               // set by the launcher
  const int8_t* xq;         // int8 activations [ntok][x_tok_stride]
  const float* xs;          // activation scales [ntok][xs_tok_stride]
  const float* xf;          // f32 activations [ntok][x_tok_stride] (F16 / lm_head)
  uint64_t x_tok_stride, xs_tok_stride;
  uint32_t ntok;            // tokens in this pass (<= 8)
  float* out;
  uint64_t out_tok_stride;
  uint32_t quirk_cols;      // EPI_QUIRK: columns below this add, the rest store
  int* err;
  // PRO_NORM: f32 residual rows [ntok][x_tok_stride] and the norm weight
  int pro;
  const float* xres;
  const float* norm_w;
  float eps;
  // EPI_SWIGLU_Q8: quantized h [ntok][rows/2] + scales [ntok][rows/64], and
  // one arrival counter per (token, block), zero between launches
  int8_t* hq;
  float* hs;
  unsigned int* hcount;
  // EPI_ARGMAX: per-CTA winners, arrival counter (zero between launches),
  // output id slot (hist[state->steps] or hist[0]) and the step state
  float* am_val;
  uint32_t* am_idx;
  unsigned int* am_count;
  uint32_t* am_out;
  StepState* state;
  // EPI_ARGMAX over a vocabulary shard (nullable): the winner is published as
  // {value f32, global index u32 (rows + am_base), first-logit-NaN u32}
  // instead of updating am_out / state
  float* am_shard;
  uint32_t am_base;
  // Tensor parallel, single-token passes (tp_mode). Inboxes are [world][rows]
  // 8-byte entries {f32 value, u32 flag} at byte offset tp_inbox_off of every
  // rank's exchange region; the flag of this pass is
  // *tp_epoch * tp_nsites + tp_site + 1. 1 = push epilogue: each output row
  // goes into every rank's inbox (slot of this rank) as one 8-byte store;
  // 2 = all-reduce prologue (with PRO_NORM): each thread waits (bounded)
  // until its entries of every rank carry the flag, takes the rows as
  // xres + the sum of the ranks' values (in rank order), CTA 0 stores them to
  // tp_xout.
  int tp_mode;
  uint32_t tp_rank, tp_world, tp_site, tp_nsites;
  uint8_t* tp_base[8];
  uint64_t tp_inbox_off;
  const uint32_t* tp_epoch;
  float* tp_xout;
  // Dynamic scheduling (nullable): [next row set, CTAs done] counters, zero
  // between launches; CTAs claim 8-row sets from it instead of a static range.
  // Used by the launcher only for single-token passes with >= 4 sets per CTA.
  unsigned int* work;
  // timeline tracing (nullable): 8 slots per CTA in globaltimer nanoseconds:
  // entry, activations staged, wait released, consumers done, and for the
  // RMSNorm prologue: first token's rows loaded, norm factor ready, warp 0's
  // and the last warp's rows quantized
  uint64_t* trace;
  // issued by each CTA's producer once its own copies are all issued
  L2Prefetch pf;
};
// fmt: FMT_*; scale_f16: weight scale type. Chooses NT from a.ntok.
cudaError_t matvec(const MvArgs& a, int fmt, bool scale_f16, int epi, const LaunchCfg& lc);
// The schedule matvec() picks: CTA count, and whether a single-token pass
// given row-set counters (has_work) hands out 8-row sets dynamically (worth it
// with 4 or more sets per CTA; the SwiGLU+quantize epilogue also needs whole
// sets and at most 16 per CTA). Also used to aim L2Prefetch at a launch.
constexpr uint32_t MV_ROWSET = 8;
constexpr uint32_t MV_SWIGLU_LIST = 32;  // row sets one CTA may list for its h-quantize tail
inline void matvec_schedule(uint32_t rows, int epi, uint32_t lc_grid, uint32_t ntok, bool has_work, uint32_t* grid,
                            bool* dyn) {
  const uint32_t g = lc_grid ? lc_grid : 148;
  const uint32_t unit = (epi == EPI_SWIGLU || epi == EPI_SWIGLU_Q8) ? 2u : 1u;
  *grid = g > rows / unit ? rows / unit : g;
  const uint32_t nrs = (rows + MV_ROWSET - 1) / MV_ROWSET;
  bool ok = has_work && ntok == 1 && nrs >= 4 * g;
  if (epi == EPI_SWIGLU_Q8) ok = ok && rows % MV_ROWSET == 0 && nrs <= g * (MV_SWIGLU_LIST / 2);
  *dyn = ok;
}
// Largest tokens-per-pass (1, 2, 4 or 8) whose shared-memory layout fits with
// at least two ring stages.
uint32_t matvec_max_ntok(int fmt, uint32_t K, uint32_t kc, int epi);

// ---- multi-token projections (int8 tensor-core GEMM) ----------------------
// out[t][r] = sum_g ((f32)isum * ws[r][g]) * xs[t][g] over Q8_0 / Q4_0 weight
// rows (f16 or f32 scales) and Q8_0 activation rows; epi: EPI_STORE,
// EPI_ADD, EPI_QUIRK (quirk_cols) or EPI_SWIGLU_Q8 (interleaved gate/up rows,
// rows % 128 == 0: h quantized into hq [ntok][rows/2] / hs [ntok][rows/64],
// and h as f32 into out when out is not null).
struct GemmArgs {
  const uint8_t* wq;
  const uint8_t* ws;
  uint32_t rows, K, row_bytes, scale_row_bytes;
  const int8_t* xq;
  const float* xs;
  uint64_t x_stride, xs_stride;  // bytes / floats per token row
  uint32_t ntok;
  float* out;
  uint64_t out_stride;
  uint32_t quirk_cols;
  int8_t* hq;
  float* hs;
  int* err;  // device error word (bounded waits of the tensor-memory GEMM)
  float neg_zero;  // -0.0f, set by gemm_tc (an addend the compiler cannot see through)
};
bool gemm_supported(const GemmArgs& a, int fmt, bool scale_f16, int epi);
cudaError_t gemm_q(const GemmArgs& a, int fmt, bool scale_f16, int epi, const LaunchCfg& lc);
// The same contraction on the 5th-generation tensor cores (tcgen05.mma
// kind::i8, TMA-fed, accumulators in tensor memory; Q8_0 weights, 128 x 128
// tiles), bit-identical to gemm_q. Needs the 16-byte alignments of TMA.
bool gemm_tc_supported(const GemmArgs& a, int fmt, bool scale_f16, int epi);
cudaError_t gemm_tc(const GemmArgs& a, bool scale_f16, int epi, const LaunchCfg& lc);

// Multi-token F16 projections on the tensor cores (matmul_f32,
// weight_type.rs:228-270: out[t][r] = sum_k (f32)w[r][k] * x[t][k]). f16_split
// writes each token's f32 row (or its RMSNorm, norm_w non-null, computed as
// the matvec prologue computes it) as x * 2^e = hi + lo, two f16 rows, with e
// the power of two that puts the row's max |x| in [2^14, 2^15); the GEMM runs
// mma.sync m16n8k16 (f16 x f16 -> f32) on w*hi and w*lo into one f32
// accumulator and scales by 2^-e. Epilogues: EPI_STORE, EPI_ADD, EPI_QUIRK,
// EPI_SWIGLU (interleaved gate/up rows, f32 h [ntok][rows/2]).
struct GemmF16Args {
  const uint8_t* w;          // f16 weight rows
  uint32_t rows, K, row_bytes;
  const float* x;            // f32 activation rows (the residual rows when norm_w is set)
  uint64_t x_stride;         // floats per token row
  const float* norm_w;       // nullable: RMSNorm weights
  float eps;
  uint32_t ntok;
  uint16_t* hi;              // workspace [ntok][K] f16 each
  uint16_t* lo;
  int* exps;                 // workspace [ntok]
  float* out;
  uint64_t out_stride;
  uint32_t quirk_cols;
};
// Workspace bytes of a pass: hi and lo rows plus the exponents.
inline uint64_t gemm_f16_workspace_bytes(uint32_t ntok, uint32_t K) {
  return (uint64_t)ntok * K * 4 + (uint64_t)ntok * 4 + 256;
}
bool gemm_f16_supported(const GemmF16Args& a, int epi);
// f16_split then the GEMM: two launches.
cudaError_t gemm_f16(const GemmF16Args& a, int epi, const LaunchCfg& lc);

// ---- activations ------------------------------------------------------------
// Bit-exact Q8_0 quantization of nblocks 32-element blocks (warp per block).
cudaError_t quantize_q8(const float* x, int8_t* q, float* s, uint64_t nblocks, const LaunchCfg& lc);
// RMSNorm (util.rs:389-426) of ntok rows of `dim`, then Q8_0 quantization of
// the normalized rows into q/s (if q != null) and/or the f32 rows into y.
cudaError_t rmsnorm_quant(const float* x, const float* w, uint32_t ntok, uint32_t dim, float eps, int8_t* q,
                          float* s, float* y, const LaunchCfg& lc);

// Embedding rows (base_transformer.rs:143-161 over the dequantized table of
// transformer_llama_gguf.rs:453-489): x[t] = row(tokens[t]) as f32, zeros for
// out-of-range ids. tokens: device ids; if tok_from_state, tokens[0] is read
// from state->token.
struct StepState {
  int32_t pos;    // position of the token being processed
  int32_t token;  // token id being processed
  int32_t next;   // greedy id produced by this step
  int32_t steps;  // number of device steps executed
};
cudaError_t embed(int fmt, const uint8_t* wq, const uint8_t* ws, uint32_t row_bytes, uint32_t scale_row_bytes,
                  bool sf16, uint32_t dim, uint32_t vocab, const uint32_t* tokens, const StepState* state, uint32_t ntok,
                  float* x, const LaunchCfg& lc);

// RoPE + KV-cache write. qkv: [ntok][att_dim + 2 kv_dim] (q | k | v) from the
// fused projection; q_out: [ntok][att_dim] rotated; k/v rows go to
// kcache/vcache [ctx][kv_dim] (layer base) at positions pos0 + t. pos0 comes
// from state->pos when state != null. cs: cos/sin table [ctx][head_size/2].
cudaError_t rope_kv(const float* qkv, uint32_t ntok, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_size,
                    int rope_mode, const float2* cs, uint32_t ctx_len, const StepState* state, uint32_t pos0,
                    float* q_out, float* kcache, float* vcache, const LaunchCfg& lc);

// Causal GQA attention (forward.rs:299-400) for ntok queries at positions
// pos0..pos0+ntok-1 over kcache/vcache [ctx][kv_dim], bit-identical to the
// reference's sequence of f32 operations: 8-lane dot products, max, the
// correctly rounded exp, the softmax sum in position order, 1/sum, and the
// 8-lane P.V sums over the batch's seq_len = pos0 + ntok with the sequential
// tail. The scores and weights go through `part` ([ntok][n_heads][seq_len]
// floats, attention_scratch_floats). The output is quantized per 32-block into
// q8/s8 (Q8_0) and/or written as f32 into out.
struct AttnArgs {
  const float* q;
  const float* kcache;
  const float* vcache;
  uint32_t ntok, n_heads, n_kv_heads, head_size, kv_dim;
  const StepState* state;
  uint32_t pos0;
  float scale;
  uint32_t n_splits;  // unused (kept for the argument layout)
  float* part;  // scores / weights scratch [ntok][n_heads][pos0 + ntok]
  float* out;   // [ntok][n_heads*head_size] f32 (nullable)
  int8_t* q8;   // [ntok][n_heads*head_size] (nullable)
  float* s8;    // [ntok][n_heads*head_size/32]
};
cudaError_t attention(const AttnArgs& a, const LaunchCfg& lc);
// Row stride (floats) and size of `part` for attention(): one row of
// seq_len = pos0 + ntok weights per (query row, head), rows 16-byte aligned.
#if defined(__CUDACC__)
#define YL_KHD __host__ __device__
#else
#define YL_KHD
#endif
YL_KHD inline uint64_t attention_scratch_stride(uint32_t ntok, uint32_t pos0) {
  return ((uint64_t)pos0 + ntok + 3) / 4 * 4;
}
YL_KHD inline uint64_t attention_scratch_floats(uint32_t ntok, uint32_t n_heads, uint32_t pos0) {
  return (uint64_t)ntok * n_heads * attention_scratch_stride(ntok, pos0);
}

// Batch-1 decode attention with RoPE and the KV-cache write fused in:
// q and the new k/v rows are taken unrotated from `qkv` ([att | k | v]),
// rotated with cs[pos], the new k/v rows written at `pos`. One thread-block
// cluster of n_splits CTAs per KV head: the CTAs split the scores, then the
// output 32-blocks; scores and weights of every query head go through
// sc[head][sc_stride] (sc_stride >= pos + 1). Bit-identical to the
// reference's operation sequence, like attention(); the output is quantized
// per 32-block in the same kernel.
struct AttnDecodeArgs {
  const float* qkv;
  const float2* cs;  // [ctx][head_size/2]
  int rope_mode;
  float* kcache;
  float* vcache;
  uint32_t n_heads, n_kv_heads, head_size, kv_dim;
  const StepState* state;
  uint32_t pos0;
  float scale;
  uint32_t n_splits;      // cluster size, 1..16
  // Cache rows below pos were written by work that completed before the
  // preceding kernel started (a graph replay): fetch them before waiting.
  int early_kv;
  float* out;             // [n_heads*head_size] f32 (nullable)
  int8_t* q8;             // (nullable)
  float* s8;
  // timeline tracing (nullable): 8 slots per CTA in globaltimer nanoseconds:
  // entry, wait released, partials visible, done, q rotated, first key tile
  // in shared memory, partial ready, merge done
  uint64_t* trace;
  // issued by thread 0 of every CTA at entry (HBM is otherwise idle while
  // attention runs)
  L2Prefetch pf;
  float* sc;           // scores / weights scratch [n_heads][sc_stride]
  uint32_t sc_stride;
  // Independent sequences in one launch (batched decode of several
  // sessions): when nseq > 0, the CTAs of grid row y serve sequence y: its
  // layer caches kseq[y] / vseq[y], its position pseq[y], row y of qkv
  // (qkv_stride floats apart), out / q8 / s8 (n_heads*head_size apart) and
  // scratch sc + y * sc_seq_stride. kcache, vcache, state and pos0 are unused.
  uint32_t nseq;
  float* kseq[YL_MAX_BATCH];
  float* vseq[YL_MAX_BATCH];
  uint32_t pseq[YL_MAX_BATCH];
  uint64_t qkv_stride, sc_seq_stride;
};
// Cluster size for the decode attention: 16 when n_kv_heads clusters of 16
// can be resident at once, else 8.
uint32_t attention_decode_splits(uint32_t n_kv_heads, uint32_t head_size);
cudaError_t attention_decode(const AttnDecodeArgs& a, const LaunchCfg& lc);

// ---- tensor parallelism over peer memory --------------------------------
// Every rank owns one "exchange region" (cudaMalloc, shared by CUDA IPC) with
// the same layout; base[r] is rank r's region as mapped in this process.
// Flags: [sites][world] u32, written by peers (flag[site][src] = epoch).
struct TpArgs {
  uint8_t* base[8];
  uint32_t rank, world;
  uint32_t site;
  uint64_t flags_off;
  const uint32_t* epoch;  // this rank's completed-step counter (the step's epoch is *epoch + 1)
  int* err;
};
// All-reduce + residual add: x[i] += sum over ranks r (in rank order) of
// rank r's partial [n] at byte offset part_off of its region.
cudaError_t tp_allreduce_add(const TpArgs& t, uint64_t part_off, uint32_t n, float* x, const LaunchCfg& lc);
// Vocabulary-parallel greedy id: combines the ranks' published winners
// ({value, global index, first-logit NaN} at lm_off), writes the id to
// hist[state ? state->steps : 0], advances state like EPI_ARGMAX, increments
// *epoch (the step's last collective), and with logits != null gathers every
// rank's slice [vl] (at logit_off) into logits[V].
// pepoch (nullable): the single-token step counter of the push exchanges,
// incremented here after a decode step.
cudaError_t tp_argmax(const TpArgs& t, uint64_t lm_off, uint64_t logit_off, uint32_t vl, float* logits,
                      uint32_t* hist, StepState* state, uint32_t* epoch, uint32_t* pepoch, const LaunchCfg& lc);

// Greedy argmax over n logits (sampler.rs:67-79: the lowest index among equal
// maxima). Writes out[0]; with state != null also state->next/token/pos/steps
// for the device-resident decode loop.
cudaError_t argmax(const float* logits, uint32_t n, uint32_t* out, StepState* state, const LaunchCfg& lc);

// Starts a device-resident decode run: state = {pos, token, next 0, steps 0}
// (one thread; the values are launch arguments, so nothing is staged on the host).
cudaError_t set_step_state(StepState* state, int32_t pos, int32_t token, const LaunchCfg& lc);

// ---- device sampler (sampler.rs:117-180) ----------------------------------
struct SampleArgs {
  float* logits = nullptr;  // [V] on the device; overwritten (x/T, then probabilities) like Sampler::sample
  uint32_t V = 0, ntiles = 0;  // ntiles = sample_tiles(V)
  float temperature = 0.f, top_p = 0.f;
  float cutoff = 0.f;  // (1 - top_p) / (V - 1), computed in f32 as the reference does
  float rand = 0.f;    // random_f32(seed); the reference's generator never advances
  int topp = 0;        // 1: sample_topp, 0: sample_mult
  float* tile_val = nullptr;     // [ntiles]
  uint32_t* tile_cnt = nullptr;  // [ntiles]
  float* misc = nullptr;         // [0] softmax sum, [1] kept count (bits)
  float* prefix = nullptr;       // [V] cumulative sums of the sorted entries
  uint32_t* out = nullptr;       // sampled id (device)
  int* err = nullptr;
  // the persistent probability_idx array (prob, index) of the sampler, two
  // buffers for the radix sort; zero at creation
  float* sbuf_prob[2] = {nullptr, nullptr};
  uint32_t* sbuf_idx[2] = {nullptr, nullptr};
  float* sprob = nullptr;        // the current buffer (set by sample())
  uint32_t* sidx = nullptr;
  void* sort_temp = nullptr;
  size_t sort_temp_bytes = 0;
};
uint32_t sample_tiles(uint32_t V);
size_t sample_sort_temp_bytes(uint32_t V);
// Enqueues one Sampler::sample; *cur selects the current persistent buffer
// and is updated by the sort.
cudaError_t sample(SampleArgs& a, int* cur, const LaunchCfg& lc);
}  // namespace k
}  // namespace yl
