/*
 * yallma3_b200 — C-ABI of the B200-native quantized-weight forward path.
 *
 * This header is the drop-in boundary for yallma3-mini-inference's hot path.
 * Each entry point names the reference item it replaces (path:line inside the
 * reference project). All entry points are plain C: pointers and sizes only,
 * no C++ or torch types. Device pointers are CUDA global-memory addresses on
 * the current device; `stream` is a cudaStream_t passed as void* (NULL = the
 * legacy default stream).
 *
 * Errors: every function that can fail returns int (YL_OK = 0, negative =
 * error) and never aborts; yl_last_error() returns a thread-local message for
 * the last failure on the calling thread. (The reference panics across its
 * FFI; lib.rs:135-152 only returns false for load failures.)
 *
 * Threading: a yl_model may be shared by many threads (the reference's
 * `Transformer: Send + Sync`, transformer.rs:19). A yl_session is used by one
 * thread at a time (the reference passes `&mut InferenceSession`).
 */
#ifndef YALLMA3_B200_H
#define YALLMA3_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
enum yl_status {
  YL_OK = 0,
  YL_ERR_ARG = -1,         /* bad argument (null pointer, size, range) */
  YL_ERR_IO = -2,          /* file cannot be opened / read */
  YL_ERR_FORMAT = -3,      /* malformed file, or format/variant mismatch
                              (the reference panics: weight_type.rs:88,104) */
  YL_ERR_CUDA = -4,        /* CUDA runtime error */
  YL_ERR_OOM = -5,         /* device allocation failed */
  YL_ERR_RANGE = -6,       /* position beyond the session's ctx_len */
  YL_ERR_TIMEOUT = -7,     /* a bounded device wait expired */
  YL_ERR_UNSUPPORTED = -8, /* valid request the device path does not support */
  YL_ERR_COMM = -9         /* tensor-parallel communicator error */
};

/* WeightFormat (weight_type.rs:17-22). */
enum yl_weight_format { YL_Q8_0 = 0, YL_Q4_0 = 1, YL_F16 = 2 };

/* Scale element type of a yl_qtensor. */
enum yl_scale_type { YL_SCALE_F32 = 0, YL_SCALE_F16 = 1 };

/* Q4_0 decode semantics: GGML order (element j is the low nibble of byte j,
 * element j+16 the high nibble) with value (q - 8) * d. The reference's own
 * decode (interleaved nibbles, no -8, transformer_llama_gguf.rs:394-405) is
 * not GGML-conformant and exists only in the oracle as a documented mode. */
enum yl_q4_mode { YL_Q4_GGML = 0 };

/* RoPE variants: util.rs:653-718 `rope_gguf` (pairs 2k,2k+1) and
 * util.rs:589-635 `rope` (pairs j, j+hd/2, llama3 frequency scaling). */
enum yl_rope_mode { YL_ROPE_GGUF = 0, YL_ROPE_LLAMA3 = 1 };

const char* yl_last_error(void);
/* Library version string, e.g. "yallma3_b200 0.1 sm_100a". */
const char* yl_version(void);

/* ---- quantized tensors (weight_type.rs:24-50, quantization.rs:23-27) -----
 *
 * Two kinds share one struct:
 *  - activation tensors (rows == 0): the reference's flat containers.
 *    Q8_0 / Q4_0: `quant` int8[len], `scale` f32[len/gs]. F16 format keeps
 *    activations unquantized: `quant` f32[len], `scale` NULL
 *    (F16Kernel::quantize copies, forward.rs:78-81).
 *  - weight tensors (rows > 0, cols = row length): the repacked HBM layout.
 *    Q8_0: `quant` int8 [rows][cols]; Q4_0: `quant` GGML nibbles
 *    [rows][cols/2] (byte j of a block: low nibble = element j, high nibble =
 *    element j+16, value (q-8)*d); F16: `quant` f16 [rows][cols].
 *    `scale` [rows][scale_stride] of f16 (or f32), scale_stride padded so that
 *    every row starts on a 16-byte boundary.
 * Memory is owned by the library when allocated with yl_qtensor_alloc*.
 */
typedef struct yl_qtensor {
  int32_t fmt;         /* yl_weight_format */
  int32_t scale_type;  /* yl_scale_type */
  uint64_t len;        /* element count */
  uint64_t gs;         /* group size (32 on the device path) */
  uint64_t rows, cols; /* weights: matrix shape; activations: 0, 0 */
  uint64_t scale_stride;
  void* quant;
  void* scale;
  int32_t owned;       /* 1 if freed by yl_qtensor_free */
  int32_t flags;       /* bit 0: an f16 scale is +-inf (set by yl_qtensor_upload) */
} yl_qtensor;

/* new_workspace_buffer (weight_type.rs:108-120): zeroed activation tensor. */
int yl_qtensor_alloc(int fmt, uint64_t len, uint64_t gs, yl_qtensor* out);
/* Weight tensor [rows][cols] in the repacked layout (zeroed). */
int yl_qtensor_alloc_weight(int fmt, int scale_type, uint64_t rows, uint64_t cols, uint64_t gs,
                            yl_qtensor* out);
int yl_qtensor_free(yl_qtensor* t);
/* Copy host data in the reference container layout into `t`:
 *  Q8_0/Q4_0 activation or weight: q int8[len] (for Q4_0 weights: signed
 *  values q-8 in [-8,7]), scales f32[len/gs]; F16: values f32[len] (weights
 *  are rounded to f16; activations stay f32), scales NULL. Weight scales are
 *  stored as f16 when t->scale_type == YL_SCALE_F16 (exact only if every scale
 *  is an f16 value, as for GGUF weights). */
int yl_qtensor_upload(yl_qtensor* t, const int8_t* q, const float* scales, const float* values);
/* Inverse of yl_qtensor_upload (host buffers sized as above). */
int yl_qtensor_download(const yl_qtensor* t, int8_t* q, float* scales, float* values);

/* quantization.rs:29-52 `quantize`: per group of gs, scale = absmax/127 (f32),
 * q = round-half-away(x/scale) saturated to int8, NaN -> 0. Bit-exact with the
 * reference. x, q, scale are device pointers; floor(n/gs) groups are written. */
int yl_quantize_q8_0(const float* x, int8_t* q, float* scale, uint64_t n, uint32_t gs, void* stream);
/* weight_type.rs:76-90 `quantize(fmt, dst, x, n, gs)`: format dispatch into
 * an activation tensor (YL_ERR_FORMAT on a variant mismatch). */
int yl_quantize(int fmt, yl_qtensor* dst, const float* x, uint64_t n, uint32_t gs, void* stream);
/* weight_type.rs:92-106 `matmul(out, x, w, n, o, gs)` with the batch made
 * explicit (the reference infers it as out.len()/o). out: device f32
 * [batch][o]. accumulate = 1 reproduces the reference's store semantics
 * exactly (columns < 4*floor(o/4) add into out, the rest overwrite,
 * weight_type.rs:190-201 and :207-224, inside matmul_q8_slices :122-226);
 * accumulate = 0 overwrites every column. Q8_0 / Q4_0: batches of 5 or more
 * rows run on the int8 tensor-core GEMM, smaller ones on the matvec; both
 * fold the per-block int32 dots in the reference's order, so with
 * accumulate = 0 the results equal the reference's bit for bit. With
 * accumulate = 1 a quad column gets its initial value plus the folded row
 * (the reference adds every block term into the initial value in turn):
 * within 1e-5 of the sum of |terms| and |initial value|. F16 weights: below
 * 16 rows the matvec with f32 products summed in lane-parallel order; from 16
 * rows the f16 tensor-core GEMM on the activations split into two f16 parts
 * (stream-ordered scratch of 4 bytes per activation element; the matvec when
 * it cannot be had). Both within 1e-5 of the sum of |terms|. */
int yl_matmul(float* out, const yl_qtensor* x, const yl_qtensor* w, uint64_t n, uint64_t o, uint64_t gs,
              uint64_t batch, int accumulate, void* stream);

/* forward.rs:299-400 `fused_attention`: causal GQA attention of `batch` query
 * rows at positions start_pos..start_pos+batch-1 over key/value caches
 * [seq_len][kv_dim] (queries already rotated, caches already holding the new
 * rows, seq_len = start_pos + batch as in forward.rs:135). Scores use
 * attn_scale, masked positions are excluded, the softmax runs over the whole
 * visible row. sq/output: [batch][n_heads*head_size]. All device pointers,
 * 16-byte aligned. The result is bit-identical to the reference's: the same
 * f32 operations in the same order (8-lane dot products, the softmax sum in
 * position order, 8-lane P.V sums split at seq_len/8, exp correctly rounded).
 * seq_len must equal start_pos + batch. The reference takes its softmax
 * scratch from the caller (`scores`); here the weights live in a workspace of
 * batch * n_heads * round_up(seq_len, 4) floats that this function allocates
 * and frees on `stream`. head_size 64 or 128, n_heads/n_kv_heads <= 8. */
int yl_fused_attention(float* output, const float* sq, const float* key_cache, const float* value_cache,
                       uint64_t seq_len, uint64_t batch, uint64_t n_heads, uint64_t n_kv_heads, uint64_t head_size,
                       uint32_t start_pos, uint64_t kv_dim, float attn_scale, void* stream);

/* No counterpart in the reference: an addition of this library.
 * yl_fused_attention without any allocation, for callers that cannot call
 * cudaMalloc or cudaMallocAsync where attention runs (an engine whose memory
 * manager owns all device memory, or a latency-critical loop that must not
 * risk the allocator's implicit synchronization or out-of-memory failures).
 * Same arguments and result as yl_fused_attention; its workspace lives in a
 * fixed device array of YL_ATTN_STATIC_BYTES (1 MiB) that every GPU loading
 * this library holds until the process exits. A call whose workspace would
 * not fit (batch * n_heads * round_up(seq_len, 4) * 4 bytes) fails with
 * YL_ERR_UNSUPPORTED. Every call resolves the array's device address on the
 * current device (cudaGetSymbolAddress, which allocates nothing), so calls
 * after a cudaDeviceReset find the reloaded array; the first call on a device
 * also loads this library's kernels there, so make that first call before
 * any stream capture. All calls share the array: calls that overlap on the
 * GPU (other streams, other threads) race on it; serialize them. */
#define YL_ATTN_STATIC_BYTES (1u << 20)
int yl_fused_attention_static(float* output, const float* sq, const float* key_cache, const float* value_cache,
                              uint64_t seq_len, uint64_t batch, uint64_t n_heads, uint64_t n_kv_heads,
                              uint64_t head_size, uint32_t start_pos, uint64_t kv_dim, float attn_scale, void* stream);

/* ---- model and sessions (transformer.rs:19-69, lib.rs:107-133) ---------- */
typedef struct yl_model yl_model;
typedef struct yl_session yl_session;

/* TransformerShape (base_transformer.rs:25-44) plus the device-path switches. */
typedef struct yl_shape {
  uint32_t dim, hidden_dim, n_heads, head_size, n_kv_heads, vocab_size, n_layers, ctx_len;
  float rms_norm_eps, rope_theta;
  uint32_t group_size;
  float rope_freq_scale, rope_ext_factor, rope_attn_factor;
  uint32_t rope_original_ctx_len;
  float attention_scale;
  int32_t weight_format; /* yl_weight_format */
  int32_t rope_mode;     /* yl_rope_mode */
  int32_t untied_lm_head;
  int32_t tp_rank, tp_size;
  int32_t _pad;
} yl_shape;

/* Batched decode of independent sessions (no reference counterpart: the
 * reference serves one session per forward_x call, each user holding their
 * own InferenceSession, main.rs:23-32, with Transformer: Send + Sync,
 * transformer.rs:19). One yl_batch_forward call is one decode step for n
 * distinct sessions of the batch's model: token tokens[i] at position
 * positions[i] of sessions[i]. The projections run once over the n stacked
 * rows (weights streamed once per 8 rows on the matvec, once per 64 on the
 * GEMM from 16 rows) and the attention is one launch over every session's own
 * KV cache and position; each session's results equal a yl_forward_x step of
 * that session alone, bit for bit. logits_out (nullable): n x vocab floats,
 * row i for session i; ids_out (nullable): the n greedy ids. Each session's
 * pos becomes positions[i] + 1. n <= max_sessions <= 16; one GPU. */
typedef struct yl_batch yl_batch;
int yl_batch_create(const yl_model* m, uint32_t max_sessions, yl_batch** out);
int yl_batch_free(yl_batch* b);
int yl_batch_forward(yl_batch* b, yl_session* const* sessions, uint32_t n, const uint32_t* tokens,
                     const uint32_t* positions, float* logits_out, uint32_t* ids_out);

/* Process-wide options of the device path (no reference counterpart), read
 * by launches made after the call:
 *  "gemm"        1 = batches of 5+ tokens on the int8 tensor-core GEMM (default)
 *  "gemm_tc"     1 = Q8_0 batches on the tcgen05 / tensor-memory kernel
 *                (bit-identical, not faster; default 0, env YL_GEMM_TC)
 *  "gemm_tc_min" token count from which gemm_tc applies (default 96)
 *  "gemm_f16_min" F16 passes of this many tokens on the f16 tensor-core GEMM
 *                (default 16, env YL_GEMM_F16_MIN; 0 = the matvec at every N)
 * YL_ERR_ARG for an unknown key. */
int yl_config_set(const char* key, int64_t value);

/* lib.rs:107-133 `load_transformer(path, sequential, max_ctx_len, fmt_override)`.
 * Dispatch by extension:
 *  - .gguf (architecture must be "llama"; fmt_override = -1 keeps
 *    general.file_type);
 *  - .safetensors with config.json beside it (transformer_llama_st.rs): MLX
 *    affine 8-bit weights are requantized to symmetric Q8 with f32 scales
 *    (util.rs:451-518), F16 weights when config.json has no "quantization"
 *    section; a "Q4_0" quant_type gives YL_ERR_UNSUPPORTED (the reference
 *    runs its Q4_0 kernel on requantized Q8 tensors there). BOS/EOS come
 *    from tokenizer.json, else tokenizer.bin;
 *  - .lmrs (transformer_llama_lmrs.rs): Q8 with f32 scales whatever the
 *    override; tokenizer.bin beside it supplies BOS/EOS.
 * Quantized files must use groups of 32 (YL_ERR_UNSUPPORTED otherwise).
 * `sequential` selects nothing on the device path: the forward is
 * forward.rs's llama_forward_x for every format. Weights are parsed on the
 * host, repacked and uploaded to the current CUDA device. */
int yl_load_transformer(const char* path, int sequential, uint32_t max_ctx_len, int fmt_override,
                        yl_model** out);
/* Tensor parallelism (no counterpart in the reference, which runs on one
 * CPU; this is the Megatron split of forward.rs:154-279 for one NVSwitch
 * box). Rank tp_rank of tp_size (2..8, one process per GPU, the device
 * current) loads its shard: q/k/v heads and gate/up rows by rank, wo and
 * down along their inputs, lm_head by vocabulary rows; embeddings and norms
 * whole. Needs KV heads, ffn/64 and vocabulary divisible by tp_size.
 * Sessions of such a model exchange partial sums over NVLink peer memory
 * after wo and down, and per-rank greedy winners after the lm_head: create
 * the session on every rank, collect every rank's yl_session_tp_handle (64
 * bytes) in rank order, and pass the array to yl_session_tp_connect. Every
 * rank must then make the same forward/decode calls in the same order (the
 * exchange waits for all ranks, bounded: a missing rank gives
 * YL_ERR_TIMEOUT). */
int yl_load_transformer_tp(const char* path, uint32_t max_ctx_len, int fmt_override, int tp_rank, int tp_size,
                           yl_model** out);
int yl_session_tp_handle(yl_session* s, void* handle_out);
int yl_session_tp_connect(yl_session* s, const void* handles);
/* The split itself, without a GPU: first row / row count of this rank's q
 * rows, k (= v) rows, gate (= up) rows and vocabulary rows. */
typedef struct yl_tp_split {
  uint32_t q_rows0, q_rows, kv_rows0, kv_rows, ffn_rows0, ffn_rows, vocab0, vocab_rows;
} yl_tp_split;
int yl_tp_plan(const yl_shape* shape, int tp_rank, int tp_size, yl_tp_split* out);
int yl_model_free(yl_model* m);
const char* yl_model_name(const yl_model* m);            /* Transformer::name */
uint64_t yl_model_vocab_size(const yl_model* m);         /* Transformer::vocab_size */
uint32_t yl_model_max_ctx_len(const yl_model* m);        /* Transformer::max_ctx_len */
uint32_t yl_model_eos_token(const yl_model* m);          /* Transformer::eos_token */
uint32_t yl_model_bos_token(const yl_model* m);          /* Transformer::bos_token */
int yl_model_shape(const yl_model* m, yl_shape* out);
/* Bytes of device memory the model's weights occupy. */
uint64_t yl_model_device_bytes(const yl_model* m);
/* base_transformer.rs:129-161: host f32 copies; out-of-range ids give zeros. */
int yl_get_embeddings(const yl_model* m, uint32_t token, float* out);
int yl_get_embeddings_batch(const yl_model* m, const uint32_t* tokens, uint64_t n, float* out);
/* Device view of one weight matrix: which = 0 wq, 1 wk, 2 wv, 3 wo, 4 w1 (gate),
 * 5 w2 (down), 6 w3 (up), 7 lm_head (tied embedding or output.weight).
 * The view aliases model memory (owned = 0). */
int yl_model_weight(const yl_model* m, uint32_t layer, int which, yl_qtensor* out);

/* InferenceSession (base_transformer.rs:78-105): device KV cache f32
 * [n_layers][ctx_len][kv_dim] for keys and values, zeroed. */
int yl_create_session(const yl_model* m, yl_session** out);
int yl_session_reset(yl_session* s);
int yl_session_free(yl_session* s);
uint32_t yl_session_pos(const yl_session* s);
int yl_session_set_pos(yl_session* s, uint32_t pos);
/* Device pointers of the session's KV cache (for inspection). */
int yl_session_kv(const yl_session* s, float** key_cache, float** value_cache, uint64_t* elems);

/* Transformer::forward_x (transformer.rs:44-53; forward.rs:282-297).
 * tokens: host array of n ids at positions start_pos..start_pos+n-1. Writes the
 * last token's logits to logits_out (host, vocab floats) and/or its greedy id
 * (sampler.rs:67-79 semantics: lowest index among equal maxima) to
 * argmax_out; either may be NULL. Like the reference, the caller advances the
 * session position; this call does not. */
int yl_forward_x(const yl_model* m, yl_session* s, const uint32_t* tokens, uint64_t n, uint32_t start_pos,
                 float* logits_out, uint32_t* argmax_out);
/* Device-resident greedy decode: n_steps batch-1 steps starting with
 * `first_token` at `start_pos`, each step feeding its argmax to the next,
 * without host round trips (one CUDA graph launch per step). tokens_out:
 * host array of n_steps ids (NULL allowed). Runs on `stream`; returns after
 * enqueueing when sync == 0 (tokens_out must then be NULL). */
int yl_decode_greedy(const yl_model* m, yl_session* s, uint32_t first_token, uint32_t start_pos,
                     uint32_t n_steps, uint32_t* tokens_out, void* stream, int sync);
/* Number of kernel launches one batch-1 decode step issues (the decode
 * graph's kernels: 5 per layer + 2, + 1 with tensor parallelism, + 2 per layer
 * more when the tensor-parallel exchange runs as separate kernels). */
int yl_decode_step_launches(const yl_model* m, uint32_t* out);
/* The decode step's attention kernel on its own, with the model's RoPE table,
 * head layout and attention scale (no reference counterpart as one function:
 * it fuses the batch-1 RoPE of q/k and the cache write of forward.rs:154-175
 * with fused_attention, forward.rs:299-400). qkv: device [q (heads*hd) | k |
 * v] of one token, unrotated; key_cache/value_cache: device [>= pos+1][kv_dim]
 * (one layer); the new k/v rows are rotated and written at `pos`, then the
 * token attends to positions 0..pos. out: f32 [heads*hd] and/or out_q/out_s:
 * its Q8_0 blocks (either may be NULL, not both). */
int yl_model_attention_decode(const yl_model* m, const float* qkv, float* key_cache, float* value_cache, uint32_t pos,
                              float* out, int8_t* out_q, float* out_s, void* stream);
/* Diagnostic (no reference counterpart): the kernel nodes of this session's
 * captured decode graph, counted in the graph itself (builds the graph if
 * needed; with_logits selects the tensor-parallel graph that also gathers
 * the logits). Equals yl_decode_step_launches for the graph without logits. */
int yl_session_decode_graph_launches(yl_session* s, int with_logits, uint32_t* out);
/* Diagnostic: runs one batch-1 decode step of `token` at `pos` launch by
 * launch (no graph, no programmatic dependent launch) with CUDA events
 * between launches, and writes each launch's device time in microseconds to
 * us_out (up to cap entries; *n_out = launches). Order: embedding, then per
 * layer qkv, attention, wo, gate/up, down, then lm_head. */
int yl_profile_decode_step(const yl_model* m, yl_session* s, uint32_t token, uint32_t pos, float* us_out,
                           uint32_t cap, uint32_t* n_out);
/* Diagnostic, in a build with YL_WITH_TRACE=1 only (YL_ERR_UNSUPPORTED
 * otherwise): runs one batch-1 decode step of `token` at `pos` exactly as the
 * decode graph does (one graph, programmatic dependent launch) while every
 * matvec and attention CTA stamps the GPU's nanosecond global timer:
 * out[launch * 8192 + cta * 8 + i], i = 0 entry, 1 activations staged
 * (attention: wait released), 2 wait on the preceding kernel released
 * (attention: every slice's scores visible), 3 done; RMSNorm prologues also 6
 * warp 0's rows quantized, 7 the last warp's (4, 5: the tensor-parallel
 * prologue's rows loaded, norm factor ready); attention also 4 q rotated,
 * 5 first key tile in shared memory, 6 slice scores written, 7 softmax sums
 * done (0 where not stamped). Launch order as yl_profile_decode_step; the
 * embedding launch (index 0) is not stamped. Writes up to cap values;
 * *n_launches = launches. */
int yl_trace_decode_step(const yl_model* m, yl_session* s, uint32_t token, uint32_t pos, uint64_t* out,
                         uint64_t cap, uint32_t* n_launches);

/* ---- reference FFI (lib.rs:135-152) -------------------------------------- */
/* Loads into a process-global slot (guarded by a mutex here; `static mut` in
 * the reference). Returns false on any error. */
bool load_transformer_ffi(const char* model_path);

/* infer_ffi / free_string as the reference documents them (README.md:88-92,
 * PoC_Bun_load.js:12-38; the reference declares but never implements them).
 * infer_ffi runs one fresh conversation on the model load_transformer_ffi
 * loaded, the way the reference's console does (main.rs:149-214): the prompt,
 * trimmed of Unicode white space at both ends as the console trims its line,
 * is tokenized with the model's tokenizer into the chat prompt of
 * yl_tokenizer_chat_prompt with an empty system prompt (the GGUF file's chat
 * template when it has one, else the built-in format), prefilled,
 * and tokens are sampled on the device and decoded one at a time until EOS,
 * the context length or the token limit. The reply (the decoded pieces
 * concatenated, each piece decoded on its own as the console prints it) is
 * returned as a malloc'ed UTF-8 string to be released with free_string.
 * NULL on any error (no model loaded, empty (after trimming) or non-UTF-8 prompt, prompt longer
 * than the context; yl_last_error() says which). Calls are serialized by a
 * mutex. Every call is a fresh conversation: the session's buffers persist
 * but its cache is reset, whereas the console continues one conversation
 * across turns (main.rs:223-226 never resets its only session); the sampler
 * keeps its state across calls, as the console's does. */
const char* infer_ffi(const char* prompt);
void free_string(const char* s);
/* Sampling of infer_ffi. Defaults are the console's Sampler::new(vocab, 0.7,
 * 0.9, 42) (main.rs:135) and no token limit (max_tokens 0). Takes effect at the
 * next infer_ffi call (a changed setting starts a fresh sampler). */
int yl_infer_config(float temperature, float top_p, uint64_t seed, uint32_t max_tokens);

/* ---- tokenizer (tokenizer.rs) -------------------------------------------- */
/* Host-side byte-level BPE tokenizer, loaded from the files the reference's
 * loaders read: a .gguf file's tokenizer.ggml.* metadata
 * (Tokenizer::from_gguf_parts, tokenizer.rs:78-132), tokenizer.json
 * (from_json, :134-217) else tokenizer.bin (new, :219-262) beside a
 * .safetensors file, tokenizer.bin beside a .lmrs file. Needs no GPU.
 * A GGUF file's chat template (tokenizer.chat_template) is parsed at load
 * (set_chat_template, tokenizer.rs:408-416) and rendered by the prompts
 * below with minijinja's semantics (the reference's template engine); a
 * template that does not parse makes those calls fail with the parse error
 * (the reference panics at load). */
typedef struct yl_tokenizer yl_tokenizer;
int yl_tokenizer_load(const char* model_path, yl_tokenizer** out);
int yl_tokenizer_free(yl_tokenizer* t);
/* Transformer::tokenizer(): the model's tokenizer, loaded from the model's
 * file at the first call and owned by the model. */
int yl_model_tokenizer(const yl_model* m, const yl_tokenizer** out);
/* vocabulary size, BOS, EOS, whether a chat template is present */
int yl_tokenizer_info(const yl_tokenizer* t, uint32_t* vocab_size, uint32_t* bos, uint32_t* eos, int* has_template);
/* Tokenizer::encode(text, bos, eos) (tokenizer.rs:338-392). text: non-empty
 * UTF-8 (YL_ERR_ARG otherwise). Writes up to cap ids; *n_out = the full count
 * (YL_ERR_RANGE when it exceeds cap). */
int yl_tokenizer_encode(const yl_tokenizer* t, const char* text, int bos, int eos, uint32_t* ids, uint64_t cap,
                        uint64_t* n_out);
/* Tokenizer::decode (tokenizer.rs:523-551): UTF-8 bytes (invalid sequences
 * replaced by U+FFFD), NUL-terminated when it fits; *n_out = byte count
 * without the terminator (YL_ERR_RANGE when n_out + 1 exceeds cap). */
int yl_tokenizer_decode(const yl_tokenizer* t, const uint32_t* ids, uint64_t n, char* out, uint64_t cap,
                        uint64_t* n_out);
/* The console's prompt of a fresh conversation (main.rs:149-153,177).
 * Without a chat template: apply_system_template(system) then
 * apply_turn_template(user, true), no-template branches (tokenizer.rs:475-521);
 * YL_ERR_FORMAT when a Llama-3 vocabulary does not encode "user" /
 * "assistant" as single tokens (a panic in the reference). With a template:
 * [BOS] when add_bos_token, the rendered system turn when system is non-empty
 * (apply_system_template), the rendered turn of [user, empty assistant] with
 * add_generation_prompt, less a trailing <|eot_id|> (apply_turn_template).
 * Template errors as yl_chat_template_render. */
int yl_tokenizer_chat_prompt(const yl_tokenizer* t, const char* system, const char* user, uint32_t* ids,
                             uint64_t cap, uint64_t* n_out);
/* The pieces the prompt above is made of, as the reference's Tokenizer has
 * them. encode_wrap_n_header (tokenizer.rs:277-297): with a Llama-3 vocabulary
 * [<|begin_of_text|>] if wrap, the header in <|start_header_id|> ..
 * <|end_header_id|> "\n\n" if non-empty, the text, ["\n\n", <|eot_id|>] if
 * wrap; otherwise [BOS] if wrap and add_bos_token, then the text. */
int yl_tokenizer_encode_wrap_n_header(const yl_tokenizer* t, const char* text, const char* header,
                                      int begin_of_text_wrap, uint32_t* ids, uint64_t cap, uint64_t* n_out);
/* set_chat_template (tokenizer.rs:408-416): parses and installs a chat
 * template (errors as yl_chat_template_render's parse step; on an error the
 * tokenizer is unchanged, where the reference panics). Not concurrently with
 * other calls on the same tokenizer. */
int yl_tokenizer_set_chat_template(yl_tokenizer* t, const char* tmpl);
/* apply_system_template (tokenizer.rs:477-495) and
 * apply_turn_template(user, add_empty_assistant) (:497-539). */
int yl_tokenizer_apply_system_template(const yl_tokenizer* t, const char* system, uint32_t* ids, uint64_t cap,
                                       uint64_t* n_out);
int yl_tokenizer_apply_turn_template(const yl_tokenizer* t, const char* user, int add_empty_assistant, uint32_t* ids,
                                     uint64_t cap, uint64_t* n_out);
/* Tokenizer::render_chat_template (tokenizer.rs:418-436): the chat template
 * rendered with {messages: [{role, content}] x n_messages,
 * add_generation_prompt}, then encode_template_output (:438-473): at each '<'
 * the longest vocabulary entry matching there is one id, the text up to the
 * next '<' goes through encode(text, false, false). *n_out = 0 when the
 * tokenizer has no template or the text is empty. */
int yl_tokenizer_render_chat(const yl_tokenizer* t, const char* const* roles, const char* const* contents,
                             uint64_t n_messages, int add_generation_prompt, uint32_t* ids, uint64_t cap,
                             uint64_t* n_out);
/* The text step alone: renders template source with the same context
 * (minijinja 2.20 at default settings: no trim_blocks / lstrip_blocks, one
 * trailing newline of the source dropped, lenient undefined values, no
 * Python-style string methods). Output as yl_tokenizer_decode. Errors:
 * YL_ERR_FORMAT where minijinja fails (syntax; an undefined value under
 * attribute access or arithmetic; an unknown filter, test, function or method;
 * a type error), YL_ERR_UNSUPPORTED for a construct this renderer does not
 * implement (floats, macros, call / filter / with blocks, includes, the less
 * common builtin filters), YL_ERR_ARG for text that is not UTF-8.
 * Parsing and rendering run on an internal thread with an 8 MiB stack and
 * bound nesting (more than ~250 nested parentheses, expressions deeper than
 * 1000 nodes, blocks nested more than 200 deep: YL_ERR_FORMAT). */
int yl_chat_template_render(const char* tmpl, const char* const* roles, const char* const* contents,
                            uint64_t n_messages, int add_generation_prompt, char* out, uint64_t cap,
                            uint64_t* n_out);

/* ---- device sampler (sampler.rs:41-180) ---------------------------------- */
/* Sampler::new(vocab_size, temperature, top_p, seed): device state (the
 * persistent (prob, index) array, zeroed) on the current CUDA device. A
 * sampler is used by one thread at a time (the reference's `&mut self`). */
typedef struct yl_sampler yl_sampler;
int yl_sampler_create(uint32_t vocab_size, float temperature, float top_p, uint64_t seed, yl_sampler** out);
int yl_sampler_free(yl_sampler* s);
/* Sampler::sample(&mut logits): logits is a DEVICE row of vocab_size floats
 * and is overwritten as the reference overwrites its slice (divided by the
 * temperature, then the probabilities; untouched at temperature 0). The id is
 * written to *id_out (host) after the stream synchronizes; with id_out NULL
 * the call returns once the work is enqueued and yl_sampler_result() reads the
 * id later. stream NULL: the legacy default stream. */
int yl_sampler_sample(yl_sampler* s, float* logits, uint32_t* id_out, void* stream);
int yl_sampler_result(yl_sampler* s, uint32_t* id_out);
/* The session's logits row on the device after its latest yl_forward_x (the
 * last token's logits; single-GPU models). */
int yl_session_logits(const yl_session* s, float** logits);

/* ---- synthetic model files (test and bench inputs) ----------------------- */
typedef struct yl_synth_config {
  uint32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, context_length;
  float rope_theta, rms_norm_eps;
  int32_t weight_format; /* yl_weight_format */
  int32_t tied;          /* 0 writes output.weight */
  int32_t llama3_scaling;
  float llama3_factor, llama3_low, llama3_high;
  uint32_t llama3_orig_ctx;
  uint64_t seed;
  float weight_std;
  int32_t threads;
} yl_synth_config;
/* Writes a GGUF v3 llama model with weights ~ N(0, weight_std) from a
 * counter-based generator (seeded), norms = 1.0, a dummy token list. */
int yl_synth_write_gguf(const char* path, const yl_synth_config* cfg);

#ifdef __cplusplus
}
#endif
#endif /* YALLMA3_B200_H */
