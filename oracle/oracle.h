/*
 * CPU ORACLE — test infrastructure only.
 *
 * A C++ restatement of the yallma3-mini-inference CPU forward path, used as the
 * parity checker for the CUDA path and as the timed CPU baseline in bench.py.
 * Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline / --impl
 * reference legs) may load it. The product library never links or calls it.
 *
 * Pinning: the reference is Rust (rayon/wide/half/memmap2) and cannot be built
 * in this environment (no cargo/rustc, no crate sources). The oracle is pinned
 * against every known-answer and property test the reference ships for this
 * path: tests/matmul_q8_tests.rs:30-53 (remainder-column KAT) and the rms_norm /
 * silu property tests in tests/simd_tests.rs:87-340. Everything else follows the
 * reference source line by line (citations on each function). Two details are
 * third-party and therefore "parity unpinned" at the ULP level: the horizontal
 * order of wide::f32x8::reduce_add (wide 0.7.33) and wide's f32x8 exp used by the
 * SiLU in forward.rs:230. The oracle uses a pairwise 8-lane fold and libm expf.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* WeightFormat (weight_type.rs:17-22). */
enum { ORC_Q8_0 = 0, ORC_Q4_0 = 1, ORC_F16 = 2 };

/* Q4_0 decoding modes. GGML: element j = low nibble of byte j, element j+16 =
 * high nibble, value (q-8)*d, Q8_0 activations (the GGML semantics the
 * benchmark configurations define).
 * REF: the literal reference decode (transformer_llama_gguf.rs:394-405: lo->2j,
 * hi->2j+1, no -8) with the +-7 activation quantizer (weight_type.rs:52-74). */
enum { ORC_Q4_GGML = 0, ORC_Q4_REF = 1 };

/* RoPE variants (util.rs:589-635 `rope`, util.rs:653-718 `rope_gguf`). */
enum { ORC_ROPE_GGUF = 0, ORC_ROPE_LLAMA3 = 1 };

/* TransformerShape (base_transformer.rs:25-44) plus the switches above. */
typedef struct orc_shape {
  uint32_t dim, hidden_dim, n_heads, head_size, n_kv_heads, vocab_size, n_layers, ctx_len;
  float rms_norm_eps, rope_theta;
  uint32_t group_size;
  float rope_freq_scale, rope_ext_factor, rope_attn_factor;
  uint32_t rope_original_ctx_len;
  float attention_scale;
  int32_t weight_format;  /* ORC_Q8_0 / ORC_Q4_0 / ORC_F16 */
  int32_t rope_mode;      /* ORC_ROPE_GGUF / ORC_ROPE_LLAMA3 */
  float llama3_old_ctx;   /* rope(): old_context_len (reference: ctx_len) */
  int32_t q4_mode;        /* ORC_Q4_GGML / ORC_Q4_REF */
  int32_t untied_lm_head; /* 1 when output.weight was read */
  uint32_t bos, eos;
} orc_shape;

/* ---- numeric kernels ---------------------------------------------------- */
void orc_set_threads(int n);
/* Sensitivity probe (test infrastructure): flags != 0 perturbs the oracle by
 * at most one rounding step. Bit 0: the rmsnorm sum of squares is accumulated
 * in double instead of the reference's 8-lane f32 fold. Bit 1: exp is the C
 * library's expf (within 0.502 ulp) instead of the correctly rounded e^x.
 * Used only to measure how far a model's logits move under a 1-ulp change
 * (how sensitive a test model is to activation-quantization flips);
 * 0 = the faithful restatement. */
void orc_set_probe(int flags);
int orc_get_threads(void);

void orc_quantize_q8(int8_t* q, float* scale, const float* x, size_t n, uint32_t gs);
void orc_quantize_q4_ref(int8_t* q, float* scale, const float* x, size_t n, uint32_t gs);
void orc_matmul_q8_slices(float* xout, size_t out_len, const int8_t* x, const float* x_scale,
                          const int8_t* w, const float* w_scale, size_t n, size_t o, size_t gs);
void orc_matmul_f32(float* xout, size_t out_len, const float* x, const float* w, size_t n, size_t o);
void orc_block_dots(int32_t* out, const int8_t* x, const int8_t* w, size_t batch, size_t n, size_t o,
                    size_t gs);
void orc_rmsnorm(float* o, const float* x, const float* weight, size_t size, float eps, int add_unit_offset);
void orc_rms_norm_scalar(float* x, size_t n, const float* weight, float eps, int add_unit_offset);
void orc_silu(float* x, size_t n);
void orc_rope(const orc_shape* s, float* sq, float* k, uint32_t pos);
void orc_rope_gguf(const orc_shape* s, float* sq, float* k, uint32_t pos);
void orc_fused_attention(float* output, float* scores, const float* sq, const float* key_cache,
                         const float* value_cache, size_t seq_len, size_t batch, size_t n_heads,
                         size_t n_kv_heads, size_t head_size, uint32_t start_pos, size_t kv_dim,
                         float attn_scale);
uint32_t orc_argmax(const float* p, size_t n);
float orc_f16_to_f32(uint16_t h);

/* ---- model / session ----------------------------------------------------- */
typedef struct orc_model orc_model;
typedef struct orc_session orc_session;

/* fmt_override: -1 = from general.file_type. q4_mode: ORC_Q4_*. Returns NULL on
 * error; orc_last_error() tells why. */
orc_model* orc_model_load(const char* path, uint32_t max_ctx_len, int fmt_override, int q4_mode);
void orc_model_free(orc_model* m);
const char* orc_last_error(void);
int orc_model_shape(const orc_model* m, orc_shape* out);
int orc_get_embeddings(const orc_model* m, uint32_t token, float* out);
orc_session* orc_session_new(const orc_model* m);
void orc_session_free(orc_session* s);
void orc_session_reset(orc_session* s);
float* orc_session_key_cache(orc_session* s);
float* orc_session_value_cache(orc_session* s);
size_t orc_session_cache_len(const orc_session* s);
/* llama_forward_x (forward.rs:119-297). logits: vocab floats. Returns 0 on success. */
int orc_forward_x(const orc_model* m, orc_session* s, const uint32_t* tokens, size_t n, uint32_t start_pos,
                  float* logits);

#ifdef __cplusplus
}
#endif
