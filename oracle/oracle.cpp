/*
 * CPU ORACLE — test infrastructure only (see oracle.h for the contract).
 *
 * Restates the reference CPU path of yallma3-mini-inference line by line.
 * All citations are path:line inside the reference project (src_llm/...).
 * Build: -O3 -ffp-contract=off, no -ffast-math, so that every f32 operation is
 * one IEEE-rounded operation in the same order as the Rust code (Rust never
 * contracts a*b+c into an FMA).
 */
#include "oracle.h"

#include <fcntl.h>
#include <omp.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;
int g_probe = 0;

/* Rust `f as i8`: saturating, NaN -> 0. */
inline int8_t rust_f32_as_i8(float v) {
  if (v != v) return 0;
  if (v >= 127.0f) return 127;
  if (v <= -128.0f) return -128;
  return (int8_t)v;
}

/* e^x rounded to nearest float. The reference calls `f32::exp` in the
 * softmax (forward.rs:358, the platform libm's expf) and wide's f32x8 exp in
 * the SiLU (forward.rs:230, wide 0.7.33, not vendored; f32::exp for a scalar
 * tail, :235). Neither is pinned
 * to the bit: glibc's expf is within 0.502 ulp and, checked over all 2^32
 * float inputs (tests/test_expf_exact.py), differs from the correctly rounded
 * value by one ulp on 170,648 of them. The oracle defines exp as the correctly
 * rounded value, computed through the C library's double exp (whose error is
 * far below half a float ulp; the same test finds it equal to an x87
 * long-double evaluation on every input). Probe bit 1 switches back to the
 * C library's expf to measure what that choice moves. */
inline float exp_f32(float x) {
  if (g_probe & 2) return expf(x);
  return (float)exp((double)x);
}

/* wide::f32x8::reduce_add (wide 0.7.33, not vendored; order unpinned).
 * Assumed: (lo4 + hi4) folded pairwise, the SSE horizontal-sum idiom. */
inline float reduce_add8(const float l[8]) {
  float a0 = l[0] + l[4], a1 = l[1] + l[5], a2 = l[2] + l[6], a3 = l[3] + l[7];
  float b0 = a0 + a2, b1 = a1 + a3;
  return b0 + b1;
}

/* 8-lane partial dot (f32x8 `sum += a*b` then reduce_add, then scalar tail),
 * the pattern of forward.rs:265-277, :332-343 and util.rs:399-408. */
inline float dot8(const float* a, const float* b, size_t n) {
  size_t n_simd = n / 8;
  float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t s = 0; s < n_simd; ++s)
    for (int l = 0; l < 8; ++l) {
      float p = a[s * 8 + l] * b[s * 8 + l];
      lanes[l] = lanes[l] + p;
    }
  float acc = reduce_add8(lanes);
  for (size_t d = n_simd * 8; d < n; ++d) {
    float p = a[d] * b[d];
    acc = acc + p;
  }
  return acc;
}

}  // namespace

extern "C" {

float orc_f16_to_f32(uint16_t h) {
  /* half::f16::to_f32 (half 2.7.1): exact widening. */
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

void orc_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
void orc_set_probe(int flags) { g_probe = flags; }
int orc_get_threads(void) { return omp_get_max_threads(); }

/* quantization.rs:29-52 */
void orc_quantize_q8(int8_t* q, float* scale_out, const float* x, size_t n, uint32_t gs) {
  uint32_t num_groups = (uint32_t)n / gs;
  const float q_max = 127.0f;
  for (uint32_t group = 0; group < num_groups; ++group) {
    float wmax = 0.0f;
    for (uint32_t i = 0; i < gs; ++i) {
      float val = fabsf(x[group * gs + i]);
      if (val > wmax) wmax = val;
    }
    float scale = wmax / q_max;
    scale_out[group] = scale;
    for (uint32_t i = 0; i < gs; ++i) {
      float quant_value = x[group * gs + i] / scale;
      q[group * gs + i] = rust_f32_as_i8(roundf(quant_value));
    }
  }
}

/* weight_type.rs:52-74 (`q4_0_quantize`, the reference's +-7 quantizer) */
void orc_quantize_q4_ref(int8_t* q, float* scale_out, const float* x, size_t n, uint32_t gs) {
  uint32_t num_groups = (uint32_t)n / gs;
  const float q_max = 7.0f;
  for (uint32_t group = 0; group < num_groups; ++group) {
    float wmax = 0.0f;
    for (uint32_t i = 0; i < gs; ++i) {
      float val = fabsf(x[group * gs + i]);
      if (val > wmax) wmax = val;
    }
    float scale = wmax / q_max;
    scale_out[group] = scale;
    for (uint32_t i = 0; i < gs; ++i) {
      float quant_value = x[group * gs + i] / scale;
      int8_t qv = rust_f32_as_i8(roundf(quant_value));
      q[group * gs + i] = qv < -7 ? -7 : (qv > 7 ? 7 : qv);
    }
  }
}

/* weight_type.rs:122-226 (`matmul_q8_slices`). Quirks kept: quad columns use
 * `+=` into out (:190-201), remainder columns use `=` (:207-224); the quad path
 * only sees floor(remaining/8)*8 elements of a group (:147-155, no scalar
 * tail); batch rows = out_len / o (par_chunks_exact_mut, :135). */
void orc_matmul_q8_slices(float* xout, size_t out_len, const int8_t* x, const float* x_scale,
                          const int8_t* w, const float* w_scale, size_t n, size_t o, size_t gs) {
  if (o == 0) return;
  size_t rows = out_len / o;
  size_t quads = o / 4;
  for (size_t row_idx = 0; row_idx < rows; ++row_idx) {
    float* elem = xout + row_idx * o;
    size_t xi = row_idx * n;
#pragma omp parallel for schedule(static)
    for (long long cc = 0; cc < (long long)quads; ++cc) {
      size_t col_chunk = (size_t)cc;
      size_t ni[4];
      for (int c = 0; c < 4; ++c) ni[c] = (col_chunk * 4 + c) * n;
      size_t group_start = 0;
      while (group_start < n) {
        size_t group_end = group_start + gs < n ? group_start + gs : n;
        size_t remaining = group_end - group_start;
        size_t n_simd = remaining / 8;
        uint32_t ival[4] = {0, 0, 0, 0}; /* i32x8 lanes, wrapping; the lane fold is exact */
        for (size_t s = 0; s < n_simd; ++s) {
          size_t base = group_start + s * 8;
          for (int l = 0; l < 8; ++l) {
            int32_t xv = x[xi + base + l];
            for (int c = 0; c < 4; ++c) ival[c] += (uint32_t)(xv * (int32_t)w[ni[c] + base + l]);
          }
        }
        for (int c = 0; c < 4; ++c) {
          float t = (float)(int32_t)ival[c] * w_scale[(ni[c] + group_start) / gs];
          t = t * x_scale[(xi + group_start) / gs];
          elem[col_chunk * 4 + c] = elem[col_chunk * 4 + c] + t;
        }
        group_start = group_end;
      }
    }
    size_t handled = quads * 4;
    for (size_t col = handled; col < o; ++col) {
      size_t ni0 = col * n;
      float sum = 0.0f;
      size_t group_start = 0;
      while (group_start < n) {
        size_t group_end = group_start + gs < n ? group_start + gs : n;
        int32_t block_sum = 0;
        for (size_t k = group_start; k < group_end; ++k) block_sum += (int32_t)x[xi + k] * (int32_t)w[ni0 + k];
        float t = (float)block_sum * w_scale[(ni0 + group_start) / gs];
        t = t * x_scale[(xi + group_start) / gs];
        sum = sum + t;
        group_start = group_end;
      }
      elem[col] = sum;
    }
  }
}

/* weight_type.rs:228-270 (`matmul_f32`): sequential f32 sums, `=` semantics. */
void orc_matmul_f32(float* xout, size_t out_len, const float* x, const float* w, size_t n, size_t o) {
  if (o == 0) return;
  size_t rows = out_len / o;
  size_t quads = o / 4;
  for (size_t row_idx = 0; row_idx < rows; ++row_idx) {
    float* elem = xout + row_idx * o;
    size_t xi = row_idx * n;
#pragma omp parallel for schedule(static)
    for (long long cc = 0; cc < (long long)quads; ++cc) {
      size_t w_base = (size_t)cc * 4;
      float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
      for (size_t i = 0; i < n; ++i) {
        float xv = x[xi + i];
        float p0 = xv * w[(w_base + 0) * n + i];
        float p1 = xv * w[(w_base + 1) * n + i];
        float p2 = xv * w[(w_base + 2) * n + i];
        float p3 = xv * w[(w_base + 3) * n + i];
        s0 = s0 + p0; s1 = s1 + p1; s2 = s2 + p2; s3 = s3 + p3;
      }
      elem[w_base + 0] = s0; elem[w_base + 1] = s1; elem[w_base + 2] = s2; elem[w_base + 3] = s3;
    }
    for (size_t col = quads * 4; col < o; ++col) {
      float sum = 0.0f;
      for (size_t i = 0; i < n; ++i) {
        float p = x[xi + i] * w[col * n + i];
        sum = sum + p;
      }
      elem[col] = sum;
    }
  }
}

/* Per-block int32 dot products Σ x_q·w_q of weight_type.rs:150-201 (the value
 * of `ival.reduce_add()`), laid out [batch][o][n/gs]. Checker for the
 * bit-exactness of the device block dots. */
void orc_block_dots(int32_t* out, const int8_t* x, const int8_t* w, size_t batch, size_t n, size_t o,
                    size_t gs) {
  size_t nb = n / gs;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)(batch * o); ++r) {
    size_t b = (size_t)r / o, c = (size_t)r % o;
    for (size_t g = 0; g < nb; ++g) {
      int32_t s = 0;
      for (size_t k = 0; k < gs; ++k) s += (int32_t)x[b * n + g * gs + k] * (int32_t)w[c * n + g * gs + k];
      out[r * nb + g] = s;
    }
  }
}

/* util.rs:389-426 (`rmsnorm`, the SIMD norm used by forward.rs). No tail loop:
 * only the first floor(size/8)*8 outputs are written. */
void orc_rmsnorm(float* o, const float* x, const float* weight, size_t size, float eps, int add_unit_offset) {
  size_t n_simd = size / 8;
  float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t j = 0; j < n_simd; ++j)
    for (int l = 0; l < 8; ++l) {
      float p = x[j * 8 + l] * x[j * 8 + l];
      lanes[l] = lanes[l] + p;
    }
  float ss = reduce_add8(lanes);
  if (g_probe & 1) {
    double sd = 0.0;
    for (size_t i = 0; i < n_simd * 8; ++i) sd += (double)x[i] * (double)x[i];
    ss = (float)sd;
  }
  ss = ss / (float)size;
  ss = ss + eps;
  ss = 1.0f / sqrtf(ss);
  for (size_t j = 0; j < n_simd; ++j)
    for (int l = 0; l < 8; ++l) {
      float xv = x[j * 8 + l], wv = weight[j * 8 + l];
      float sx = ss * xv;
      o[j * 8 + l] = add_unit_offset ? (1.0f + wv) * sx : wv * sx;
    }
}

/* util.rs:428-444 (`rms_norm`, scalar; the function the reference's own
 * tests pin in tests/simd_tests.rs:87-247). */
void orc_rms_norm_scalar(float* x, size_t n, const float* weight, float eps, int add_unit_offset) {
  float nf = (float)n;
  float sum_sq = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float p = x[i] * x[i];
    sum_sq = sum_sq + p;
  }
  float rms = sqrtf(sum_sq / nf + eps);
  for (size_t i = 0; i < n; ++i) x[i] = (x[i] / rms) * (add_unit_offset ? 1.0f + weight[i] : weight[i]);
}

/* util.rs:446-450 */
void orc_silu(float* x, size_t n) {
  for (size_t i = 0; i < n; ++i) x[i] = x[i] / (1.0f + exp_f32(-x[i]));
}

/* util.rs:589-635 (`rope`, half-split pairs, llama3 scaling 32/1/4 hard-coded).
 * old_context_len is shape.ctx_len in the reference; the oracle takes it from
 * s->llama3_old_ctx (set to ctx_len for the literal reference behaviour). */
void orc_rope(const orc_shape* s, float* sq, float* k, uint32_t pos) {
  const float rope_factor = 32.0f, low_freq_factor = 1.0f, high_freq_factor = 4.0f;
  float old_context_len = s->llama3_old_ctx;
  float low_freq_wavelen = old_context_len / low_freq_factor;
  float high_freq_wavelen = old_context_len / high_freq_factor;
  float rope_theta = s->rope_theta;
  size_t head_size = s->head_size, half = head_size / 2;
  for (size_t j = 0; j < half; ++j) {
    size_t head_dim = j * 2;
    float freq = powf(rope_theta, -((float)head_dim) / (float)head_size);
    float wavelen = (2.0f * (float)M_PI) / freq;
    if (wavelen > low_freq_wavelen) {
      freq = freq / rope_factor;
    } else if (wavelen <= low_freq_wavelen && wavelen >= high_freq_wavelen) {
      float smooth = (old_context_len / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor);
      freq = (1.0f - smooth) * freq / rope_factor + smooth * freq;
    }
    float val = (float)pos * freq;
    float fcr = cosf(val), fci = sinf(val);
    for (size_t h = 0; h < s->n_heads; ++h) {
      size_t off = h * head_size + j;
      float v0 = sq[off], v1 = sq[off + half];
      sq[off] = v0 * fcr - v1 * fci;
      sq[off + half] = v0 * fci + v1 * fcr;
    }
    for (size_t h = 0; h < s->n_kv_heads; ++h) {
      size_t off = h * head_size + j;
      float v0 = k[off], v1 = k[off + half];
      k[off] = v0 * fcr - v1 * fci;
      k[off + half] = v0 * fci + v1 * fcr;
    }
  }
}

/* util.rs:720-724 */
static float rope_yarn_ramp(float low, float high, float i0) {
  float y = (i0 * 0.5f - low) / fmaxf(high - low, 0.001f);
  return 1.0f - fminf(1.0f, fmaxf(y, 0.0f));
}

/* util.rs:653-718 (`rope_gguf`, consecutive pairs, YaRN terms). */
void orc_rope_gguf(const orc_shape* s, float* sq, float* k, uint32_t pos) {
  float rope_theta = s->rope_theta;
  size_t head_size = s->head_size;
  float freq_scale = s->rope_freq_scale, ext_factor = s->rope_ext_factor, attn_factor = s->rope_attn_factor;
  float n_ctx_orig = (float)s->rope_original_ctx_len;
  const float beta_fast = 32.0f, beta_slow = 1.0f;
  size_t n_pairs = head_size / 2;
  float theta_scale = powf(rope_theta, -2.0f / (float)head_size);
  float corr_start = fmaf(logf(n_ctx_orig / (beta_fast * 2.0f * (float)M_PI)), (float)head_size, 0.0f) /
                     (2.0f * logf(rope_theta));
  corr_start = fmaxf(floorf(corr_start), 0.0f);
  float corr_end = fmaf(logf(n_ctx_orig / (beta_slow * 2.0f * (float)M_PI)), (float)head_size, 0.0f) /
                   (2.0f * logf(rope_theta));
  float corr_dims_1 = fminf(corr_start, corr_end) + fminf(corr_end, (float)n_pairs) - fmaxf(corr_start, 0.0f);
  float theta = (float)pos;
  for (size_t kp = 0; kp < n_pairs; ++kp) {
    const float ff = 1.0f;
    float theta_interp = freq_scale * theta / ff;
    float t = theta_interp;
    if (ext_factor != 0.0f) {
      float i0 = (float)(kp * 2);
      float ramp_mix = rope_yarn_ramp(corr_start, corr_dims_1, i0) * ext_factor;
      t = theta_interp * (1.0f - ramp_mix) + theta / ff * ramp_mix;
    }
    float cos_t = cosf(t) * attn_factor, sin_t = sinf(t) * attn_factor;
    size_t col0 = kp * 2;
    for (size_t h = 0; h < s->n_heads; ++h) {
      size_t off = h * head_size + col0;
      float v0 = sq[off], v1 = sq[off + 1];
      sq[off] = v0 * cos_t - v1 * sin_t;
      sq[off + 1] = v0 * sin_t + v1 * cos_t;
    }
    for (size_t h = 0; h < s->n_kv_heads; ++h) {
      size_t off = h * head_size + col0;
      float v0 = k[off], v1 = k[off + 1];
      k[off] = v0 * cos_t - v1 * sin_t;
      k[off + 1] = v0 * sin_t + v1 * cos_t;
    }
    theta = theta * theta_scale;
  }
}

/* forward.rs:299-400 (`fused_attention`). Score rows are indexed qh*batch+t1;
 * masked positions get -1e10; the softmax runs over the whole row. */
void orc_fused_attention(float* output, float* scores, const float* sq, const float* key_cache,
                         const float* value_cache, size_t seq_len, size_t batch, size_t n_heads,
                         size_t n_kv_heads, size_t head_size, uint32_t start_pos, size_t kv_dim,
                         float attn_scale) {
  size_t kv_mul = n_heads / n_kv_heads;
  long long rows = (long long)(n_heads * batch);
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < rows; ++idx) {
    float* score_row = scores + (size_t)idx * seq_len;
    size_t qh = (size_t)idx / batch, t1 = (size_t)idx % batch;
    size_t kvh = qh / kv_mul;
    size_t abs_pos = (size_t)start_pos + t1;
    size_t max_t2 = abs_pos < seq_len - 1 ? abs_pos : seq_len - 1;
    const float* q = sq + t1 * (n_heads * head_size) + qh * head_size;
    float max_score = -1e10f;
    for (size_t t2 = 0; t2 <= max_t2; ++t2) {
      const float* kk = key_cache + t2 * kv_dim + kvh * head_size;
      float sum = dot8(q, kk, head_size);
      float s_val = sum * attn_scale;
      score_row[t2] = s_val;
      if (s_val > max_score) max_score = s_val;
    }
    for (size_t t2 = max_t2 + 1; t2 < seq_len; ++t2) score_row[t2] = -1e10f;
    float sum_exp = 0.0f;
    for (size_t t2 = 0; t2 < seq_len; ++t2) {
      float e = exp_f32(score_row[t2] - max_score);
      score_row[t2] = e;
      sum_exp = sum_exp + e;
    }
    float inv_sum = sum_exp > 0.0f ? 1.0f / sum_exp : 0.0f;
    for (size_t t2 = 0; t2 < seq_len; ++t2) score_row[t2] = score_row[t2] * inv_sum;
  }
#pragma omp parallel for schedule(static)
  for (long long tt = 0; tt < (long long)batch; ++tt) {
    size_t t1 = (size_t)tt;
    float* out_token = output + t1 * n_heads * head_size;
    for (size_t qh = 0; qh < n_heads; ++qh) {
      size_t kvh = qh / kv_mul;
      size_t out_base = qh * head_size;
      size_t s_base = qh * (batch * seq_len) + t1 * seq_len;
      for (size_t d = 0; d < head_size; ++d) {
        size_t n_simd = seq_len / 8;
        float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (size_t c = 0; c < n_simd; ++c) {
          size_t t2 = c * 8;
          for (int l = 0; l < 8; ++l) {
            float p = scores[s_base + t2 + l] * value_cache[(t2 + l) * kv_dim + kvh * head_size + d];
            lanes[l] = lanes[l] + p;
          }
        }
        float sum = reduce_add8(lanes);
        for (size_t t2 = n_simd * 8; t2 < seq_len; ++t2) {
          float p = scores[s_base + t2] * value_cache[t2 * kv_dim + kvh * head_size + d];
          sum = sum + p;
        }
        out_token[out_base + d] = sum;
      }
    }
  }
}

/* sampler.rs:67-79: first index with a strictly greater value wins. */
uint32_t orc_argmax(const float* p, size_t n) {
  uint32_t max_i = 0;
  float max_p = p[0];
  for (size_t i = 1; i < n; ++i)
    if (p[i] > max_p) { max_i = (uint32_t)i; max_p = p[i]; }
  return max_i;
}

}  // extern "C"

/* ======================= GGUF loader + model ============================== */
namespace {

struct QT { /* QuantizedTensor (weight_type.rs:30-36) */
  std::vector<int8_t> q;
  std::vector<float> s;
  std::vector<float> f; /* F16 variant, stored as f32 */
};

struct GVal {
  uint32_t type = 0;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string str;
  std::vector<GVal> arr;
};

struct TInfo {
  std::string name;
  uint32_t type;
  uint64_t off;
  size_t n;
};

struct Reader {
  const uint8_t* p;
  size_t size, off = 0;
  bool ok = true;
  bool need(size_t k) {
    if (off + k > size) { ok = false; return false; }
    return true;
  }
  uint64_t rd(size_t k) {
    if (!need(k)) return 0;
    uint64_t v = 0;
    memcpy(&v, p + off, k);
    off += k;
    return v;
  }
  std::string str() {
    uint64_t len = rd(8);
    if (!ok || !need(len)) return "";
    std::string s((const char*)p + off, len);
    off += len;
    return s;
  }
  /* transformer_llama_gguf.rs:80-107 */
  GVal value(uint32_t t, int depth = 0) {
    GVal v;
    v.type = t;
    switch (t) {
      case 0: v.u = rd(1); break;
      case 1: v.i = (int8_t)rd(1); break;
      case 2: v.u = rd(2); break;
      case 3: v.i = (int16_t)rd(2); break;
      case 4: v.u = rd(4); break;
      case 5: v.i = (int32_t)rd(4); break;
      case 6: { uint32_t b = (uint32_t)rd(4); float f; memcpy(&f, &b, 4); v.f = f; break; }
      case 7: v.u = rd(1) != 0; break;
      case 8: v.str = str(); break;
      case 9: {
        uint32_t et = (uint32_t)rd(4);
        uint64_t len = rd(8);
        if (depth > 2 || !ok) { ok = false; break; }
        v.u = len;
        if (et == 8 && len > 0) {
          v.arr.reserve(len);
        }
        for (uint64_t k = 0; k < len && ok; ++k) v.arr.push_back(value(et, depth + 1));
        break;
      }
      case 10: v.u = rd(8); break;
      case 11: v.i = (int64_t)rd(8); break;
      case 12: { uint64_t b = rd(8); double d; memcpy(&d, &b, 8); v.f = d; break; }
      default: ok = false;
    }
    return v;
  }
};

}  // namespace

struct orc_model {
  orc_shape shape;
  std::vector<float> token_embedding; /* f32 (transformer_llama_gguf.rs:453-489) */
  std::vector<float> lm_head;         /* output.weight dequantized (deviation D2) or empty */
  std::vector<QT> wq, wk, wv, wo, w1, w2, w3;
  std::vector<std::vector<float>> w_rms_att, w_rms_post_att;
  std::vector<float> w_rms_final;
};

struct orc_session {
  std::vector<float> key_cache, value_cache; /* base_transformer.rs:82-98 */
  uint32_t pos = 0;
};

namespace {

bool meta_u64(const std::map<std::string, GVal>& m, const char* k, uint64_t* out) {
  auto it = m.find(k);
  if (it == m.end()) return false;
  if (it->second.type == 10 || it->second.type == 4) { *out = it->second.u; return true; }
  return false;
}
bool meta_f32(const std::map<std::string, GVal>& m, const char* k, float* out) {
  auto it = m.find(k);
  if (it == m.end()) return false;
  if (it->second.type == 6 || it->second.type == 12) { *out = (float)it->second.f; return true; }
  return false;
}

/* transformer_llama_gguf.rs:345-421, with the Q4_0 decode switch (D1). */
bool load_qt(const uint8_t* base, const TInfo& ti, int q4_mode, QT* out) {
  const uint8_t* p = base + ti.off;
  size_t n = ti.n;
  size_t blocks = (n + 31) / 32;
  if (ti.type == 8) { /* Q8_0: f16 d + 32 i8 */
    out->q.assign(n, 0);
    out->s.assign(blocks, 0.f);
    for (size_t b = 0; b < blocks; ++b) {
      const uint8_t* bp = p + b * 34;
      uint16_t h = (uint16_t)(bp[0] | (bp[1] << 8));
      out->s[b] = orc_f16_to_f32(h);
      for (size_t j = 0; j < 32; ++j)
        if (b * 32 + j < n) out->q[b * 32 + j] = (int8_t)bp[2 + j];
    }
    return true;
  }
  if (ti.type == 2) { /* Q4_0: f16 d + 16 bytes of nibbles */
    out->q.assign(n, 0);
    out->s.assign(blocks, 0.f);
    for (size_t b = 0; b < blocks; ++b) {
      const uint8_t* bp = p + b * 18;
      uint16_t h = (uint16_t)(bp[0] | (bp[1] << 8));
      out->s[b] = orc_f16_to_f32(h);
      for (size_t j = 0; j < 16; ++j) {
        uint8_t byte = bp[2 + j];
        int lo = byte & 0x0F, hi = (byte >> 4) & 0x0F;
        if (q4_mode == ORC_Q4_REF) { /* :394-405 literal */
          if (b * 32 + j * 2 < n) out->q[b * 32 + j * 2] = (int8_t)lo;
          if (b * 32 + j * 2 + 1 < n) out->q[b * 32 + j * 2 + 1] = (int8_t)hi;
        } else { /* GGML: j <- lo, j+16 <- hi, value q-8 */
          if (b * 32 + j < n) out->q[b * 32 + j] = (int8_t)(lo - 8);
          if (b * 32 + j + 16 < n) out->q[b * 32 + j + 16] = (int8_t)(hi - 8);
        }
      }
    }
    return true;
  }
  if (ti.type == 1) { /* F16 */
    out->f.resize(n);
    for (size_t i = 0; i < n; ++i) out->f[i] = orc_f16_to_f32((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8)));
    return true;
  }
  g_err = "unsupported tensor type for " + ti.name;
  return false;
}

/* transformer_llama_gguf.rs:459-489: E_f32 = q * scale per 32-group. */
std::vector<float> dequant(const QT& t, size_t gs) {
  if (!t.f.empty()) return t.f;
  std::vector<float> e(t.q.size());
  for (size_t i = 0; i < t.q.size(); ++i) e[i] = (float)t.q[i] * t.s[i / gs];
  return e;
}

}  // namespace

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }

static orc_model* load_gguf(const char* path, uint32_t max_ctx_len, int fmt_override, int q4_mode) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) { g_err = std::string("cannot open ") + path; return nullptr; }
  struct stat st;
  fstat(fd, &st);
  size_t size = (size_t)st.st_size;
  void* mp = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (mp == MAP_FAILED) { g_err = "mmap failed"; return nullptr; }
  std::unique_ptr<void, std::function<void(void*)>> guard(mp, [size](void* q) { munmap(q, size); });
  Reader r{(const uint8_t*)mp, size};
  /* :188-199 */
  if (r.rd(4) != 0x46554747u) { g_err = "Not a GGUF file (bad magic)"; return nullptr; }
  if (r.rd(4) != 3) { g_err = "Only GGUF version 3 is supported"; return nullptr; }
  uint64_t tensor_count = r.rd(8), kv_count = r.rd(8);
  std::map<std::string, GVal> meta;
  for (uint64_t i = 0; i < kv_count && r.ok; ++i) {
    std::string key = r.str();
    uint32_t t = (uint32_t)r.rd(4);
    meta[key] = r.value(t);
  }
  if (!r.ok) { g_err = "truncated GGUF metadata"; return nullptr; }
  auto arch = meta.find("general.architecture");
  if (arch == meta.end() || arch->second.str != "llama") { g_err = "Architecture must be 'llama'"; return nullptr; }
  /* :218-287 */
  orc_shape s;
  memset(&s, 0, sizeof(s));
  uint64_t v;
  if (!meta_u64(meta, "llama.embedding_length", &v)) { g_err = "missing llama.embedding_length"; return nullptr; }
  s.dim = (uint32_t)v;
  if (!meta_u64(meta, "llama.feed_forward_length", &v)) { g_err = "missing feed_forward_length"; return nullptr; }
  s.hidden_dim = (uint32_t)v;
  if (!meta_u64(meta, "llama.block_count", &v)) { g_err = "missing block_count"; return nullptr; }
  s.n_layers = (uint32_t)v;
  if (!meta_u64(meta, "llama.attention.head_count", &v)) { g_err = "missing head_count"; return nullptr; }
  s.n_heads = (uint32_t)v;
  s.n_kv_heads = meta_u64(meta, "llama.attention.head_count_kv", &v) ? (uint32_t)v : s.n_heads;
  if (!meta_f32(meta, "llama.attention.layer_norm_rms_epsilon", &s.rms_norm_eps)) { g_err = "missing rms eps"; return nullptr; }
  uint64_t file_type = meta_u64(meta, "general.file_type", &v) ? v : 7;
  if (!meta_f32(meta, "llama.rope.freq_base", &s.rope_theta)) s.rope_theta = 10000.0f;
  if (!meta_u64(meta, "llama.context_length", &v)) { g_err = "missing context_length"; return nullptr; }
  uint32_t seq_len = (uint32_t)v;
  if (s.n_heads == 0 || s.dim % s.n_heads) { g_err = "dim must be divisible by n_heads"; return nullptr; }
  s.head_size = s.dim / s.n_heads;
  s.ctx_len = seq_len < max_ctx_len ? seq_len : max_ctx_len;
  auto toks = meta.find("tokenizer.ggml.tokens");
  if (toks == meta.end() || toks->second.type != 9) { g_err = "tokenizer.ggml.tokens missing"; return nullptr; }
  s.vocab_size = (uint32_t)toks->second.arr.size();
  float raw;
  if (!meta_f32(meta, "llama.rope.scaling.factor", &raw)) raw = 1.0f;
  s.rope_freq_scale = raw != 0.0f ? 1.0f / raw : 1.0f;
  if (!meta_f32(meta, "llama.rope.scaling.ext_factor", &s.rope_ext_factor)) s.rope_ext_factor = 0.0f;
  if (!meta_f32(meta, "llama.rope.scaling.attn_factor", &s.rope_attn_factor)) s.rope_attn_factor = 1.0f;
  s.rope_original_ctx_len =
      meta_u64(meta, "llama.rope.scaling.original_context_length", &v) ? (uint32_t)v : seq_len;
  if (!meta_f32(meta, "llama.attention.scale", &s.attention_scale)) s.attention_scale = 0.0f;
  s.group_size = 32;
  /* Deviation D3: llama3-type scaling selects the half-split rope() math with
   * old_context_len = original_context_length. */
  auto sct = meta.find("llama.rope.scaling.type");
  s.rope_mode = (sct != meta.end() && sct->second.str == "llama3") ? ORC_ROPE_LLAMA3 : ORC_ROPE_GGUF;
  s.llama3_old_ctx = (float)s.rope_original_ctx_len;
  int fmt;
  if (fmt_override >= 0) fmt = fmt_override;
  else if (file_type == 1) fmt = ORC_F16;
  else if (file_type == 2) fmt = ORC_Q4_0;
  else if (file_type == 7) fmt = ORC_Q8_0;
  else { g_err = "Unsupported GGUF file_type"; return nullptr; }
  s.weight_format = fmt;
  s.q4_mode = q4_mode;
  auto bos = meta.find("tokenizer.ggml.bos_token_id");
  s.bos = bos != meta.end() ? (uint32_t)(bos->second.type == 5 || bos->second.type == 11 ? bos->second.i : bos->second.u) : 128000u;
  auto eos = meta.find("tokenizer.ggml.eos_token_id");
  s.eos = eos != meta.end() ? (uint32_t)(eos->second.type == 5 || eos->second.type == 11 ? eos->second.i : eos->second.u) : 128009u;

  /* :298-330 tensor infos and data start */
  std::vector<TInfo> infos;
  for (uint64_t i = 0; i < tensor_count && r.ok; ++i) {
    TInfo ti;
    ti.name = r.str();
    uint32_t nd = (uint32_t)r.rd(4);
    ti.n = 1;
    for (uint32_t d = 0; d < nd; ++d) ti.n *= (size_t)r.rd(8);
    ti.type = (uint32_t)r.rd(4);
    ti.off = r.rd(8);
    infos.push_back(ti);
  }
  if (!r.ok) { g_err = "truncated tensor infos"; return nullptr; }
  uint64_t alignment = meta_u64(meta, "general.alignment", &v) ? v : 32;
  uint64_t data_start = (r.off + alignment - 1) / alignment * alignment;
  std::map<std::string, TInfo> tmap;
  for (auto& ti : infos) { ti.off += data_start; tmap[ti.name] = ti; }
  auto get = [&](const std::string& nm, TInfo* out) {
    auto it = tmap.find(nm);
    if (it == tmap.end()) { g_err = "Missing tensor: " + nm; return false; }
    *out = it->second;
    return true;
  };
  const uint8_t* base = (const uint8_t*)mp;
  std::unique_ptr<orc_model> m(new orc_model());
  m->shape = s;
  TInfo ti;
  QT emb;
  if (!get("token_embd.weight", &ti) || !load_qt(base, ti, q4_mode, &emb)) return nullptr;
  m->token_embedding = dequant(emb, 32);
  if (tmap.count("output.weight")) { /* deviation D2 */
    QT lm;
    if (!get("output.weight", &ti) || !load_qt(base, ti, q4_mode, &lm)) return nullptr;
    m->lm_head = dequant(lm, 32);
    m->shape.untied_lm_head = 1;
  }
  auto f32t = [&](const std::string& nm, std::vector<float>* out) {
    TInfo t;
    if (!get(nm, &t)) return false;
    if (t.type != 0) { g_err = "Expected F32 tensor " + nm; return false; }
    out->resize(t.n);
    memcpy(out->data(), base + t.off, t.n * 4);
    return true;
  };
  if (!f32t("output_norm.weight", &m->w_rms_final)) return nullptr;
  size_t L = s.n_layers;
  m->w_rms_att.resize(L); m->w_rms_post_att.resize(L);
  m->wq.resize(L); m->wk.resize(L); m->wv.resize(L); m->wo.resize(L);
  m->w1.resize(L); m->w2.resize(L); m->w3.resize(L);
  for (size_t l = 0; l < L; ++l) {
    std::string p = "blk." + std::to_string(l) + ".";
    if (!f32t(p + "attn_norm.weight", &m->w_rms_att[l])) return nullptr;
    if (!f32t(p + "ffn_norm.weight", &m->w_rms_post_att[l])) return nullptr;
    struct { const char* nm; QT* dst; } list[] = {
        {"attn_q", &m->wq[l]}, {"attn_k", &m->wk[l]}, {"attn_v", &m->wv[l]}, {"attn_output", &m->wo[l]},
        {"ffn_gate", &m->w1[l]}, {"ffn_down", &m->w2[l]}, {"ffn_up", &m->w3[l]}};
    for (auto& e : list) {
      if (!get(p + e.nm + ".weight", &ti) || !load_qt(base, ti, q4_mode, e.dst)) return nullptr;
      bool is_f = !e.dst->f.empty();
      if ((fmt == ORC_F16) != is_f) { g_err = "format/variant mismatch"; return nullptr; }
    }
  }
  return m.release();
}

/* Loaders of the other two model files (below): safetensors + config.json
 * (transformer_llama_st.rs:41-372) and lm.rs (transformer_llama_lmrs.rs:56-439). */
static orc_model* load_st(const char* path, uint32_t max_ctx_len, int fmt_override);
static orc_model* load_lmrs(const char* path, uint32_t max_ctx_len);

/* lib.rs:107-133: dispatch by file extension. */
orc_model* orc_model_load(const char* path, uint32_t max_ctx_len, int fmt_override, int q4_mode) {
  std::string p(path);
  size_t dot = p.rfind('.'), slash = p.rfind('/');
  std::string ext = (dot == std::string::npos || (slash != std::string::npos && dot < slash)) ? "" : p.substr(dot + 1);
  if (ext == "gguf") return load_gguf(path, max_ctx_len, fmt_override, q4_mode);
  if (ext == "safetensors") return load_st(path, max_ctx_len, fmt_override);
  if (ext == "lmrs") return load_lmrs(path, max_ctx_len);
  g_err = "Unsupported model extension for path: " + p;
  return nullptr;
}

void orc_model_free(orc_model* m) { delete m; }

int orc_model_shape(const orc_model* m, orc_shape* out) {
  if (!m || !out) return -1;
  *out = m->shape;
  return 0;
}

/* base_transformer.rs:129-141 */
int orc_get_embeddings(const orc_model* m, uint32_t token, float* out) {
  size_t dim = m->shape.dim;
  size_t idx = (size_t)token * dim;
  if (idx + dim <= m->token_embedding.size()) memcpy(out, &m->token_embedding[idx], dim * 4);
  else memset(out, 0, dim * 4);
  return 0;
}

/* base_transformer.rs:88-98 */
orc_session* orc_session_new(const orc_model* m) {
  orc_session* s = new orc_session();
  size_t kv_dim = (size_t)m->shape.n_kv_heads * m->shape.head_size;
  size_t n = (size_t)m->shape.n_layers * m->shape.ctx_len * kv_dim;
  s->key_cache.assign(n, 0.f);
  s->value_cache.assign(n, 0.f);
  return s;
}
void orc_session_free(orc_session* s) { delete s; }
void orc_session_reset(orc_session* s) { /* :100-104 */
  std::fill(s->key_cache.begin(), s->key_cache.end(), 0.f);
  std::fill(s->value_cache.begin(), s->value_cache.end(), 0.f);
  s->pos = 0;
}
float* orc_session_key_cache(orc_session* s) { return s->key_cache.data(); }
float* orc_session_value_cache(orc_session* s) { return s->value_cache.data(); }
size_t orc_session_cache_len(const orc_session* s) { return s->key_cache.size(); }

}  // extern "C"

namespace {

/* ForwardKernel (forward.rs:25-92): format-specific quantize and matmul. */
struct Act {
  std::vector<int8_t> q;
  std::vector<float> s, f;
};

void fk_quantize(const orc_shape& sh, Act* dst, const float* x, size_t n) {
  uint32_t gs = sh.group_size;
  if (sh.weight_format == ORC_F16) { /* F16Kernel::quantize copies (:78-81) */
    if (dst->f.size() < n) dst->f.resize(n);
    memcpy(dst->f.data(), x, n * 4);
    return;
  }
  if (dst->q.size() < n) dst->q.resize(n);
  if (dst->s.size() < n / gs) dst->s.resize(n / gs);
  if (sh.weight_format == ORC_Q4_0 && sh.q4_mode == ORC_Q4_REF) orc_quantize_q4_ref(dst->q.data(), dst->s.data(), x, n, gs);
  else orc_quantize_q8(dst->q.data(), dst->s.data(), x, n, gs);
}

void fk_matmul(const orc_shape& sh, float* out, size_t out_len, const Act& x, const QT& w, size_t n, size_t o) {
  if (sh.weight_format == ORC_F16) orc_matmul_f32(out, out_len, x.f.data(), w.f.data(), n, o);
  else orc_matmul_q8_slices(out, out_len, x.q.data(), x.s.data(), w.q.data(), w.s.data(), n, o, sh.group_size);
}

}  // namespace

extern "C" int orc_forward_x(const orc_model* m, orc_session* sess, const uint32_t* tokens, size_t batch,
                             uint32_t start_pos, float* logits) {
  /* forward.rs:119-280 */
  const orc_shape& sh = m->shape;
  if (batch == 0) { g_err = "empty token batch"; return -1; }
  if ((size_t)start_pos + batch > sh.ctx_len) { g_err = "position beyond ctx_len"; return -1; }
  size_t dim = sh.dim, hidden_dim = sh.hidden_dim;
  size_t att_dim = (size_t)sh.n_heads * sh.head_size;
  size_t kv_dim = (size_t)sh.n_kv_heads * sh.head_size;
  size_t seq_len = (size_t)start_pos + batch;
  std::vector<float> x(batch * dim);
  for (size_t t = 0; t < batch; ++t) orc_get_embeddings(m, tokens[t], &x[t * dim]);
  std::vector<float> xn(batch * dim), sq(batch * att_dim), scores(sh.n_heads * batch * seq_len),
      att(batch * att_dim), hg(batch * hidden_dim), hu(batch * hidden_dim), ffn(batch * dim);
  Act xq;
  float attn_scale = sh.attention_scale != 0.0f ? sh.attention_scale : 1.0f / sqrtf((float)sh.head_size);
  size_t total = batch * dim;
  for (size_t layer = 0; layer < sh.n_layers; ++layer) {
    size_t cache_off = layer * (size_t)sh.ctx_len * kv_dim;
    size_t write_off = (size_t)start_pos * kv_dim;
    for (size_t t = 0; t < batch; ++t)
      orc_rmsnorm(&xn[t * dim], &x[t * dim], m->w_rms_att[layer].data(), dim, sh.rms_norm_eps, 0);
    fk_quantize(sh, &xq, xn.data(), batch * dim);
    std::fill(sq.begin(), sq.end(), 0.f);
    fk_matmul(sh, sq.data(), batch * att_dim, xq, m->wq[layer], dim, att_dim);
    float* k = &sess->key_cache[cache_off + write_off];
    float* v = &sess->value_cache[cache_off + write_off];
    fk_matmul(sh, k, batch * kv_dim, xq, m->wk[layer], dim, kv_dim);
    fk_matmul(sh, v, batch * kv_dim, xq, m->wv[layer], dim, kv_dim);
    for (size_t t = 0; t < batch; ++t) {
      if (sh.rope_mode == ORC_ROPE_LLAMA3) orc_rope(&sh, &sq[t * att_dim], k + t * kv_dim, start_pos + (uint32_t)t);
      else orc_rope_gguf(&sh, &sq[t * att_dim], k + t * kv_dim, start_pos + (uint32_t)t);
    }
    orc_fused_attention(att.data(), scores.data(), sq.data(), &sess->key_cache[cache_off],
                        &sess->value_cache[cache_off], seq_len, batch, sh.n_heads, sh.n_kv_heads, sh.head_size,
                        start_pos, kv_dim, attn_scale);
    fk_quantize(sh, &xq, att.data(), batch * att_dim);
    std::fill(ffn.begin(), ffn.end(), 0.f);
    fk_matmul(sh, ffn.data(), batch * dim, xq, m->wo[layer], att_dim, dim);
    for (size_t i = 0; i < total; ++i) x[i] = x[i] + ffn[i]; /* :195-204 */
    for (size_t t = 0; t < batch; ++t)
      orc_rmsnorm(&xn[t * dim], &x[t * dim], m->w_rms_post_att[layer].data(), dim, sh.rms_norm_eps, 0);
    fk_quantize(sh, &xq, xn.data(), batch * dim);
    std::fill(hg.begin(), hg.end(), 0.f);
    std::fill(hu.begin(), hu.end(), 0.f);
    fk_matmul(sh, hg.data(), batch * hidden_dim, xq, m->w1[layer], dim, hidden_dim);
    fk_matmul(sh, hu.data(), batch * hidden_dim, xq, m->w3[layer], dim, hidden_dim);
    for (size_t i = 0; i < batch * hidden_dim; ++i) { /* :221-237 (correctly rounded exp; wide exp unpinned) */
      float g = hg[i];
      float silu = g / (1.0f + exp_f32(-g));
      hg[i] = silu * hu[i];
    }
    fk_quantize(sh, &xq, hg.data(), batch * hidden_dim);
    std::fill(ffn.begin(), ffn.end(), 0.f);
    fk_matmul(sh, ffn.data(), batch * dim, xq, m->w2[layer], hidden_dim, dim);
    for (size_t i = 0; i < total; ++i) x[i] = x[i] + ffn[i]; /* :244-253 */
  }
  for (size_t t = 0; t < batch; ++t)
    orc_rmsnorm(&xn[t * dim], &x[t * dim], m->w_rms_final.data(), dim, sh.rms_norm_eps, 0);
  /* :261-279, last token only; the reference's single-threaded loop is kept. */
  const float* last = &xn[(batch - 1) * dim];
  const std::vector<float>& E = m->lm_head.empty() ? m->token_embedding : m->lm_head;
  for (size_t vv = 0; vv < sh.vocab_size; ++vv) logits[vv] = dot8(last, &E[vv * dim], dim);
  return 0;
}

/* ===================== safetensors and lm.rs loaders ====================== */
namespace {

/* A JSON value: the subset the two loaders read (serde_json semantics for
 * as_u64: non-negative integer literals only; as_f64: any number). */
struct JV {
  char t = 'n'; /* n null, b bool, d number, s string, a array, o object */
  double num = 0;
  bool uint_lit = false;
  unsigned long long u = 0;
  std::string s;
  std::vector<JV> a;
  std::vector<std::pair<std::string, JV>> o;
  const JV* at(const char* k) const { /* last duplicate wins */
    const JV* r = nullptr;
    if (t == 'o')
      for (auto& kv : o)
        if (kv.first == k) r = &kv.second;
    return r;
  }
};

struct JP {
  const char* p;
  const char* e;
  bool ok = true;
  void sp() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
  bool str(std::string* out) {
    if (p >= e || *p != '"') return ok = false;
    ++p;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return ok = false;
        char c = *p++;
        if (c == 'u') {
          if (e - p < 4) return ok = false;
          unsigned cp = (unsigned)strtoul(std::string(p, 4).c_str(), nullptr, 16);
          p += 4;
          if (cp >= 0xD800 && cp < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            unsigned lo = (unsigned)strtoul(std::string(p + 2, 4).c_str(), nullptr, 16);
            p += 6;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          if (cp < 0x80) out->push_back((char)cp);
          else if (cp < 0x800) { out->push_back((char)(0xC0 | (cp >> 6))); out->push_back((char)(0x80 | (cp & 63))); }
          else if (cp < 0x10000) {
            out->push_back((char)(0xE0 | (cp >> 12)));
            out->push_back((char)(0x80 | ((cp >> 6) & 63)));
            out->push_back((char)(0x80 | (cp & 63)));
          } else {
            out->push_back((char)(0xF0 | (cp >> 18)));
            out->push_back((char)(0x80 | ((cp >> 12) & 63)));
            out->push_back((char)(0x80 | ((cp >> 6) & 63)));
            out->push_back((char)(0x80 | (cp & 63)));
          }
        } else {
          const char* from = "\"\\/bfnrt";
          const char* to = "\"\\/\b\f\n\r\t";
          const char* f = strchr(from, c);
          if (!f || !c) return ok = false;
          out->push_back(to[f - from]);
        }
      } else {
        out->push_back(*p++);
      }
    }
    if (p >= e) return ok = false;
    ++p;
    return true;
  }
  JV val(int depth) {
    JV v;
    sp();
    if (p >= e || depth > 64) { ok = false; return v; }
    if (*p == '{') {
      v.t = 'o';
      ++p;
      sp();
      if (p < e && *p == '}') { ++p; return v; }
      while (ok) {
        sp();
        std::string k;
        if (!str(&k)) break;
        sp();
        if (p >= e || *p != ':') { ok = false; break; }
        ++p;
        JV x = val(depth + 1);
        v.o.emplace_back(k, x);
        sp();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; break; }
        ok = false;
      }
    } else if (*p == '[') {
      v.t = 'a';
      ++p;
      sp();
      if (p < e && *p == ']') { ++p; return v; }
      while (ok) {
        v.a.push_back(val(depth + 1));
        sp();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; break; }
        ok = false;
      }
    } else if (*p == '"') {
      v.t = 's';
      str(&v.s);
    } else if (e - p >= 4 && !strncmp(p, "true", 4)) {
      v.t = 'b'; p += 4;
    } else if (e - p >= 5 && !strncmp(p, "false", 5)) {
      v.t = 'b'; p += 5;
    } else if (e - p >= 4 && !strncmp(p, "null", 4)) {
      p += 4;
    } else {
      const char* b = p;
      while (p < e && strchr("+-0123456789.eE", *p)) ++p;
      std::string tok(b, p - b);
      if (tok.empty()) { ok = false; return v; }
      v.t = 'd';
      v.num = strtod(tok.c_str(), nullptr);
      bool digits = tok.find_first_not_of("0123456789") == std::string::npos;
      if (digits && tok.size() < 20) { v.uint_lit = true; v.u = strtoull(tok.c_str(), nullptr, 10); }
    }
    return v;
  }
};

bool json_read(const char* p, size_t n, JV* out) {
  JP jp{p, p + n};
  *out = jp.val(0);
  jp.sp();
  return jp.ok && jp.p == jp.e;
}

bool read_file(const std::string& path, std::string* out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[65536];
  size_t k;
  while ((k = fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, k);
  fclose(f);
  return true;
}

std::string parent_dir(const std::string& p) {
  size_t k = p.rfind('/');
  return k == std::string::npos ? "." : p.substr(0, k);
}

/* Tokenizer::new header (tokenizer.rs:223-228) / Tokenizer::from_json added
 * tokens (tokenizer.rs:179-186): BOS and EOS only. */
bool tokenizer_ids(const std::string& dir, bool try_json, uint32_t* bos, uint32_t* eos) {
  std::string t;
  if (try_json && read_file(dir + "/tokenizer.json", &t)) {
    JV root;
    if (!json_read(t.data(), t.size(), &root)) { g_err = "bad tokenizer.json"; return false; }
    const JV* added = root.at("added_tokens");
    if (!added || added->t != 'a') { g_err = "tokenizer.json: no added_tokens"; return false; }
    *bos = 128000u;
    *eos = 128009u;
    for (auto& tk : added->a) {
      const JV* c = tk.at("content");
      const JV* id = tk.at("id");
      if (!c || c->t != 's' || !id || !id->uint_lit) { g_err = "tokenizer.json: bad added token"; return false; }
      if (c->s == "<|begin_of_text|>") *bos = (uint32_t)id->u;
      if (c->s == "<|end_of_text|>" || c->s == "<|eot_id|>") *eos = (uint32_t)id->u;
    }
    return true;
  }
  t.clear();
  if (!read_file(dir + "/tokenizer.bin", &t)) { g_err = "cannot open " + dir + "/tokenizer.bin"; return false; }
  if (t.size() < 16) { g_err = "tokenizer.bin too short"; return false; }
  memcpy(bos, t.data() + 8, 4);
  memcpy(eos, t.data() + 12, 4);
  return true;
}

/* Rust `f as i32`: NaN -> 0, saturating. */
inline int32_t rust_f32_as_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return (int32_t)v;
}

/* util.rs:451-518 load_q8_tensor_st: unpack the u32-packed u8 quants, then
 * per group: dequantize (q as u8) * scale + bias, symmetric requantize. */
void load_q8_tensor_st(const uint8_t* data, size_t rows, size_t cols, size_t gs, size_t w_off, size_t s_off,
                       size_t b_off, QT* out) {
  size_t n = rows * cols, groups = n / gs, packed_cols = cols / 4;
  std::vector<int8_t> vals(n);
  for (size_t r = 0; r < rows; ++r)
    for (size_t pc = 0; pc < packed_cols; ++pc) {
      uint32_t packed;
      memcpy(&packed, data + w_off + (r * packed_cols + pc) * 4, 4);
      size_t dst = r * cols + pc * 4;
      for (int b = 0; b < 4; ++b) vals[dst + b] = (int8_t)(uint8_t)(packed >> (8 * b));
    }
  out->q.assign(n, 0);
  out->s.assign(groups, 0.0f);
  std::vector<float> deq(gs);
  for (size_t g = 0; g < groups; ++g) {
    uint16_t sb, bb;
    memcpy(&sb, data + s_off + g * 2, 2);
    memcpy(&bb, data + b_off + g * 2, 2);
    float scale = orc_f16_to_f32(sb), bias = orc_f16_to_f32(bb);
    size_t start = g * gs, end = start + gs < n ? start + gs : n;
    float max_abs = 0.0f;
    for (size_t i = start; i < end; ++i) {
      float f = (float)(uint8_t)vals[i] * scale + bias;
      deq[i - start] = f;
      float a = fabsf(f);
      if (a > max_abs) max_abs = a;
    }
    float sym = max_abs == 0.0f ? 1.0f : max_abs / 127.0f;
    out->s[g] = sym;
    for (size_t i = start; i < end; ++i) {
      int32_t q = rust_f32_as_i32(roundf(deq[i - start] / sym));
      out->q[i] = (int8_t)(q < -128 ? -128 : q > 127 ? 127 : q);
    }
  }
}

struct StInfo {
  std::string dtype;
  size_t off = 0, len = 0;
};

}  // namespace

static orc_model* load_st(const char* path, uint32_t max_ctx_len, int fmt_override) {
  std::string dir = parent_dir(path), text;
  if (!read_file(dir + "/config.json", &text)) { g_err = "cannot open " + dir + "/config.json"; return nullptr; }
  JV cfg;
  if (!json_read(text.data(), text.size(), &cfg)) { g_err = "bad config.json"; return nullptr; }
  auto u = [&](const char* k, uint32_t* v) {
    const JV* j = cfg.at(k);
    if (!j || !j->uint_lit) { g_err = std::string("config.json: ") + k; return false; }
    *v = (uint32_t)j->u;
    return true;
  };
  auto f = [&](const char* k, float* v) {
    const JV* j = cfg.at(k);
    if (!j || j->t != 'd') { g_err = std::string("config.json: ") + k; return false; }
    *v = (float)j->num;
    return true;
  };
  orc_shape s;
  memset(&s, 0, sizeof(s));
  uint32_t max_seq_len;
  /* transformer_llama_st.rs:50-59 */
  if (!u("hidden_size", &s.dim) || !u("intermediate_size", &s.hidden_dim) || !u("num_attention_heads", &s.n_heads) ||
      !u("num_key_value_heads", &s.n_kv_heads) || !u("head_dim", &s.head_size) ||
      !u("num_hidden_layers", &s.n_layers) || !u("vocab_size", &s.vocab_size) || !f("rms_norm_eps", &s.rms_norm_eps) ||
      !f("rope_theta", &s.rope_theta) || !u("max_position_embeddings", &max_seq_len))
    return nullptr;
  /* :62-91 */
  const JV* q = cfg.at("quantization");
  uint32_t gs = 32;
  if (q && q->at("group_size") && q->at("group_size")->uint_lit) gs = (uint32_t)q->at("group_size")->u;
  int fmt;
  if (fmt_override >= 0) fmt = fmt_override;
  else if (!q) fmt = ORC_F16;
  else {
    const JV* qt = q->at("quant_type");
    fmt = (qt && qt->t == 's' && qt->s == "Q4_0") ? ORC_Q4_0 : ORC_Q8_0;
  }
  if (fmt == ORC_Q4_0) { g_err = "safetensors Q4_0 has no defined result (Q8 tensors under the Q4_0 kernel)"; return nullptr; }
  if (fmt == ORC_F16) gs = 32;
  /* :97-117 */
  s.ctx_len = max_seq_len < max_ctx_len ? max_seq_len : max_ctx_len;
  s.group_size = gs;
  s.rope_freq_scale = 1.0f;
  s.rope_ext_factor = 0.0f;
  s.rope_attn_factor = 1.0f;
  s.rope_original_ctx_len = s.ctx_len;
  s.attention_scale = 0.0f;
  s.weight_format = fmt;
  s.rope_mode = ORC_ROPE_LLAMA3; /* the ST forward calls util::rope */
  s.llama3_old_ctx = (float)s.ctx_len;
  s.q4_mode = ORC_Q4_GGML;
  /* :347-352 tokenizer.json, else tokenizer.bin */
  if (!tokenizer_ids(dir, true, &s.bos, &s.eos)) return nullptr;
  /* :122-157 safetensors header */
  int fd = open(path, O_RDONLY);
  if (fd < 0) { g_err = std::string("cannot open ") + path; return nullptr; }
  struct stat st;
  fstat(fd, &st);
  size_t size = (size_t)st.st_size;
  if (size < 8) { close(fd); g_err = "short safetensors file"; return nullptr; }
  void* mp = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (mp == MAP_FAILED) { g_err = "mmap failed"; return nullptr; }
  std::unique_ptr<void, std::function<void(void*)>> guard(mp, [size](void* x) { munmap(x, size); });
  const uint8_t* data = (const uint8_t*)mp;
  uint64_t hlen;
  memcpy(&hlen, data, 8);
  if (hlen > size - 8) { g_err = "bad safetensors header length"; return nullptr; }
  JV hdr;
  if (!json_read((const char*)data + 8, hlen, &hdr) || hdr.t != 'o') { g_err = "bad safetensors header"; return nullptr; }
  size_t data_start = 8 + hlen;
  std::map<std::string, StInfo> tensors;
  for (auto& kv : hdr.o) {
    if (kv.first == "__metadata__") continue;
    const JV* dt = kv.second.at("dtype");
    const JV* offs = kv.second.at("data_offsets");
    if (!dt || dt->t != 's' || !offs || offs->t != 'a' || offs->a.size() != 2) { g_err = "bad entry " + kv.first; return nullptr; }
    StInfo ti;
    ti.dtype = dt->s;
    ti.off = data_start + (size_t)offs->a[0].u;
    ti.len = (size_t)(offs->a[1].u - offs->a[0].u);
    if (ti.off + ti.len > size) { g_err = "tensor out of bounds " + kv.first; return nullptr; }
    tensors[kv.first] = ti;
  }
  auto need = [&](const std::string& nm, size_t bytes, const char* dtype, size_t* off) {
    auto it = tensors.find(nm);
    if (it == tensors.end()) { g_err = "Missing tensor: " + nm; return false; }
    if (dtype && it->second.dtype != dtype) { g_err = "dtype of " + nm; return false; }
    if (it->second.len < bytes) { g_err = "short tensor " + nm; return false; }
    *off = it->second.off;
    return true;
  };
  auto f16vec = [&](size_t off, size_t n, std::vector<float>* out) { /* :162-170 load_f16_vec */
    out->resize(n);
    for (size_t i = 0; i < n; ++i) {
      uint16_t h;
      memcpy(&h, data + off + 2 * i, 2);
      (*out)[i] = orc_f16_to_f32(h);
    }
  };
  bool quant = fmt != ORC_F16;
  /* :280-300 load_q: MLX affine (weight, scales, biases) or an F16 tensor */
  auto load_q = [&](const std::string& stem, size_t rows, size_t cols, QT* out) {
    size_t w, sc, bi;
    if (!quant) {
      if (!need(stem + ".weight", rows * cols * 2, "F16", &w)) return false;
      f16vec(w, rows * cols, &out->f);
      return true;
    }
    if (!need(stem + ".weight", rows * cols, nullptr, &w) || !need(stem + ".scales", rows * cols / gs * 2, nullptr, &sc) ||
        !need(stem + ".biases", rows * cols / gs * 2, nullptr, &bi))
      return false;
    load_q8_tensor_st(data, rows, cols, gs, w, sc, bi, out);
    return true;
  };
  std::unique_ptr<orc_model> m(new orc_model());
  m->shape = s;
  size_t dim = s.dim, qr = (size_t)s.n_heads * s.head_size, kvr = (size_t)s.n_kv_heads * s.head_size;
  size_t off;
  /* :172-178 final norm, :181-199 layer norms */
  if (!need("model.norm.weight", dim * 2, "F16", &off)) return nullptr;
  f16vec(off, dim, &m->w_rms_final);
  size_t L = s.n_layers;
  m->w_rms_att.resize(L); m->w_rms_post_att.resize(L);
  for (size_t l = 0; l < L; ++l) {
    std::string p = "model.layers." + std::to_string(l) + ".";
    if (!need(p + "input_layernorm.weight", dim * 2, "F16", &off)) return nullptr;
    f16vec(off, dim, &m->w_rms_att[l]);
    if (!need(p + "post_attention_layernorm.weight", dim * 2, "F16", &off)) return nullptr;
    f16vec(off, dim, &m->w_rms_post_att[l]);
  }
  /* :213-251 token embedding: F16 as is, else requantized and dequantized q * scale */
  QT emb;
  if (!load_q("model.embed_tokens", s.vocab_size, dim, &emb)) return nullptr;
  m->token_embedding = dequant(emb, gs);
  /* :280-316 */
  m->wq.resize(L); m->wk.resize(L); m->wv.resize(L); m->wo.resize(L);
  m->w1.resize(L); m->w2.resize(L); m->w3.resize(L);
  for (size_t l = 0; l < L; ++l) {
    std::string p = "model.layers." + std::to_string(l) + ".";
    if (!load_q(p + "self_attn.q_proj", qr, dim, &m->wq[l]) || !load_q(p + "self_attn.k_proj", kvr, dim, &m->wk[l]) ||
        !load_q(p + "self_attn.v_proj", kvr, dim, &m->wv[l]) || !load_q(p + "self_attn.o_proj", dim, qr, &m->wo[l]) ||
        !load_q(p + "mlp.gate_proj", s.hidden_dim, dim, &m->w1[l]) ||
        !load_q(p + "mlp.down_proj", dim, s.hidden_dim, &m->w2[l]) ||
        !load_q(p + "mlp.up_proj", s.hidden_dim, dim, &m->w3[l]))
      return nullptr;
  }
  return m.release();
}

static orc_model* load_lmrs(const char* path, uint32_t max_ctx_len) {
  std::string dir = parent_dir(path);
  orc_shape s;
  memset(&s, 0, sizeof(s));
  /* transformer_llama_lmrs.rs:62-66: the file must exist; tokenizer.bin first */
  struct stat st;
  if (stat(path, &st) != 0) { g_err = std::string("Model file does not exist: ") + path; return nullptr; }
  if (!tokenizer_ids(dir, false, &s.bos, &s.eos)) return nullptr;
  int fd = open(path, O_RDONLY);
  if (fd < 0) { g_err = std::string("cannot open ") + path; return nullptr; }
  size_t size = (size_t)st.st_size;
  if (size < 256) { close(fd); g_err = "Model not in lm.rs format."; return nullptr; }
  void* mp = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (mp == MAP_FAILED) { g_err = "mmap failed"; return nullptr; }
  std::unique_ptr<void, std::function<void(void*)>> guard(mp, [size](void* x) { munmap(x, size); });
  const uint8_t* raw = (const uint8_t*)mp;
  /* :72-77 magic */
  if (memcmp(raw, "lmrs", 4) != 0) { g_err = "Model not in lm.rs format."; return nullptr; }
  /* :31-47, :81-88: packed TransformerArgs at 8..55 */
  const uint8_t* c = raw + 8;
  uint32_t seq_len;
  memcpy(&s.dim, c + 0, 4);
  memcpy(&s.hidden_dim, c + 4, 4);
  memcpy(&s.n_layers, c + 8, 4);
  memcpy(&s.n_heads, c + 12, 4);
  memcpy(&s.head_size, c + 16, 4);
  memcpy(&s.n_kv_heads, c + 20, 4);
  memcpy(&s.vocab_size, c + 24, 4);
  memcpy(&seq_len, c + 28, 4);
  memcpy(&s.rms_norm_eps, c + 32, 4);
  memcpy(&s.rope_theta, c + 36, 4);
  memcpy(&s.group_size, c + 42, 4);
  /* :111-120 */
  if (s.dim == 0 || s.hidden_dim == 0 || s.n_heads == 0 || s.n_layers == 0) {
    g_err = "Invalid model configuration: critical dimensions cannot be zero";
    return nullptr;
  }
  if (seq_len == 0 || s.vocab_size == 0) {
    g_err = "Invalid model configuration: sequence length and vocab size must be positive";
    return nullptr;
  }
  if (s.group_size == 0) { g_err = "group_size 0"; return nullptr; }
  /* :122-148 */
  s.ctx_len = seq_len < max_ctx_len ? seq_len : max_ctx_len;
  s.rope_freq_scale = 1.0f;
  s.rope_ext_factor = 0.0f;
  s.rope_attn_factor = 1.0f;
  s.rope_original_ctx_len = s.ctx_len;
  s.attention_scale = 0.0f;
  s.weight_format = ORC_Q8_0; /* :101-109 */
  s.rope_mode = ORC_ROPE_LLAMA3;
  s.llama3_old_ctx = (float)s.ctx_len;
  s.q4_mode = ORC_Q4_GGML;
  size_t gs = s.group_size, dim = s.dim, hd = s.hidden_dim, L = s.n_layers;
  size_t qsz = (size_t)s.n_heads * s.head_size * dim, kvsz = (size_t)s.n_kv_heads * s.head_size * dim;
  /* total bytes the tensors need, so that a short file is an error */
  size_t need = 256 + (size_t)s.vocab_size * dim + (size_t)s.vocab_size * dim / gs * 4 + 2 * L * dim * 4 + dim * 4 +
                L * (2 * (qsz + qsz / gs * 4) + 2 * (kvsz + kvsz / gs * 4) + 3 * (hd * dim + hd * dim / gs * 4));
  if (need > size) { g_err = "lm.rs file shorter than its tensors"; return nullptr; }
  std::unique_ptr<orc_model> m(new orc_model());
  m->shape = s;
  size_t off = 256;
  /* util.rs:547-573 load_q8_tenstor_lmrs: quants then f32 scales */
  auto q8 = [&](size_t n, QT* out) {
    out->q.resize(n);
    memcpy(out->q.data(), raw + off, n);
    off += n;
    out->s.resize(n / gs);
    memcpy(out->s.data(), raw + off, n / gs * 4);
    off += n / gs * 4;
  };
  auto f32v = [&](std::vector<float>* out) {
    out->resize(dim);
    memcpy(out->data(), raw + off, dim * 4);
    off += dim * 4;
  };
  QT emb;
  q8((size_t)s.vocab_size * dim, &emb);
  /* :176-181 emb_tab[i] = q[i] * scale[i / group_size] */
  m->token_embedding = dequant(emb, gs);
  m->w_rms_att.resize(L); m->w_rms_post_att.resize(L);
  m->wq.resize(L); m->wk.resize(L); m->wv.resize(L); m->wo.resize(L);
  m->w1.resize(L); m->w2.resize(L); m->w3.resize(L);
  for (size_t l = 0; l < L; ++l) f32v(&m->w_rms_att[l]);
  for (size_t l = 0; l < L; ++l) q8(qsz, &m->wq[l]);
  for (size_t l = 0; l < L; ++l) q8(kvsz, &m->wk[l]);
  for (size_t l = 0; l < L; ++l) q8(kvsz, &m->wv[l]);
  for (size_t l = 0; l < L; ++l) q8(qsz, &m->wo[l]);
  for (size_t l = 0; l < L; ++l) f32v(&m->w_rms_post_att[l]);
  for (size_t l = 0; l < L; ++l) q8(hd * dim, &m->w1[l]);
  for (size_t l = 0; l < L; ++l) q8(hd * dim, &m->w2[l]);
  for (size_t l = 0; l < L; ++l) q8(hd * dim, &m->w3[l]);
  f32v(&m->w_rms_final);
  return m.release();
}
