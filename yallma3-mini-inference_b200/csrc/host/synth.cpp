// Synthetic GGUF v3 writer: seeded random-init LLaMA models in Q8_0, Q4_0 or
// F16, with the metadata keys the GGUF loader reads
// (transformer_llama_gguf.rs:215-287, :584-641) and the tensor names it loads
// (:453-551). Weights ~ N(0, std) come from a counter-based generator
// (splitmix64 + Box-Muller), so any element can be produced independently and
// the file is identical for any thread count.
#include <cmath>
#include <cstdio>
#include <string>
#include <thread>
#include <vector>

#include "common.h"

namespace {

inline uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Element i of tensor `tid`: two normals per 64-bit draw.
inline float normal_at(uint64_t key, uint64_t i, float std) {
  uint64_t r = splitmix64(key + (i >> 1));
  float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
  float u2 = ((float)((r >> 8) & 0xFFFFFFu) + 0.5f) * (1.0f / 16777216.0f);
  float rad = sqrtf(-2.0f * logf(u1));
  float ang = 6.2831853f * u2;
  return std * rad * ((i & 1) ? sinf(ang) : cosf(ang));
}

struct Buf {
  std::vector<uint8_t> b;
  void u8(uint8_t v) { b.push_back(v); }
  void u32(uint32_t v) { for (int k = 0; k < 4; ++k) b.push_back((uint8_t)(v >> (8 * k))); }
  void u64(uint64_t v) { for (int k = 0; k < 8; ++k) b.push_back((uint8_t)(v >> (8 * k))); }
  void f32(float f) { uint32_t v; memcpy(&v, &f, 4); u32(v); }
  void str(const std::string& s) { u64(s.size()); b.insert(b.end(), s.begin(), s.end()); }
  void kv_u32(const std::string& k, uint32_t v) { str(k); u32(4); u32(v); }
  void kv_f32(const std::string& k, float v) { str(k); u32(6); f32(v); }
  void kv_str(const std::string& k, const std::string& v) { str(k); u32(8); str(v); }
};

struct TensorSpec {
  std::string name;
  uint64_t rows, cols;  // cols = row length (GGUF ne0)
  uint32_t ggml_type;   // 0 F32, 1 F16, 2 Q4_0, 8 Q8_0
  int rng_id;           // -1: constant 1.0 (norms)
  uint64_t offset = 0, nbytes = 0;
};

uint64_t tensor_bytes(uint32_t type, uint64_t n) {
  switch (type) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 2: return n / 32 * 18;
    case 8: return n / 32 * 34;
  }
  return 0;
}

// Encodes blocks [b0, b1) of tensor `t` into `dst` (points at block b0).
void encode_blocks(const TensorSpec& t, uint64_t key, float std, uint64_t b0, uint64_t b1, uint8_t* dst) {
  float w[32];
  for (uint64_t b = b0; b < b1; ++b) {
    for (int j = 0; j < 32; ++j) w[j] = t.rng_id < 0 ? 1.0f : normal_at(key, b * 32 + j, std);
    if (t.ggml_type == 0) {
      memcpy(dst, w, 128);
      dst += 128;
    } else if (t.ggml_type == 1) {
      for (int j = 0; j < 32; ++j) {
        uint16_t h = yl::f32_to_f16(w[j]);
        dst[2 * j] = (uint8_t)h;
        dst[2 * j + 1] = (uint8_t)(h >> 8);
      }
      dst += 64;
    } else if (t.ggml_type == 8) {  // Q8_0: d = absmax/127 (f16), q = round(w/d)
      float amax = 0.f;
      for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(w[j]));
      float d = amax / 127.0f;
      float id = d != 0.f ? 1.0f / d : 0.f;
      uint16_t dh = yl::f32_to_f16(d);
      dst[0] = (uint8_t)dh;
      dst[1] = (uint8_t)(dh >> 8);
      for (int j = 0; j < 32; ++j) {
        int q = (int)roundf(w[j] * id);
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        dst[2 + j] = (uint8_t)(int8_t)q;
      }
      dst += 34;
    } else {  // Q4_0: m = element of largest |w| (signed), d = m/-8, q = clamp(round(w/d)+8, 0, 15)
      float amax = 0.f, m = 0.f;
      for (int j = 0; j < 32; ++j)
        if (fabsf(w[j]) > amax) { amax = fabsf(w[j]); m = w[j]; }
      float d = m / -8.0f;
      float id = d != 0.f ? 1.0f / d : 0.f;
      uint16_t dh = yl::f32_to_f16(d);
      dst[0] = (uint8_t)dh;
      dst[1] = (uint8_t)(dh >> 8);
      for (int j = 0; j < 16; ++j) {
        int lo = (int)roundf(w[j] * id) + 8, hi = (int)roundf(w[j + 16] * id) + 8;
        lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
        hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
        dst[2 + j] = (uint8_t)(lo | (hi << 4));
      }
      dst += 18;
    }
  }
}

}  // namespace

extern "C" int yl_synth_write_gguf(const char* path, const yl_synth_config* c) {
  if (!path || !c) return yl::fail(YL_ERR_ARG, "null argument");
  if (c->dim % 32 || c->hidden_dim % 32 || c->n_heads == 0 || c->dim % c->n_heads || c->n_kv_heads == 0 ||
      c->n_heads % c->n_kv_heads || c->vocab_size == 0)
    return yl::fail(YL_ERR_ARG, "invalid synthetic shape");
  uint32_t wtype = c->weight_format == YL_Q8_0 ? 8 : c->weight_format == YL_Q4_0 ? 2 : 1;
  uint32_t ftype = c->weight_format == YL_Q8_0 ? 7 : c->weight_format == YL_Q4_0 ? 2 : 1;
  uint64_t d = c->dim, f = c->hidden_dim, hd = d / c->n_heads, kvd = hd * c->n_kv_heads;
  std::vector<TensorSpec> ts;
  ts.push_back({"token_embd.weight", c->vocab_size, d, wtype, 0});
  ts.push_back({"output_norm.weight", 1, d, 0, -1});
  if (!c->tied) ts.push_back({"output.weight", c->vocab_size, d, wtype, 1 + 7 * (int)c->n_layers});
  for (uint32_t l = 0; l < c->n_layers; ++l) {
    std::string p = "blk." + std::to_string(l) + ".";
    int r = 1 + 7 * (int)l;
    ts.push_back({p + "attn_norm.weight", 1, d, 0, -1});
    ts.push_back({p + "attn_q.weight", d, d, wtype, r + 0});
    ts.push_back({p + "attn_k.weight", kvd, d, wtype, r + 1});
    ts.push_back({p + "attn_v.weight", kvd, d, wtype, r + 2});
    ts.push_back({p + "attn_output.weight", d, d, wtype, r + 3});
    ts.push_back({p + "ffn_norm.weight", 1, d, 0, -1});
    ts.push_back({p + "ffn_gate.weight", f, d, wtype, r + 4});
    ts.push_back({p + "ffn_up.weight", f, d, wtype, r + 5});
    ts.push_back({p + "ffn_down.weight", d, f, wtype, r + 6});
  }
  const uint64_t align = 32;
  uint64_t off = 0;
  for (auto& t : ts) {
    t.nbytes = tensor_bytes(t.ggml_type, t.rows * t.cols);
    t.offset = off;
    off = yl::round_up(off + t.nbytes, align);
  }
  Buf h;
  h.u32(0x46554747u);
  h.u32(3);
  h.u64(ts.size());
  uint64_t nkv = 16 + (c->llama3_scaling ? 5 : 0);
  h.u64(nkv);
  h.kv_str("general.architecture", "llama");
  h.kv_str("general.name", "yallma3-b200-synthetic");
  h.kv_u32("general.file_type", ftype);
  h.kv_u32("general.alignment", (uint32_t)align);
  h.kv_u32("llama.context_length", c->context_length);
  h.kv_u32("llama.embedding_length", c->dim);
  h.kv_u32("llama.block_count", c->n_layers);
  h.kv_u32("llama.feed_forward_length", c->hidden_dim);
  h.kv_u32("llama.attention.head_count", c->n_heads);
  h.kv_u32("llama.attention.head_count_kv", c->n_kv_heads);
  h.kv_f32("llama.attention.layer_norm_rms_epsilon", c->rms_norm_eps);
  h.kv_f32("llama.rope.freq_base", c->rope_theta);
  if (c->llama3_scaling) {
    h.kv_str("llama.rope.scaling.type", "llama3");
    h.kv_f32("llama.rope.scaling.factor", c->llama3_factor);
    h.kv_f32("llama.rope.scaling.low_freq_factor", c->llama3_low);
    h.kv_f32("llama.rope.scaling.high_freq_factor", c->llama3_high);
    h.kv_u32("llama.rope.scaling.original_context_length", c->llama3_orig_ctx);
  }
  h.kv_str("tokenizer.ggml.model", "gpt2");
  h.str("tokenizer.ggml.tokens");
  h.u32(9);
  h.u32(8);
  h.u64(c->vocab_size);
  for (uint32_t v = 0; v < c->vocab_size; ++v) h.str("<t" + std::to_string(v) + ">");
  uint32_t bos = c->vocab_size > 128009 ? 128000 : 1, eos = c->vocab_size > 128009 ? 128009 : 2;
  h.kv_u32("tokenizer.ggml.bos_token_id", bos);
  h.kv_u32("tokenizer.ggml.eos_token_id", eos);
  for (auto& t : ts) {
    h.str(t.name);
    bool vec = t.rows == 1;
    h.u32(vec ? 1 : 2);
    h.u64(t.cols);
    if (!vec) h.u64(t.rows);
    h.u32(t.ggml_type);
    h.u64(t.offset);
  }
  while (h.b.size() % align) h.u8(0);
  FILE* fp = fopen(path, "wb");
  if (!fp) return yl::fail(YL_ERR_IO, std::string("cannot create ") + path);
  bool ok = fwrite(h.b.data(), 1, h.b.size(), fp) == h.b.size();
  int nthreads = c->threads > 0 ? c->threads : (int)std::thread::hardware_concurrency();
  if (nthreads < 1) nthreads = 1;
  uint64_t written = 0;
  std::vector<uint8_t> chunk;
  const uint64_t blocks_per_chunk = 1u << 20;  // 32M elements per parallel chunk
  for (auto& t : ts) {
    if (!ok) break;
    std::vector<uint8_t> pad(t.offset - written, 0);
    if (!pad.empty()) ok = fwrite(pad.data(), 1, pad.size(), fp) == pad.size();
    written = t.offset;
    uint64_t key = splitmix64(c->seed * 0x9E3779B97F4A7C15ull + (uint64_t)(t.rng_id + 1) * 0xD1B54A32D192ED03ull);
    uint64_t nblocks = t.rows * t.cols / 32, bpb = t.nbytes / nblocks;
    for (uint64_t b0 = 0; b0 < nblocks && ok; b0 += blocks_per_chunk) {
      uint64_t b1 = b0 + blocks_per_chunk < nblocks ? b0 + blocks_per_chunk : nblocks;
      chunk.resize((b1 - b0) * bpb);
      std::vector<std::thread> th;
      uint64_t per = (b1 - b0 + nthreads - 1) / nthreads;
      for (int k = 0; k < nthreads; ++k) {
        uint64_t s = b0 + k * per, e = s + per < b1 ? s + per : b1;
        if (s >= e) break;
        th.emplace_back(encode_blocks, std::cref(t), key, c->weight_std, s, e, chunk.data() + (s - b0) * bpb);
      }
      for (auto& x : th) x.join();
      ok = fwrite(chunk.data(), 1, chunk.size(), fp) == chunk.size();
      written += chunk.size();
    }
  }
  if (fclose(fp) != 0) ok = false;
  if (!ok) return yl::fail(YL_ERR_IO, std::string("write failed: ") + path);
  return YL_OK;
}
