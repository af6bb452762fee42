// Loaders for the two other model files of the reference, into the same
// split HBM layout as GGUF (int8 quant rows + scale rows, scales f32 here):
//  - safetensors + config.json (transformer_llama_st.rs:41-372): MLX affine
//    8-bit groups requantized to symmetric Q8 (util.rs:451-518), or raw F16
//    weights when config.json has no "quantization" section;
//  - lm.rs files (transformer_llama_lmrs.rs:56-439): Q8 with f32 scales.
// Both run the llama forward (forward.rs:119-297) with the half-split rope()
// of util.rs:589-635 (old context length = ctx_len) and a tied lm_head.
#include <sys/stat.h>

#include <algorithm>
#include <cmath>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>

#include "json.h"
#include "model.h"
#include "upload.h"

namespace yl {

namespace {

bool file_exists(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

std::string dir_of(const std::string& p) {
  const size_t k = p.rfind('/');
  return k == std::string::npos ? std::string(".") : p.substr(0, k);
}

int read_text(const std::string& path, std::string* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return fail(YL_ERR_IO, "cannot open " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  *out = ss.str();
  return YL_OK;
}

uint32_t le32(const uint8_t* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}

// BOS / EOS ids of the tokenizer the reference loads beside the model:
// tokenizer.bin keeps them at bytes 8..16 (tokenizer.rs:223-228);
// tokenizer.json names them among its added tokens, defaults 128000 / 128009
// (tokenizer.rs:179-186).
int tokenizer_bin_ids(const std::string& path, uint32_t* bos, uint32_t* eos) {
  std::string t;
  int rc = read_text(path, &t);
  if (rc) return rc;
  if (t.size() < 16) return fail(YL_ERR_FORMAT, "tokenizer.bin is shorter than its 16-byte header");
  *bos = le32((const uint8_t*)t.data() + 8);
  *eos = le32((const uint8_t*)t.data() + 12);
  return YL_OK;
}

int tokenizer_json_ids(const std::string& path, uint32_t* bos, uint32_t* eos) {
  std::string t, err;
  int rc = read_text(path, &t);
  if (rc) return rc;
  Json root;
  if (!json_parse(t.data(), t.size(), &root, &err)) return fail(YL_ERR_FORMAT, "tokenizer.json: " + err);
  const Json* added = root.get("added_tokens");
  if (!added || added->kind != Json::ARR) return fail(YL_ERR_FORMAT, "tokenizer.json: no added_tokens array");
  *bos = 128000u;
  *eos = 128009u;
  for (const Json& tk : added->arr) {
    const Json* c = tk.get("content");
    const Json* id = tk.get("id");
    uint64_t v;
    if (!c || !c->as_str() || !id || !id->as_u64(&v)) return fail(YL_ERR_FORMAT, "tokenizer.json: bad added token");
    if (*c->as_str() == "<|begin_of_text|>") *bos = (uint32_t)v;
    if (*c->as_str() == "<|end_of_text|>" || *c->as_str() == "<|eot_id|>") *eos = (uint32_t)v;
  }
  return YL_OK;
}

// Rust's `f as i32`: truncation toward zero, NaN to 0, saturating.
int32_t rust_f32_as_i32(float f) {
  if (f != f) return 0;
  if (f >= 2147483648.0f) return INT32_MAX;
  if (f <= -2147483648.0f) return INT32_MIN;
  return (int32_t)f;
}

// util.rs:480-515, one group of 32: MLX affine u8 quants q with an f16 scale
// and bias are dequantized as q * scale + bias (a product and a sum, each
// rounded to f32), then requantized symmetrically: scale = max|v| / 127 (1
// when every value is 0), quant = round-half-away-from-zero(v / scale)
// clamped to [-128, 127]. Returns the new scale.
float requant_group32(const uint8_t* q, float scale, float bias, int8_t* out) {
  float deq[32];
  float max_abs = 0.0f;
  for (int i = 0; i < 32; ++i) {
    const volatile float prod = (float)q[i] * scale;  // no contraction into a fused multiply-add
    const float f = prod + bias;
    deq[i] = f;
    const float a = fabsf(f);
    if (a > max_abs) max_abs = a;
  }
  const float sym = max_abs == 0.0f ? 1.0f : max_abs / 127.0f;
  for (int i = 0; i < 32; ++i) {
    const int32_t v = rust_f32_as_i32(roundf(deq[i] / sym));
    out[i] = (int8_t)std::min(127, std::max(-128, v));
  }
  return sym;
}

struct StTensor {
  std::string dtype;
  std::vector<uint64_t> shape;
  uint64_t off = 0, nbytes = 0;  // absolute file offset, byte length
};

// A (rows x cols) projection as stored in the safetensors file: MLX affine
// (weight u32 [rows][cols/4] = the u8 quants in order, scales and biases f16
// [rows][cols/32]) or F16 [rows][cols].
struct StMatrix {
  const uint8_t* w = nullptr;
  const uint8_t* sc = nullptr;
  const uint8_t* bi = nullptr;
  uint32_t rows = 0, cols = 0;
  // row r into the device layout (quants, and f32 scales when quantized)
  void fill(uint32_t r, uint8_t* dq, uint8_t* ds) const {
    if (!sc) {
      memcpy(dq, w + (uint64_t)r * cols * 2, (size_t)cols * 2);
      return;
    }
    const uint32_t nb = cols / 32;
    float* s = reinterpret_cast<float*>(ds);
    for (uint32_t j = 0; j < nb; ++j) {
      const uint64_t g = (uint64_t)r * nb + j;
      uint16_t hs, hb;
      memcpy(&hs, sc + 2 * g, 2);
      memcpy(&hb, bi + 2 * g, 2);
      s[j] = requant_group32(w + (uint64_t)r * cols + 32 * j, f16_to_f32(hs), f16_to_f32(hb),
                             reinterpret_cast<int8_t*>(dq) + 32 * j);
    }
  }
};

}  // namespace

int model_load_st(const char* path, uint32_t max_ctx_len, int fmt_override, Model** out) {
  const std::string mpath(path), dir = dir_of(mpath);
  // config.json (transformer_llama_st.rs:46-93)
  std::string text, err;
  int rc = read_text(dir + "/config.json", &text);
  if (rc) return rc;
  Json cfg;
  if (!json_parse(text.data(), text.size(), &cfg, &err)) return fail(YL_ERR_FORMAT, "config.json: " + err);
  auto u64_of = [&](const char* k, uint32_t* v) -> int {
    const Json* j = cfg.get(k);
    uint64_t x;
    if (!j || !j->as_u64(&x) || x > UINT32_MAX) return fail(YL_ERR_FORMAT, std::string("config.json: ") + k + " missing or not an unsigned integer");
    *v = (uint32_t)x;
    return YL_OK;
  };
  auto f64_of = [&](const char* k, float* v) -> int {
    const Json* j = cfg.get(k);
    double x;
    if (!j || !j->as_f64(&x)) return fail(YL_ERR_FORMAT, std::string("config.json: ") + k + " missing or not a number");
    *v = (float)x;
    return YL_OK;
  };
  std::unique_ptr<Model> m(new Model());
  m->path = mpath;
  m->name = "TransformerLlamaSt";
  yl_shape& s = m->shape;
  uint32_t seq_len = 0;
  if ((rc = u64_of("hidden_size", &s.dim)) || (rc = u64_of("intermediate_size", &s.hidden_dim)) ||
      (rc = u64_of("num_attention_heads", &s.n_heads)) || (rc = u64_of("num_key_value_heads", &s.n_kv_heads)) ||
      (rc = u64_of("head_dim", &s.head_size)) || (rc = u64_of("num_hidden_layers", &s.n_layers)) ||
      (rc = u64_of("vocab_size", &s.vocab_size)) || (rc = f64_of("rms_norm_eps", &s.rms_norm_eps)) ||
      (rc = f64_of("rope_theta", &s.rope_theta)) || (rc = u64_of("max_position_embeddings", &seq_len)))
    return rc;
  // weight format: the override, else the "quantization" section (absent: F16)
  const Json* qsec = cfg.get("quantization");
  uint32_t gs = 32;
  if (qsec) {
    const Json* g = qsec->get("group_size");
    uint64_t x;
    if (g && g->as_u64(&x)) gs = (uint32_t)x;
  }
  int fmt;
  if (fmt_override >= 0) {
    fmt = fmt_override;
  } else if (!qsec) {
    fmt = YL_F16;
  } else {
    const Json* qt = qsec->get("quant_type");
    fmt = (qt && qt->as_str() && *qt->as_str() == "Q4_0") ? YL_Q4_0 : YL_Q8_0;
  }
  if (fmt == YL_Q4_0)
    return fail(YL_ERR_UNSUPPORTED,
                "safetensors Q4_0: the reference loads these tensors as requantized Q8 and then runs its Q4_0 "
                "kernel on them (a format mismatch), so there is no defined result to reproduce");
  if (fmt == YL_F16) gs = 32;
  s.group_size = gs;
  s.weight_format = fmt;
  s.ctx_len = std::min(seq_len, max_ctx_len);
  s.rope_freq_scale = 1.0f;
  s.rope_ext_factor = 0.0f;
  s.rope_attn_factor = 1.0f;
  s.rope_original_ctx_len = s.ctx_len;
  s.attention_scale = 0.0f;
  s.rope_mode = YL_ROPE_LLAMA3;
  s.tp_rank = 0;
  s.tp_size = 1;
  if (s.n_heads == 0 || s.n_layers == 0 || s.dim == 0 || s.vocab_size == 0)
    return fail(YL_ERR_FORMAT, "config.json: zero dimension");
  if ((rc = check_device_shape(s, 1))) return rc;
  set_rank_split(m.get(), 0, 1);
  // the tokenizer the reference loads beside the model supplies BOS / EOS
  // (transformer_llama_st.rs:347-352, :394-400)
  if (file_exists(dir + "/tokenizer.json")) rc = tokenizer_json_ids(dir + "/tokenizer.json", &m->bos, &m->eos);
  else rc = tokenizer_bin_ids(dir + "/tokenizer.bin", &m->bos, &m->eos);
  if (rc) return rc;

  // safetensors header (:123-157): u64 length, JSON {name: {dtype, shape, data_offsets}}
  Mapped mp;
  if ((rc = map_file(path, &mp))) return rc;
  const uint8_t* base = mp.data();
  if (mp.size < 8) return fail(YL_ERR_FORMAT, "safetensors file shorter than its header length");
  uint64_t hlen;
  memcpy(&hlen, base, 8);
  if (hlen > mp.size - 8) return fail(YL_ERR_FORMAT, "safetensors header runs past the end of the file");
  Json hdr;
  if (!json_parse((const char*)base + 8, hlen, &hdr, &err)) return fail(YL_ERR_FORMAT, "safetensors header: " + err);
  if (hdr.kind != Json::OBJ) return fail(YL_ERR_FORMAT, "safetensors header is not an object");
  const uint64_t data_start = 8 + hlen;
  std::map<std::string, StTensor> tensors;
  for (const auto& kv : hdr.obj) {
    if (kv.first == "__metadata__") continue;
    const Json* dt = kv.second.get("dtype");
    const Json* sh = kv.second.get("shape");
    const Json* offs = kv.second.get("data_offsets");
    StTensor t;
    uint64_t a, b;
    if (!dt || !dt->as_str() || !sh || sh->kind != Json::ARR || !offs || offs->kind != Json::ARR ||
        offs->arr.size() != 2 || !offs->arr[0].as_u64(&a) || !offs->arr[1].as_u64(&b) || b < a)
      return fail(YL_ERR_FORMAT, "safetensors header: bad entry " + kv.first);
    t.dtype = *dt->as_str();
    for (const Json& d : sh->arr) {
      uint64_t x;
      if (!d.as_u64(&x)) return fail(YL_ERR_FORMAT, "safetensors header: bad shape of " + kv.first);
      t.shape.push_back(x);
    }
    if (b > mp.size - data_start) return fail(YL_ERR_FORMAT, "tensor out of file bounds: " + kv.first);
    t.off = data_start + a;
    t.nbytes = b - a;
    tensors[kv.first] = t;
  }
  auto get = [&](const std::string& nm, const char* dtype, uint64_t nbytes, const uint8_t** p) -> int {
    auto it = tensors.find(nm);
    if (it == tensors.end()) return fail(YL_ERR_FORMAT, "Missing tensor: " + nm);
    if (dtype && it->second.dtype != dtype)
      return fail(YL_ERR_FORMAT, "Expected " + std::string(dtype) + " tensor " + nm + ", got " + it->second.dtype);
    if (it->second.nbytes < nbytes) return fail(YL_ERR_FORMAT, "tensor smaller than its shape needs: " + nm);
    *p = base + it->second.off;
    return YL_OK;
  };
  const bool quant = fmt != YL_F16;
  // a projection `stem` (.weight, and .scales/.biases when quantized) of rows x cols
  auto matrix = [&](const std::string& stem, uint32_t rows, uint32_t cols, StMatrix* mx) -> int {
    mx->rows = rows;
    mx->cols = cols;
    const uint64_t n = (uint64_t)rows * cols;
    if (!quant) return get(stem + ".weight", "F16", n * 2, &mx->w);
    int r;
    if ((r = get(stem + ".weight", nullptr, n, &mx->w)) || (r = get(stem + ".scales", nullptr, n / 32 * 2, &mx->sc)) ||
        (r = get(stem + ".biases", nullptr, n / 32 * 2, &mx->bi)))
      return r;
    return YL_OK;
  };
  const uint32_t d = s.dim, att = s.n_heads * s.head_size, kvd = s.n_kv_heads * s.head_size, f = s.hidden_dim;
  StMatrix emb;
  if ((rc = matrix("model.embed_tokens", s.vocab_size, d, &emb))) return rc;
  struct LayerSrc {
    StMatrix q, k, v, o, gate, down, up;
    const uint8_t *att_norm = nullptr, *ffn_norm = nullptr;
  };
  std::vector<LayerSrc> ls(s.n_layers);
  const uint8_t* final_norm;
  if ((rc = get("model.norm.weight", "F16", (uint64_t)d * 2, &final_norm))) return rc;
  for (uint32_t l = 0; l < s.n_layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    LayerSrc& L = ls[l];
    if ((rc = get(p + "input_layernorm.weight", "F16", (uint64_t)d * 2, &L.att_norm)) ||
        (rc = get(p + "post_attention_layernorm.weight", "F16", (uint64_t)d * 2, &L.ffn_norm)) ||
        (rc = matrix(p + "self_attn.q_proj", att, d, &L.q)) || (rc = matrix(p + "self_attn.k_proj", kvd, d, &L.k)) ||
        (rc = matrix(p + "self_attn.v_proj", kvd, d, &L.v)) || (rc = matrix(p + "self_attn.o_proj", d, att, &L.o)) ||
        (rc = matrix(p + "mlp.gate_proj", f, d, &L.gate)) || (rc = matrix(p + "mlp.down_proj", d, f, &L.down)) ||
        (rc = matrix(p + "mlp.up_proj", f, d, &L.up)))
      return rc;
  }

  // upload
  YL_CUDA_TRY(cudaGetDevice(&m->device));
  YL_CUDA_TRY(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, m->device));
  Uploader up{m.get()};
  const bool sf16 = false;
  auto norm = [&](const uint8_t* src, float** dst) -> int {
    std::vector<float> v(d);
    for (uint32_t i = 0; i < d; ++i) {
      uint16_t h;
      memcpy(&h, src + 2 * i, 2);
      v[i] = f16_to_f32(h);
    }
    return up.f32(v.data(), d, dst);
  };
  if ((rc = up.rows(fmt, sf16, s.vocab_size, d, [&](uint32_t r, uint8_t* q, uint8_t* sc) { emb.fill(r, q, sc); },
                    &m->emb)))
    return rc;
  m->lm = m->emb;  // tied lm_head (forward.rs:261-279 reads the token embedding)
  if ((rc = norm(final_norm, &m->rms_final))) return rc;
  m->layers.resize(s.n_layers);
  for (uint32_t l = 0; l < s.n_layers; ++l) {
    const LayerSrc& L = ls[l];
    Layer& D = m->layers[l];
    if ((rc = norm(L.att_norm, &D.rms_att)) || (rc = norm(L.ffn_norm, &D.rms_ffn))) return rc;
    rc = up.rows(fmt, sf16, att + 2 * kvd, d, [&](uint32_t r, uint8_t* q, uint8_t* sc) {
      if (r < att) L.q.fill(r, q, sc);
      else if (r < att + kvd) L.k.fill(r - att, q, sc);
      else L.v.fill(r - att - kvd, q, sc);
    }, &D.wqkv);
    if (rc) return rc;
    if ((rc = up.rows(fmt, sf16, d, att, [&](uint32_t r, uint8_t* q, uint8_t* sc) { L.o.fill(r, q, sc); }, &D.wo)))
      return rc;
    rc = up.rows(fmt, sf16, 2 * f, d, [&](uint32_t r, uint8_t* q, uint8_t* sc) {
      if (r & 1) L.up.fill(r / 2, q, sc);
      else L.gate.fill(r / 2, q, sc);
    }, &D.w13);
    if (rc) return rc;
    if ((rc = up.rows(fmt, sf16, d, f, [&](uint32_t r, uint8_t* q, uint8_t* sc) { L.down.fill(r, q, sc); }, &D.w2)))
      return rc;
  }
  // util.rs:589-635: llama3 scaling constants 32 / 1 / 4, old context = ctx_len
  if ((rc = finish_model(m.get(), up, 32.0f, 1.0f, 4.0f, (float)s.ctx_len))) return rc;
  *out = m.release();
  return YL_OK;
}

int model_load_lmrs(const char* path, uint32_t max_ctx_len, int fmt_override, Model** out) {
  (void)fmt_override;  // lm.rs files are Q8_0 whatever the override (transformer_llama_lmrs.rs:101-109)
  const std::string mpath(path), dir = dir_of(mpath);
  Mapped mp;
  int rc = map_file(path, &mp);
  if (rc) return rc;
  const uint8_t* base = mp.data();
  std::unique_ptr<Model> m(new Model());
  m->path = mpath;
  m->name = "TransformerLlamaLmrs";
  // the reference reads tokenizer.bin first (:66), for BOS / EOS
  if ((rc = tokenizer_bin_ids(dir + "/tokenizer.bin", &m->bos, &m->eos))) return rc;
  if (mp.size < 256 || memcmp(base, "lmrs", 4) != 0) return fail(YL_ERR_FORMAT, "Model not in lm.rs format.");
  // packed TransformerArgs at bytes 8..55 (:31-47)
  const uint8_t* h = base + 8;
  yl_shape& s = m->shape;
  s.dim = le32(h + 0);
  s.hidden_dim = le32(h + 4);
  s.n_layers = le32(h + 8);
  s.n_heads = le32(h + 12);
  s.head_size = le32(h + 16);
  s.n_kv_heads = le32(h + 20);
  s.vocab_size = le32(h + 24);
  const uint32_t seq_len = le32(h + 28);
  memcpy(&s.rms_norm_eps, h + 32, 4);
  memcpy(&s.rope_theta, h + 36, 4);
  s.group_size = le32(h + 42);  // after q_type (u8) and model_type (u8)
  if (s.dim == 0 || s.hidden_dim == 0 || s.n_heads == 0 || s.n_layers == 0)
    return fail(YL_ERR_FORMAT, "Invalid model configuration: critical dimensions cannot be zero");
  if (seq_len == 0 || s.vocab_size == 0)
    return fail(YL_ERR_FORMAT, "Invalid model configuration: sequence length and vocab size must be positive");
  s.weight_format = YL_Q8_0;
  s.ctx_len = std::min(seq_len, max_ctx_len);
  s.rope_freq_scale = 1.0f;
  s.rope_ext_factor = 0.0f;
  s.rope_attn_factor = 1.0f;
  s.rope_original_ctx_len = s.ctx_len;
  s.attention_scale = 0.0f;
  s.rope_mode = YL_ROPE_LLAMA3;
  s.tp_rank = 0;
  s.tp_size = 1;
  if ((rc = check_device_shape(s, 1))) return rc;
  set_rank_split(m.get(), 0, 1);
  // Tensor order from byte 256 (:161-438): embedding; attention norms of
  // every layer; wq, wk, wv, wo of every layer (each int8 quants then f32
  // scales); ffn norms; w1 (gate), w2 (down), w3 (up); final norm.
  const uint32_t d = s.dim, att = s.n_heads * s.head_size, kvd = s.n_kv_heads * s.head_size, f = s.hidden_dim;
  const uint32_t L = s.n_layers;
  uint64_t off = 256;
  struct Q8Src {
    uint64_t off = 0;
    uint32_t rows = 0, cols = 0;
  };
  auto take_q8 = [&](uint32_t rows, uint32_t cols) {
    Q8Src t{off, rows, cols};
    off += (uint64_t)rows * cols + (uint64_t)rows * cols / 32 * 4;
    return t;
  };
  auto take_f32 = [&](uint64_t n) {
    const uint64_t o = off;
    off += n * 4;
    return o;
  };
  const Q8Src emb = take_q8(s.vocab_size, d);
  std::vector<uint64_t> att_norm(L), ffn_norm(L);
  std::vector<Q8Src> wq(L), wk(L), wv(L), wo(L), w1(L), w2(L), w3(L);
  for (uint32_t l = 0; l < L; ++l) att_norm[l] = take_f32(d);
  for (uint32_t l = 0; l < L; ++l) wq[l] = take_q8(att, d);
  for (uint32_t l = 0; l < L; ++l) wk[l] = take_q8(kvd, d);
  for (uint32_t l = 0; l < L; ++l) wv[l] = take_q8(kvd, d);
  for (uint32_t l = 0; l < L; ++l) wo[l] = take_q8(d, att);
  for (uint32_t l = 0; l < L; ++l) ffn_norm[l] = take_f32(d);
  for (uint32_t l = 0; l < L; ++l) w1[l] = take_q8(f, d);
  for (uint32_t l = 0; l < L; ++l) w2[l] = take_q8(d, f);
  for (uint32_t l = 0; l < L; ++l) w3[l] = take_q8(f, d);
  const uint64_t final_norm = take_f32(d);
  if (off > mp.size) return fail(YL_ERR_FORMAT, "lm.rs file is shorter than its tensors (" + std::to_string(off) +
                                                    " bytes needed, " + std::to_string(mp.size) + " present)");
  // row r of a Q8 tensor: cols quants at off + r*cols, cols/32 f32 scales after all quants
  auto fill = [&](const Q8Src& t, uint32_t r, uint8_t* q, uint8_t* sc) {
    memcpy(q, base + t.off + (uint64_t)r * t.cols, t.cols);
    memcpy(sc, base + t.off + (uint64_t)t.rows * t.cols + (uint64_t)r * (t.cols / 32) * 4, (size_t)t.cols / 32 * 4);
  };

  YL_CUDA_TRY(cudaGetDevice(&m->device));
  YL_CUDA_TRY(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, m->device));
  Uploader up{m.get()};
  auto f32v = [&](uint64_t o, float** dst) {
    std::vector<float> v(d);
    memcpy(v.data(), base + o, (size_t)d * 4);  // the file's offsets need not be 4-byte aligned
    return up.f32(v.data(), d, dst);
  };
  if ((rc = up.rows(YL_Q8_0, false, s.vocab_size, d, [&](uint32_t r, uint8_t* q, uint8_t* sc) { fill(emb, r, q, sc); },
                    &m->emb)))
    return rc;
  m->lm = m->emb;
  if ((rc = f32v(final_norm, &m->rms_final))) return rc;
  m->layers.resize(L);
  for (uint32_t l = 0; l < L; ++l) {
    Layer& D = m->layers[l];
    if ((rc = f32v(att_norm[l], &D.rms_att)) || (rc = f32v(ffn_norm[l], &D.rms_ffn))) return rc;
    rc = up.rows(YL_Q8_0, false, att + 2 * kvd, d, [&](uint32_t r, uint8_t* q, uint8_t* sc) {
      if (r < att) fill(wq[l], r, q, sc);
      else if (r < att + kvd) fill(wk[l], r - att, q, sc);
      else fill(wv[l], r - att - kvd, q, sc);
    }, &D.wqkv);
    if (rc) return rc;
    if ((rc = up.rows(YL_Q8_0, false, d, att, [&](uint32_t r, uint8_t* q, uint8_t* sc) { fill(wo[l], r, q, sc); },
                      &D.wo)))
      return rc;
    rc = up.rows(YL_Q8_0, false, 2 * f, d, [&](uint32_t r, uint8_t* q, uint8_t* sc) {
      if (r & 1) fill(w3[l], r / 2, q, sc);
      else fill(w1[l], r / 2, q, sc);
    }, &D.w13);
    if (rc) return rc;
    if ((rc = up.rows(YL_Q8_0, false, d, f, [&](uint32_t r, uint8_t* q, uint8_t* sc) { fill(w2[l], r, q, sc); },
                      &D.w2)))
      return rc;
  }
  if ((rc = finish_model(m.get(), up, 32.0f, 1.0f, 4.0f, (float)s.ctx_len))) return rc;
  *out = m.release();
  return YL_OK;
}

}  // namespace yl
