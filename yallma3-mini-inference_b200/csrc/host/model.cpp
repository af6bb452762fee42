// GGUF loading (transformer_llama_gguf.rs:183-655) into the repacked HBM
// layout, sessions (base_transformer.rs:78-105) and the device forward
// (forward.rs:119-297) with a CUDA-graph batch-1 decode step.
#include "model.h"
#include "upload.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <functional>
#include <map>
#include <memory>
#include <thread>

namespace yl {

namespace {

struct GVal {
  uint32_t type = 0;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string str;
  uint64_t arr_len = 0;
  uint32_t arr_type = 0;
};

struct Cursor {
  const uint8_t* p;
  size_t size, off;
  bool ok = true;
  uint64_t rd(size_t k) {
    if (off + k > size) { ok = false; return 0; }
    uint64_t v = 0;
    memcpy(&v, p + off, k);
    off += k;
    return v;
  }
  std::string str() {
    uint64_t n = rd(8);
    if (!ok || n > size - off) { ok = false; return ""; }  // (off + n could wrap)
    std::string s((const char*)p + off, n);
    off += n;
    return s;
  }
  void skip_str() {
    uint64_t n = rd(8);
    if (!ok || n > size - off) { ok = false; return; }
    off += n;
  }
  // GGUF value of type t (transformer_llama_gguf.rs:80-107). Arrays keep only
  // their length and element type (the token list is counted, not stored).
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
        v.arr_type = (uint32_t)rd(4);
        v.arr_len = rd(8);
        if (depth > 1) { ok = false; break; }
        for (uint64_t k = 0; k < v.arr_len && ok; ++k) {
          if (v.arr_type == 8) skip_str();
          else value(v.arr_type, depth + 1);
        }
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

struct TInfo {
  std::string name;
  uint32_t type = 0;  // GGML type
  uint64_t off = 0;   // absolute file offset
  uint64_t ne0 = 0, ne1 = 1;
  uint64_t n = 0;
};

bool meta_u(const std::map<std::string, GVal>& m, const char* k, uint64_t* out) {
  auto it = m.find(k);
  if (it == m.end() || !(it->second.type == 4 || it->second.type == 10)) return false;
  *out = it->second.u;
  return true;
}
bool meta_f(const std::map<std::string, GVal>& m, const char* k, float* out) {
  auto it = m.find(k);
  if (it == m.end() || !(it->second.type == 6 || it->second.type == 12)) return false;
  *out = (float)it->second.f;
  return true;
}
uint32_t meta_id(const std::map<std::string, GVal>& m, const char* k, uint32_t dflt) {
  auto it = m.find(k);
  if (it == m.end()) return dflt;
  switch (it->second.type) {
    case 4: case 10: return (uint32_t)it->second.u;
    case 5: case 11: return (uint32_t)it->second.i;
  }
  return dflt;
}

}  // namespace

Model::~Model() {
  for (void* p : allocs) cudaFree(p);
}

namespace {
Tunables& tunables_mut() {
  static Tunables t = [] {
    Tunables x;
    if (const char* e = getenv("YL_MV_KC_BYTES")) x.kc_bytes = (uint32_t)atoi(e);
    if (const char* e = getenv("YL_MV_SMEM")) x.smem = (uint32_t)atoi(e);
    if (const char* e = getenv("YL_PDL")) x.pdl = atoi(e) != 0;
    if (const char* e = getenv("YL_MV_GRID_MULT")) x.grid_mult = std::max(1, atoi(e));
    if (const char* e = getenv("YL_LM_LIMBS")) x.limbs = atoi(e) != 0;
    if (const char* e = getenv("YL_TP_FUSED")) x.tp_fused = atoi(e) != 0;
    if (const char* e = getenv("YL_GEMM")) x.gemm = atoi(e) != 0;
    if (const char* e = getenv("YL_GEMM_MIN")) x.gemm_min = (uint32_t)std::max(2, atoi(e));
    if (const char* e = getenv("YL_GEMM_TC")) x.gemm_tc = atoi(e) != 0;
    if (const char* e = getenv("YL_GEMM_TC_MIN")) x.gemm_tc_min = (uint32_t)std::max(1, atoi(e));
    if (const char* e = getenv("YL_GEMM_F16_MIN")) x.gemm_f16_min = (uint32_t)std::max(0, atoi(e));
    if (const char* e = getenv("YL_PF_MB")) x.pf_bytes = (uint64_t)std::max(0, atoi(e)) << 20;
    return x;
  }();
  return t;
}
}  // namespace

const Tunables& tunables() { return tunables_mut(); }

int set_tunable(const std::string& key, int64_t value) {
  Tunables& t = tunables_mut();
  if (key == "gemm_tc") t.gemm_tc = value != 0;
  else if (key == "gemm_tc_min") t.gemm_tc_min = (uint32_t)std::max<int64_t>(1, value);
  else if (key == "gemm") t.gemm = value != 0;
  else if (key == "gemm_f16_min") t.gemm_f16_min = (uint32_t)std::max<int64_t>(0, value);
  else return fail(YL_ERR_ARG, "unknown option " + key);
  return YL_OK;
}

int model_load_gguf(const char* path, uint32_t max_ctx_len, int fmt_override, int tp_rank, int tp_size, Model** out) {
  if (tp_size < 1 || tp_size > 8 || tp_rank < 0 || tp_rank >= tp_size) return fail(YL_ERR_ARG, "bad tensor-parallel rank/size");
  Mapped mp;
  int rc = map_file(path, &mp);
  if (rc) return rc;
  const uint8_t* base = mp.data();
  Cursor c{base, mp.size, 0};
  if (c.rd(4) != 0x46554747u) return fail(YL_ERR_FORMAT, "Not a GGUF file (bad magic)");
  const uint64_t version = c.rd(4);
  if (version != 3) return fail(YL_ERR_FORMAT, "Only GGUF version 3 is supported, got " + std::to_string(version));
  const uint64_t n_tensors = c.rd(8), n_kv = c.rd(8);
  std::map<std::string, GVal> meta;
  for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
    std::string key = c.str();
    uint32_t t = (uint32_t)c.rd(4);
    meta[key] = c.value(t);
  }
  if (!c.ok) return fail(YL_ERR_FORMAT, "truncated GGUF metadata");
  auto arch = meta.find("general.architecture");
  if (arch == meta.end() || arch->second.str != "llama")
    return fail(YL_ERR_FORMAT, "Unsupported GGUF architecture (must be 'llama')");

  std::unique_ptr<Model> m(new Model());
  m->path = path;
  yl_shape& s = m->shape;
  uint64_t v;
  if (!meta_u(meta, "llama.embedding_length", &v)) return fail(YL_ERR_FORMAT, "Missing llama.embedding_length");
  s.dim = (uint32_t)v;
  if (!meta_u(meta, "llama.feed_forward_length", &v)) return fail(YL_ERR_FORMAT, "Missing llama.feed_forward_length");
  s.hidden_dim = (uint32_t)v;
  if (!meta_u(meta, "llama.block_count", &v)) return fail(YL_ERR_FORMAT, "Missing llama.block_count");
  s.n_layers = (uint32_t)v;
  if (!meta_u(meta, "llama.attention.head_count", &v)) return fail(YL_ERR_FORMAT, "Missing head_count");
  s.n_heads = (uint32_t)v;
  s.n_kv_heads = meta_u(meta, "llama.attention.head_count_kv", &v) ? (uint32_t)v : s.n_heads;
  if (!meta_f(meta, "llama.attention.layer_norm_rms_epsilon", &s.rms_norm_eps))
    return fail(YL_ERR_FORMAT, "Missing layer_norm_rms_epsilon");
  const uint64_t file_type = meta_u(meta, "general.file_type", &v) ? v : 7;
  if (!meta_f(meta, "llama.rope.freq_base", &s.rope_theta)) s.rope_theta = 10000.0f;
  if (!meta_u(meta, "llama.context_length", &v)) return fail(YL_ERR_FORMAT, "Missing llama.context_length");
  const uint32_t seq_len = (uint32_t)v;
  if (s.n_heads == 0 || s.dim % s.n_heads) return fail(YL_ERR_FORMAT, "dim must be divisible by n_heads");
  s.head_size = s.dim / s.n_heads;
  s.ctx_len = std::min(seq_len, max_ctx_len);
  auto toks = meta.find("tokenizer.ggml.tokens");
  if (toks == meta.end() || toks->second.type != 9) return fail(YL_ERR_FORMAT, "tokenizer.ggml.tokens not found");
  s.vocab_size = (uint32_t)toks->second.arr_len;
  float raw = 1.0f;
  if (!meta_f(meta, "llama.rope.scaling.factor", &raw)) raw = 1.0f;
  s.rope_freq_scale = raw != 0.0f ? 1.0f / raw : 1.0f;
  if (!meta_f(meta, "llama.rope.scaling.ext_factor", &s.rope_ext_factor)) s.rope_ext_factor = 0.0f;
  if (!meta_f(meta, "llama.rope.scaling.attn_factor", &s.rope_attn_factor)) s.rope_attn_factor = 1.0f;
  s.rope_original_ctx_len = meta_u(meta, "llama.rope.scaling.original_context_length", &v) ? (uint32_t)v : seq_len;
  if (!meta_f(meta, "llama.attention.scale", &s.attention_scale)) s.attention_scale = 0.0f;
  s.group_size = 32;
  auto sct = meta.find("llama.rope.scaling.type");
  s.rope_mode = (sct != meta.end() && sct->second.str == "llama3") ? YL_ROPE_LLAMA3 : YL_ROPE_GGUF;
  float l3_factor = 32.0f, l3_low = 1.0f, l3_high = 4.0f;
  meta_f(meta, "llama.rope.scaling.factor", &l3_factor);
  meta_f(meta, "llama.rope.scaling.low_freq_factor", &l3_low);
  meta_f(meta, "llama.rope.scaling.high_freq_factor", &l3_high);
  int fmt;
  if (fmt_override >= 0) fmt = fmt_override;
  else if (file_type == 1) fmt = YL_F16;
  else if (file_type == 2) fmt = YL_Q4_0;
  else if (file_type == 7) fmt = YL_Q8_0;
  else return fail(YL_ERR_FORMAT, "Unsupported GGUF file_type " + std::to_string(file_type));
  s.weight_format = fmt;
  s.tp_rank = tp_rank;
  s.tp_size = tp_size;
  m->bos = meta_id(meta, "tokenizer.ggml.bos_token_id", 128000u);
  m->eos = meta_id(meta, "tokenizer.ggml.eos_token_id", 128009u);
  if ((rc = check_device_shape(s, tp_size))) return rc;
  set_rank_split(m.get(), tp_rank, tp_size);

  std::map<std::string, TInfo> tmap;
  for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
    TInfo ti;
    ti.name = c.str();
    const uint32_t nd = (uint32_t)c.rd(4);
    ti.n = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      uint64_t e = c.rd(8);
      if (d == 0) ti.ne0 = e;
      else if (d == 1) ti.ne1 = e;
      ti.n *= e;
    }
    ti.type = (uint32_t)c.rd(4);
    ti.off = c.rd(8);
    tmap[ti.name] = ti;
  }
  if (!c.ok) return fail(YL_ERR_FORMAT, "truncated tensor infos");
  const uint64_t alignment = meta_u(meta, "general.alignment", &v) ? v : 32;
  if (alignment == 0 || (alignment & (alignment - 1))) return fail(YL_ERR_FORMAT, "GGUF alignment must be a power of 2");
  const uint64_t data_start = (c.off + alignment - 1) / alignment * alignment;
  for (auto& kv : tmap) kv.second.off += data_start;
  auto bytes_of = [](uint32_t type, uint64_t n) -> uint64_t {
    switch (type) {
      case 0: return n * 4;
      case 1: return n * 2;
      case 2: return n / 32 * 18;
      case 8: return n / 32 * 34;
    }
    return 0;
  };
  for (auto& kv : tmap) {
    const uint64_t nb = bytes_of(kv.second.type, kv.second.n);
    if (nb == 0 || kv.second.off > mp.size || nb > mp.size - kv.second.off)  // (off + nb could wrap)
      return fail(YL_ERR_FORMAT, "tensor out of file bounds: " + kv.first);
  }
  auto get = [&](const std::string& nm, const TInfo** out_ti) -> int {
    auto it = tmap.find(nm);
    if (it == tmap.end()) return fail(YL_ERR_FORMAT, "Missing tensor: " + nm);
    *out_ti = &it->second;
    return YL_OK;
  };
  const uint32_t want_type = fmt == YL_Q8_0 ? 8 : fmt == YL_Q4_0 ? 2 : 1;

  YL_CUDA_TRY(cudaGetDevice(&m->device));
  YL_CUDA_TRY(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, m->device));
  Uploader up{m.get()};
  const uint32_t d = s.dim, att = s.n_heads * s.head_size, kvd = s.n_kv_heads * s.head_size, f = s.hidden_dim;
  auto row_ptr = [&](const TInfo* ti, uint32_t cols, uint32_t r) {
    return base + ti->off + bytes_of(ti->type, (uint64_t)r * cols);
  };
  auto check = [&](const TInfo* ti, uint64_t rows, uint64_t cols) -> int {
    if (ti->type != want_type) return fail(YL_ERR_FORMAT, "format/variant mismatch in " + ti->name);
    if (ti->n != rows * cols) return fail(YL_ERR_FORMAT, "unexpected element count in " + ti->name);
    return YL_OK;
  };
  const TInfo* te;
  if ((rc = get("token_embd.weight", &te))) return rc;
  if (te->n != (uint64_t)s.vocab_size * d) return fail(YL_ERR_FORMAT, "token_embd.weight shape mismatch");
  if ((rc = up.gguf(te->type, s.vocab_size, d, [&](uint32_t r) { return row_ptr(te, d, r); }, &m->emb))) return rc;
  m->lm = m->emb;  // this rank's vocabulary rows of the tied table
  m->lm.rows = m->l_vocab;
  m->lm.q = m->emb.q + (uint64_t)m->vocab0 * m->emb.row_bytes;
  if (m->emb.s) m->lm.s = m->emb.s + (uint64_t)m->vocab0 * m->emb.scale_row_bytes;
  auto out_it = tmap.find("output.weight");
  if (out_it != tmap.end()) {  // untied lm_head (resolved deviation D2)
    const TInfo* to = &out_it->second;
    if (to->n != (uint64_t)s.vocab_size * d) return fail(YL_ERR_FORMAT, "output.weight shape mismatch");
    if ((rc = up.gguf(to->type, m->l_vocab, d, [&](uint32_t r) { return row_ptr(to, d, m->vocab0 + r); }, &m->lm)))
      return rc;
    s.untied_lm_head = 1;
  }
  auto f32t = [&](const std::string& nm, uint64_t n, float** dst) -> int {
    const TInfo* t;
    int r = get(nm, &t);
    if (r) return r;
    if (t->type != 0 || t->n != n) return fail(YL_ERR_FORMAT, "Expected F32 tensor " + nm);
    return up.f32((const float*)(base + t->off), n, dst);
  };
  if ((rc = f32t("output_norm.weight", d, &m->rms_final))) return rc;
  m->layers.resize(s.n_layers);
  for (uint32_t l = 0; l < s.n_layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    Layer& L = m->layers[l];
    if ((rc = f32t(p + "attn_norm.weight", d, &L.rms_att))) return rc;
    if ((rc = f32t(p + "ffn_norm.weight", d, &L.rms_ffn))) return rc;
    const TInfo *tq, *tk, *tv, *to, *tg, *tu, *tdn;
    if ((rc = get(p + "attn_q.weight", &tq)) || (rc = get(p + "attn_k.weight", &tk)) ||
        (rc = get(p + "attn_v.weight", &tv)) || (rc = get(p + "attn_output.weight", &to)) ||
        (rc = get(p + "ffn_gate.weight", &tg)) || (rc = get(p + "ffn_up.weight", &tu)) ||
        (rc = get(p + "ffn_down.weight", &tdn)))
      return rc;
    if ((rc = check(tq, att, d)) || (rc = check(tk, kvd, d)) || (rc = check(tv, kvd, d)) || (rc = check(to, d, att)) ||
        (rc = check(tg, f, d)) || (rc = check(tu, f, d)) || (rc = check(tdn, d, f)))
      return rc;
    // this rank's rows / columns (the whole matrices at one rank)
    const uint32_t hs = s.head_size, la = m->l_heads * hs, lk = m->l_kv * hs, lf = m->l_ffn;
    const uint32_t qa0 = (uint32_t)tp_rank * la, kv0 = (uint32_t)tp_rank * lk, f0 = (uint32_t)tp_rank * lf;
    rc = up.gguf(want_type, la + 2 * lk, d, [&](uint32_t r) {
      if (r < la) return row_ptr(tq, d, qa0 + r);
      if (r < la + lk) return row_ptr(tk, d, kv0 + r - la);
      return row_ptr(tv, d, kv0 + r - la - lk);
    }, &L.wqkv);
    if (rc) return rc;
    if ((rc = up.gguf(want_type, d, la, [&](uint32_t r) { return row_ptr(to, att, r) + bytes_of(want_type, qa0); },
                        &L.wo)))
      return rc;
    rc = up.gguf(want_type, 2 * lf, d,
                   [&](uint32_t r) { return (r & 1) ? row_ptr(tu, d, f0 + r / 2) : row_ptr(tg, d, f0 + r / 2); }, &L.w13);
    if (rc) return rc;
    if ((rc = up.gguf(want_type, d, lf, [&](uint32_t r) { return row_ptr(tdn, f, r) + bytes_of(want_type, f0); },
                        &L.w2)))
      return rc;
  }
  if ((rc = finish_model(m.get(), up, l3_factor, l3_low, l3_high, (float)s.rope_original_ctx_len))) return rc;
  *out = m.release();
  return YL_OK;
}

// ------------------------------ sessions ---------------------------------

Session::~Session() {
  if (graph) cudaGraphExecDestroy(graph);
  if (graph_lg) cudaGraphExecDestroy(graph_lg);
  if (stream) cudaStreamSynchronize(stream);
  for (void* p : tp_opened) cudaIpcCloseMemHandle(p);
  if (tp_region) cudaFree(tp_region);
  if (stream) cudaStreamDestroy(stream);
  for (void* p : allocs) cudaFree(p);
  if (ascr) cudaFree(ascr);
  if (logits_h) cudaFreeHost(logits_h);
  if (hist_h) cudaFreeHost(hist_h);
}

namespace {
int salloc(Session* s, size_t bytes, void** out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 256));
  if (e != cudaSuccess) return fail(YL_ERR_OOM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  s->allocs.push_back(p);
  *out = p;
  return YL_OK;
}

// Grows the per-token workspace to hold `n` tokens.
int ensure_cap(Session* s, uint32_t n) {
  if (n <= s->cap) return YL_OK;
  const yl_shape& sh = s->m->shape;
  const uint64_t att = (uint64_t)sh.n_heads * sh.head_size, kvd = (uint64_t)sh.n_kv_heads * sh.head_size;
  const uint64_t wmax = std::max<uint64_t>({sh.dim, att, sh.hidden_dim});
  const uint32_t cap = std::max(n, 8u);
  void* p;
  int rc;
  if ((rc = salloc(s, cap * sh.dim * 4ull, &p))) return rc;
  s->x = (float*)p;
  if ((rc = salloc(s, cap * wmax * 4ull, &p))) return rc;
  s->xf = (float*)p;
  if ((rc = salloc(s, cap * wmax, &p))) return rc;
  s->xq = (int8_t*)p;
  if ((rc = salloc(s, cap * (wmax / 32) * 4ull, &p))) return rc;
  s->xs = (float*)p;
  if ((rc = salloc(s, cap * (att + 2 * kvd) * 4ull, &p))) return rc;
  s->qkv = (float*)p;
  if ((rc = salloc(s, cap * att * 4ull, &p))) return rc;
  s->q = (float*)p;
  if ((rc = salloc(s, cap * (uint64_t)sh.hidden_dim * 4ull, &p))) return rc;
  s->h = (float*)p;
  if ((rc = salloc(s, cap * (uint64_t)sh.hidden_dim, &p))) return rc;
  s->hq = (int8_t*)p;
  if ((rc = salloc(s, cap * (uint64_t)(sh.hidden_dim / 32) * 4ull, &p))) return rc;
  s->hs = (float*)p;
  if ((rc = salloc(s, cap * (uint64_t)(sh.hidden_dim / 32) * 4ull, &p))) return rc;
  s->hcount = (unsigned int*)p;
  YL_CUDA_TRY(cudaMemset(s->hcount, 0, cap * (uint64_t)(sh.hidden_dim / 32) * 4ull));
  if ((rc = salloc(s, cap * 4ull, &p))) return rc;
  s->tok = (uint32_t*)p;
  if (sh.weight_format == YL_F16 && s->m->tp_size == 1) {
    if ((rc = salloc(s, k::gemm_f16_workspace_bytes(cap, (uint32_t)wmax), &p))) return rc;
    s->f16ws = p;
  }
  s->cap = cap;
  return YL_OK;
}
}  // namespace

int session_create(const Model* m, Session** out) { return session_create_ex(m, true, out); }

int session_create_ex(const Model* m, bool with_kv, Session** out) {
  std::unique_ptr<Session> s(new Session());
  s->m = m;
  s->device = m->device;
  YL_CUDA_TRY(cudaSetDevice(m->device));
  YL_CUDA_TRY(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
  const yl_shape& sh = m->shape;
  const uint64_t kvd = (uint64_t)m->l_kv * sh.head_size;  // this rank's KV heads
  s->kv_elems = with_kv ? (uint64_t)sh.n_layers * sh.ctx_len * kvd : 0;
  void* p;
  int rc;
  if (with_kv) {
    if ((rc = salloc(s.get(), s->kv_elems * 4, &p))) return rc;
    s->kcache = (float*)p;
    if ((rc = salloc(s.get(), s->kv_elems * 4, &p))) return rc;
    s->vcache = (float*)p;
    YL_CUDA_TRY(cudaMemset(s->kcache, 0, s->kv_elems * 4));
    YL_CUDA_TRY(cudaMemset(s->vcache, 0, s->kv_elems * 4));
  }
  if ((rc = salloc(s.get(), (uint64_t)sh.vocab_size * 4, &p))) return rc;
  s->logits = (float*)p;
  // decode attention: one cluster of n_splits CTAs per KV head; the scores /
  // weights of every local query head over the context
  s->n_splits = k::attention_decode_splits(m->l_kv, sh.head_size);
  s->part_stride = (uint32_t)round_up(sh.ctx_len, 4);
  if ((rc = salloc(s.get(), (uint64_t)m->l_heads * s->part_stride * 4, &p))) return rc;
  s->part = (float*)p;
  if ((rc = salloc(s.get(), ((uint64_t)sh.n_layers + 1) * 2 * 4, &p))) return rc;
  s->work = (unsigned int*)p;
  YL_CUDA_TRY(cudaMemset(s->work, 0, ((uint64_t)sh.n_layers + 1) * 2 * 4));
  if ((rc = salloc(s.get(), ((uint64_t)sh.ctx_len + 1) * 4, &p))) return rc;
  s->hist = (uint32_t*)p;
  const uint64_t am_slots = (uint64_t)m->num_sms * 8;
  if ((rc = salloc(s.get(), am_slots * 4, &p))) return rc;
  s->am_val = (float*)p;
  if ((rc = salloc(s.get(), am_slots * 4, &p))) return rc;
  s->am_idx = (uint32_t*)p;
  if ((rc = salloc(s.get(), sizeof(unsigned int), &p))) return rc;
  s->am_count = (unsigned int*)p;
  YL_CUDA_TRY(cudaMemset(s->am_count, 0, sizeof(unsigned int)));
  if ((rc = salloc(s.get(), sizeof(k::StepState), &p))) return rc;
  s->state = (k::StepState*)p;
  if ((rc = salloc(s.get(), sizeof(int), &p))) return rc;
  s->err = (int*)p;
  YL_CUDA_TRY(cudaMemset(s->err, 0, sizeof(int)));
  YL_CUDA_TRY(cudaMemset(s->state, 0, sizeof(k::StepState)));
  YL_CUDA_TRY(cudaMallocHost(&s->logits_h, (uint64_t)sh.vocab_size * 4));
  YL_CUDA_TRY(cudaMallocHost(&s->hist_h, ((uint64_t)sh.ctx_len + 1) * 4));
  if ((rc = ensure_cap(s.get(), 8))) return rc;
  if (m->tp_size > 1) {
    // exchange region: flags [2 L + 1][world], partials [2][tp_cap][dim],
    // the lm_head winner slot, and this rank's logits slice
    s->tp_cap = 512;
    const uint64_t world = (uint64_t)m->tp_size;
    s->tp_flags_off = 0;
    uint64_t off = round_up((2ull * sh.n_layers + 1) * world * 4, 256);
    s->tp_part_off[0] = off;
    off += round_up((uint64_t)s->tp_cap * sh.dim * 4, 256);
    s->tp_part_off[1] = off;
    off += round_up((uint64_t)s->tp_cap * sh.dim * 4, 256);
    s->tp_lm_off = off;
    off += 256;
    s->tp_inbox_off[0] = off;
    off += round_up(world * sh.dim * 8, 256);
    s->tp_inbox_off[1] = off;
    off += round_up(world * sh.dim * 8, 256);
    s->tp_logit_off = off;
    off += round_up((uint64_t)m->l_vocab * 4, 256);
    s->tp_bytes = off;
    YL_CUDA_TRY(cudaMalloc(&p, s->tp_bytes));  // plain cudaMalloc: exportable through CUDA IPC
    s->tp_region = (uint8_t*)p;
    YL_CUDA_TRY(cudaMemset(s->tp_region, 0, s->tp_bytes));
    if ((rc = salloc(s.get(), 8, &p))) return rc;
    s->tp_epoch = (uint32_t*)p;
    s->tp_pepoch = s->tp_epoch + 1;
    YL_CUDA_TRY(cudaMemset(s->tp_epoch, 0, 8));
    if ((rc = salloc(s.get(), (uint64_t)sh.dim * 4, &p))) return rc;
    s->x2 = (float*)p;
  }
  *out = s.release();
  return YL_OK;
}

int session_tp_handle(Session* s, void* handle_out) {
  if (s->m->tp_size < 2) return fail(YL_ERR_ARG, "session is not tensor-parallel");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  cudaIpcMemHandle_t h;
  YL_CUDA_TRY(cudaIpcGetMemHandle(&h, s->tp_region));
  memcpy(handle_out, &h, sizeof(h));
  return YL_OK;
}

int session_tp_connect(Session* s, const void* handles) {
  const Model* m = s->m;
  if (m->tp_size < 2) return fail(YL_ERR_ARG, "session is not tensor-parallel");
  if (s->tp_ready) return fail(YL_ERR_ARG, "session already connected");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  for (int r = 0; r < m->tp_size; ++r) {
    if (r == m->tp_rank) {
      s->tp_base[r] = s->tp_region;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, (const uint8_t*)handles + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(YL_ERR_COMM, std::string("opening rank ") + std::to_string(r) +
                                                       "'s exchange region: " + cudaGetErrorString(e));
    s->tp_opened.push_back(p);
    s->tp_base[r] = (uint8_t*)p;
  }
  s->tp_ready = true;
  return YL_OK;
}

int session_reset(Session* s) {
  YL_CUDA_TRY(cudaSetDevice(s->device));
  YL_CUDA_TRY(cudaMemsetAsync(s->kcache, 0, s->kv_elems * 4, s->stream));
  YL_CUDA_TRY(cudaMemsetAsync(s->vcache, 0, s->kv_elems * 4, s->stream));
  YL_CUDA_TRY(cudaStreamSynchronize(s->stream));
  s->pos = 0;
  return YL_OK;
}

// ------------------------------ forward ------------------------------------

int run_matvec(const DevWeight& w, bool f32act, const int8_t* xq, const float* xs, const float* xf, uint64_t x_stride,
               uint64_t xs_stride, uint32_t ntok, float* out, uint64_t out_stride, int epi, uint32_t quirk_cols,
               int* err, cudaStream_t st, bool pdl, int num_sms) {
  return run_matvec_ex(w, f32act, xq, xs, xf, x_stride, xs_stride, ntok, out, out_stride, epi, quirk_cols, err, st,
                       pdl, num_sms, MvExtra(), nullptr);
}

int run_matvec_ex(const DevWeight& w, bool f32act, const int8_t* xq, const float* xs, const float* xf,
                  uint64_t x_stride, uint64_t xs_stride, uint32_t ntok, float* out, uint64_t out_stride, int epi,
                  uint32_t quirk_cols, int* err, cudaStream_t st, bool pdl, int num_sms, const MvExtra& ex,
                  uint32_t* launches) {
  const Tunables& tu = tunables();
  int fmt;
  uint32_t kc;
  if (w.fmt == YL_Q8_0) {
    fmt = f32act ? k::FMT_Q8F : k::FMT_Q8;
    // f32 activations out of the norm prologue run as three int8 limbs (dp4a)
    if (f32act && tu.limbs && ex.pro == k::PRO_NORM && w.cols <= 8192) fmt = k::FMT_Q8X;
    kc = tu.kc_bytes;
  }
  else if (w.fmt == YL_Q4_0) { fmt = f32act ? k::FMT_Q4F : k::FMT_Q4; kc = tu.kc_bytes * 2; }
  else { fmt = k::FMT_F16; kc = tu.kc_bytes / 2; }
  if (tu.kc_bytes == 0) kc = (uint32_t)round_up(w.cols, 256);  // whole rows
  kc = std::max<uint32_t>(256, kc / 256 * 256);
  k::LaunchCfg lc;
  lc.stream = st;
  lc.pdl = pdl;
  lc.grid = (uint32_t)num_sms * tu.grid_mult;
  lc.smem_budget = tu.smem;
  // several tokens of an F16 model: the f16 tensor-core GEMM, its activation
  // split (with the RMSNorm prologue) as a separate kernel
  if (f32act && fmt == k::FMT_F16 && tu.gemm && tu.gemm_f16_min && ntok >= tu.gemm_f16_min && ex.tp_mode == 0 &&
      ex.f16ws && (ex.pro == k::PRO_LOAD || (ex.pro == k::PRO_NORM && ex.xres && ex.norm_w))) {
    k::GemmF16Args g{};
    g.w = w.q;
    g.rows = w.rows;
    g.K = w.cols;
    g.row_bytes = w.row_bytes;
    g.x = ex.pro == k::PRO_NORM ? ex.xres : xf;
    g.x_stride = x_stride;
    g.norm_w = ex.pro == k::PRO_NORM ? ex.norm_w : nullptr;
    g.eps = ex.eps;
    g.ntok = ntok;
    g.hi = static_cast<uint16_t*>(ex.f16ws);
    g.lo = g.hi + (uint64_t)ntok * w.cols;
    g.exps = reinterpret_cast<int*>(g.lo + (uint64_t)ntok * w.cols);
    g.out = out;
    g.out_stride = out_stride;
    g.quirk_cols = quirk_cols;
    if (k::gemm_f16_supported(g, epi)) {
      cudaError_t e = k::gemm_f16(g, epi, lc);
      if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("f16 gemm launch: ") + cudaGetErrorString(e));
      if (launches) *launches += 2;
      return YL_OK;
    }
  }
  // several tokens with int8 activations: the tensor-core GEMM (weights read
  // once per 64 tokens), with the RMSNorm prologue as a separate kernel
  if (!f32act && tu.gemm && ntok >= tu.gemm_min && ex.tp_mode == 0 && (fmt == k::FMT_Q8 || fmt == k::FMT_Q4) &&
      (ex.pro == k::PRO_LOAD || (ex.pro == k::PRO_NORM && ex.gq && ex.gs && ex.xres && ex.norm_w))) {
    k::GemmArgs g{};
    g.wq = w.q;
    g.ws = w.s;
    g.rows = w.rows;
    g.K = w.cols;
    g.row_bytes = w.row_bytes;
    g.scale_row_bytes = w.scale_row_bytes;
    g.xq = ex.pro == k::PRO_NORM ? ex.gq : xq;
    g.xs = ex.pro == k::PRO_NORM ? ex.gs : xs;
    g.x_stride = ex.pro == k::PRO_NORM ? w.cols : x_stride;
    g.xs_stride = ex.pro == k::PRO_NORM ? w.cols / 32 : xs_stride;
    g.ntok = ntok;
    g.out = out;
    g.out_stride = out_stride;
    g.quirk_cols = quirk_cols;
    g.hq = ex.hq;
    g.hs = ex.hs;
    g.err = err;
    if (k::gemm_supported(g, fmt, w.sf16, epi)) {
      if (ex.pro == k::PRO_NORM) {
        cudaError_t e = k::rmsnorm_quant(ex.xres, ex.norm_w, ntok, w.cols, ex.eps, ex.gq, ex.gs, nullptr, lc);
        if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("rmsnorm_quant launch: ") + cudaGetErrorString(e));
        if (launches) ++*launches;
      }
      const bool tc = tu.gemm_tc && ntok >= tu.gemm_tc_min && w.no_inf_scales && k::gemm_tc_supported(g, fmt, w.sf16, epi);
      cudaError_t e = tc ? k::gemm_tc(g, w.sf16, epi, lc) : k::gemm_q(g, fmt, w.sf16, epi, lc);
      if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("gemm launch: ") + cudaGetErrorString(e));
      if (launches) ++*launches;
      return YL_OK;
    }
  }
  const uint32_t kc_eff = std::min<uint32_t>(kc, (uint32_t)round_up(w.cols, 256));
  const uint32_t group = k::matvec_max_ntok(fmt, w.cols, kc_eff, epi);
  if (group == 0) return fail(YL_ERR_UNSUPPORTED, "matvec row length too large for shared memory");
  for (uint32_t t0 = 0; t0 < ntok; t0 += group) {
    k::MvArgs a{};
    a.wq = w.q;
    a.ws = w.s;
    a.rows = w.rows;
    a.K = w.cols;
    a.row_bytes = w.row_bytes;
    a.scale_row_bytes = w.scale_row_bytes;
    a.kc = kc_eff;
    a.xq = xq ? xq + t0 * x_stride : nullptr;
    a.xs = xs ? xs + t0 * xs_stride : nullptr;
    a.xf = xf ? xf + t0 * x_stride : nullptr;
    a.x_tok_stride = x_stride;
    a.xs_tok_stride = xs_stride;
    a.ntok = std::min(group, ntok - t0);
    a.out = out + t0 * out_stride;
    a.out_tok_stride = out_stride;
    a.quirk_cols = quirk_cols;
    a.err = err;
    a.pro = ex.pro;
    a.xres = ex.xres ? ex.xres + t0 * x_stride : nullptr;
    a.norm_w = ex.norm_w;
    a.eps = ex.eps;
    a.hq = ex.hq ? ex.hq + t0 * (uint64_t)(w.rows / 2) : nullptr;
    a.hs = ex.hs ? ex.hs + t0 * (uint64_t)(w.rows / 64) : nullptr;
    a.hcount = ex.hcount ? ex.hcount + t0 * (uint64_t)(w.rows / 64) : nullptr;
    a.am_val = ex.am_val;
    a.am_idx = ex.am_idx;
    a.am_count = ex.am_count;
    a.am_out = ex.am_out;
    a.state = ex.state;
    a.trace = ex.trace;
    a.work = ex.work;
    a.am_shard = ex.am_shard;
    a.am_base = ex.am_base;
    if (t0 + group >= ntok) a.pf = ex.pf;  // the last pass of this site prefetches for the next one
    a.tp_mode = ex.tp_mode;
    if (ex.tp_mode) {
      for (int r = 0; r < 8; ++r) a.tp_base[r] = ex.tp->base[r];
      a.tp_rank = ex.tp->rank;
      a.tp_world = ex.tp->world;
      a.tp_epoch = ex.tp_epoch;
      a.tp_inbox_off = ex.tp_inbox_off;
      a.tp_site = ex.tp_site;
      a.tp_nsites = ex.tp_nsites;
      a.tp_xout = ex.tp_xout;
    }
    cudaError_t e = k::matvec(a, fmt, w.sf16, epi, lc);
    if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("matvec launch: ") + cudaGetErrorString(e));
    if (launches) ++*launches;
  }
  return YL_OK;
}

namespace {

// Enqueues the full forward for n tokens (already on device in s->tok unless
// from_state). from_state: batch-1 step whose token/pos live in s->state
// (graph capture). pdl: launch with programmatic dependent launch.
int enqueue_forward(Session* s, uint32_t n, uint32_t start_pos, bool from_state, bool pdl, uint32_t* launches,
                    bool want_logits = true) {
  const Model* m = s->m;
  const yl_shape& sh = m->shape;
  // this rank's attention width, KV width and ffn rows (the whole model at one rank)
  const uint32_t d = sh.dim, att = m->l_heads * sh.head_size, kvd = m->l_kv * sh.head_size, f = m->l_ffn;
  const bool tp = m->tp_size > 1;
  if (tp && !s->tp_ready) return fail(YL_ERR_ARG, "tensor-parallel session is not connected to its peers");
  if (tp && n > s->tp_cap) return fail(YL_ERR_ARG, "too many tokens for the exchange buffers in one pass");
  k::TpArgs tpa{};
  if (tp) {
    for (int r = 0; r < m->tp_size; ++r) tpa.base[r] = s->tp_base[r];
    tpa.rank = (uint32_t)m->tp_rank;
    tpa.world = (uint32_t)m->tp_size;
    tpa.flags_off = s->tp_flags_off;
    tpa.epoch = s->tp_epoch;
    tpa.err = s->err;
  }
  const bool f32act = sh.weight_format == YL_F16;
  const k::StepState* st = from_state ? s->state : nullptr;
  k::LaunchCfg lc;
  lc.stream = s->stream;
  lc.pdl = pdl;
  uint32_t nl = 0;
  cudaError_t e;
  int rc;
// With s->prof set (profiling), an event is recorded after every launch.
#define YL_MARK()                                   \
  do {                                              \
    if (s->prof) {                                  \
      cudaEvent_t ev_;                              \
      YL_CUDA_TRY(cudaEventCreate(&ev_));           \
      s->prof->push_back(ev_);                      \
      YL_CUDA_TRY(cudaEventRecordWithFlags(ev_, s->stream, cudaEventRecordExternal)); \
    }                                               \
  } while (0)
#define YL_LAUNCH(expr)                                                                   \
  do {                                                                                    \
    e = (expr);                                                                           \
    if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e)); \
    ++nl;                                                                                 \
    YL_MARK();                                                                            \
  } while (0)
// timeline stamps of the launch about to be enqueued (launch index nl)
#define YL_TRACE() (s->trace_on ? s->trace + (uint64_t)nl * TRACE_STRIDE : nullptr)
  MvExtra plain;
#define YL_MV(...)                                                   \
  do {                                                               \
    plain.trace = YL_TRACE();                                        \
    if ((rc = run_matvec_ex(__VA_ARGS__, plain, nullptr))) return rc; \
    nl += 1;                                                         \
    YL_MARK();                                                       \
  } while (0)

  YL_MARK();
  YL_LAUNCH(k::embed(m->emb.fmt == YL_Q8_0 ? k::FMT_Q8 : m->emb.fmt == YL_Q4_0 ? k::FMT_Q4 : k::FMT_F16, m->emb.q,
                     m->emb.s, m->emb.row_bytes, m->emb.scale_row_bytes, m->emb.sf16, d, sh.vocab_size, s->tok, st, n, s->x, lc));
  const bool decode = n == 1;
  // Decode streams every weight once per token. Each weight-streaming launch
  // (and the attention kernel, during which HBM would idle) prefetches into
  // L2 the first rows the next weight-streaming launch reads, aimed at that
  // launch's own schedule (its CTAs' static ranges, or its first row sets).
  const uint32_t mv_grid = (uint32_t)m->num_sms * tunables().grid_mult;
  auto pf_for = [&](const DevWeight& w, int epi, bool has_work) {
    k::L2Prefetch p;
    const uint64_t budget = tunables().pf_bytes;
    if (!decode || budget == 0 || !w.q || w.rows == 0) return p;
    uint32_t g;
    bool dyn;
    k::matvec_schedule(w.rows, epi, mv_grid, 1, has_work, &g, &dyn);
    if (g == 0) return p;
    const uint64_t per_row = (uint64_t)w.row_bytes + w.scale_row_bytes;
    const uint64_t rows = std::min<uint64_t>(w.rows, std::max<uint64_t>(1, budget / per_row));
    p.q = w.q;
    p.s = w.s;
    p.rows = w.rows;
    p.row_bytes = w.row_bytes;
    p.srow_bytes = w.scale_row_bytes;
    p.unit = (epi == k::EPI_SWIGLU || epi == k::EPI_SWIGLU_Q8) ? 2u : 1u;
    p.dyn = dyn ? 1u : 0u;
    p.slots = dyn ? mv_grid : g;
    uint64_t each = (rows + p.slots - 1) / p.slots;
    if (dyn) each = round_up(each, k::MV_ROWSET);
    p.rows_each = (uint32_t)each;
    return p;
  };
  const int epi_ffn = f32act ? k::EPI_SWIGLU : k::EPI_SWIGLU_Q8;
  const int epi_res = tp ? k::EPI_STORE : k::EPI_ADD;
  MvExtra norm;
  norm.pro = k::PRO_NORM;
  norm.xres = s->x;
  norm.eps = sh.rms_norm_eps;
  norm.gq = decode ? nullptr : s->xq;  // multi-token passes: normalized rows for the GEMM
  norm.gs = decode ? nullptr : s->xs;
  norm.f16ws = decode ? nullptr : s->f16ws;  // F16 models: split rows for the f16 GEMM
  plain.f16ws = norm.f16ws;
  // Tensor-parallel single-token steps: wo and down push their partial rows
  // into every rank's inbox in their epilogue, and the next RMSNorm prologue
  // all-reduces them into the residual, which alternates between two rows
  // (xcur is read, the other written by CTA 0). Multi-token passes (and
  // YL_TP_FUSED=0) all-reduce with a separate exchange kernel instead.
  const bool tp_push = tp && decode && tunables().tp_fused;
  float* xcur = s->x;
  float* xalt = s->x2;
  auto tp_pull = [&](MvExtra& ex, uint32_t site) {  // all-reduce prologue of the site's pushes
    ex.tp_mode = 2;
    ex.tp = &tpa;
    ex.tp_epoch = s->tp_pepoch;
    ex.tp_inbox_off = s->tp_inbox_off[site & 1];
    ex.tp_site = site;
    ex.tp_nsites = 2 * sh.n_layers;
    ex.tp_xout = xalt;
  };
  auto tp_push_ex = [&](MvExtra& ex, uint32_t site) {  // push epilogue into the site's inboxes
    ex = MvExtra();
    ex.tp_mode = 1;
    ex.tp = &tpa;
    ex.tp_epoch = s->tp_pepoch;
    ex.tp_inbox_off = s->tp_inbox_off[site & 1];
    ex.tp_site = site;
    ex.tp_nsites = 2 * sh.n_layers;
  };
  auto own_inbox = [&](uint32_t site) {
    return (float*)(s->tp_region + s->tp_inbox_off[site & 1]);  // not written: the entries are pushed
  };
  for (uint32_t l = 0; l < sh.n_layers; ++l) {
    const Layer& L = m->layers[l];
    float* kc = s->kcache + (uint64_t)l * sh.ctx_len * kvd;
    float* vc = s->vcache + (uint64_t)l * sh.ctx_len * kvd;
    // ---- attention block (forward.rs:154-204) ----
    // RMSNorm + quantize fused into the QKV projection's prologue
    norm.norm_w = L.rms_att;
    norm.hq = nullptr;
    norm.hs = nullptr;
    norm.hcount = nullptr;
    norm.trace = YL_TRACE();
    norm.work = nullptr;
    norm.xres = xcur;
    norm.tp_mode = 0;
    norm.pf = pf_for(L.wo, epi_res, false);
    if (tp_push && l > 0) tp_pull(norm, 2 * (l - 1) + 1);
    if ((rc = run_matvec_ex(L.wqkv, f32act, nullptr, nullptr, nullptr, d, d / 32, n, s->qkv, att + 2 * kvd,
                            k::EPI_STORE, 0, s->err, s->stream, pdl, m->num_sms, norm, &nl)))
      return rc;
    YL_MARK();
    if (norm.tp_mode == 2) std::swap(xcur, xalt);
    if (decode) {
      // RoPE, KV write, split attention, merge and quantize in one kernel
      k::AttnDecodeArgs ad{};
      ad.qkv = s->qkv;
      ad.cs = m->rope_cs;
      ad.rope_mode = sh.rope_mode;
      ad.kcache = kc;
      ad.vcache = vc;
      ad.n_heads = m->l_heads;
      ad.n_kv_heads = m->l_kv;
      ad.head_size = sh.head_size;
      ad.kv_dim = kvd;
      ad.state = st;
      ad.pos0 = start_pos;
      ad.scale = m->attn_scale;
      ad.n_splits = s->n_splits;
      ad.sc = s->part;
      ad.sc_stride = s->part_stride;
      ad.early_kv = from_state ? 1 : 0;
      ad.trace = YL_TRACE();
      ad.pf = pf_for(L.w13, epi_ffn, true);
      ad.out = f32act ? s->xf : nullptr;
      ad.q8 = f32act ? nullptr : s->xq;
      ad.s8 = s->xs;
      YL_LAUNCH(k::attention_decode(ad, lc));
    } else {
      YL_LAUNCH(k::rope_kv(s->qkv, n, m->l_heads, m->l_kv, sh.head_size, sh.rope_mode, m->rope_cs, sh.ctx_len,
                           st, start_pos, s->q, kc, vc, lc));
      k::AttnArgs aa{};
      aa.q = s->q;
      aa.kcache = kc;
      aa.vcache = vc;
      aa.ntok = n;
      aa.n_heads = m->l_heads;
      aa.n_kv_heads = m->l_kv;
      aa.head_size = sh.head_size;
      aa.kv_dim = kvd;
      aa.state = st;
      aa.pos0 = start_pos;
      aa.scale = m->attn_scale;
      aa.n_splits = 1;
      if (s->ascr_floats < k::attention_scratch_floats(n, m->l_heads, start_pos))
        return fail(YL_ERR_ARG, "attention scratch not sized for this pass");
      aa.part = s->ascr;
      aa.out = f32act ? s->xf : nullptr;
      aa.q8 = f32act ? nullptr : s->xq;
      aa.s8 = s->xs;
      YL_LAUNCH(k::attention(aa, lc));
    }
    // wo projection + residual add (tensor-parallel: this rank's partial
    // sums, all-reduced over peer memory into the replicated residual)
    plain.pf = pf_for(L.w13, epi_ffn, true);
    if (tp_push) {
      MvExtra px;
      tp_push_ex(px, 2 * l);
      px.trace = YL_TRACE();
      px.pf = plain.pf;
      if ((rc = run_matvec_ex(L.wo, f32act, s->xq, s->xs, s->xf, att, att / 32, n, own_inbox(2 * l), d, k::EPI_STORE,
                              0, s->err, s->stream, pdl, m->num_sms, px, &nl)))
        return rc;
      YL_MARK();
    } else if (tp) {
      YL_MV(L.wo, f32act, s->xq, s->xs, s->xf, att, att / 32, n, (float*)(s->tp_region + s->tp_part_off[0]), d,
            k::EPI_STORE, 0, s->err, s->stream, pdl, m->num_sms);
      tpa.site = 2 * l;
      YL_LAUNCH(k::tp_allreduce_add(tpa, s->tp_part_off[0], n * d, s->x, lc));
    } else {
      YL_MV(L.wo, f32act, s->xq, s->xs, s->xf, att, att / 32, n, s->x, d, k::EPI_ADD, 0, s->err, s->stream, pdl,
            m->num_sms);
    }
    // ---- feed-forward block (forward.rs:206-253) ----
    // RMSNorm + quantize in the prologue, SwiGLU in the epilogue (row pairs:
    // any CTA split keeps gate and up together), which for quantized formats
    // also quantizes h once (forward.rs:240). F16Kernel's quantize is a copy
    // (forward.rs:78-81), so the F16 path keeps h in f32.
    norm.norm_w = L.rms_ffn;
    norm.hq = f32act ? nullptr : s->hq;
    norm.hs = f32act ? nullptr : s->hs;
    norm.hcount = f32act ? nullptr : s->hcount;
    norm.trace = YL_TRACE();
    norm.work = decode ? s->work + 2ull * l : nullptr;  // one launch per step at this site
    norm.xres = xcur;
    norm.tp_mode = 0;
    norm.pf = pf_for(L.w2, epi_res, false);
    if (tp_push) tp_pull(norm, 2 * l);
    if ((rc = run_matvec_ex(L.w13, f32act, nullptr, nullptr, nullptr, d, d / 32, n, s->h, f,
                            f32act ? k::EPI_SWIGLU : k::EPI_SWIGLU_Q8, 0, s->err, s->stream, pdl, m->num_sms, norm,
                            &nl)))
      return rc;
    YL_MARK();
    if (norm.tp_mode == 2) std::swap(xcur, xalt);
    // down projection + residual add
    plain.pf = l + 1 < sh.n_layers ? pf_for(m->layers[l + 1].wqkv, k::EPI_STORE, false)
                                   : pf_for(m->lm, k::EPI_ARGMAX, true);
    if (tp_push) {
      MvExtra px;
      tp_push_ex(px, 2 * l + 1);
      px.trace = YL_TRACE();
      px.pf = plain.pf;
      if ((rc = run_matvec_ex(L.w2, f32act, s->hq, s->hs, s->h, f, f / 32, n, own_inbox(2 * l + 1), d, k::EPI_STORE, 0,
                              s->err, s->stream, pdl, m->num_sms, px, &nl)))
        return rc;
      YL_MARK();
    } else if (tp) {
      YL_MV(L.w2, f32act, s->hq, s->hs, s->h, f, f / 32, n, (float*)(s->tp_region + s->tp_part_off[1]), d,
            k::EPI_STORE, 0, s->err, s->stream, pdl, m->num_sms);
      tpa.site = 2 * l + 1;
      YL_LAUNCH(k::tp_allreduce_add(tpa, s->tp_part_off[1], n * d, s->x, lc));
    } else {
      YL_MV(L.w2, f32act, s->hq, s->hs, s->h, f, f / 32, n, s->x, d, k::EPI_ADD, 0, s->err, s->stream, pdl,
            m->num_sms);
    }
  }
  // final norm (prologue), lm_head on the last token and greedy id
  // (forward.rs:256-279, sampler.rs:67-79)
  {
    MvExtra fin;
    fin.pro = k::PRO_NORM;
    fin.xres = xcur + (uint64_t)(n - 1) * d;
    if (tp_push) tp_pull(fin, 2 * sh.n_layers - 1);
    fin.norm_w = m->rms_final;
    fin.eps = sh.rms_norm_eps;
    fin.am_val = s->am_val;
    fin.am_idx = s->am_idx;
    fin.am_count = s->am_count;
    fin.am_out = tp ? nullptr : s->hist;
    fin.state = (from_state && !tp) ? s->state : nullptr;
    fin.trace = YL_TRACE();
    fin.work = s->work + 2ull * sh.n_layers;  // lm_head: one launch per forward
    fin.pf = pf_for(m->layers[0].wqkv, k::EPI_STORE, false);  // the next decode step starts there
    // tensor-parallel: this rank's vocabulary rows; the winner is published
    // in the exchange region and combined across ranks
    fin.am_shard = tp ? (float*)(s->tp_region + s->tp_lm_off) : nullptr;
    fin.am_base = m->vocab0;
    float* lg = tp ? (float*)(s->tp_region + s->tp_logit_off) : s->logits;
    if ((rc = run_matvec_ex(m->lm, true, nullptr, nullptr, nullptr, d, 0, 1, lg, m->l_vocab, k::EPI_ARGMAX, 0, s->err,
                            s->stream, pdl, m->num_sms, fin, &nl)))
      return rc;
    YL_MARK();
    if (tp) {
      tpa.site = 2 * sh.n_layers;
      YL_LAUNCH(k::tp_argmax(tpa, s->tp_lm_off, s->tp_logit_off, m->l_vocab, want_logits ? s->logits : nullptr,
                             s->hist, from_state ? s->state : nullptr, s->tp_epoch, tp_push ? s->tp_pepoch : nullptr,
                             lc));
    }
  }
#undef YL_LAUNCH
#undef YL_MV
#undef YL_MARK
#undef YL_TRACE
  if (launches) *launches = nl;
  return YL_OK;
}

}  // namespace

int forward(Session* s, const uint32_t* tokens_host, uint32_t n, uint32_t start_pos, bool want_logits) {
  const yl_shape& sh = s->m->shape;
  if (n == 0) return fail(YL_ERR_ARG, "empty token batch");
  if ((uint64_t)start_pos + n > sh.ctx_len) return fail(YL_ERR_RANGE, "position beyond ctx_len");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  // tensor-parallel passes are limited by the exchange buffers: a longer
  // prompt runs in chunks (causal attention over the cache makes that exact)
  const uint32_t chunk = s->m->tp_size > 1 ? s->tp_cap : n;
  for (uint32_t t0 = 0; t0 < n; t0 += chunk) {
    const uint32_t nc = std::min(chunk, n - t0);
    int rc = ensure_cap(s, nc);
    if (rc) return rc;
    // multi-token attention keeps every (row, head) weight row of the pass
    const uint64_t need = nc > 1 ? k::attention_scratch_floats(nc, s->m->l_heads, start_pos + t0) : 0;
    if (need > s->ascr_floats) {
      YL_CUDA_TRY(cudaStreamSynchronize(s->stream));
      if (s->ascr) cudaFree(s->ascr);
      s->ascr = nullptr;
      s->ascr_floats = 0;
      YL_CUDA_TRY(cudaMalloc(&s->ascr, need * 4));
      s->ascr_floats = need;
    }
    YL_CUDA_TRY(cudaMemcpyAsync(s->tok, tokens_host + t0, (uint64_t)nc * 4, cudaMemcpyHostToDevice, s->stream));
    rc = enqueue_forward(s, nc, start_pos + t0, false, tunables().pdl, nullptr, want_logits && t0 + nc == n);
    if (rc) return rc;
  }
  return YL_OK;
}

// ------------------------------ batched sessions ---------------------------

Batch::~Batch() {
  if (ws) {
    cudaStreamSynchronize(ws->stream);
    delete ws;
  }
  if (tok_h) cudaFreeHost(tok_h);
}

int batch_create(const Model* m, uint32_t cap, Batch** out) {
  if (cap == 0 || cap > k::YL_MAX_BATCH)
    return fail(YL_ERR_ARG, "a batch carries 1 to " + std::to_string(k::YL_MAX_BATCH) + " sessions");
  if (m->tp_size > 1) return fail(YL_ERR_UNSUPPORTED, "batched decode runs on one GPU (not tensor parallel)");
  YL_CUDA_TRY(cudaSetDevice(m->device));
  std::unique_ptr<Batch> b(new Batch());
  b->m = m;
  b->cap = cap;
  int rc = session_create_ex(m, false, &b->ws);
  if (rc) return rc;
  Session* w = b->ws;
  if ((rc = ensure_cap(w, cap))) return rc;
  const yl_shape& sh = m->shape;
  void* p;
  if ((rc = salloc(w, (uint64_t)cap * m->l_heads * w->part_stride * 4, &p))) return rc;
  b->sc = (float*)p;
  if ((rc = salloc(w, (uint64_t)cap * sh.vocab_size * 4, &p))) return rc;
  b->logits = (float*)p;
  if ((rc = salloc(w, (uint64_t)cap * 4, &p))) return rc;
  b->ids = (uint32_t*)p;
  YL_CUDA_TRY(cudaMallocHost(&b->tok_h, (uint64_t)(2 * cap + 1) * 4));
  *out = b.release();
  return YL_OK;
}

int forward_batch(Batch* b, Session* const* ss, uint32_t n, const uint32_t* tokens, const uint32_t* pos) {
  const Model* m = b->m;
  const yl_shape& sh = m->shape;
  if (n == 0 || n > b->cap) return fail(YL_ERR_ARG, "batch of " + std::to_string(n) + " sessions, capacity " + std::to_string(b->cap));
  for (uint32_t i = 0; i < n; ++i) {
    if (!ss[i] || ss[i]->m != m) return fail(YL_ERR_ARG, "session missing or of another model");
    if (pos[i] >= sh.ctx_len) return fail(YL_ERR_RANGE, "position beyond ctx_len");
    for (uint32_t j = 0; j < i; ++j)
      if (ss[j] == ss[i]) return fail(YL_ERR_ARG, "a session appears twice in one batch");
  }
  Session* w = b->ws;
  YL_CUDA_TRY(cudaSetDevice(m->device));
  for (uint32_t i = 0; i < n; ++i) YL_CUDA_TRY(cudaStreamSynchronize(ss[i]->stream));  // their caches are settled
  memcpy(b->tok_h, tokens, (uint64_t)n * 4);
  YL_CUDA_TRY(cudaMemcpyAsync(w->tok, b->tok_h, (uint64_t)n * 4, cudaMemcpyHostToDevice, w->stream));
  const uint32_t d = sh.dim, att = m->l_heads * sh.head_size, kvd = m->l_kv * sh.head_size, f = m->l_ffn;
  const bool f32act = sh.weight_format == YL_F16;
  const bool pdl = tunables().pdl;
  k::LaunchCfg lc;
  lc.stream = w->stream;
  lc.pdl = pdl;
  int rc;
  cudaError_t e = k::embed(m->emb.fmt == YL_Q8_0 ? k::FMT_Q8 : m->emb.fmt == YL_Q4_0 ? k::FMT_Q4 : k::FMT_F16, m->emb.q,
                           m->emb.s, m->emb.row_bytes, m->emb.scale_row_bytes, m->emb.sf16, d, sh.vocab_size, w->tok,
                           nullptr, n, w->x, lc);
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("embed launch: ") + cudaGetErrorString(e));
  MvExtra norm, plain;
  norm.pro = k::PRO_NORM;
  norm.xres = w->x;
  norm.eps = sh.rms_norm_eps;
  norm.gq = w->xq;  // 16+ rows: normalized rows for the GEMM
  norm.gs = w->xs;
  norm.f16ws = w->f16ws;
  plain.f16ws = w->f16ws;
  for (uint32_t l = 0; l < sh.n_layers; ++l) {
    const Layer& L = m->layers[l];
    // attention block: the stacked rows' projections, then every session's
    // RoPE, cache write and attention over its own cache in one launch
    norm.norm_w = L.rms_att;
    norm.hq = nullptr;
    norm.hs = nullptr;
    norm.hcount = nullptr;
    if ((rc = run_matvec_ex(L.wqkv, f32act, nullptr, nullptr, nullptr, d, d / 32, n, w->qkv, att + 2 * kvd,
                            k::EPI_STORE, 0, w->err, w->stream, pdl, m->num_sms, norm, nullptr)))
      return rc;
    k::AttnDecodeArgs ad{};
    ad.qkv = w->qkv;
    ad.cs = m->rope_cs;
    ad.rope_mode = sh.rope_mode;
    ad.n_heads = m->l_heads;
    ad.n_kv_heads = m->l_kv;
    ad.head_size = sh.head_size;
    ad.kv_dim = kvd;
    ad.scale = m->attn_scale;
    ad.n_splits = w->n_splits;
    ad.sc = b->sc;
    ad.sc_stride = w->part_stride;
    ad.early_kv = 0;
    ad.out = f32act ? w->xf : nullptr;
    ad.q8 = f32act ? nullptr : w->xq;
    ad.s8 = w->xs;
    ad.nseq = n;
    for (uint32_t i = 0; i < n; ++i) {
      ad.kseq[i] = ss[i]->kcache + (uint64_t)l * sh.ctx_len * kvd;
      ad.vseq[i] = ss[i]->vcache + (uint64_t)l * sh.ctx_len * kvd;
      ad.pseq[i] = pos[i];
    }
    ad.qkv_stride = att + 2 * kvd;
    ad.sc_seq_stride = (uint64_t)m->l_heads * w->part_stride;
    if ((e = k::attention_decode(ad, lc)) != cudaSuccess)
      return fail(YL_ERR_CUDA, std::string("batched attention launch: ") + cudaGetErrorString(e));
    if ((rc = run_matvec_ex(L.wo, f32act, w->xq, w->xs, w->xf, att, att / 32, n, w->x, d, k::EPI_ADD, 0, w->err,
                            w->stream, pdl, m->num_sms, plain, nullptr)))
      return rc;
    // feed-forward block
    norm.norm_w = L.rms_ffn;
    norm.hq = f32act ? nullptr : w->hq;
    norm.hs = f32act ? nullptr : w->hs;
    norm.hcount = f32act ? nullptr : w->hcount;
    if ((rc = run_matvec_ex(L.w13, f32act, nullptr, nullptr, nullptr, d, d / 32, n, w->h, f,
                            f32act ? k::EPI_SWIGLU : k::EPI_SWIGLU_Q8, 0, w->err, w->stream, pdl, m->num_sms, norm,
                            nullptr)))
      return rc;
    if ((rc = run_matvec_ex(L.w2, f32act, w->hq, w->hs, w->h, f, f / 32, n, w->x, d, k::EPI_ADD, 0, w->err, w->stream,
                            pdl, m->num_sms, plain, nullptr)))
      return rc;
  }
  // every row's final norm, lm_head and greedy id (forward.rs:256-279)
  for (uint32_t i = 0; i < n; ++i) {
    MvExtra fin;
    fin.pro = k::PRO_NORM;
    fin.xres = w->x + (uint64_t)i * d;
    fin.norm_w = m->rms_final;
    fin.eps = sh.rms_norm_eps;
    fin.am_val = w->am_val;
    fin.am_idx = w->am_idx;
    fin.am_count = w->am_count;
    fin.am_out = b->ids + i;
    fin.work = w->work + 2ull * sh.n_layers;
    if ((rc = run_matvec_ex(m->lm, true, nullptr, nullptr, nullptr, d, 0, 1, b->logits + (uint64_t)i * sh.vocab_size,
                            m->l_vocab, k::EPI_ARGMAX, 0, w->err, w->stream, pdl, m->num_sms, fin, nullptr)))
      return rc;
  }
  for (uint32_t i = 0; i < n; ++i) ss[i]->pos = pos[i] + 1;
  return YL_OK;
}

int profile_step(Session* s, uint32_t token, uint32_t pos, float* us, uint32_t cap, uint32_t* n_out) {
  const yl_shape& sh = s->m->shape;
  if (pos >= sh.ctx_len) return fail(YL_ERR_RANGE, "position beyond ctx_len");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  int rc = ensure_cap(s, 8);
  if (rc) return rc;
  YL_CUDA_TRY(cudaMemcpyAsync(s->tok, &token, 4, cudaMemcpyHostToDevice, s->stream));
  YL_CUDA_TRY(cudaStreamSynchronize(s->stream));
  // Captured as a graph (event-record nodes between kernel nodes) so that the
  // host's launch pacing does not enter the measured gaps.
  std::vector<cudaEvent_t> evs;
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ge = nullptr;
  YL_CUDA_TRY(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  s->prof = &evs;
  rc = enqueue_forward(s, 1, pos, false, false, nullptr);
  s->prof = nullptr;
  cudaError_t e = cudaStreamEndCapture(s->stream, &g);
  if (e == cudaSuccess && rc == YL_OK) e = cudaGraphInstantiate(&ge, g, 0);
  if (e == cudaSuccess && rc == YL_OK) e = cudaGraphLaunch(ge, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (ge) cudaGraphExecDestroy(ge);
  if (g) cudaGraphDestroy(g);
  uint32_t n = 0;
  for (size_t i = 1; i < evs.size(); ++i) {
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, evs[i - 1], evs[i]);
    if (n < cap && us) us[n] = ms * 1000.0f;
    ++n;
  }
  for (cudaEvent_t ev : evs) cudaEventDestroy(ev);
  if (rc) return rc;
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("profile: ") + cudaGetErrorString(e));
  if (n_out) *n_out = n;
  return YL_OK;
}

int trace_step(Session* s, uint32_t token, uint32_t pos, uint64_t* out, uint64_t cap, uint32_t* n_launches) {
  const yl_shape& sh = s->m->shape;
  if (!YL_WITH_TRACE)
    return fail(YL_ERR_UNSUPPORTED, "timeline stamps are compiled in only by a diagnostics build (YL_WITH_TRACE=1)");
  if (pos >= sh.ctx_len) return fail(YL_ERR_RANGE, "position beyond ctx_len");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  int rc = ensure_cap(s, 8);
  if (rc) return rc;
  const uint64_t n_max = 7ull * sh.n_layers + 6;
  if (!s->trace) {
    void* p = nullptr;
    if ((rc = salloc(s, n_max * TRACE_STRIDE * 8, &p))) return rc;
    s->trace = (uint64_t*)p;
  }
  YL_CUDA_TRY(cudaMemsetAsync(s->trace, 0, n_max * TRACE_STRIDE * 8, s->stream));
  {
    k::LaunchCfg lc;
    lc.stream = s->stream;
    YL_CUDA_TRY(k::set_step_state(s->state, (int32_t)pos, (int32_t)token, lc));
  }
  YL_CUDA_TRY(cudaStreamSynchronize(s->stream));
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ge = nullptr;
  uint32_t nl = 0;
  YL_CUDA_TRY(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  s->trace_on = true;
  rc = enqueue_forward(s, 1, 0, true, tunables().pdl, &nl);
  s->trace_on = false;
  cudaError_t e = cudaStreamEndCapture(s->stream, &g);
  if (e == cudaSuccess && rc == YL_OK) e = cudaGraphInstantiate(&ge, g, 0);
  if (e == cudaSuccess && rc == YL_OK) e = cudaGraphLaunch(ge, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (ge) cudaGraphExecDestroy(ge);
  if (g) cudaGraphDestroy(g);
  if (rc) return rc;
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("trace: ") + cudaGetErrorString(e));
  const uint64_t n = std::min<uint64_t>(cap, (uint64_t)nl * TRACE_STRIDE);
  if (out && n) YL_CUDA_TRY(cudaMemcpy(out, s->trace, n * 8, cudaMemcpyDeviceToHost));
  if (n_launches) *n_launches = nl;
  return YL_OK;
}

int ensure_decode_graph(Session* s, bool logits) {
  // tensor-parallel: a second graph gathers the full logits for callers that
  // read them (one model rank holds only its vocabulary slice)
  if (logits && s->m->tp_size > 1) {
    if (s->graph_lg) return YL_OK;
    cudaGraphExec_t keep = s->graph;
    s->graph = nullptr;
    int rc = capture_decode_graph(s, true);
    s->graph_lg = s->graph;
    s->graph = keep;
    return rc;
  }
  return capture_decode_graph(s, false);
}

int capture_decode_graph(Session* s, bool gather) {
  if (s->graph) return YL_OK;
  YL_CUDA_TRY(cudaSetDevice(s->device));
  int rc = ensure_cap(s, 8);
  if (rc) return rc;
  cudaGraph_t g = nullptr;
  YL_CUDA_TRY(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  uint32_t nl = 0;
  rc = enqueue_forward(s, 1, 0, true, tunables().pdl, &nl, gather);
  cudaError_t e = cudaStreamEndCapture(s->stream, &g);
  if (rc) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  // the kernel nodes the capture recorded (the launch count of one step)
  size_t nn = 0;
  e = cudaGraphGetNodes(g, nullptr, &nn);
  std::vector<cudaGraphNode_t> nodes(nn);
  if (e == cudaSuccess && nn) e = cudaGraphGetNodes(g, nodes.data(), &nn);
  uint32_t kernels = 0;
  for (size_t i = 0; e == cudaSuccess && i < nn; ++i) {
    cudaGraphNodeType t;
    e = cudaGraphNodeGetType(nodes[i], &t);
    if (e == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
  }
  if (e != cudaSuccess) { cudaGraphDestroy(g); return fail(YL_ERR_CUDA, std::string("graph nodes: ") + cudaGetErrorString(e)); }
  e = cudaGraphInstantiate(&s->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) { s->graph = nullptr; return fail(YL_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e)); }
  if (kernels != nl) return fail(YL_ERR_CUDA, "decode graph holds " + std::to_string(kernels) + " kernels, " +
                                                  std::to_string(nl) + " were enqueued");
  if (gather) s->graph_launches_lg = kernels;
  else s->graph_launches = kernels;
  return YL_OK;
}

}  // namespace yl
