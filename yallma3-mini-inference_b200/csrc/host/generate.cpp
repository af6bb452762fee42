// C-ABI of the tokenizer (tokenizer.rs) and of the device sampler
// (sampler.rs), the pieces of the reference's generation loop (main.rs:186-214)
// around the forward pass.
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "../kernels/kernels.h"
#include "chat_template.h"
#include "common.h"
#include "generate.h"
#include "tokenizer.h"

using yl::fail;
using yl::guarded;

struct yl_sampler {
  int device = 0;
  uint32_t V = 0;
  float temperature = 0.f, top_p = 0.f;
  uint64_t seed = 0;
  yl::k::SampleArgs a;
  int cur = 0;
  void* block = nullptr;      // one device allocation for every buffer
  uint32_t* out_h = nullptr;  // page-locked id
  cudaStream_t last = nullptr;
  bool pending = false;
};

namespace yl {

// random_f32(seed) of sampler.rs:81-91 (xorshift of the seed, never advanced)
float sampler_rand(uint64_t state) {
  state ^= state >> 12;
  state ^= state << 25;
  state ^= state >> 27;
  const uint32_t r = (uint32_t)((state * 0x2545F4914F6CDD1Dull) >> 32);
  return (float)(r >> 8) / 16777216.0f;
}

int sampler_run(yl_sampler* s, float* logits, cudaStream_t st) {
  s->a.logits = logits;
  k::LaunchCfg lc;
  lc.stream = st;
  cudaError_t e = k::sample(s->a, &s->cur, lc);
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("sampler launch: ") + cudaGetErrorString(e));
  YL_CUDA_TRY(cudaMemcpyAsync(s->out_h, s->a.out, 4, cudaMemcpyDeviceToHost, st));
  YL_CUDA_TRY(cudaMemcpyAsync(s->out_h + 1, s->a.err, 4, cudaMemcpyDeviceToHost, st));
  s->last = st;
  s->pending = true;
  return YL_OK;
}

int sampler_wait(yl_sampler* s, uint32_t* id) {
  if (!s->pending) return fail(YL_ERR_ARG, "no sample has been taken");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  YL_CUDA_TRY(cudaStreamSynchronize(s->last));
  s->pending = false;
  if (s->out_h[1]) {
    cudaMemsetAsync(s->a.err, 0, 4, s->last);
    cudaStreamSynchronize(s->last);
    return fail(YL_ERR_RANGE, "top-p kept no entry (the reference's n0 - 1 underflows)");
  }
  if (id) *id = s->out_h[0];
  return YL_OK;
}

}  // namespace yl

extern "C" {

int yl_sampler_create(uint32_t vocab_size, float temperature, float top_p, uint64_t seed, yl_sampler** out) {
  if (!out || vocab_size < 2) return fail(YL_ERR_ARG, "null output or vocab_size < 2");
  if (!(temperature >= 0.0f)) return fail(YL_ERR_ARG, "temperature must be >= 0");
  auto* s = new yl_sampler();
  cudaGetDevice(&s->device);
  s->V = vocab_size;
  s->temperature = temperature;
  s->top_p = top_p;
  s->seed = seed;
  yl::k::SampleArgs& a = s->a;
  a.V = vocab_size;
  a.ntiles = yl::k::sample_tiles(vocab_size);
  a.temperature = temperature;
  a.top_p = top_p;
  a.topp = (top_p <= 0.0f || top_p >= 1.0f) ? 0 : 1;
  a.cutoff = (1.0f - top_p) / (float)(vocab_size - 1);
  a.rand = yl::sampler_rand(seed);
  a.sort_temp_bytes = yl::k::sample_sort_temp_bytes(vocab_size);
  const uint64_t V = vocab_size, T = a.ntiles;
  uint64_t off = 0;
  auto carve = [&](uint64_t bytes) {
    const uint64_t o = off;
    off = yl::round_up(off + bytes, 256);
    return o;
  };
  const uint64_t o_tv = carve(T * 4), o_tc = carve(T * 4), o_misc = carve(16), o_pre = carve(V * 4),
                 o_out = carve(4), o_err = carve(4), o_p0 = carve(V * 4), o_p1 = carve(V * 4), o_i0 = carve(V * 4),
                 o_i1 = carve(V * 4), o_tmp = carve(a.sort_temp_bytes);
  cudaError_t e = cudaMalloc(&s->block, off);
  if (e == cudaSuccess) e = cudaMemset(s->block, 0, off);  // probability_idx starts as {0.0, 0}
  if (e == cudaSuccess) e = cudaMallocHost((void**)&s->out_h, 8);
  if (e != cudaSuccess) {
    if (s->block) cudaFree(s->block);
    delete s;
    return fail(e == cudaErrorMemoryAllocation ? YL_ERR_OOM : YL_ERR_CUDA,
                std::string("sampler buffers: ") + cudaGetErrorString(e));
  }
  uint8_t* b = (uint8_t*)s->block;
  a.tile_val = (float*)(b + o_tv);
  a.tile_cnt = (uint32_t*)(b + o_tc);
  a.misc = (float*)(b + o_misc);
  a.prefix = (float*)(b + o_pre);
  a.out = (uint32_t*)(b + o_out);
  a.err = (int*)(b + o_err);
  a.sbuf_prob[0] = (float*)(b + o_p0);
  a.sbuf_prob[1] = (float*)(b + o_p1);
  a.sbuf_idx[0] = (uint32_t*)(b + o_i0);
  a.sbuf_idx[1] = (uint32_t*)(b + o_i1);
  a.sort_temp = b + o_tmp;
  *out = s;
  return YL_OK;
}

int yl_sampler_free(yl_sampler* s) {
  if (!s) return YL_OK;
  cudaSetDevice(s->device);
  if (s->pending && s->last) cudaStreamSynchronize(s->last);
  if (s->block) cudaFree(s->block);
  if (s->out_h) cudaFreeHost(s->out_h);
  delete s;
  return YL_OK;
}

int yl_sampler_sample(yl_sampler* s, float* logits, uint32_t* id_out, void* stream) {
  if (!s || !logits) return fail(YL_ERR_ARG, "null argument");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  int rc = yl::sampler_run(s, logits, (cudaStream_t)stream);
  if (rc || !id_out) return rc;
  return yl::sampler_wait(s, id_out);
}

int yl_sampler_result(yl_sampler* s, uint32_t* id_out) {
  if (!s || !id_out) return fail(YL_ERR_ARG, "null argument");
  return yl::sampler_wait(s, id_out);
}

int yl_tokenizer_load(const char* model_path, yl_tokenizer** out) {
  if (!model_path || !out) return fail(YL_ERR_ARG, "null argument");
  std::unique_ptr<yl::Tokenizer> t;
  int rc = guarded([&] { return yl::tokenizer_load(model_path, &t); });
  if (rc) return rc;
  auto* h = new yl_tokenizer();
  h->t = std::move(*t);
  *out = h;
  return YL_OK;
}

int yl_tokenizer_free(yl_tokenizer* t) {
  delete t;
  return YL_OK;
}

int yl_tokenizer_info(const yl_tokenizer* t, uint32_t* vocab_size, uint32_t* bos, uint32_t* eos, int* has_template) {
  if (!t) return fail(YL_ERR_ARG, "null tokenizer");
  if (vocab_size) *vocab_size = (uint32_t)t->t.vocab.size();
  if (bos) *bos = t->t.bos;
  if (eos) *eos = t->t.eos;
  if (has_template) *has_template = t->t.has_template ? 1 : 0;
  return YL_OK;
}

static int copy_ids(const std::vector<uint32_t>& v, uint32_t* ids, uint64_t cap, uint64_t* n_out) {
  if (n_out) *n_out = v.size();
  if (v.size() > cap) return fail(YL_ERR_RANGE, "output holds fewer ids than the result");
  if (ids && !v.empty()) memcpy(ids, v.data(), v.size() * 4);
  return YL_OK;
}

int yl_tokenizer_encode(const yl_tokenizer* t, const char* text, int bos, int eos, uint32_t* ids, uint64_t cap,
                        uint64_t* n_out) {
  if (!t || !text) return fail(YL_ERR_ARG, "null argument");
  std::vector<uint32_t> v;
  int rc = guarded([&] { return yl::tok_encode(t->t, text, bos != 0, eos != 0, &v); });
  if (rc) return rc;
  return copy_ids(v, ids, cap, n_out);
}

int yl_tokenizer_decode(const yl_tokenizer* t, const uint32_t* ids, uint64_t n, char* out, uint64_t cap,
                        uint64_t* n_out) {
  if (!t || (!ids && n)) return fail(YL_ERR_ARG, "null argument");
  std::string s;
  const int rc = guarded([&] {
    s = yl::tok_decode(t->t, ids, (size_t)n);
    return YL_OK;
  });
  if (rc) return rc;
  if (n_out) *n_out = s.size();
  if (s.size() + 1 > cap) return fail(YL_ERR_RANGE, "output buffer too small");
  if (out) {
    memcpy(out, s.data(), s.size());
    out[s.size()] = '\0';
  }
  return YL_OK;
}

int yl_tokenizer_chat_prompt(const yl_tokenizer* t, const char* system, const char* user, uint32_t* ids,
                             uint64_t cap, uint64_t* n_out) {
  if (!t || !user) return fail(YL_ERR_ARG, "null argument");
  std::vector<uint32_t> v;
  int rc = guarded([&] { return yl::tok_chat_prompt(t->t, system ? system : "", user, &v); });
  if (rc) return rc;
  return copy_ids(v, ids, cap, n_out);
}

int yl_tokenizer_encode_wrap_n_header(const yl_tokenizer* t, const char* text, const char* header,
                                      int begin_of_text_wrap, uint32_t* ids, uint64_t cap, uint64_t* n_out) {
  if (!t || !text || !header) return fail(YL_ERR_ARG, "null argument");
  std::vector<uint32_t> v;
  int rc = guarded([&] { return yl::tok_encode_wrap_n_header(t->t, text, header, begin_of_text_wrap != 0, &v); });
  if (rc) return rc;
  return copy_ids(v, ids, cap, n_out);
}

int yl_tokenizer_set_chat_template(yl_tokenizer* t, const char* tmpl) {
  if (!t || !tmpl) return fail(YL_ERR_ARG, "null argument");
  return guarded([&] { return yl::tok_set_chat_template(&t->t, tmpl); });
}

int yl_tokenizer_apply_system_template(const yl_tokenizer* t, const char* system, uint32_t* ids, uint64_t cap,
                                       uint64_t* n_out) {
  if (!t || !system) return fail(YL_ERR_ARG, "null argument");
  std::vector<uint32_t> v;
  int rc = guarded([&] { return yl::tok_apply_system_template(t->t, system, &v); });
  if (rc) return rc;
  return copy_ids(v, ids, cap, n_out);
}

int yl_tokenizer_apply_turn_template(const yl_tokenizer* t, const char* user, int add_empty_assistant, uint32_t* ids,
                                     uint64_t cap, uint64_t* n_out) {
  if (!t || !user) return fail(YL_ERR_ARG, "null argument");
  std::vector<uint32_t> v;
  int rc = guarded([&] { return yl::tok_apply_turn_template(t->t, user, add_empty_assistant != 0, &v); });
  if (rc) return rc;
  return copy_ids(v, ids, cap, n_out);
}

static int gather_messages(const char* const* roles, const char* const* contents, uint64_t n,
                           yl::ChatMessages* out) {
  if (n && (!roles || !contents)) return fail(YL_ERR_ARG, "null message arrays");
  for (uint64_t i = 0; i < n; ++i) {
    if (!roles[i] || !contents[i]) return fail(YL_ERR_ARG, "null message");
    out->push_back({roles[i], contents[i]});
  }
  return YL_OK;
}

int yl_tokenizer_render_chat(const yl_tokenizer* t, const char* const* roles, const char* const* contents,
                             uint64_t n_messages, int add_generation_prompt, uint32_t* ids, uint64_t cap,
                             uint64_t* n_out) {
  if (!t) return fail(YL_ERR_ARG, "null tokenizer");
  yl::ChatMessages msgs;
  int rc = gather_messages(roles, contents, n_messages, &msgs);
  if (rc) return rc;
  std::vector<uint32_t> v;
  if ((rc = guarded([&] { return yl::tok_render_chat(t->t, msgs, add_generation_prompt != 0, &v); }))) return rc;
  return copy_ids(v, ids, cap, n_out);
}

int yl_chat_template_render(const char* tmpl, const char* const* roles, const char* const* contents,
                            uint64_t n_messages, int add_generation_prompt, char* out, uint64_t cap,
                            uint64_t* n_out) {
  if (!tmpl) return fail(YL_ERR_ARG, "null template");
  yl::ChatMessages msgs;
  int rc = gather_messages(roles, contents, n_messages, &msgs);
  if (rc) return rc;
  std::shared_ptr<const yl::ChatTemplate> t;
  if ((rc = yl::chat_template_parse(tmpl, &t))) return rc;
  std::string s;
  if ((rc = yl::chat_template_render(*t, msgs, add_generation_prompt != 0, &s))) return rc;
  if (n_out) *n_out = s.size();
  if (s.size() + 1 > cap) return fail(YL_ERR_RANGE, "output buffer too small");
  if (out) {
    memcpy(out, s.data(), s.size());
    out[s.size()] = '\0';
  }
  return YL_OK;
}

}  // extern "C"
