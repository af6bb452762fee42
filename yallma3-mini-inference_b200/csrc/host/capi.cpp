// extern "C" entry points declared in include/yallma3.h.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "generate.h"
#include "model.h"

struct yl_model {
  yl::Model* m;
};
struct yl_session {
  yl::Session* s;
};
struct yl_batch {
  yl::Batch* b;
};

namespace yl {
namespace {
thread_local std::string g_last_error;
}
void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
}  // namespace yl

using namespace yl;

extern "C" {

const char* yl_last_error(void) { return g_last_error.c_str(); }
const char* yl_version(void) { return "yallma3_b200 0.1 sm_100a"; }

// ------------------------------- qtensors --------------------------------

static uint64_t w_row_bytes(int fmt, uint64_t cols) {
  return fmt == YL_Q8_0 ? cols : fmt == YL_Q4_0 ? cols / 2 : cols * 2;
}

int yl_qtensor_alloc(int fmt, uint64_t len, uint64_t gs, yl_qtensor* out) {
  if (!out || gs == 0) return fail(YL_ERR_ARG, "null output or zero group size");
  if (fmt != YL_Q8_0 && fmt != YL_Q4_0 && fmt != YL_F16) return fail(YL_ERR_ARG, "unknown format");
  if (len > (1ull << 40)) return fail(YL_ERR_ARG, "len too large");  // (len * 4 must not wrap)
  yl_qtensor t{};
  t.fmt = fmt;
  t.scale_type = YL_SCALE_F32;
  t.len = len;
  t.gs = gs;
  t.owned = 1;
  const uint64_t qbytes = fmt == YL_F16 ? len * 4 : len;
  YL_CUDA_TRY(cudaMalloc(&t.quant, std::max<uint64_t>(qbytes, 16)));
  YL_CUDA_TRY(cudaMemset(t.quant, 0, std::max<uint64_t>(qbytes, 16)));
  if (fmt != YL_F16) {
    YL_CUDA_TRY(cudaMalloc(&t.scale, std::max<uint64_t>(len / gs * 4, 16)));
    YL_CUDA_TRY(cudaMemset(t.scale, 0, std::max<uint64_t>(len / gs * 4, 16)));
  }
  *out = t;
  return YL_OK;
}

int yl_qtensor_alloc_weight(int fmt, int scale_type, uint64_t rows, uint64_t cols, uint64_t gs, yl_qtensor* out) {
  if (!out) return fail(YL_ERR_ARG, "null output");
  if (fmt != YL_Q8_0 && fmt != YL_Q4_0 && fmt != YL_F16) return fail(YL_ERR_ARG, "unknown format");
  if (gs != 32) return fail(YL_ERR_UNSUPPORTED, "device weights use group size 32");
  if (rows == 0 || cols == 0 || cols % 32) return fail(YL_ERR_ARG, "cols must be a non-zero multiple of 32");
  if (rows > 0xFFFFFFFFull || cols > 0x3FFFFFFFull) return fail(YL_ERR_ARG, "shape too large");
  yl_qtensor t{};
  t.fmt = fmt;
  t.scale_type = scale_type == YL_SCALE_F16 ? YL_SCALE_F16 : YL_SCALE_F32;
  t.len = rows * cols;
  t.gs = gs;
  t.rows = rows;
  t.cols = cols;
  t.owned = 1;
  const uint64_t rb = w_row_bytes(fmt, cols);
  YL_CUDA_TRY(cudaMalloc(&t.quant, rows * rb));
  YL_CUDA_TRY(cudaMemset(t.quant, 0, rows * rb));
  if (fmt != YL_F16) {
    const uint64_t ssz = t.scale_type == YL_SCALE_F16 ? 2 : 4;
    t.scale_stride = round_up(cols / 32 * ssz, 16) / ssz;
    YL_CUDA_TRY(cudaMalloc(&t.scale, rows * t.scale_stride * ssz));
    YL_CUDA_TRY(cudaMemset(t.scale, 0, rows * t.scale_stride * ssz));
  }
  *out = t;
  return YL_OK;
}

int yl_qtensor_free(yl_qtensor* t) {
  if (!t) return fail(YL_ERR_ARG, "null tensor");
  if (t->owned) {
    if (t->quant) cudaFree(t->quant);
    if (t->scale) cudaFree(t->scale);
  }
  t->quant = t->scale = nullptr;
  return YL_OK;
}

int yl_qtensor_upload(yl_qtensor* t, const int8_t* q, const float* scales, const float* values) {
  if (!t || !t->quant) return fail(YL_ERR_ARG, "null tensor");
  if (t->rows == 0) {  // activation container
    if (t->fmt == YL_F16) {
      if (!values) return fail(YL_ERR_ARG, "F16 activations need values");
      YL_CUDA_TRY(cudaMemcpy(t->quant, values, t->len * 4, cudaMemcpyHostToDevice));
    } else {
      if (!q || !scales) return fail(YL_ERR_ARG, "quantized activations need q and scales");
      YL_CUDA_TRY(cudaMemcpy(t->quant, q, t->len, cudaMemcpyHostToDevice));
      YL_CUDA_TRY(cudaMemcpy(t->scale, scales, t->len / t->gs * 4, cudaMemcpyHostToDevice));
    }
    return YL_OK;
  }
  const uint64_t rows = t->rows, cols = t->cols, nb = cols / 32, rb = w_row_bytes(t->fmt, cols);
  std::vector<uint8_t> hq(rows * rb);
  if (t->fmt == YL_F16) {
    if (!values) return fail(YL_ERR_ARG, "F16 weights need values");
    uint16_t* h = (uint16_t*)hq.data();
    for (uint64_t i = 0; i < rows * cols; ++i) h[i] = f32_to_f16(values[i]);
    YL_CUDA_TRY(cudaMemcpy(t->quant, hq.data(), hq.size(), cudaMemcpyHostToDevice));
    return YL_OK;
  }
  if (!q || !scales) return fail(YL_ERR_ARG, "quantized weights need q and scales");
  for (uint64_t r = 0; r < rows; ++r) {
    const int8_t* src = q + r * cols;
    uint8_t* dst = hq.data() + r * rb;
    if (t->fmt == YL_Q8_0) {
      memcpy(dst, src, cols);
    } else {  // Q4_0: signed values q-8 in [-8, 7] -> GGML nibbles
      for (uint64_t b = 0; b < nb; ++b)
        for (int j = 0; j < 16; ++j) {
          int lo = src[b * 32 + j] + 8, hi = src[b * 32 + 16 + j] + 8;
          if (lo < 0 || lo > 15 || hi < 0 || hi > 15) return fail(YL_ERR_ARG, "Q4_0 value out of [-8, 7]");
          dst[b * 16 + j] = (uint8_t)(lo | (hi << 4));
        }
    }
  }
  YL_CUDA_TRY(cudaMemcpy(t->quant, hq.data(), hq.size(), cudaMemcpyHostToDevice));
  const uint64_t ssz = t->scale_type == YL_SCALE_F16 ? 2 : 4;
  std::vector<uint8_t> hs(rows * t->scale_stride * ssz, 0);
  t->flags &= ~1;
  for (uint64_t r = 0; r < rows; ++r)
    for (uint64_t b = 0; b < nb; ++b) {
      const float sv = scales[r * nb + b];
      if (ssz == 2) {
        const uint16_t h = f32_to_f16(sv);
        ((uint16_t*)hs.data())[r * t->scale_stride + b] = h;
        if ((h & 0x7FFFu) == 0x7C00u) t->flags |= 1;
      } else {
        ((float*)hs.data())[r * t->scale_stride + b] = sv;
      }
    }
  YL_CUDA_TRY(cudaMemcpy(t->scale, hs.data(), hs.size(), cudaMemcpyHostToDevice));
  return YL_OK;
}

int yl_qtensor_download(const yl_qtensor* t, int8_t* q, float* scales, float* values) {
  if (!t || !t->quant) return fail(YL_ERR_ARG, "null tensor");
  if (t->rows == 0) {
    if (t->fmt == YL_F16) {
      if (values) YL_CUDA_TRY(cudaMemcpy(values, t->quant, t->len * 4, cudaMemcpyDeviceToHost));
    } else {
      if (q) YL_CUDA_TRY(cudaMemcpy(q, t->quant, t->len, cudaMemcpyDeviceToHost));
      if (scales) YL_CUDA_TRY(cudaMemcpy(scales, t->scale, t->len / t->gs * 4, cudaMemcpyDeviceToHost));
    }
    return YL_OK;
  }
  const uint64_t rows = t->rows, cols = t->cols, nb = cols / 32, rb = w_row_bytes(t->fmt, cols);
  std::vector<uint8_t> hq(rows * rb);
  YL_CUDA_TRY(cudaMemcpy(hq.data(), t->quant, hq.size(), cudaMemcpyDeviceToHost));
  if (t->fmt == YL_F16) {
    if (values)
      for (uint64_t i = 0; i < rows * cols; ++i) values[i] = f16_to_f32(((uint16_t*)hq.data())[i]);
    return YL_OK;
  }
  if (q)
    for (uint64_t r = 0; r < rows; ++r) {
      const uint8_t* src = hq.data() + r * rb;
      int8_t* dst = q + r * cols;
      if (t->fmt == YL_Q8_0) memcpy(dst, src, cols);
      else
        for (uint64_t b = 0; b < nb; ++b)
          for (int j = 0; j < 16; ++j) {
            dst[b * 32 + j] = (int8_t)((src[b * 16 + j] & 0xF) - 8);
            dst[b * 32 + 16 + j] = (int8_t)((src[b * 16 + j] >> 4) - 8);
          }
    }
  if (scales) {
    const uint64_t ssz = t->scale_type == YL_SCALE_F16 ? 2 : 4;
    std::vector<uint8_t> hs(rows * t->scale_stride * ssz);
    YL_CUDA_TRY(cudaMemcpy(hs.data(), t->scale, hs.size(), cudaMemcpyDeviceToHost));
    for (uint64_t r = 0; r < rows; ++r)
      for (uint64_t b = 0; b < nb; ++b)
        scales[r * nb + b] = ssz == 2 ? f16_to_f32(((uint16_t*)hs.data())[r * t->scale_stride + b])
                                      : ((float*)hs.data())[r * t->scale_stride + b];
  }
  return YL_OK;
}

// ------------------------------- quantize / matmul -----------------------

int yl_quantize_q8_0(const float* x, int8_t* q, float* scale, uint64_t n, uint32_t gs, void* stream) {
  if (gs != 32) return fail(YL_ERR_UNSUPPORTED, "the device quantizer uses group size 32");
  if (n / gs == 0) return YL_OK;
  if (!x || !q || !scale) return fail(YL_ERR_ARG, "null pointer");
  k::LaunchCfg lc;
  lc.stream = (cudaStream_t)stream;
  cudaError_t e = k::quantize_q8(x, q, scale, n / gs, lc);
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("quantize: ") + cudaGetErrorString(e));
  return YL_OK;
}

int yl_quantize(int fmt, yl_qtensor* dst, const float* x, uint64_t n, uint32_t gs, void* stream) {
  if (!dst || !x) return fail(YL_ERR_ARG, "null pointer");
  if (dst->fmt != fmt || dst->rows != 0) return fail(YL_ERR_FORMAT, "quantize: format/variant mismatch");
  if (n > dst->len) return fail(YL_ERR_ARG, "n exceeds the destination length");
  if (fmt == YL_F16) {  // F16Kernel::quantize copies (forward.rs:78-81)
    YL_CUDA_TRY(cudaMemcpyAsync(dst->quant, x, n * 4, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    return YL_OK;
  }
  // Q8_0, and Q4_0 activations quantized as Q8_0 (GGML semantics)
  return yl_quantize_q8_0(x, (int8_t*)dst->quant, (float*)dst->scale, n, gs, stream);
}

// The library's own stream-ordered memory pool per device (yl_matmul's F16
// scratch): it keeps freed blocks (no release threshold), so repeated calls
// reuse them instead of mapping memory every time. Null if it cannot be made.
static cudaMemPool_t scratch_pool(int dev) {
  static std::mutex mu;
  static std::vector<std::pair<int, cudaMemPool_t>> pools;
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& p : pools)
    if (p.first == dev) return p.second;
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = dev;
  cudaMemPool_t pool = nullptr;
  if (cudaMemPoolCreate(&pool, &props) == cudaSuccess) {
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  } else {
    (void)cudaGetLastError();
    pool = nullptr;
  }
  pools.push_back({dev, pool});
  return pool;
}

int yl_matmul(float* out, const yl_qtensor* x, const yl_qtensor* w, uint64_t n, uint64_t o, uint64_t gs,
              uint64_t batch, int accumulate, void* stream) {
  if (!out || !x || !w) return fail(YL_ERR_ARG, "null pointer");
  if (x->fmt != w->fmt) return fail(YL_ERR_FORMAT, "matmul: format/variant mismatch or mixed formats");
  if (w->rows == 0) return fail(YL_ERR_ARG, "w must be a weight tensor (yl_qtensor_alloc_weight)");
  if (x->rows != 0) return fail(YL_ERR_ARG, "x must be an activation tensor");
  if (w->rows != o || w->cols != n) return fail(YL_ERR_ARG, "w shape does not match (o, n)");
  if (gs != 32 || w->gs != 32) return fail(YL_ERR_UNSUPPORTED, "device matmul uses group size 32");
  if (batch == 0 || o == 0) return YL_OK;
  if (n == 0 || batch > 0xFFFFFFFFull) return fail(YL_ERR_ARG, "n must be positive and batch below 2^32");
  if (batch > x->len / n) return fail(YL_ERR_ARG, "x is shorter than batch * n");  // (batch * n could wrap)
  DevWeight dw;
  dw.fmt = w->fmt;
  dw.sf16 = w->scale_type == YL_SCALE_F16;
  dw.rows = (uint32_t)o;
  dw.cols = (uint32_t)n;
  dw.row_bytes = (uint32_t)w_row_bytes(w->fmt, n);
  dw.scale_row_bytes = w->fmt == YL_F16 ? 0 : (uint32_t)(w->scale_stride * (dw.sf16 ? 2 : 4));
  dw.q = (uint8_t*)w->quant;
  dw.s = (uint8_t*)w->scale;
  dw.no_inf_scales = (w->flags & 1) == 0;
  const bool f32act = w->fmt == YL_F16;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t st = (cudaStream_t)stream;
  MvExtra ex;
  // F16 batches for the f16 tensor-core GEMM: its split rows in stream-ordered
  // scratch from the library's pool (without it, the matvec runs)
  const Tunables& tu = tunables();
  if (f32act && tu.gemm && tu.gemm_f16_min && batch >= tu.gemm_f16_min && batch <= 0xFFFFFFFFull) {
    cudaMemPool_t pool = scratch_pool(dev);
    if (!pool || cudaMallocFromPoolAsync(&ex.f16ws, k::gemm_f16_workspace_bytes((uint32_t)batch, (uint32_t)n), pool,
                                         st) != cudaSuccess) {
      (void)cudaGetLastError();
      ex.f16ws = nullptr;
    }
  }
  const int rc = run_matvec_ex(dw, f32act, f32act ? nullptr : (const int8_t*)x->quant,
                               f32act ? nullptr : (const float*)x->scale, f32act ? (const float*)x->quant : nullptr, n,
                               n / 32, (uint32_t)batch, out, o, accumulate ? k::EPI_QUIRK : k::EPI_STORE,
                               (uint32_t)(o / 4 * 4), nullptr, st, false, sms, ex, nullptr);
  if (ex.f16ws) cudaFreeAsync(ex.f16ws, st);
  return rc;
}

}  // extern "C"

namespace yl {
int check_attention_args(const float* output, const float* sq, const float* kc, const float* vc, uint64_t seq_len,
                         uint64_t batch, uint64_t n_heads, uint64_t n_kv_heads, uint64_t head_size,
                         uint32_t start_pos, uint64_t kv_dim) {
  if (!output || !sq || !kc || !vc) return fail(YL_ERR_ARG, "null pointer");
  if (batch == 0) return fail(YL_ERR_ARG, "empty batch");
  if (batch > 0xFFFFFFFFull || seq_len > 0xFFFFFFFFull || n_heads > 0xFFFFull || kv_dim > 0xFFFFFFFFull)
    return fail(YL_ERR_ARG, "batch, seq_len or kv_dim beyond 32 bits, or more than 65535 heads");
  if (head_size != 64 && head_size != 128) return fail(YL_ERR_UNSUPPORTED, "head_size must be 64 or 128");
  if (n_kv_heads == 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > 8)
    return fail(YL_ERR_UNSUPPORTED, "n_heads must be a multiple (at most 8x) of n_kv_heads");
  if (kv_dim < n_kv_heads * head_size) return fail(YL_ERR_ARG, "kv_dim smaller than n_kv_heads * head_size");
  if ((uint64_t)start_pos + batch > seq_len) return fail(YL_ERR_RANGE, "start_pos + batch exceeds seq_len");
  // the reference calls it with seq_len = start_pos + batch (forward.rs:135),
  // which also fixes its 8-lane / tail split of the P.V sums
  if ((uint64_t)start_pos + batch != seq_len) return fail(YL_ERR_ARG, "seq_len must equal start_pos + batch");
  if (((uintptr_t)kc | (uintptr_t)vc | (uintptr_t)sq) % 16 || kv_dim % 4)
    return fail(YL_ERR_ARG, "queries and caches must be 16-byte aligned");
  return YL_OK;
}
}  // namespace yl

extern "C" {

int yl_fused_attention(float* output, const float* sq, const float* key_cache, const float* value_cache,
                       uint64_t seq_len, uint64_t batch, uint64_t n_heads, uint64_t n_kv_heads, uint64_t head_size,
                       uint32_t start_pos, uint64_t kv_dim, float attn_scale, void* stream) {
  int rc = check_attention_args(output, sq, key_cache, value_cache, seq_len, batch, n_heads, n_kv_heads, head_size,
                                start_pos, kv_dim);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  k::AttnArgs a{};
  a.q = sq;
  a.kcache = key_cache;
  a.vcache = value_cache;
  a.ntok = (uint32_t)batch;
  a.n_heads = (uint32_t)n_heads;
  a.n_kv_heads = (uint32_t)n_kv_heads;
  a.head_size = (uint32_t)head_size;
  a.kv_dim = (uint32_t)kv_dim;
  a.pos0 = start_pos;
  a.scale = attn_scale;
  a.n_splits = 1;
  a.out = output;
  void* ws = nullptr;
  YL_CUDA_TRY(cudaMallocAsync(&ws, k::attention_scratch_floats((uint32_t)batch, (uint32_t)n_heads, start_pos) * 4, st));
  a.part = (float*)ws;
  k::LaunchCfg lc;
  lc.stream = st;
  cudaError_t e = k::attention(a, lc);
  if (ws) cudaFreeAsync(ws, st);
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
  return YL_OK;
}

// ------------------------------- model -----------------------------------

int yl_config_set(const char* key, int64_t value) {
  if (!key) return fail(YL_ERR_ARG, "null key");
  return set_tunable(key, value);
}

int yl_load_transformer(const char* path, int sequential, uint32_t max_ctx_len, int fmt_override, yl_model** out) {
  (void)sequential;
  if (!path || !out) return fail(YL_ERR_ARG, "null argument");
  std::string p(path);
  const size_t dot = p.rfind('.'), slash = p.rfind('/');
  const std::string ext = dot == std::string::npos || (slash != std::string::npos && dot < slash) ? "" : p.substr(dot + 1);
  if (fmt_override < -1 || fmt_override > YL_F16) return fail(YL_ERR_ARG, "bad format override");
  Model* m = nullptr;
  int rc;
  if (ext == "gguf") rc = guarded([&] { return model_load_gguf(path, max_ctx_len, fmt_override, 0, 1, &m); });
  else if (ext == "safetensors") rc = guarded([&] { return model_load_st(path, max_ctx_len, fmt_override, &m); });
  else if (ext == "lmrs") rc = guarded([&] { return model_load_lmrs(path, max_ctx_len, fmt_override, &m); });
  else return fail(YL_ERR_ARG, "Unsupported model extension for path: " + p);
  if (rc) return rc;
  *out = new yl_model{m};
  return YL_OK;
}

int yl_load_transformer_tp(const char* path, uint32_t max_ctx_len, int fmt_override, int tp_rank, int tp_size,
                           yl_model** out) {
  if (!path || !out) return fail(YL_ERR_ARG, "null argument");
  std::string p(path);
  if (p.size() < 5 || p.substr(p.size() - 5) != ".gguf") return fail(YL_ERR_ARG, "tensor-parallel load needs a .gguf");
  if (fmt_override < -1 || fmt_override > YL_F16) return fail(YL_ERR_ARG, "bad format override");
  Model* m = nullptr;
  int rc = guarded([&] { return model_load_gguf(path, max_ctx_len, fmt_override, tp_rank, tp_size, &m); });
  if (rc) return rc;
  *out = new yl_model{m};
  return YL_OK;
}

int yl_session_tp_handle(yl_session* sp, void* handle_out) {
  if (!sp || !handle_out) return fail(YL_ERR_ARG, "null argument");
  return session_tp_handle(sp->s, handle_out);
}

int yl_session_tp_connect(yl_session* sp, const void* handles) {
  if (!sp || !handles) return fail(YL_ERR_ARG, "null argument");
  return session_tp_connect(sp->s, handles);
}

int yl_tp_plan(const yl_shape* shape, int tp_rank, int tp_size, yl_tp_split* out) {
  if (!shape || !out) return fail(YL_ERR_ARG, "null argument");
  if (tp_size < 1 || tp_size > 8 || tp_rank < 0 || tp_rank >= tp_size) return fail(YL_ERR_ARG, "bad rank/size");
  const uint32_t N = (uint32_t)tp_size, r = (uint32_t)tp_rank, hs = shape->head_size;
  if (shape->n_kv_heads == 0 || shape->n_kv_heads % N || shape->n_heads % shape->n_kv_heads ||
      shape->hidden_dim % (64 * N) || shape->vocab_size % N)
    return fail(YL_ERR_UNSUPPORTED, "tensor parallelism needs KV heads, ffn/64 and vocabulary divisible by the ranks");
  out->q_rows0 = r * (shape->n_heads / N) * hs;
  out->q_rows = (shape->n_heads / N) * hs;
  out->kv_rows0 = r * (shape->n_kv_heads / N) * hs;
  out->kv_rows = (shape->n_kv_heads / N) * hs;
  out->ffn_rows0 = r * (shape->hidden_dim / N);
  out->ffn_rows = shape->hidden_dim / N;
  out->vocab0 = r * (shape->vocab_size / N);
  out->vocab_rows = shape->vocab_size / N;
  return YL_OK;
}

int yl_model_free(yl_model* m) {
  if (!m) return fail(YL_ERR_ARG, "null model");
  delete m->m;
  delete m;
  return YL_OK;
}
const char* yl_model_name(const yl_model* m) { return m ? m->m->name.c_str() : ""; }
uint64_t yl_model_vocab_size(const yl_model* m) { return m ? m->m->shape.vocab_size : 0; }
uint32_t yl_model_max_ctx_len(const yl_model* m) { return m ? m->m->shape.ctx_len : 2048; }
uint32_t yl_model_eos_token(const yl_model* m) { return m ? m->m->eos : 0; }
uint32_t yl_model_bos_token(const yl_model* m) { return m ? m->m->bos : 0; }
int yl_model_shape(const yl_model* m, yl_shape* out) {
  if (!m || !out) return fail(YL_ERR_ARG, "null argument");
  *out = m->m->shape;
  return YL_OK;
}
uint64_t yl_model_device_bytes(const yl_model* m) { return m ? m->m->device_bytes : 0; }

int yl_get_embeddings_batch(const yl_model* m, const uint32_t* tokens, uint64_t n, float* out) {
  if (!m || (!tokens && n) || (!out && n)) return fail(YL_ERR_ARG, "null argument");
  if (n == 0) return YL_OK;
  if (n > 0xFFFFFFFFull) return fail(YL_ERR_ARG, "more than 2^32 - 1 tokens");
  const Model* mm = m->m;
  const uint32_t d = mm->shape.dim;
  YL_CUDA_TRY(cudaSetDevice(mm->device));
  uint32_t* tk = nullptr;
  float* x = nullptr;
  YL_CUDA_TRY(cudaMalloc(&tk, n * 4));
  cudaError_t e = cudaMalloc(&x, n * d * 4ull);
  if (e == cudaSuccess) e = cudaMemcpy(tk, tokens, n * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    k::LaunchCfg lc;
    e = k::embed(mm->emb.fmt == YL_Q8_0 ? k::FMT_Q8 : mm->emb.fmt == YL_Q4_0 ? k::FMT_Q4 : k::FMT_F16, mm->emb.q,
                 mm->emb.s, mm->emb.row_bytes, mm->emb.scale_row_bytes, mm->emb.sf16, d, mm->shape.vocab_size, tk, nullptr,
                 (uint32_t)n, x, lc);
  }
  if (e == cudaSuccess) e = cudaMemcpy(out, x, n * d * 4ull, cudaMemcpyDeviceToHost);
  cudaFree(tk);
  cudaFree(x);
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("get_embeddings: ") + cudaGetErrorString(e));
  return YL_OK;
}
int yl_get_embeddings(const yl_model* m, uint32_t token, float* out) {
  return yl_get_embeddings_batch(m, &token, 1, out);
}

int yl_model_weight(const yl_model* m, uint32_t layer, int which, yl_qtensor* out) {
  if (!m || !out) return fail(YL_ERR_ARG, "null argument");
  const Model* mm = m->m;
  const DevWeight* w = nullptr;
  yl_qtensor t{};
  if (which == 7) {
    w = &mm->lm;
  } else {
    if (layer >= mm->layers.size() || which < 0 || which > 6) return fail(YL_ERR_ARG, "bad layer or weight id");
    const Layer& L = mm->layers[layer];
    switch (which) {
      case 0: case 1: case 2: w = &L.wqkv; break;
      case 3: w = &L.wo; break;
      case 4: case 6: w = &L.w13; break;
      case 5: w = &L.w2; break;
    }
  }
  t.fmt = w->fmt;
  t.scale_type = YL_SCALE_F16;
  t.gs = 32;
  t.cols = w->cols;
  t.scale_stride = w->scale_row_bytes / 2;
  t.owned = 0;
  uint64_t r0 = 0, nr = w->rows, stride = 1;
  const yl_shape& s = mm->shape;
  const uint64_t att = (uint64_t)s.n_heads * s.head_size, kvd = (uint64_t)s.n_kv_heads * s.head_size;
  if (which == 0) nr = att;
  if (which == 1) { r0 = att; nr = kvd; }
  if (which == 2) { r0 = att + kvd; nr = kvd; }
  if (which == 4 || which == 6) {
    // gate/up rows are interleaved in HBM; expose the fused pair matrix
    r0 = 0;
    nr = w->rows;
    stride = 1;
  }
  (void)stride;
  t.rows = nr;
  t.len = nr * w->cols;
  t.quant = w->q + r0 * w->row_bytes;
  t.scale = w->s ? w->s + r0 * w->scale_row_bytes : nullptr;
  *out = t;
  return YL_OK;
}

// ------------------------------- sessions --------------------------------

int yl_create_session(const yl_model* m, yl_session** out) {
  if (!m || !out) return fail(YL_ERR_ARG, "null argument");
  Session* s = nullptr;
  int rc = guarded([&] { return session_create(m->m, &s); });
  if (rc) return rc;
  *out = new yl_session{s};
  return YL_OK;
}
int yl_session_reset(yl_session* s) {
  if (!s) return fail(YL_ERR_ARG, "null session");
  return session_reset(s->s);
}
int yl_session_free(yl_session* s) {
  if (!s) return fail(YL_ERR_ARG, "null session");
  delete s->s;
  delete s;
  return YL_OK;
}
uint32_t yl_session_pos(const yl_session* s) { return s ? s->s->pos : 0; }

int yl_batch_create(const yl_model* m, uint32_t max_sessions, yl_batch** out) {
  if (!m || !out) return fail(YL_ERR_ARG, "null argument");
  Batch* b = nullptr;
  int rc = guarded([&] { return batch_create(m->m, max_sessions, &b); });
  if (rc) return rc;
  *out = new yl_batch{b};
  return YL_OK;
}

int yl_batch_free(yl_batch* b) {
  if (!b) return fail(YL_ERR_ARG, "null batch");
  delete b->b;
  delete b;
  return YL_OK;
}

int yl_batch_forward(yl_batch* bp, yl_session* const* sessions, uint32_t n, const uint32_t* tokens,
                     const uint32_t* positions, float* logits_out, uint32_t* ids_out) {
  if (!bp || !sessions || !tokens || !positions) return fail(YL_ERR_ARG, "null argument");
  Batch* b = bp->b;
  if (n == 0 || n > b->cap) return fail(YL_ERR_ARG, "batch size out of range");
  Session* ss[k::YL_MAX_BATCH];
  for (uint32_t i = 0; i < n; ++i) {
    if (!sessions[i]) return fail(YL_ERR_ARG, "null session");
    ss[i] = sessions[i]->s;
  }
  int rc = forward_batch(b, ss, n, tokens, positions);
  if (rc) return rc;
  Session* w = b->ws;
  const uint64_t V = b->m->shape.vocab_size;
  if (logits_out)
    YL_CUDA_TRY(cudaMemcpyAsync(logits_out, b->logits, (uint64_t)n * V * 4, cudaMemcpyDeviceToHost, w->stream));
  YL_CUDA_TRY(cudaMemcpyAsync(b->tok_h + b->cap, b->ids, (uint64_t)n * 4, cudaMemcpyDeviceToHost, w->stream));
  YL_CUDA_TRY(cudaMemcpyAsync(b->tok_h + 2 * b->cap, w->err, 4, cudaMemcpyDeviceToHost, w->stream));
  YL_CUDA_TRY(cudaStreamSynchronize(w->stream));
  if (const int herr = (int)b->tok_h[2 * b->cap]) {
    cudaMemsetAsync(w->err, 0, sizeof(int), w->stream);
    cudaStreamSynchronize(w->stream);
    return fail(YL_ERR_TIMEOUT, "a bounded device wait expired (error word " + std::to_string(herr) + ")");
  }
  if (ids_out) memcpy(ids_out, b->tok_h + b->cap, (uint64_t)n * 4);
  return YL_OK;
}
int yl_session_set_pos(yl_session* s, uint32_t pos) {
  if (!s) return fail(YL_ERR_ARG, "null session");
  if (pos > s->s->m->shape.ctx_len) return fail(YL_ERR_RANGE, "position beyond ctx_len");
  s->s->pos = pos;
  return YL_OK;
}
int yl_session_kv(const yl_session* s, float** key_cache, float** value_cache, uint64_t* elems) {
  if (!s) return fail(YL_ERR_ARG, "null session");
  if (key_cache) *key_cache = s->s->kcache;
  if (value_cache) *value_cache = s->s->vcache;
  if (elems) *elems = s->s->kv_elems;
  return YL_OK;
}

static int check_err(Session* s) {
  int herr = 0;
  YL_CUDA_TRY(cudaMemcpy(&herr, s->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (herr) {
    cudaMemset(s->err, 0, sizeof(int));
    return fail(YL_ERR_TIMEOUT, "a bounded device wait expired (error word " + std::to_string(herr) + ")");
  }
  return YL_OK;
}

int yl_forward_x(const yl_model* m, yl_session* sp, const uint32_t* tokens, uint64_t n, uint32_t start_pos,
                 float* logits_out, uint32_t* argmax_out) {
  if (!m || !sp || (!tokens && n)) return fail(YL_ERR_ARG, "null argument");
  if (sp->s->m != m->m) return fail(YL_ERR_ARG, "session belongs to another model");
  Session* s = sp->s;
  const yl_shape& sh = m->m->shape;
  if (n == 0) return fail(YL_ERR_ARG, "empty token batch");
  if ((uint64_t)start_pos + n > sh.ctx_len) return fail(YL_ERR_RANGE, "position beyond ctx_len");
  YL_CUDA_TRY(cudaSetDevice(s->device));
  int rc;
  const bool lg_graph = logits_out && m->m->tp_size > 1;
  if (n == 1) {  // batch-1 step through the captured decode graph
    if ((rc = ensure_decode_graph(s, lg_graph))) return rc;
    k::LaunchCfg lc;
    lc.stream = s->stream;
    YL_CUDA_TRY(k::set_step_state(s->state, (int32_t)start_pos, (int32_t)tokens[0], lc));
    YL_CUDA_TRY(cudaGraphLaunch(lg_graph ? s->graph_lg : s->graph, s->stream));
  } else {
    if ((rc = forward(s, tokens, (uint32_t)n, start_pos, logits_out != nullptr))) return rc;
  }
  // logits straight into a page-locked caller buffer, else through the
  // session's page-locked staging buffer; the greedy id and the error word
  // come back with the same synchronization (error word in the last slot of
  // hist_h, which batch-1 calls never use for ids)
  bool direct = false;
  if (logits_out) {
    cudaPointerAttributes pa{};
    direct = cudaPointerGetAttributes(&pa, logits_out) == cudaSuccess && pa.type == cudaMemoryTypeHost;
    cudaGetLastError();
    YL_CUDA_TRY(cudaMemcpyAsync(direct ? logits_out : s->logits_h, s->logits, (uint64_t)sh.vocab_size * 4,
                                cudaMemcpyDeviceToHost, s->stream));
  }
  YL_CUDA_TRY(cudaMemcpyAsync(s->hist_h, s->hist, 4, cudaMemcpyDeviceToHost, s->stream));
  YL_CUDA_TRY(cudaMemcpyAsync(s->hist_h + sh.ctx_len, s->err, 4, cudaMemcpyDeviceToHost, s->stream));
  YL_CUDA_TRY(cudaStreamSynchronize(s->stream));
  if (const int herr = (int)s->hist_h[sh.ctx_len]) {
    cudaMemsetAsync(s->err, 0, sizeof(int), s->stream);
    cudaStreamSynchronize(s->stream);
    return fail(YL_ERR_TIMEOUT, "a bounded device wait expired (error word " + std::to_string(herr) + ")");
  }
  if (logits_out && !direct) memcpy(logits_out, s->logits_h, (uint64_t)sh.vocab_size * 4);
  if (argmax_out) *argmax_out = s->hist_h[0];
  return YL_OK;
}

int yl_decode_greedy(const yl_model* m, yl_session* sp, uint32_t first_token, uint32_t start_pos, uint32_t n_steps,
                     uint32_t* tokens_out, void* stream, int sync) {
  if (!m || !sp) return fail(YL_ERR_ARG, "null argument");
  Session* s = sp->s;
  const yl_shape& sh = m->m->shape;
  if ((uint64_t)start_pos + n_steps > sh.ctx_len) return fail(YL_ERR_RANGE, "position beyond ctx_len");
  if (!sync && tokens_out) return fail(YL_ERR_ARG, "tokens_out needs sync");
  if (n_steps == 0) return YL_OK;
  YL_CUDA_TRY(cudaSetDevice(s->device));
  int rc;
  if ((rc = ensure_decode_graph(s))) return rc;
  cudaStream_t st = stream ? (cudaStream_t)stream : s->stream;
  // the start state is a launch argument, not a host staging buffer, so a
  // second call made before this one's work ran cannot overwrite it
  k::LaunchCfg lc;
  lc.stream = st;
  YL_CUDA_TRY(k::set_step_state(s->state, (int32_t)start_pos, (int32_t)first_token, lc));
  for (uint32_t i = 0; i < n_steps; ++i) YL_CUDA_TRY(cudaGraphLaunch(s->graph, st));
  if (!sync) return YL_OK;
  if (tokens_out)
    YL_CUDA_TRY(cudaMemcpyAsync(s->hist_h, s->hist, (uint64_t)n_steps * 4, cudaMemcpyDeviceToHost, st));
  YL_CUDA_TRY(cudaStreamSynchronize(st));
  if ((rc = check_err(s))) return rc;
  if (tokens_out) memcpy(tokens_out, s->hist_h, (uint64_t)n_steps * 4);
  return YL_OK;
}

int yl_decode_step_launches(const yl_model* m, uint32_t* out) {
  if (!m || !out) return fail(YL_ERR_ARG, "null argument");
  const uint32_t L = m->m->shape.n_layers;
  // embedding; per layer qkv (+ RMSNorm prologue), decode attention (RoPE,
  // cache write, merge, quantize), wo, gate/up (+ RMSNorm, SwiGLU, quantize),
  // down; lm_head (+ RMSNorm, argmax). Tensor parallel: the winners' combine,
  // and two exchange kernels per layer unless the exchange is fused.
  uint32_t n = 1 + 5 * L + 1;
  if (m->m->tp_size > 1) n += 1 + (tunables().tp_fused ? 0 : 2 * L);
  *out = n;
  return YL_OK;
}

int yl_model_attention_decode(const yl_model* m, const float* qkv, float* key_cache, float* value_cache, uint32_t pos,
                              float* out, int8_t* out_q, float* out_s, void* stream) {
  if (!m || !qkv || !key_cache || !value_cache || (!out && !out_q)) return fail(YL_ERR_ARG, "null argument");
  if (out_q && !out_s) return fail(YL_ERR_ARG, "quantized output needs its scales");
  const Model* mm = m->m;
  const yl_shape& sh = mm->shape;
  if (pos >= sh.ctx_len) return fail(YL_ERR_RANGE, "position beyond the model's ctx_len (RoPE table rows)");
  YL_CUDA_TRY(cudaSetDevice(mm->device));
  k::AttnDecodeArgs ad{};
  ad.qkv = qkv;
  ad.cs = mm->rope_cs;
  ad.rope_mode = sh.rope_mode;
  ad.kcache = key_cache;
  ad.vcache = value_cache;
  ad.n_heads = mm->l_heads;
  ad.n_kv_heads = mm->l_kv;
  ad.head_size = sh.head_size;
  ad.kv_dim = mm->l_kv * sh.head_size;
  ad.pos0 = pos;
  ad.scale = mm->attn_scale;
  ad.n_splits = k::attention_decode_splits(mm->l_kv, sh.head_size);
  ad.out = out;
  ad.q8 = out_q;
  ad.s8 = out_s;
  ad.sc_stride = (uint32_t)round_up((uint64_t)pos + 1, 4);
  k::LaunchCfg lc;
  lc.stream = (cudaStream_t)stream;
  void* ws = nullptr;
  YL_CUDA_TRY(cudaMallocAsync(&ws, (uint64_t)mm->l_heads * ad.sc_stride * 4, lc.stream));
  ad.sc = (float*)ws;
  cudaError_t e = k::attention_decode(ad, lc);
  cudaFreeAsync(ws, lc.stream);
  if (e != cudaSuccess) return fail(YL_ERR_CUDA, std::string("decode attention launch: ") + cudaGetErrorString(e));
  return YL_OK;
}

int yl_session_decode_graph_launches(yl_session* sp, int with_logits, uint32_t* out) {
  if (!sp || !out) return fail(YL_ERR_ARG, "null argument");
  Session* s = sp->s;
  const bool lg = with_logits && s->m->tp_size > 1;
  int rc = ensure_decode_graph(s, lg);
  if (rc) return rc;
  *out = lg ? s->graph_launches_lg : s->graph_launches;
  return YL_OK;
}

int yl_profile_decode_step(const yl_model* m, yl_session* sp, uint32_t token, uint32_t pos, float* us_out,
                           uint32_t cap, uint32_t* n_out) {
  if (!m || !sp) return fail(YL_ERR_ARG, "null argument");
  if (sp->s->m != m->m) return fail(YL_ERR_ARG, "session belongs to another model");
  return profile_step(sp->s, token, pos, us_out, cap, n_out);
}

int yl_trace_decode_step(const yl_model* m, yl_session* sp, uint32_t token, uint32_t pos, uint64_t* out,
                         uint64_t cap, uint32_t* n_launches) {
  if (!m || !sp) return fail(YL_ERR_ARG, "null argument");
  if (sp->s->m != m->m) return fail(YL_ERR_ARG, "session belongs to another model");
  return trace_step(sp->s, token, pos, out, cap, n_launches);
}

// ------------------------------- reference FFI ---------------------------

static std::mutex g_ffi_mu;
static yl_model* g_current = nullptr;  // CURRENT_TRANSFORMER (lib.rs:48)
// infer_ffi's conversation state on g_current, and its sampling settings
static yl_session* g_ffi_sess = nullptr;
static yl_sampler* g_ffi_smp = nullptr;
static float g_ffi_temp = 0.7f, g_ffi_topp = 0.9f;  // Sampler::new(vocab, 0.7, 0.9, 42) (main.rs:135)
static uint64_t g_ffi_seed = 42;
static uint32_t g_ffi_max_tokens = 0;  // 0: no limit (the console's default)

static void ffi_drop_state() {
  if (g_ffi_sess) yl_session_free(g_ffi_sess);
  if (g_ffi_smp) yl_sampler_free(g_ffi_smp);
  g_ffi_sess = nullptr;
  g_ffi_smp = nullptr;
}

bool load_transformer_ffi(const char* model_path) {
  if (!model_path) return false;
  yl_model* m = nullptr;
  // lib.rs:143: load_transformer(path, false, u32::MAX, None)
  if (yl_load_transformer(model_path, 0, 0xFFFFFFFFu, -1, &m) != YL_OK) return false;
  std::lock_guard<std::mutex> lk(g_ffi_mu);
  ffi_drop_state();
  if (g_current) yl_model_free(g_current);
  g_current = m;
  return true;
}

int yl_infer_config(float temperature, float top_p, uint64_t seed, uint32_t max_tokens) {
  if (!(temperature >= 0.0f)) return fail(YL_ERR_ARG, "temperature must be >= 0");
  std::lock_guard<std::mutex> lk(g_ffi_mu);
  if (temperature != g_ffi_temp || top_p != g_ffi_topp || seed != g_ffi_seed) {
    if (g_ffi_smp) yl_sampler_free(g_ffi_smp);
    g_ffi_smp = nullptr;
  }
  g_ffi_temp = temperature;
  g_ffi_topp = top_p;
  g_ffi_seed = seed;
  g_ffi_max_tokens = max_tokens;
  return YL_OK;
}

int yl_model_tokenizer(const yl_model* m, const yl_tokenizer** out) {
  if (!m || !out) return fail(YL_ERR_ARG, "null argument");
  std::lock_guard<std::mutex> lk(m->m->tok_mu);
  if (!m->m->tok) {
    yl_tokenizer* t = nullptr;
    int rc = yl_tokenizer_load(m->m->path.c_str(), &t);
    if (rc) return rc;
    m->m->tok.reset(t);
  }
  *out = m->m->tok.get();
  return YL_OK;
}

int yl_session_logits(const yl_session* s, float** logits) {
  if (!s || !logits) return fail(YL_ERR_ARG, "null argument");
  if (s->s->m->tp_size > 1) return fail(YL_ERR_UNSUPPORTED, "the logits row of a tensor-parallel session is a shard");
  *logits = s->s->logits;
  return YL_OK;
}

// The prompt as the console takes it: str::trim (Unicode White_Space at both
// ends, main.rs:165,173); a prompt that is not UTF-8 is left to the
// tokenizer's error.
static std::string trim_prompt(const std::string& p) {
  std::vector<uint32_t> cps;
  std::vector<size_t> offs;
  if (!utf8_code_points(p, &cps, &offs)) return p;
  size_t a = 0, b = cps.size();
  while (a < b && is_white_space(cps[a])) ++a;
  while (b > a && is_white_space(cps[b - 1])) --b;
  return p.substr(offs[a], offs[b] - offs[a]);
}

// One conversation turn of the console (main.rs:163-214) on the device.
static int ffi_generate(const char* prompt_in, std::string* reply) {
  if (!g_current) return fail(YL_ERR_ARG, "no model loaded (load_transformer_ffi)");
  if (!prompt_in) return fail(YL_ERR_ARG, "null prompt");
  const std::string prompt = trim_prompt(prompt_in);
  if (prompt.empty()) return fail(YL_ERR_ARG, "empty prompt");  // the console skips such a line
  const Model* mm = g_current->m;
  if (mm->tp_size > 1) return fail(YL_ERR_UNSUPPORTED, "infer_ffi runs single-GPU models");
  const yl_tokenizer* tk = nullptr;
  int rc = yl_model_tokenizer(g_current, &tk);
  if (rc) return rc;
  std::vector<uint32_t> ids;
  if ((rc = tok_chat_prompt(tk->t, "", prompt, &ids))) return rc;
  const uint32_t ctx = mm->shape.ctx_len;
  if (ids.empty() || ids.size() > ctx) return fail(YL_ERR_RANGE, "prompt longer than the context");
  YL_CUDA_TRY(cudaSetDevice(mm->device));
  if (!g_ffi_sess && (rc = yl_create_session(g_current, &g_ffi_sess))) return rc;
  if (!g_ffi_smp && (rc = yl_sampler_create(mm->shape.vocab_size, g_ffi_temp, g_ffi_topp, g_ffi_seed, &g_ffi_smp)))
    return rc;
  if ((rc = yl_session_reset(g_ffi_sess))) return rc;
  Session* s = g_ffi_sess->s;
  // prefill, then sample from the last token's logits (they stay on the device)
  if ((rc = yl_forward_x(g_current, g_ffi_sess, ids.data(), ids.size(), 0, nullptr, nullptr))) return rc;
  uint32_t pos = (uint32_t)ids.size(), next = 0, gen = 0;
  if ((rc = sampler_run(g_ffi_smp, s->logits, s->stream)) || (rc = sampler_wait(g_ffi_smp, &next))) return rc;
  const uint32_t max_gen = g_ffi_max_tokens ? g_ffi_max_tokens : 0xFFFFFFFFu;
  while (next != mm->eos && pos < ctx && gen < max_gen) {
    *reply += tok_decode(tk->t, &next, 1);
    if ((rc = yl_forward_x(g_current, g_ffi_sess, &next, 1, pos, nullptr, nullptr))) return rc;
    ++pos;
    ++gen;
    if ((rc = sampler_run(g_ffi_smp, s->logits, s->stream)) || (rc = sampler_wait(g_ffi_smp, &next))) return rc;
  }
  return YL_OK;
}

const char* infer_ffi(const char* prompt) {
  std::lock_guard<std::mutex> lk(g_ffi_mu);
  std::string reply;
  if (guarded([&] { return ffi_generate(prompt, &reply); }) != YL_OK) return nullptr;
  char* out = (char*)malloc(reply.size() + 1);
  if (!out) {
    fail(YL_ERR_OOM, "reply buffer");
    return nullptr;
  }
  memcpy(out, reply.data(), reply.size());
  out[reply.size()] = '\0';
  return out;
}

void free_string(const char* s) { free((void*)s); }

}  // extern "C"
