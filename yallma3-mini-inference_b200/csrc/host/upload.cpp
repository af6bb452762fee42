// Shared loader pieces: file mapping, the repacking upload, the RoPE table
// (util.rs:589-635 rope, util.rs:653-718 rope_gguf) and the device-path
// shape checks.
#include "upload.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <thread>
#include <vector>

namespace yl {

int map_file(const char* path, Mapped* out) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(YL_ERR_IO, std::string("cannot open ") + path);
  struct stat stt;
  if (fstat(fd, &stt) != 0) { close(fd); return fail(YL_ERR_IO, "fstat failed"); }
  out->size = (size_t)stt.st_size;
  out->p = out->size ? mmap(nullptr, out->size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  close(fd);
  if (out->p == MAP_FAILED) return fail(YL_ERR_IO, std::string("cannot map ") + path);
  madvise(out->p, out->size, MADV_SEQUENTIAL);
  return YL_OK;
}

void parallel_for(uint64_t n, const std::function<void(uint64_t, uint64_t)>& fn) {
  unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  if (n < 4096) nt = 1;
  std::vector<std::thread> th;
  uint64_t per = (n + nt - 1) / nt;
  for (unsigned k = 0; k < nt; ++k) {
    uint64_t a = k * per, b = std::min(n, a + per);
    if (a >= b) break;
    th.emplace_back(fn, a, b);
  }
  for (auto& t : th) t.join();
}

Uploader::~Uploader() {
  if (stage) cudaFreeHost(stage);
}

int Uploader::alloc(size_t bytes, void** out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 256));
  if (e != cudaSuccess) return fail(YL_ERR_OOM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  m->allocs.push_back(p);
  m->device_bytes += bytes;
  *out = p;
  return YL_OK;
}

int Uploader::ensure_stage(size_t bytes) {
  if (bytes <= stage_bytes) return YL_OK;
  if (stage) cudaFreeHost(stage);
  stage = nullptr;
  YL_CUDA_TRY(cudaMallocHost(&stage, bytes));
  stage_bytes = bytes;
  return YL_OK;
}

int Uploader::rows(int fmt, bool sf16, uint32_t nrows, uint32_t cols, const RowFill& fill, DevWeight* w) {
  if (cols % 32) return fail(YL_ERR_FORMAT, "row length must be a multiple of 32");
  w->rows = nrows;
  w->cols = cols;
  w->fmt = fmt;
  w->sf16 = sf16;
  const uint32_t nb = cols / 32;
  if (fmt == YL_Q8_0) w->row_bytes = cols;
  else if (fmt == YL_Q4_0) w->row_bytes = cols / 2;
  else if (fmt == YL_F16) w->row_bytes = cols * 2;
  else return fail(YL_ERR_FORMAT, "unsupported weight format " + std::to_string(fmt));
  w->scale_row_bytes = fmt == YL_F16 ? 0 : (uint32_t)round_up((uint64_t)nb * (sf16 ? 2 : 4), 16);
  void* q;
  int rc = alloc((size_t)nrows * w->row_bytes, &q);
  if (rc) return rc;
  w->q = (uint8_t*)q;
  w->s = nullptr;
  if (w->scale_row_bytes) {
    void* s;
    if ((rc = alloc((size_t)nrows * w->scale_row_bytes, &s))) return rc;
    w->s = (uint8_t*)s;
  }
  std::atomic<bool> inf_scale{false};
  const size_t per_row = (size_t)w->row_bytes + w->scale_row_bytes;
  const uint32_t chunk_rows = (uint32_t)std::max<size_t>(1, (64u << 20) / per_row);
  if ((rc = ensure_stage((size_t)std::min(chunk_rows, std::max(nrows, 1u)) * per_row))) return rc;
  for (uint32_t r0 = 0; r0 < nrows; r0 += chunk_rows) {
    const uint32_t nr = std::min(chunk_rows, nrows - r0);
    uint8_t* sq = stage;
    uint8_t* ss = stage + (size_t)nr * w->row_bytes;
    parallel_for(nr, [&](uint64_t a, uint64_t b) {
      for (uint64_t r = a; r < b; ++r) {
        uint8_t* ds = w->scale_row_bytes ? ss + r * w->scale_row_bytes : nullptr;
        if (ds) memset(ds, 0, w->scale_row_bytes);  // the padding past cols/32 scales
        fill(r0 + (uint32_t)r, sq + r * w->row_bytes, ds);
        if (ds && sf16)
          for (uint32_t b = 0; b < nb; ++b) {
            uint16_t h;
            memcpy(&h, ds + 2 * b, 2);
            if ((h & 0x7FFFu) == 0x7C00u) inf_scale = true;
          }
      }
    });
    YL_CUDA_TRY(cudaMemcpy(w->q + (size_t)r0 * w->row_bytes, sq, (size_t)nr * w->row_bytes, cudaMemcpyHostToDevice));
    if (w->scale_row_bytes)
      YL_CUDA_TRY(cudaMemcpy(w->s + (size_t)r0 * w->scale_row_bytes, ss, (size_t)nr * w->scale_row_bytes,
                             cudaMemcpyHostToDevice));
  }
  w->no_inf_scales = !inf_scale;
  return YL_OK;
}

int Uploader::gguf(uint32_t ggml_type, uint32_t nrows, uint32_t cols,
                   const std::function<const uint8_t*(uint32_t)>& src_row, DevWeight* w) {
  int fmt;
  if (ggml_type == 8) fmt = YL_Q8_0;
  else if (ggml_type == 2) fmt = YL_Q4_0;
  else if (ggml_type == 1) fmt = YL_F16;
  else return fail(YL_ERR_FORMAT, "unsupported tensor type " + std::to_string(ggml_type));
  const uint32_t nb = cols / 32;
  const uint32_t bsz = fmt == YL_Q8_0 ? 34 : 18, qb = fmt == YL_Q8_0 ? 32 : 16;
  return rows(fmt, true, nrows, cols, [&](uint32_t r, uint8_t* dq, uint8_t* ds) {
    const uint8_t* src = src_row(r);
    if (fmt == YL_F16) {
      memcpy(dq, src, (size_t)cols * 2);
      return;
    }
    // a GGUF block is {f16 scale, quants}: quants and scales go to their own rows
    for (uint32_t b = 0; b < nb; ++b) {
      const uint8_t* blk = src + (size_t)b * bsz;
      ds[2 * b] = blk[0];
      ds[2 * b + 1] = blk[1];
      memcpy(dq + (size_t)b * qb, blk + 2, qb);
    }
  }, w);
}

int Uploader::f32(const float* src, uint64_t n, float** out) {
  void* p;
  int rc = alloc(n * 4, &p);
  if (rc) return rc;
  YL_CUDA_TRY(cudaMemcpy(p, src, n * 4, cudaMemcpyHostToDevice));
  *out = (float*)p;
  return YL_OK;
}

int check_device_shape(const yl_shape& s, int tp_size) {
  // bounds far above any real model that keep every size the loaders compute
  // from a file's header (sums of rows x cols over the layers) clear of
  // 64-bit overflow
  if (s.dim > (1u << 20) || s.hidden_dim > (1u << 22) || s.vocab_size > (1u << 23) || s.n_layers > 4096 ||
      s.n_heads > 4096)
    return fail(YL_ERR_UNSUPPORTED, "model shape beyond the supported bounds (dim, ffn, vocabulary, layers, heads)");
  if (s.dim % 32 || s.hidden_dim % 32 || s.head_size % 32 || s.n_kv_heads == 0 || s.n_heads % s.n_kv_heads)
    return fail(YL_ERR_UNSUPPORTED, "device path needs dim, ffn and head_size multiples of 32 and GQA grouping");
  if (s.head_size != 64 && s.head_size != 128) return fail(YL_ERR_UNSUPPORTED, "head_size must be 64 or 128");
  if (s.n_heads / s.n_kv_heads > 8) return fail(YL_ERR_UNSUPPORTED, "more than 8 query heads per KV head");
  if (s.ctx_len == 0) return fail(YL_ERR_ARG, "ctx_len is 0");
  if (s.weight_format != YL_F16 && s.group_size != 32)
    return fail(YL_ERR_UNSUPPORTED, "device quantization uses groups of 32, the file has " + std::to_string(s.group_size));
  // Megatron split: heads (q and KV) and ffn rows by rank, wo/down along K,
  // lm_head by vocabulary rows; activation and weight blocks of 32 never
  // straddle ranks (the ffn slice is a multiple of 64 for the SwiGLU pairs)
  const uint32_t N = (uint32_t)tp_size;
  if (s.n_kv_heads % N || s.hidden_dim % (64 * N) || s.vocab_size % N)
    return fail(YL_ERR_UNSUPPORTED, "tensor parallelism needs KV heads, ffn/64 and vocabulary divisible by the ranks");
  return YL_OK;
}

void set_rank_split(Model* m, int tp_rank, int tp_size) {
  const yl_shape& s = m->shape;
  const uint32_t N = (uint32_t)tp_size;
  m->tp_rank = tp_rank;
  m->tp_size = tp_size;
  m->l_heads = s.n_heads / N;
  m->l_kv = s.n_kv_heads / N;
  m->l_ffn = s.hidden_dim / N;
  m->l_vocab = s.vocab_size / N;
  m->vocab0 = m->l_vocab * (uint32_t)tp_rank;
}

namespace {

// RoPE (cos, sin) table per (position, pair), by the reference formulas:
// util.rs:653-718 (rope_gguf, theta iterated by *= theta_scale) or
// util.rs:589-635 (rope with llama3 frequency scaling).
void rope_table(const yl_shape& s, float llama3_factor, float llama3_low, float llama3_high, float old_ctx,
                std::vector<float2>* out) {
  const uint32_t hs = s.head_size, half = hs / 2;
  out->assign((size_t)s.ctx_len * half, float2{0.f, 0.f});
  if (s.rope_mode == YL_ROPE_GGUF) {
    const float theta_scale = powf(s.rope_theta, -2.0f / (float)hs);
    const float n_ctx_orig = (float)s.rope_original_ctx_len;
    const float beta_fast = 32.0f, beta_slow = 1.0f;
    float corr_start = fmaf(logf(n_ctx_orig / (beta_fast * 2.0f * (float)M_PI)), (float)hs, 0.0f) /
                       (2.0f * logf(s.rope_theta));
    corr_start = fmaxf(floorf(corr_start), 0.0f);
    const float corr_end = fmaf(logf(n_ctx_orig / (beta_slow * 2.0f * (float)M_PI)), (float)hs, 0.0f) /
                           (2.0f * logf(s.rope_theta));
    const float corr_dims_1 = fminf(corr_start, corr_end) + fminf(corr_end, (float)half) - fmaxf(corr_start, 0.0f);
    parallel_for(s.ctx_len, [&](uint64_t a, uint64_t b) {
      for (uint64_t pos = a; pos < b; ++pos) {
        float theta = (float)pos;
        for (uint32_t kp = 0; kp < half; ++kp) {
          const float theta_interp = s.rope_freq_scale * theta / 1.0f;
          float t = theta_interp;
          if (s.rope_ext_factor != 0.0f) {
            const float y = ((float)(kp * 2) * 0.5f - corr_start) / fmaxf(corr_dims_1 - corr_start, 0.001f);
            const float ramp = (1.0f - fminf(1.0f, fmaxf(y, 0.0f))) * s.rope_ext_factor;
            t = theta_interp * (1.0f - ramp) + theta / 1.0f * ramp;
          }
          (*out)[pos * half + kp] = float2{cosf(t) * s.rope_attn_factor, sinf(t) * s.rope_attn_factor};
          theta = theta * theta_scale;
        }
      }
    });
  } else {
    const float low_wl = old_ctx / llama3_low, high_wl = old_ctx / llama3_high;
    std::vector<float> freq(half);
    for (uint32_t j = 0; j < half; ++j) {
      float f = powf(s.rope_theta, -((float)(j * 2)) / (float)hs);
      const float wl = (2.0f * (float)M_PI) / f;
      if (wl > low_wl) {
        f = f / llama3_factor;
      } else if (wl <= low_wl && wl >= high_wl) {
        const float sm = (old_ctx / wl - llama3_low) / (llama3_high - llama3_low);
        f = (1.0f - sm) * f / llama3_factor + sm * f;
      }
      freq[j] = f;
    }
    parallel_for(s.ctx_len, [&](uint64_t a, uint64_t b) {
      for (uint64_t pos = a; pos < b; ++pos)
        for (uint32_t j = 0; j < half; ++j) {
          const float v = (float)pos * freq[j];
          (*out)[pos * half + j] = float2{cosf(v), sinf(v)};
        }
    });
  }
}

}  // namespace

int finish_model(Model* m, Uploader& up, float llama3_factor, float llama3_low, float llama3_high, float old_ctx) {
  std::vector<float2> cs;
  rope_table(m->shape, llama3_factor, llama3_low, llama3_high, old_ctx, &cs);
  void* csd;
  int rc = up.alloc(cs.size() * sizeof(float2), &csd);
  if (rc) return rc;
  YL_CUDA_TRY(cudaMemcpy(csd, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice));
  m->rope_cs = (float2*)csd;
  const yl_shape& s = m->shape;
  m->attn_scale = s.attention_scale != 0.0f ? s.attention_scale : 1.0f / sqrtf((float)s.head_size);
  return YL_OK;
}

}  // namespace yl
