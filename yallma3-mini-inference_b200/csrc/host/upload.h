// Host-side pieces shared by the model-file loaders (GGUF, safetensors,
// lm.rs): file mapping, the repacking upload into the split HBM layout, the
// RoPE table and the checks of what the device path supports.
#pragma once
#include <sys/mman.h>

#include <functional>

#include "model.h"

namespace yl {

// Read-only private mapping of a whole file.
struct Mapped {
  void* p = MAP_FAILED;
  size_t size = 0;
  ~Mapped() { if (p != MAP_FAILED) munmap(p, size); }
  const uint8_t* data() const { return static_cast<const uint8_t*>(p); }
};
int map_file(const char* path, Mapped* out);

// Runs fn(begin, end) over [0, n) split across up to 32 host threads.
void parallel_for(uint64_t n, const std::function<void(uint64_t, uint64_t)>& fn);

// Fills one logical row: its packed quants (row_bytes) and, for quantized
// formats, its scales (cols/32 f16 or f32 values, as the weight's sf16 says).
using RowFill = std::function<void(uint32_t row, uint8_t* q, uint8_t* s)>;

// Uploads weight matrices into the device layout: quants [rows][row_bytes]
// and scales [rows][scale_row_bytes] (rows 16-byte aligned), through a
// pinned staging buffer filled by host threads.
struct Uploader {
  Model* m;
  uint8_t* stage = nullptr;
  size_t stage_bytes = 0;
  ~Uploader();
  int alloc(size_t bytes, void** out);
  int ensure_stage(size_t bytes);
  // fmt: YL_Q8_0 / YL_Q4_0 (blocks of 32, scales f16 when sf16 else f32) or YL_F16
  int rows(int fmt, bool sf16, uint32_t rows, uint32_t cols, const RowFill& fill, DevWeight* w);
  // rows of GGUF blocks (ggml_type 8 Q8_0, 2 Q4_0, 1 F16); src_row(r) = file address of row r
  int gguf(uint32_t ggml_type, uint32_t rows, uint32_t cols, const std::function<const uint8_t*(uint32_t)>& src_row,
           DevWeight* w);
  int f32(const float* src, uint64_t n, float** out);
};

// Device-path limits on a parsed shape (head sizes, GQA grouping, multiples
// of 32, the tensor-parallel split): YL_ERR_UNSUPPORTED with the reason.
int check_device_shape(const yl_shape& s, int tp_size);

// Fills the model's per-rank counts (heads, KV heads, ffn rows, vocabulary
// rows) for rank tp_rank of tp_size, after check_device_shape.
void set_rank_split(Model* m, int tp_rank, int tp_size);

// RoPE (cos, sin) table [ctx_len][head_size/2] uploaded to the device and
// the attention scale; llama3_* are the llama3 frequency-scaling constants
// and old_ctx its original context length.
int finish_model(Model* m, Uploader& up, float llama3_factor, float llama3_low, float llama3_high, float old_ctx);

}  // namespace yl
