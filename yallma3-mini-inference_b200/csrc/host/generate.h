// Sampler steps shared by the C-ABI (generate.cpp) and infer_ffi (capi.cpp).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "../../../include/yallma3.h"

namespace yl {
// random_f32(seed) of sampler.rs:81-91
float sampler_rand(uint64_t state);
// Enqueues Sampler::sample on logits (device) and the copy of its id.
int sampler_run(yl_sampler* s, float* logits, cudaStream_t st);
// Waits for the enqueued sample; *id = the sampled token.
int sampler_wait(yl_sampler* s, uint32_t* id);
}  // namespace yl
