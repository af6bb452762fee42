// Q4_0 weights (GGML nibble order, value (q-8)*d): int8 activations (dp4a) and
// f32 activations (lm_head).
#include "matvec.cuh"

namespace yl {
namespace k {
cudaError_t matvec_q4(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc) {
  if (fmt == FMT_Q4) return sf16 ? mv_launch<FMT_Q4, true>(a, epi, lc) : mv_launch<FMT_Q4, false>(a, epi, lc);
  return sf16 ? mv_launch<FMT_Q4F, true>(a, epi, lc) : mv_launch<FMT_Q4F, false>(a, epi, lc);
}
}  // namespace k
}  // namespace yl
