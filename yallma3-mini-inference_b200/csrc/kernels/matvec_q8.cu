// Q8_0 weights: int8 activations (dp4a), f32 activations, and f32 activations
// as three int8 limbs (the lm_head).
#include "matvec.cuh"

namespace yl {
namespace k {
cudaError_t matvec_q8(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc) {
  if (fmt == FMT_Q8) return sf16 ? mv_launch<FMT_Q8, true>(a, epi, lc) : mv_launch<FMT_Q8, false>(a, epi, lc);
  if (fmt == FMT_Q8X) return sf16 ? mv_launch<FMT_Q8X, true>(a, epi, lc) : mv_launch<FMT_Q8X, false>(a, epi, lc);
  return sf16 ? mv_launch<FMT_Q8F, true>(a, epi, lc) : mv_launch<FMT_Q8F, false>(a, epi, lc);
}
}  // namespace k
}  // namespace yl
