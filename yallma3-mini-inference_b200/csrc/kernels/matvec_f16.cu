// F16 weights with f32 activations (matmul_f32 semantics), and the format
// dispatcher of the matvec family.
#include "matvec.cuh"

namespace yl {
namespace k {
cudaError_t matvec_q8(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc);
cudaError_t matvec_q4(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc);

cudaError_t matvec(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc) {
  if (a.K % 32 || a.kc % 256 || a.kc == 0 || a.ntok == 0 || a.ntok > 8) return cudaErrorInvalidValue;
  switch (fmt) {
    case FMT_Q8:
    case FMT_Q8F: return matvec_q8(a, fmt, sf16, epi, lc);
    case FMT_Q4:
    case FMT_Q4F: return matvec_q4(a, fmt, sf16, epi, lc);
    case FMT_F16: return mv_launch<FMT_F16, true>(a, epi, lc);
  }
  return cudaErrorInvalidValue;
}
}  // namespace k
}  // namespace yl
