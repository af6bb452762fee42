// F16 weights with f32 activations (matmul_f32 semantics), and the format
// dispatcher of the matvec family.
#include "matvec.cuh"

namespace yl {
namespace k {
cudaError_t matvec_q8(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc);
cudaError_t matvec_q4(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc);

template <int FMT>
static uint32_t max_ntok_fmt(uint32_t K, uint32_t kc, int rpw) {
  const uint32_t lim = 227u * 1024u;
  const int g = rpw == 2 ? 2 : 1;  // mv_groups of the SwiGLU / other epilogues
  if (mv_layout<FMT, 8>(K, kc, rpw, 2, 4, g).total <= lim) return 8;
  if (mv_layout<FMT, 4>(K, kc, rpw, 2, 4, g).total <= lim) return 4;
  if (mv_layout<FMT, 2>(K, kc, rpw, 2, 4, g).total <= lim) return 2;
  if (mv_layout<FMT, 1>(K, kc, rpw, 2, 4, g).total <= lim) return 1;
  return 0;
}


uint32_t matvec_max_ntok(int fmt, uint32_t K, uint32_t kc, int epi) {
  const int rpw = (epi == EPI_SWIGLU || epi == EPI_SWIGLU_Q8) ? 2 : 1;
  switch (fmt) {
    case FMT_Q8: return max_ntok_fmt<FMT_Q8>(K, kc, rpw);
    case FMT_Q8F: return max_ntok_fmt<FMT_Q8F>(K, kc, rpw);
    case FMT_Q8X: return mv_layout<FMT_Q8X, 1>(K, kc, rpw, 2).total <= 227u * 1024u ? 1 : 0;
    case FMT_Q4: return max_ntok_fmt<FMT_Q4>(K, kc, rpw);
    case FMT_Q4F: return max_ntok_fmt<FMT_Q4F>(K, kc, rpw);
    case FMT_F16: return max_ntok_fmt<FMT_F16>(K, kc, rpw);
  }
  return 0;
}

cudaError_t matvec(const MvArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc) {
  if (a.K % 32 || a.kc % 256 || a.kc == 0 || a.ntok == 0 || a.ntok > 8) return cudaErrorInvalidValue;
  switch (fmt) {
    case FMT_Q8:
    case FMT_Q8F:
    case FMT_Q8X: return matvec_q8(a, fmt, sf16, epi, lc);
    case FMT_Q4:
    case FMT_Q4F: return matvec_q4(a, fmt, sf16, epi, lc);
    case FMT_F16: return mv_launch<FMT_F16, true>(a, epi, lc);
  }
  return cudaErrorInvalidValue;
}
}  // namespace k
}  // namespace yl
