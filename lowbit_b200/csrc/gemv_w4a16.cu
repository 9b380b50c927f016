// gemv_kernel instantiations for w4a16.
#include "gemv_dispatch.cuh"

namespace lbc {

#define LBC_GEMV_CASE_L(MT, CH, RT) \
  if (mt == MT && ch == CH && rt == RT) return detail::launch_one<FMT_W4A16, MT, CH, RT>(a, grid, threads, smem, st);
#define LBC_GEMV_CASE_R(MT, CH, RT) \
  if (mt == MT && ch == CH && rt == RT) return detail::occ_one<FMT_W4A16, MT, CH, RT>(threads, smem);

template <>
cudaError_t gemv_launch<FMT_W4A16>(const GemvArgs &a, int mt, int ch, int rt, dim3 grid, int threads,
                                int smem, cudaStream_t st) {
  LBC_GEMV_FP_COMBOS(LBC_GEMV_CASE_L)
  return cudaErrorInvalidConfiguration;
}

template <>
int gemv_occupancy<FMT_W4A16>(int mt, int ch, int rt, int threads, int smem) {
  LBC_GEMV_FP_COMBOS(LBC_GEMV_CASE_R)
  return 0;
}

}  // namespace lbc
