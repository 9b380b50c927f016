// Host-side dispatch of gemv_kernel instantiations: one translation unit per
// weight format (gemv_w4a16.cu, gemv_mxfp4.cu, gemv_w4a8.cu) so they compile
// in parallel.
#pragma once

#include <atomic>

#include "gemv.cuh"

namespace lbc {

// Launches gemv_kernel<FMT, mt, ch, rt>; returns cudaErrorInvalidConfiguration
// when the (mt, ch, rt) combination is not instantiated.
template <int FMT>
cudaError_t gemv_launch(const GemvArgs &a, int mt, int ch, int rt, dim3 grid, int threads,
                        int smem, cudaStream_t st);

// Resident CTAs per SM for an instantiation at this block size and dynamic
// shared memory (0 when not instantiated or not launchable).
template <int FMT>
int gemv_occupancy(int mt, int ch, int rt, int threads, int smem);

namespace detail {
// Largest dynamic shared memory size already enabled for this instantiation on
// each device, so steady-state launches (and CUDA-graph capture) issue no
// attribute calls.
template <int FMT, int MT, int CH, int RT>
cudaError_t ensure_smem(int smem) {
  static std::atomic<int> enabled[64];
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return e;
  if (d >= 0 && d < 64 && enabled[d].load(std::memory_order_relaxed) >= smem) return cudaSuccess;
  e = cudaFuncSetAttribute(gemv_kernel<FMT, MT, CH, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem);
  if (e == cudaSuccess && d >= 0 && d < 64) {
    int cur = enabled[d].load();
    while (cur < smem && !enabled[d].compare_exchange_weak(cur, smem)) {
    }
  }
  return e;
}

template <int FMT, int MT, int CH, int RT>
cudaError_t launch_one(const GemvArgs &a, dim3 grid, int threads, int smem, cudaStream_t st) {
  cudaError_t e = ensure_smem<FMT, MT, CH, RT>(smem);
  if (e != cudaSuccess) return e;
  gemv_kernel<FMT, MT, CH, RT><<<grid, threads, smem, st>>>(a);
  return cudaGetLastError();
}
template <int FMT, int MT, int CH, int RT>
int occ_one(int threads, int smem) {
  auto k = gemv_kernel<FMT, MT, CH, RT>;
  if (ensure_smem<FMT, MT, CH, RT>(smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return nb;
}
}  // namespace detail

// X-macro list of instantiated (MT, CH, RT) combinations per format family.
#define LBC_GEMV_FP_COMBOS(X) \
  X(1, 1, 1) X(1, 1, 4) X(2, 1, 1) X(2, 1, 4) X(4, 1, 1) X(4, 1, 4) \
  X(1, 2, 1) X(1, 2, 4) X(2, 2, 1) X(2, 2, 4) X(1, 4, 1) X(1, 4, 4)
#define LBC_GEMV_I8_COMBOS(X) \
  X(1, 1, 1) X(1, 1, 4) X(2, 1, 1) X(2, 1, 4) X(4, 1, 1) X(4, 1, 4) X(8, 1, 1) X(8, 1, 4) \
  X(1, 2, 1) X(1, 2, 4) X(2, 2, 1) X(2, 2, 4) X(4, 2, 1) X(4, 2, 4) \
  X(1, 4, 1) X(1, 4, 4) X(2, 4, 1) X(2, 4, 4)

}  // namespace lbc
