// Instantiations and launch of the warp-level tensor-core decode GEMV
// (gemv_mma.cuh): tokens per call (1, 2) x warps per CTA x units in flight.
#include <atomic>
#include <cstdio>

#include "gemv_mma.cuh"
#include "kernels.h"

namespace lbc {

namespace {

template <int NTOK, int NW, int JWS, bool HZ>
cudaError_t mma_ensure_smem(int smem) {
  static std::atomic<int> enabled[64];
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return e;
  if (d >= 0 && d < 64 && enabled[d].load(std::memory_order_relaxed) >= smem) return cudaSuccess;
  e = cudaFuncSetAttribute(gemv_mma_kernel<NTOK, NW, JWS, HZ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess && d >= 0 && d < 64) {
    int cur = enabled[d].load();
    while (cur < smem && !enabled[d].compare_exchange_weak(cur, smem)) {
    }
  }
  return e;
}

template <int NTOK, int NW, int JWS, bool HZ>
cudaError_t mma_launch_one(const GemvArgs &a, int ns, int grid, int smem, cudaStream_t st) {
  cudaError_t e = mma_ensure_smem<NTOK, NW, JWS, HZ>(smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3((NW + 1) * 32, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_mma_kernel<NTOK, NW, JWS, HZ>, a, ns);
}

template <int NTOK, int NW, int JWS, bool HZ>
int mma_occ_one(int smem) {
  if (mma_ensure_smem<NTOK, NW, JWS, HZ>(smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, gemv_mma_kernel<NTOK, NW, JWS, HZ>, (NW + 1) * 32,
                                                    (size_t)smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return nb;
}

}  // namespace

// instantiated (tokens, consumer warps, units per warp per stage) combinations
#define LBC_MMA_COMBOS(X) \
  X(1, 4, 2) X(1, 4, 4) X(1, 8, 1) X(1, 8, 2) X(1, 8, 4) X(1, 16, 1) X(1, 16, 2) \
  X(2, 4, 2) X(2, 8, 1) X(2, 8, 2) X(2, 16, 1)

bool mma_combo(int ntok, int nw, int jws) {
#define LBC_MMA_C(T, W, J) \
  if (ntok == T && nw == W && jws == J) return true;
  LBC_MMA_COMBOS(LBC_MMA_C)
#undef LBC_MMA_C
  return false;
}

int mma_smem_bytes(int ntok, int nw, int jws, int ns, int Kp, int N, int grid) {
  return mmv_smem_layout(ntok, nw, jws, ns, Kp / 128, (N + grid - 1) / grid).total;
}

cudaError_t mma_launch(const GemvArgs &a, int ntok, int nw, int jws, int ns, int grid, cudaStream_t st) {
  const int smem = mma_smem_bytes(ntok, nw, jws, ns, a.Kp, a.N, grid);
#define LBC_MMA_L(T, W, J) \
  if (ntok == T && nw == W && jws == J) \
    return a.zeros ? mma_launch_one<T, W, J, true>(a, ns, grid, smem, st) \
                   : mma_launch_one<T, W, J, false>(a, ns, grid, smem, st);
  LBC_MMA_COMBOS(LBC_MMA_L)
#undef LBC_MMA_L
  return cudaErrorInvalidConfiguration;
}

int mma_occupancy(int ntok, int nw, int jws, int smem) {
#define LBC_MMA_O(T, W, J) \
  if (ntok == T && nw == W && jws == J) return mma_occ_one<T, W, J, true>(smem);
  LBC_MMA_COMBOS(LBC_MMA_O)
#undef LBC_MMA_O
  return 0;
}

}  // namespace lbc
