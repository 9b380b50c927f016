// Host-side dispatch of gemv_kernel instantiations: one translation unit per
// weight format (gemv_w4a16.cu, gemv_mxfp4.cu, gemv_w4a8.cu) so they compile
// in parallel.
#pragma once

#include <atomic>
#include <cstdio>

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

// Register-streamed decode kernel (gemv_rows.cuh): whether (mt, ch, r) is
// instantiated, its launch (threads = 32 * warps, grid.y = passes) and its
// resident CTAs per SM at a block size (0 when not instantiated).
bool rows_combo(int mt, int ch, int r);
cudaError_t rows_launch(int fmt, const GemvArgs &a, int mt, int ch, int r, dim3 grid, int threads,
                        cudaStream_t st);
int rows_occupancy(int fmt, int mt, int ch, int r, int threads);
// W4A16 decode with the column-parallel all-gather fused in (a.land_peers ...);
// (mt, ch, r) in {(1,1,4), (1,2,4), (2,1,2)}; its resident CTAs per SM (0 when
// not instantiated): every CTA of the launch must be resident at once
cudaError_t rows_gather_launch(const GemvArgs &a, int mt, int ch, int r, dim3 grid, int threads, cudaStream_t st);
int rows_gather_occupancy(int mt, int ch, int r, int threads);
// W4A8 with 1-64 tokens on mma.sync.m16n8k32 s8 (gemv_i8mma.cu): nb n-blocks
// of 8 tokens per pass (grid.y passes), nw warps per CTA (nb, nw in {1, 2} x
// {4, 8}); its dynamic shared memory and resident CTAs per SM
cudaError_t i8mma_launch(const GemvArgs &a, int nb, int nw, dim3 grid, cudaStream_t st);
int i8mma_smem(int nb, int nw, int Kp);
int i8mma_occupancy(int nb, int nw, int smem);
// W4A16 decode with a fused activation prologue xm (XM_RMSNORM: a.xres, a.xout,
// a.lnw, a.eps; XM_GLU: x rows of 2 * Kp), same combinations as rows_launch
cudaError_t rows_fused_launch(const GemvArgs &a, int xm, int mt, int ch, int r, dim3 grid, int threads,
                              cudaStream_t st);

// Warp-level tensor-core decode kernel (gemv_mma.cuh), W4A16 with one or two
// tokens: whether (tokens, consumer warps, units per warp per stage) is
// instantiated, its dynamic shared memory with `ns` ring stages for a grid of
// `grid` CTAs, its launch and its resident CTAs per SM
bool mma_combo(int ntok, int nw, int jws);
int mma_smem_bytes(int ntok, int nw, int jws, int ns, int Kp, int N, int grid);
cudaError_t mma_launch(const GemvArgs &a, int ntok, int nw, int jws, int ns, int grid, cudaStream_t st);
int mma_occupancy(int ntok, int nw, int jws, int smem);

// thread-local note describing the last zero-occupancy configuration
inline char *occ_note() {
  static thread_local char buf[160] = "";
  return buf;
}

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

// Launch with programmatic stream serialization: the kernel may start (and
// stream its static weights) while the previous kernel in the stream drains;
// it waits for that kernel with griddepcontrol.wait before reading X.
template <int FMT, int MT, int CH, int RT>
cudaError_t launch_one(const GemvArgs &a, dim3 grid, int threads, int smem, cudaStream_t st) {
  cudaError_t e = ensure_smem<FMT, MT, CH, RT>(smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, MT, CH, RT>, a);
}
// Resident CTAs per SM, or -(cudaError_t) when a query failed.
template <int FMT, int MT, int CH, int RT>
int occ_one(int threads, int smem) {
  auto k = gemv_kernel<FMT, MT, CH, RT>;
  cudaError_t e = ensure_smem<FMT, MT, CH, RT>(smem);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return -(int)e;
  }
  int nb = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, threads, (size_t)smem);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return -(int)e;
  }
  if (nb == 0) {  // record why, for the caller's error message
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, k) == cudaSuccess)
      snprintf(occ_note(), 160, "regs=%d maxThreadsPerBlock=%d staticSmem=%zu maxDynSmem=%d",
               fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes, fa.maxDynamicSharedSizeBytes);
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
