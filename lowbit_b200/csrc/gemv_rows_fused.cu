// gemv_rows_kernel instantiations with a fused activation prologue (W4A16
// decode): RMSNorm of x + residual (the layer's input norm) or silu(gate) * up
// (the MLP's down projection input). Separate translation unit so the builds
// run in parallel with gemv_rows.cu.
#include "gemv_dispatch.cuh"
#include "gemv_rows.cuh"

namespace lbc {
namespace {

#define LBC_FUSED_COMBOS(X) X(1, 1, 4) X(1, 2, 4) X(1, 4, 2) X(2, 1, 2) X(2, 2, 2)

template <int XM, int MT, int CH, int R, int NW>
cudaError_t fused_nw(const GemvArgs &a, dim3 grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NW * 32, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_rows_kernel<FMT_W4A16, MT, CH, R, NW, false, XM>, a);
}

template <int XM, int MT, int CH, int R>
cudaError_t fused_one(const GemvArgs &a, dim3 grid, int threads, cudaStream_t st) {
  if constexpr (CH == 1 && MT <= 2) {
    switch (threads / 32) {
      case 9: return fused_nw<XM, MT, CH, R, 9>(a, grid, st);
      case 10: return fused_nw<XM, MT, CH, R, 10>(a, grid, st);
      case 11: return fused_nw<XM, MT, CH, R, 11>(a, grid, st);
      case 12: return fused_nw<XM, MT, CH, R, 12>(a, grid, st);
      case 13: return fused_nw<XM, MT, CH, R, 13>(a, grid, st);
      case 14: return fused_nw<XM, MT, CH, R, 14>(a, grid, st);
      case 15: return fused_nw<XM, MT, CH, R, 15>(a, grid, st);
      case 16: return fused_nw<XM, MT, CH, R, 16>(a, grid, st);
      default: break;
    }
  }
  switch (threads / 32) {
    case 1: return fused_nw<XM, MT, CH, R, 1>(a, grid, st);
    case 2: return fused_nw<XM, MT, CH, R, 2>(a, grid, st);
    case 3: return fused_nw<XM, MT, CH, R, 3>(a, grid, st);
    case 4: return fused_nw<XM, MT, CH, R, 4>(a, grid, st);
    case 5: return fused_nw<XM, MT, CH, R, 5>(a, grid, st);
    case 6: return fused_nw<XM, MT, CH, R, 6>(a, grid, st);
    case 7: return fused_nw<XM, MT, CH, R, 7>(a, grid, st);
    case 8: return fused_nw<XM, MT, CH, R, 8>(a, grid, st);
    default: return cudaErrorInvalidConfiguration;
  }
}

template <int XM>
cudaError_t fused_xm(const GemvArgs &a, int mt, int ch, int r, dim3 grid, int threads, cudaStream_t st) {
#define LBC_FUSED_L(MT, CH, R) \
  if (mt == MT && ch == CH && r == R) return fused_one<XM, MT, CH, R>(a, grid, threads, st);
  LBC_FUSED_COMBOS(LBC_FUSED_L)
#undef LBC_FUSED_L
  return cudaErrorInvalidConfiguration;
}

}  // namespace

cudaError_t rows_fused_launch(const GemvArgs &a, int xm, int mt, int ch, int r, dim3 grid, int threads,
                              cudaStream_t st) {
  if (xm == XM_RMSNORM) return fused_xm<XM_RMSNORM>(a, mt, ch, r, grid, threads, st);
  if (xm == XM_GLU) return fused_xm<XM_GLU>(a, mt, ch, r, grid, threads, st);
  return cudaErrorInvalidConfiguration;
}

}  // namespace lbc
