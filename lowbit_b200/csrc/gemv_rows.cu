// gemv_rows_kernel instantiations and launch (see gemv_rows.cuh).
#include <atomic>

#include "gemv_dispatch.cuh"
#include "gemv_rows.cuh"

namespace lbc {

namespace {

// (MT, CH, R) combinations: MT tokens per pass, CH chunks per thread, R rows per block
#define LBC_ROWS_COMBOS(X) X(1, 1, 4) X(1, 2, 4) X(1, 4, 2) X(2, 1, 2) X(2, 2, 2)
// W4A8 only: int8 activations are a quarter of fp32's registers, so 4 or 8
// tokens per pass fit (one chunk per thread)
#define LBC_ROWS_W8_COMBOS(X) X(4, 1, 4) X(8, 1, 2)

template <int FMT, int MT, int CH, int R, int NW, bool GATHER = false>
cudaError_t rows_launch_nw(const GemvArgs &a, dim3 grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NW * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_rows_kernel<FMT, MT, CH, R, NW, GATHER>, a);
}

// the row team is 1..ROWS_MAX_WARPS (8) warps, or up to ROWS_WIDE_WARPS (16)
// with one chunk per thread and one or two tokens
template <int FMT, int MT, int CH, int R, bool GATHER = false>
cudaError_t rows_launch_one(const GemvArgs &a, dim3 grid, int threads, cudaStream_t st) {
  if constexpr (CH == 1 && MT <= 2) {
    switch (threads / 32) {
      case 9: return rows_launch_nw<FMT, MT, CH, R, 9, GATHER>(a, grid, st);
      case 10: return rows_launch_nw<FMT, MT, CH, R, 10, GATHER>(a, grid, st);
      case 11: return rows_launch_nw<FMT, MT, CH, R, 11, GATHER>(a, grid, st);
      case 12: return rows_launch_nw<FMT, MT, CH, R, 12, GATHER>(a, grid, st);
      case 13: return rows_launch_nw<FMT, MT, CH, R, 13, GATHER>(a, grid, st);
      case 14: return rows_launch_nw<FMT, MT, CH, R, 14, GATHER>(a, grid, st);
      case 15: return rows_launch_nw<FMT, MT, CH, R, 15, GATHER>(a, grid, st);
      case 16: return rows_launch_nw<FMT, MT, CH, R, 16, GATHER>(a, grid, st);
      default: break;
    }
  }
  switch (threads / 32) {
    case 1: return rows_launch_nw<FMT, MT, CH, R, 1, GATHER>(a, grid, st);
    case 2: return rows_launch_nw<FMT, MT, CH, R, 2, GATHER>(a, grid, st);
    case 3: return rows_launch_nw<FMT, MT, CH, R, 3, GATHER>(a, grid, st);
    case 4: return rows_launch_nw<FMT, MT, CH, R, 4, GATHER>(a, grid, st);
    case 5: return rows_launch_nw<FMT, MT, CH, R, 5, GATHER>(a, grid, st);
    case 6: return rows_launch_nw<FMT, MT, CH, R, 6, GATHER>(a, grid, st);
    case 7: return rows_launch_nw<FMT, MT, CH, R, 7, GATHER>(a, grid, st);
    case 8: return rows_launch_nw<FMT, MT, CH, R, 8, GATHER>(a, grid, st);
    default: return cudaErrorInvalidConfiguration;
  }
}

template <int FMT, int MT, int CH, int R, int NW, bool GATHER = false>
int rows_occ_nw() {
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, gemv_rows_kernel<FMT, MT, CH, R, NW, GATHER>, NW * 32, 0) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return nb;
}

template <int FMT, int MT, int CH, int R, bool GATHER = false>
int rows_occ_one(int threads) {
  if constexpr (CH == 1 && MT <= 2) {
    switch (threads / 32) {
      case 9: return rows_occ_nw<FMT, MT, CH, R, 9, GATHER>();
      case 10: return rows_occ_nw<FMT, MT, CH, R, 10, GATHER>();
      case 11: return rows_occ_nw<FMT, MT, CH, R, 11, GATHER>();
      case 12: return rows_occ_nw<FMT, MT, CH, R, 12, GATHER>();
      case 13: return rows_occ_nw<FMT, MT, CH, R, 13, GATHER>();
      case 14: return rows_occ_nw<FMT, MT, CH, R, 14, GATHER>();
      case 15: return rows_occ_nw<FMT, MT, CH, R, 15, GATHER>();
      case 16: return rows_occ_nw<FMT, MT, CH, R, 16, GATHER>();
      default: break;
    }
  }
  switch (threads / 32) {
    case 1: return rows_occ_nw<FMT, MT, CH, R, 1, GATHER>();
    case 2: return rows_occ_nw<FMT, MT, CH, R, 2, GATHER>();
    case 3: return rows_occ_nw<FMT, MT, CH, R, 3, GATHER>();
    case 4: return rows_occ_nw<FMT, MT, CH, R, 4, GATHER>();
    case 5: return rows_occ_nw<FMT, MT, CH, R, 5, GATHER>();
    case 6: return rows_occ_nw<FMT, MT, CH, R, 6, GATHER>();
    case 7: return rows_occ_nw<FMT, MT, CH, R, 7, GATHER>();
    case 8: return rows_occ_nw<FMT, MT, CH, R, 8, GATHER>();
    default: return 0;
  }
}

template <int FMT>
cudaError_t rows_launch_fmt(const GemvArgs &a, int mt, int ch, int r, dim3 grid, int threads, cudaStream_t st) {
#define LBC_ROWS_L(MT, CH, R) \
  if (mt == MT && ch == CH && r == R) return rows_launch_one<FMT, MT, CH, R>(a, grid, threads, st);
  LBC_ROWS_COMBOS(LBC_ROWS_L)
  if constexpr (FMT == FMT_W4A8) {
    LBC_ROWS_W8_COMBOS(LBC_ROWS_L)
  }
#undef LBC_ROWS_L
  return cudaErrorInvalidConfiguration;
}

// fused all-gather variant (W4A16, one or two tokens)
cudaError_t rows_gather_launch_w4a16(const GemvArgs &a, int mt, int ch, int r, dim3 grid, int threads,
                                     cudaStream_t st) {
  if (mt == 1 && ch == 1 && r == 4) return rows_launch_one<FMT_W4A16, 1, 1, 4, true>(a, grid, threads, st);
  if (mt == 1 && ch == 2 && r == 4) return rows_launch_one<FMT_W4A16, 1, 2, 4, true>(a, grid, threads, st);
  if (mt == 2 && ch == 1 && r == 2) return rows_launch_one<FMT_W4A16, 2, 1, 2, true>(a, grid, threads, st);
  return cudaErrorInvalidConfiguration;
}

int rows_gather_occ_w4a16(int mt, int ch, int r, int threads) {
  if (mt == 1 && ch == 1 && r == 4) return rows_occ_one<FMT_W4A16, 1, 1, 4, true>(threads);
  if (mt == 1 && ch == 2 && r == 4) return rows_occ_one<FMT_W4A16, 1, 2, 4, true>(threads);
  if (mt == 2 && ch == 1 && r == 2) return rows_occ_one<FMT_W4A16, 2, 1, 2, true>(threads);
  return 0;
}

template <int FMT>
int rows_occ_fmt(int mt, int ch, int r, int threads) {
#define LBC_ROWS_O(MT, CH, R) \
  if (mt == MT && ch == CH && r == R) return rows_occ_one<FMT, MT, CH, R>(threads);
  LBC_ROWS_COMBOS(LBC_ROWS_O)
  if constexpr (FMT == FMT_W4A8) {
    LBC_ROWS_W8_COMBOS(LBC_ROWS_O)
  }
#undef LBC_ROWS_O
  return 0;
}

}  // namespace

cudaError_t rows_gather_launch(const GemvArgs &a, int mt, int ch, int r, dim3 grid, int threads, cudaStream_t st) {
  return rows_gather_launch_w4a16(a, mt, ch, r, grid, threads, st);
}

int rows_gather_occupancy(int mt, int ch, int r, int threads) {
  return rows_gather_occ_w4a16(mt, ch, r, threads);
}

bool rows_combo(int mt, int ch, int r) {
#define LBC_ROWS_C(MT, CH, R) \
  if (mt == MT && ch == CH && r == R) return true;
  LBC_ROWS_COMBOS(LBC_ROWS_C)
  LBC_ROWS_W8_COMBOS(LBC_ROWS_C)
#undef LBC_ROWS_C
  return false;
}

cudaError_t rows_launch(int fmt, const GemvArgs &a, int mt, int ch, int r, dim3 grid, int threads,
                        cudaStream_t st) {
  switch (fmt) {
    case FMT_W4A16: return rows_launch_fmt<FMT_W4A16>(a, mt, ch, r, grid, threads, st);
    case FMT_MXFP4: return rows_launch_fmt<FMT_MXFP4>(a, mt, ch, r, grid, threads, st);
    default: return rows_launch_fmt<FMT_W4A8>(a, mt, ch, r, grid, threads, st);
  }
}

int rows_occupancy(int fmt, int mt, int ch, int r, int threads) {
  switch (fmt) {
    case FMT_W4A16: return rows_occ_fmt<FMT_W4A16>(mt, ch, r, threads);
    case FMT_MXFP4: return rows_occ_fmt<FMT_MXFP4>(mt, ch, r, threads);
    default: return rows_occ_fmt<FMT_W4A8>(mt, ch, r, threads);
  }
}

}  // namespace lbc
