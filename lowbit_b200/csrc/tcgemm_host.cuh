// Host side of the tensor-core GEMM: weight tensor map and launch helpers.
#pragma once

#include <cudaTypedefs.h>

#include <cstdio>

#include "tcprefill.cuh"

namespace lbc {

// 2-D tensor map over the packed weights [N rows, Kp/2 bytes], 128 x 128-byte
// boxes, 128-byte swizzle (conflict-free per-row reads in the decoders).
inline cudaError_t make_weight_map(CUtensorMap *map, const uint8_t *qw, int N, int Kp) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)(Kp / 2), (cuuint64_t)N};
  const cuuint64_t strides[1] = {(cuuint64_t)(Kp / 2)};
  const cuuint32_t box[2] = {128, TC_ROWS};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(qw), dims, strides,
                            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// detail appended to launch errors (thread-local)
inline char *tc_launch_note() {
  static thread_local char buf[160] = "";
  return buf;
}

template <typename Kern, typename... Args>
inline cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

template <int FMT, int MT, int NPIECE>
cudaError_t tc_launch_one(const CUtensorMap &map, const TcArgs &a, int chunks, int grid_x, int smem,
                          cudaStream_t st) {
  {
    cudaError_t e = launch_pdl(tc_bblock_kernel<FMT, MT, NPIECE>, dim3(a.nkb, chunks, 1), dim3(256, 1, 1),
                               (size_t)0, st, a.x, a.xq, const_cast<uint8_t *>(a.bglob), a.M, a.Kp, a.nkb,
                               a.b_block_bytes);
    if (e != cudaSuccess) return e;
  }
  auto k = tcgemm_kernel<FMT, MT, NPIECE>;
  static int enabled[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && enabled[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    enabled[dev] = smem;
  }
  cudaError_t e = launch_pdl(k, dim3(grid_x, chunks, 1), dim3(TC_THREADS, 1, 1), (size_t)smem, st, map, a);
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, k) == cudaSuccess)
      snprintf(tc_launch_note(), 160, " [regs=%d maxThreadsPerBlock=%d smem=%d stages=%d]", fa.numRegs,
               fa.maxThreadsPerBlock, smem, a.stages);
  }
  return e;
}

}  // namespace lbc

namespace lbc {

template <int FMT>
cudaError_t tc_prefill_launch(const CUtensorMap &map, const TcArgs &a, int nch, int grid_x, int smem, cudaStream_t st) {
  {
    cudaError_t e = launch_pdl(tc_bblock_kernel<FMT, PF_TOK, 1>, dim3(a.nkb, nch, 1), dim3(256, 1, 1), (size_t)0,
                               st, a.x, a.xq, const_cast<uint8_t *>(a.bglob), a.M, a.Kp, a.nkb, a.b_block_bytes);
    if (e != cudaSuccess) return e;
  }
  auto k = a.y_peers ? tcprefill_kernel<FMT, false, true>
                     : a.ksplit > 1 ? tcprefill_kernel<FMT, true> : tcprefill_kernel<FMT, false>;
  static int enabled[3][64] = {{0}};
  const int sk = a.y_peers ? 2 : a.ksplit > 1 ? 1 : 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && enabled[sk][dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    enabled[sk][dev] = smem;
  }
  cudaError_t e = launch_pdl(k, dim3(grid_x, 1, 1), dim3(PF_THREADS, 1, 1), (size_t)smem, st, map, a);
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, k) == cudaSuccess)
      snprintf(tc_launch_note(), 160, " [prefill regs=%d maxThreadsPerBlock=%d smem=%d stages=%d]", fa.numRegs,
               fa.maxThreadsPerBlock, smem, a.stages);
    return e;
  }
  if (a.ksplit > 1)
    e = launch_pdl(tc_split_reduce_kernel, dim3(a.units, PF_TOK, 1), dim3(TC_ROWS, 1, 1), (size_t)0, st,
                   (const float *)a.partial, FMT == FMT_W4A8 ? a.xs : (const float *)nullptr, a.y, a.M, a.N, nch,
                   a.ksplit);
  return e;
}

}  // namespace lbc
