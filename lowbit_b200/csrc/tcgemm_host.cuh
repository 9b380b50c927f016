// Host side of the tensor-core GEMM: activation-block preparation kernel,
// weight tensor map, launch. Included by the per-format instantiation units.
#pragma once

#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "tcgemm.cuh"

namespace lbc {

// Element of a 128-element group that MMA column-pair position kk (0..127)
// contracts, for each format's decoder column order (see tcgemm.cuh).
__host__ __device__ inline int tc_perm(int fmt, int kk) {
  if (fmt == FMT_W4A8) {
    const int col = kk >> 2, b = kk & 3;
    return 64 * (col & 1) + 16 * (col >> 3) + 4 * ((col >> 1) & 3) + b;
  }
  const int col = kk >> 1, e = kk & 1;
  if (fmt == FMT_MXFP4)
    return 32 * (col >> 4) + 16 * e + 4 * ((col >> 2) & 3) + 2 * ((col >> 1) & 1) + (col & 1);
  const int p = col & 3;
  return 64 * (p & 1) + 16 * (col >> 4) + 4 * ((col >> 2) & 3) + (p >> 1) + 2 * e;
}

// Activation blocks for the tensor-core GEMM, one CTA per (K block, token
// chunk), one thread per contraction position; also zeroes Y (the GEMM
// accumulates into it). fp formats: each x splits exactly into three bf16
// pieces b1 + b2 + b3 (rows p*mt + t of the block); W4A8: the int8 codes.
template <int FMT>
__global__ void __launch_bounds__(256) tc_prep_kernel(const float *__restrict__ x,
                                                      const int8_t *__restrict__ xq, int M, int Kp,
                                                      int nkb, int mt, int nmma, int npiece,
                                                      uint8_t *__restrict__ bglob, int bbytes,
                                                      float *__restrict__ y, int N) {
  // the previous kernel may still read this scratch or accumulate into y
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int kb = blockIdx.x, chunk = blockIdx.y, kk = threadIdx.x;
  uint8_t *blk = bglob + ((size_t)chunk * nkb + kb) * bbytes;
  const int k = kb * 256 + (kk >> 7) * 128 + tc_perm(FMT, kk & 127);
  if (FMT == FMT_W4A8) {
    for (int n = 0; n < nmma; ++n) {
      const int m = chunk * mt + n;
      const int8_t v = (n < mt && m < M && k < Kp) ? xq[(size_t)m * Kp + k] : (int8_t)0;
      blk[(n >> 3) * 2048 + (kk >> 4) * 128 + (n & 7) * 16 + (kk & 15)] = (uint8_t)v;
    }
  } else {
    for (int t = 0; t < mt; ++t) {
      const int m = chunk * mt + t;
      const float v = (m < M && k < Kp) ? x[(size_t)m * Kp + k] : 0.f;
      const __nv_bfloat16 b1 = __float2bfloat16_rn(v);
      const float r1 = v - __bfloat162float(b1);
      const __nv_bfloat16 b2 = __float2bfloat16_rn(r1);
      const float r2 = r1 - __bfloat162float(b2);
      const __nv_bfloat16 b3 = __float2bfloat16_rn(r2);
      const __nv_bfloat16 pc[3] = {b1, b2, b3};
      for (int p = 0; p < npiece; ++p) {
        const int n = p * mt + t;
        *reinterpret_cast<__nv_bfloat16 *>(blk + (n >> 3) * 4096 + (kk >> 3) * 128 + (n & 7) * 16 +
                                           (kk & 7) * 2) = pc[p];
      }
    }
    for (int n = npiece * mt; n < nmma; ++n)
      *reinterpret_cast<uint16_t *>(blk + (n >> 3) * 4096 + (kk >> 3) * 128 + (n & 7) * 16 + (kk & 7) * 2) = 0;
  }
  const long long total = (long long)M * N;
  const long long nthr = (long long)gridDim.x * gridDim.y * blockDim.x;
  for (long long i = ((long long)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += nthr)
    y[i] = 0.f;
}

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
  auto k = tcgemm_kernel<FMT, MT, NPIECE>;
  static int enabled[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && enabled[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    enabled[dev] = smem;
  }
  return launch_pdl(k, dim3(grid_x, chunks, 1), dim3(TC_THREADS, 1, 1), (size_t)smem, st, map, a);
}

}  // namespace lbc
