// Self-test of the tcgen05 building blocks the tensor-core kernels rely on:
// TMEM allocation, tcgen05.st of an A operand (M=128), a K-major B operand in
// shared memory described by a no-swizzle descriptor, two accumulating MMAs,
// commit to an mbarrier, tcgen05.ld of the accumulator, deallocation.
// One CTA of 128 threads computes D[128,16] = A[128,K] . B[16,K]^T for small
// integer-valued A and B (exact in every format), so the host can check D
// exactly. kind 0: bf16 x bf16 -> f32 (K = 32), kind 1: s8 x s8 -> s32 (K = 64).
#include <cuda_bf16.h>

#include "../../include/lowbit_b200.h"
#include "kernels.h"
#include "tc.cuh"

namespace lbc {

__host__ __device__ inline int selftest_a(int m, int k) { return ((m * 3 + k * 5) % 11) - 5; }
__host__ __device__ inline int selftest_b(int n, int k) { return ((n * 5 + k * 7) % 13) - 6; }

__device__ __forceinline__ uint32_t bf16_bits_of_small_int(int v) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn((float)v));
}

__global__ void __launch_bounds__(128, 1) tc_selftest_kernel(int kind, int32_t *out, int *status) {
  __shared__ __align__(1024) uint8_t bsm[1024];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base_slot;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int K = kind == 0 ? 32 : 64;

  if (warp == 0) {
    tc::alloc(&tmem_base_slot, 64);
    tc::relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  // B[16, K] into the canonical K-major layout (LBO = 128 B, SBO = K/8*128 B
  // for bf16, K/16*128 B for s8)
  for (int idx = tid; idx < 16 * K; idx += 128) {
    const int n = idx / K, k = idx % K;
    const int v = selftest_b(n, k);
    if (kind == 0) {
      const int off = (n / 8) * ((K / 8) * 128) + (k / 8) * 128 + (n % 8) * 16 + (k % 8) * 2;
      *reinterpret_cast<uint16_t *>(bsm + off) = (uint16_t)bf16_bits_of_small_int(v);
    } else {
      const int off = (n / 8) * ((K / 16) * 128) + (k / 16) * 128 + (n % 8) * 16 + (k % 16);
      bsm[off] = (uint8_t)(int8_t)v;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base_slot;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

  // A: row m = tid, 16 columns of packed elements at columns [0, 16)
  uint32_t r[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (kind == 0) {
      r[j] = bf16_bits_of_small_int(selftest_a(tid, 2 * j)) |
             (bf16_bits_of_small_int(selftest_a(tid, 2 * j + 1)) << 16);
    } else {
      uint32_t w = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) w |= ((uint32_t)(uint8_t)(int8_t)selftest_a(tid, 4 * j + b)) << (8 * b);
      r[j] = w;
    }
  }
  tc::st16(tbase + lane_base + 0, r);
  tc::wait_st();
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();

  const uint32_t d_col = 32;
  if (tid == 0) {
    tc::fence_after_sync();
    for (int s = 0; s < 2; ++s) {
      const uint64_t bd = tc::smem_desc(smem_u32(bsm) + 256 * s, 128, kind == 0 ? (K / 8) * 128 : (K / 16) * 128);
      if (kind == 0)
        tc::mma_bf16_ts(tbase + d_col, tbase + 8 * s, bd, tc::idesc_bf16_f32(16), s > 0);
      else
        tc::mma_s8_ts(tbase + d_col, tbase + 8 * s, bd, tc::idesc_s8_s32(16), s > 0);
    }
    tc::commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0, status);
  tc::fence_after_sync();
  uint32_t d[16];
  tc::ld16(tbase + lane_base + d_col, d);
  tc::wait_ld();
  if (ok) {
#pragma unroll
    for (int n = 0; n < 16; ++n)
      out[tid * 16 + n] = kind == 0 ? (int32_t)__uint_as_float(d[n]) : (int32_t)d[n];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::dealloc(tbase, 64);
}

cudaError_t launch_tc_selftest(int kind, int32_t *out, int *status, cudaStream_t st) {
  tc_selftest_kernel<<<1, 128, 0, st>>>(kind, out, status);
  return cudaGetLastError();
}

}  // namespace lbc
