// Copies between pinned host memory and device memory done by SM loads and
// stores instead of the copy engines, for the host-buffer entry points
// (lbc_gemm_*_host). A kilobyte-sized activation or result copy is
// latency-bound: one small kernel reading or writing mapped host memory
// finishes sooner than a DMA transfer, and it can take part in programmatic
// dependent launch, so the GEMM that follows streams its weights while X is
// still arriving.
#include "kernels.h"

namespace {

// dst[i] = src[i] for i < n4 float4s and the n_tail floats after them.
// Launched with programmatic stream serialisation: dependents may start at
// once (they wait for this grid before reading dst), and this grid waits for
// its predecessor before reading src.
__global__ void __launch_bounds__(256) copy_f32_kernel(const float *src, float *dst, long long n4, int n_tail) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const long long stride = (long long)gridDim.x * blockDim.x;
  const float4 *s4 = reinterpret_cast<const float4 *>(src);
  float4 *d4 = reinterpret_cast<float4 *>(dst);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v;
    asm volatile("ld.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(s4 + i));
    d4[i] = v;
  }
  if (blockIdx.x == 0 && (int)threadIdx.x < n_tail) {
    float v;
    asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(src + 4 * n4 + threadIdx.x));
    dst[4 * n4 + threadIdx.x] = v;
  }
}

}  // namespace

namespace lbc {

cudaError_t launch_copy_f32(const float *src, float *dst, size_t n, int sms, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u)
    return cudaErrorMisalignedAddress;
  const long long n4 = (long long)(n / 4);
  const int tail = (int)(n % 4);
  long long blocks = (n4 + 255) / 256;
  blocks = blocks < 1 ? 1 : blocks;
  const long long cap = 2LL * (sms > 0 ? sms : 148);
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, copy_f32_kernel, src, dst, n4, tail);
}

}  // namespace lbc
