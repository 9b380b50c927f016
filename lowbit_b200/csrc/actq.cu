// Per-token int8 activation quantizer and exact int32 group accumulators.
//
// quant_act_int8 is bit-identical to the reference's lb_quant_act_int8
// (src/lowbit/csrc/dispatch.c:231-257) and to numpy's quantize_act_int8
// (src/lowbit/formats.py:236-248):
//   amax = max |x[m,k]| over the padded row (NaN never wins, as `a > amax`)
//   sc   = amax > 0 ? amax / 127 : 1          (IEEE fp32 division)
//   q    = clamp(round_half_even(x / sc), -127, 127)   (IEEE division + rint)
//   asum[m,g] = sum of the 128 codes of group g
// The file must be compiled without fast-math: both divisions are __fdiv_rn.
#include "common.cuh"
#include "kernels.h"

namespace lbc {

// one CTA per token row; a warp quantizes one 128-element group per step
__global__ void quant_act_int8_kernel(const float *x, int Kp,
                                      int8_t *__restrict__ xq, float *__restrict__ xs,
                                      int32_t *__restrict__ asum) {
  __shared__ float wmax[32];
  // let the GEMM that consumes xq start streaming its weights now; x may be
  // produced by the previous kernel, so wait for it before reading
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int m = blockIdx.x;
  const float *xr = x + (size_t)m * Kp;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;

  float amax = 0.0f;
  for (int k = tid * 4; k < Kp; k += blockDim.x * 4) {
    const float4 v = ld_act(reinterpret_cast<const float4 *>(xr + k));
    amax = fmaxf(amax, fabsf(v.x));
    amax = fmaxf(amax, fabsf(v.y));
    amax = fmaxf(amax, fabsf(v.z));
    amax = fmaxf(amax, fabsf(v.w));
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s));
  if (lane == 0) wmax[warp] = amax;
  __syncthreads();
  if (warp == 0) {
    float v = lane < nw ? wmax[lane] : 0.0f;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
    if (lane == 0) wmax[0] = v;
  }
  __syncthreads();
  amax = wmax[0];
  const float sc = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  if (tid == 0) xs[m] = sc;

  const int G = Kp >> 7;
  for (int g = warp; g < G; g += nw) {
    const int k = (g << 7) + lane * 4;
    const float4 v = ld_act(reinterpret_cast<const float4 *>(xr + k));
    const float f[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed = 0;
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float q = rintf(__fdiv_rn(f[i], sc));
      q = fminf(fmaxf(q, -127.0f), 127.0f);
      const int qi = (int)q;
      sum += qi;
      packed |= ((uint32_t)qi & 0xFFu) << (8 * i);
    }
    *reinterpret_cast<uint32_t *>(xq + (size_t)m * Kp + k) = packed;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
    if (lane == 0) asum[(size_t)m * G + g] = sum;
  }
}

// out[m,n,g] = sum_{k in g} q[n,k]*xq[m,k] - z[n,g]*asum[m,g]  (exact int32),
// the same identity as src/lowbit/csrc/kern_scalar.c:49-59. One thread per
// (m, n, g); a test/debug kernel, not a hot path.
__global__ void w4a8_group_acc_kernel(const int8_t *__restrict__ xq,
                                      const int32_t *__restrict__ asum, int M, int Kp,
                                      const uint8_t *__restrict__ qw,
                                      const uint8_t *__restrict__ zeros, int N,
                                      int32_t *__restrict__ out) {
  const int G = Kp >> 7;
  const long long total = (long long)M * N * G;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(idx % G);
    const int n = (int)((idx / G) % N);
    const int m = (int)(idx / ((long long)G * N));
    const uint4 *wp = reinterpret_cast<const uint4 *>(qw + (size_t)n * (Kp >> 1) + (size_t)g * 64);
    const uint4 *ap = reinterpret_cast<const uint4 *>(xq + (size_t)m * Kp + (size_t)g * 128);
    int acc = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // 4 chunks of 16 bytes = 32 codes each
      const uint4 w = __ldg(wp + c);
      const uint4 lo = __ldg(ap + c);      // elements 16c .. 16c+15
      const uint4 hi = __ldg(ap + 4 + c);  // elements 64+16c ..
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
      const uint32_t ll[4] = {lo.x, lo.y, lo.z, lo.w};
      const uint32_t hh[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc = dp4a_us(ww[q] & 0x0F0F0F0Fu, ll[q], acc);
        acc = dp4a_us((ww[q] >> 4) & 0x0F0F0F0Fu, hh[q], acc);
      }
    }
    const int z = zeros ? (int)zeros[(size_t)n * G + g] : 8;
    out[idx] = acc - z * asum[(size_t)m * G + g];
  }
}

cudaError_t launch_quant_act_int8(const float *x, int M, int Kp, int8_t *xq, float *xs,
                                  int32_t *asum, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(Kp <= 512 ? 128 : 256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, quant_act_int8_kernel, x, Kp, xq, xs, asum);
}

cudaError_t launch_w4a8_group_acc(const int8_t *xq, const int32_t *asum, int M, int Kp,
                                  const uint8_t *qw, const uint8_t *zeros, int N, int32_t *out,
                                  cudaStream_t st) {
  const long long total = (long long)M * N * (Kp >> 7);
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 65535LL * 16) blocks = 65535LL * 16;
  w4a8_group_acc_kernel<<<(unsigned)blocks, threads, 0, st>>>(xq, asum, M, Kp, qw, zeros, N, out);
  return cudaGetLastError();
}

}  // namespace lbc
