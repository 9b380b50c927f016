// On-device weight quantizers, bit-identical to lowbit's numpy quantizers
// (src/lowbit/formats.py:90-142 int4 g128, :175-212 MXFP4), writing the packed
// layouts the GEMMs read: a load-time path that never round-trips W through
// the host.
//
// int4 (one warp per group of 128; lane l holds elements l, l+32, l+64, l+96
// and writes packed bytes l and l+32 = codes (l, l+64) and (l+32, l+96)):
//   absmax      s = max|w| / 7, q = clip(rint(w / s), -8, 7) + 8
//   signed-max  s = w[argmax |w|] / -8 (first index on ties), same q
//   asym        s = (max(w, 0) - min(w, 0)) / 15, z = clip(rint(-min / s), 0, 15),
//               q = clip(rint(w / s) + z, 0, 15)
//   a zero scale becomes 1; padding past K gets the code that decodes to 0.
// MXFP4 (one warp per block of 32; lane j < 16 writes byte j = codes (j, j+16)):
//   e = clip(floor(log2(amax)) - 2 + 127, 0, 254) (0 for an all-zero block),
//   code = E2M1 of w / 2^(e-127): nearest, ties to the even mantissa,
//   saturating at 6, sign bit only for non-zero magnitudes.
// Divisions and rint are IEEE single precision as numpy's float32 ops are.
// floor(log2(amax)) is taken as floor of the fp32-rounded double log2, which
// equals numpy's fp32 log2 floor on every subnormal and on tested normals.
#include <cmath>
#include <cstdint>
#include <cstdio>

#include "../../include/lowbit_b200.h"
#include "kernels.h"

namespace lbc {
namespace {

constexpr int Q_THREADS = 256;

__global__ void __launch_bounds__(Q_THREADS) quant_int4_kernel(const float *w, int N, int K, int mode, uint8_t *qw,
                                                              float *scales, uint8_t *zeros) {
  const int G = (K + 127) / 128, Kp = G * 128;
  const int lane = threadIdx.x & 31;
  const long long ngroups = (long long)N * G;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long gi = wid; gi < ngroups; gi += nw) {
    const int n = (int)(gi / G), g = (int)(gi % G);
    float v[4];
    bool live[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = g * 128 + lane + 32 * u;
      live[u] = k < K;
      v[u] = live[u] ? w[(size_t)n * K + k] : 0.f;
    }
    float s;
    uint32_t z = 8;
    if (mode == 1) {  // asym
      float hi = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
      float lo = fminf(fminf(v[0], v[1]), fminf(v[2], v[3]));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      }
      hi = fmaxf(hi, 0.f);
      lo = fminf(lo, 0.f);
      s = __fdiv_rn(__fsub_rn(hi, lo), 15.f);
      if (!(s > 0.f)) s = 1.f;
      z = (uint32_t)fminf(fmaxf(rintf(__fdiv_rn(-lo, s)), 0.f), 15.f);
    } else if (mode == 2) {  // signed-max: the largest magnitude, first index on ties
      float best = -1.f;
      int bi = 0x7fffffff;
      float bv = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float a = fabsf(v[u]);
        const int idx = lane + 32 * u;
        if (a > best || (a == best && idx < bi)) {
          best = a;
          bi = idx;
          bv = v[u];
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
          bv = ov;
        }
      }
      s = __fdiv_rn(bv, -8.f);
      if (s == 0.f) s = 1.f;
    } else {  // absmax
      float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
      s = __fdiv_rn(a, 7.f);
      if (!(s > 0.f)) s = 1.f;
    }
    uint32_t c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float r = rintf(__fdiv_rn(v[u], s));
      if (mode == 1)
        c[u] = live[u] ? (uint32_t)fminf(fmaxf(__fadd_rn(r, (float)z), 0.f), 15.f) : z;
      else
        c[u] = live[u] ? (uint32_t)(fminf(fmaxf(r, -8.f), 7.f) + 8.f) : 8u;
    }
    uint8_t *row = qw + (size_t)n * (Kp / 2) + g * 64;
    row[lane] = (uint8_t)(c[0] | (c[2] << 4));
    row[lane + 32] = (uint8_t)(c[1] | (c[3] << 4));
    if (lane == 0) {
      scales[(size_t)n * G + g] = s;
      if (mode == 1) zeros[(size_t)n * G + g] = (uint8_t)z;
    }
  }
}

__device__ __forceinline__ uint32_t e2m1_code(float v) {
  const float a = fabsf(v);
  uint32_t mag = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.0f);
  const uint32_t neg = (signbit(v) && mag > 0) ? 1u : 0u;
  return mag | (neg << 3);
}

__global__ void __launch_bounds__(Q_THREADS) quant_mxfp4_kernel(const float *w, int N, int K, uint8_t *qw,
                                                               uint8_t *e8m0) {
  const int NB = (K + 31) / 32, Kp = NB * 32;
  const int lane = threadIdx.x & 31;
  const long long nblocks = (long long)N * NB;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long bi = wid; bi < nblocks; bi += nw) {
    const int n = (int)(bi / NB), b = (int)(bi % NB);
    const int k = b * 32 + lane;
    const float v = k < K ? w[(size_t)n * K + k] : 0.f;
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int e = 127;  // shared exponent 0 for an all-zero block
    if (amax > 0.f) {
      const float lg = __double2float_rn(log2((double)amax));
      e = (int)floorf(lg) - 2 + 127;
      e = e < 0 ? 0 : (e > 254 ? 254 : e);
    }
    // 2^(e - 127) for e in [0, 254]: exact in fp32 (2^-127 is subnormal)
    const float scale = ldexpf(1.0f, e - 127);
    const uint32_t c = e2m1_code(__fdiv_rn(v, scale));
    const uint32_t hi = __shfl_down_sync(0xffffffffu, c, 16);
    if (lane < 16) qw[(size_t)n * (Kp / 2) + b * 16 + lane] = (uint8_t)(c | (hi << 4));
    if (lane == 0) e8m0[(size_t)n * NB + b] = (uint8_t)e;
  }
}

int q_status(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
    set_last_error(buf);
    return LBC_ERR_CUDA;
  }
  return 0;
}

int q_grid(long long warps) {
  long long blocks = (warps * 32 + Q_THREADS - 1) / Q_THREADS;
  return (int)(blocks < 148LL * 64 ? (blocks < 1 ? 1 : blocks) : 148LL * 64);
}

}  // namespace
}  // namespace lbc

using namespace lbc;

extern "C" {

int lbc_quantize_int4(const float *w, int N, int K, int mode, uint8_t *qw, float *scales, uint8_t *zeros,
                      void *stream) {
  if (N <= 0 || K <= 0 || mode < 0 || mode > 2 || (mode == 1 && !zeros)) {
    set_last_error("quantize_int4: bad shape or mode");
    return LBC_ERR_SHAPE;
  }
  const long long groups = (long long)N * ((K + 127) / 128);
  quant_int4_kernel<<<q_grid(groups), Q_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(w, N, K, mode, qw, scales,
                                                                                          zeros);
  return q_status("quantize_int4");
}

int lbc_quantize_mxfp4(const float *w, int N, int K, uint8_t *qw, uint8_t *e8m0, void *stream) {
  if (N <= 0 || K <= 0) {
    set_last_error("quantize_mxfp4: bad shape");
    return LBC_ERR_SHAPE;
  }
  const long long blocks = (long long)N * ((K + 31) / 32);
  quant_mxfp4_kernel<<<q_grid(blocks), Q_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(w, N, K, qw, e8m0);
  return q_status("quantize_mxfp4");
}

}  // extern "C"
