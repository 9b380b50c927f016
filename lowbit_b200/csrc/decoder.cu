// Decoder-layer operators around the quantized GEMMs: the model-side path of
// the reference's numpy forward (src/lowbit/model.py:380-433) on the GPU.
//
//   rmsnorm      x <- x + residual (optional); out = x / sqrt(mean(x^2) + eps) * w
//                (src/lowbit/model.py:188-190 and the residual adds at :413, :421)
//   qkv_rope     bias add (the linear's y += b, :119-124), rotate-half RoPE on q and
//                k (:199-208), k and v appended to the KV cache (:343-345)
//   attention    causal grouped-query softmax attention over the cache (:336-361)
//   silu_mul     silu(gate) * up (:211-212, :417)
//
// Every operator reads the position from device memory, so one captured CUDA
// graph of a decode step replays at every position. Products and sums that
// the reference rounds separately are rounded separately here (__fmul_rn and
// friends keep the compiler from contracting them into fused multiply-adds).
// Activations are fp32 throughout, as in the reference.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>

#include "../../include/lowbit_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace lbc {
namespace {

constexpr int NORM_THREADS = 256;
constexpr int ATT_THREADS = 128;

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
  for (int i = 1; i < nw; ++i) t = fmaxf(t, red[i]);
  return t;
}

// one CTA per token row
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(const float *x, const float *res, float *x_out,
                                                              const float *w, float *out, int H, float eps) {
  __shared__ float red[NORM_THREADS / 32];
  const size_t row = blockIdx.x;
  const float *xr = x + row * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = xr[i];
    if (res) {
      v = __fadd_rn(v, res[row * H + i]);
      x_out[row * H + i] = v;
    }
    ss = __fmaf_rn(v, v, ss);
  }
  const float var = __fdiv_rn(block_sum(ss, red), (float)H);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = res ? x_out[row * H + i] : xr[i];
    out[row * H + i] = __fmul_rn(__fmul_rn(v, r), w[i]);
  }
}

// one CTA per token; token i = (sequence b, step t), position pos + t
__global__ void qkv_rope_kernel(const float *qkv, const float *bias, const float *cos_t, const float *sin_t,
                                const int32_t *pos_p, float *q_out, float *k_cache, float *v_cache, int T,
                                int H, int KV, int D, int S_max) {
  const int i = blockIdx.x, b = i / T, t = i % T;
  const int p = *pos_p + t;
  const int half = D / 2, W = (H + 2 * KV) * D;
  const float *row = qkv + (size_t)i * W;
  const float *cs = cos_t + (size_t)p * half, *sn = sin_t + (size_t)p * half;
  // rotated pairs (d, d + D/2) of the q heads, then of the k heads
  for (int e = threadIdx.x; e < (H + KV) * half; e += blockDim.x) {
    const int head = e / half, d = e % half;
    const int c1 = head * D + d, c2 = c1 + half;
    float x1 = row[c1], x2 = row[c2];
    if (bias) {
      x1 = __fadd_rn(x1, bias[c1]);
      x2 = __fadd_rn(x2, bias[c2]);
    }
    const float c = cs[d], s = sn[d];
    const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    if (head < H) {
      float *q = q_out + ((size_t)i * H + head) * D;
      q[d] = o1;
      q[d + half] = o2;
    } else {
      float *k = k_cache + (((size_t)b * KV + (head - H)) * S_max + p) * D;
      k[d] = o1;
      k[d + half] = o2;
    }
  }
  for (int e = threadIdx.x; e < KV * D; e += blockDim.x) {
    const int c = (H + KV) * D + e;
    float v = row[c];
    if (bias) v = __fadd_rn(v, bias[c]);
    v_cache[(((size_t)b * KV + e / D) * S_max + p) * D + e % D] = v;
  }
}

// one CTA per (token, query head): scores over keys 0..pos+t in shared memory
template <int DPL>  // head elements per lane (D = 32 * DPL)
__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const float *q, const float *k_cache,
                                                                const float *v_cache, const int32_t *pos_p,
                                                                float *out, int T, int H, int KV, int S_max,
                                                                float scale) {
  extern __shared__ float sc[];  // [S_max] scores, then [ATT_THREADS] partial outputs
  __shared__ float red[ATT_THREADS / 32];
  constexpr int D = 32 * DPL;
  const int i = blockIdx.x, h = blockIdx.y, b = i / T, t = i % T;
  const int L = *pos_p + t + 1;
  const int kvh = h / (H / KV);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float *qv = q + ((size_t)i * H + h) * D;
  float qr[DPL];
#pragma unroll
  for (int u = 0; u < DPL; ++u) qr[u] = qv[lane + 32 * u];
  const float *kb = k_cache + ((size_t)b * KV + kvh) * S_max * D;
  const float *vb = v_cache + ((size_t)b * KV + kvh) * S_max * D;
  for (int j = warp; j < L; j += nw) {
    const float *kr = kb + (size_t)j * D;
    float s = 0.f;
#pragma unroll
    for (int u = 0; u < DPL; ++u) s = __fmaf_rn(qr[u], kr[lane + 32 * u], s);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) sc[j] = __fmul_rn(s, scale);
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < L; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  mx = block_max(mx, red);
  float sum = 0.f;
  for (int j = threadIdx.x; j < L; j += blockDim.x) {
    const float e = expf(__fsub_rn(sc[j], mx));
    sc[j] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = block_sum(sum, red);
  for (int j = threadIdx.x; j < L; j += blockDim.x) sc[j] = __fdiv_rn(sc[j], sum);
  __syncthreads();
  // out[d] = sum_j p_j v_j[d]: thread (group g, element d) takes keys j = g mod groups
  const int groups = blockDim.x / D;
  const int d = threadIdx.x % D, g = threadIdx.x / D;
  float acc = 0.f;
  if (g < groups)
    for (int j = g; j < L; j += groups) acc = __fmaf_rn(sc[j], vb[(size_t)j * D + d], acc);
  float *part = sc + S_max;
  part[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < D) {
    float o = 0.f;
    for (int gg = 0; gg < groups; ++gg) o = __fadd_rn(o, part[gg * D + threadIdx.x]);
    out[((size_t)i * H + h) * D + threadIdx.x] = o;
  }
}

__global__ void silu_mul_kernel(const float *gu, float *out, int I, size_t total) {
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const size_t r = e / I, c = e % I;
    const float g = gu[r * 2 * I + c], u = gu[r * 2 * I + I + c];
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    out[e] = __fmul_rn(s, u);
  }
}

__global__ void advance_kernel(int32_t *pos, int n) { *pos += n; }

int launch_status(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
    set_last_error(buf);
    return LBC_ERR_CUDA;
  }
  return 0;
}

int shape_error(const char *msg) {
  set_last_error(msg);
  return LBC_ERR_SHAPE;
}

}  // namespace
}  // namespace lbc

using namespace lbc;

extern "C" {

int lbc_rmsnorm(const float *x, const float *residual, float *x_out, const float *w, float *out, int T, int H,
                float eps, void *stream) {
  if (T < 0 || H <= 0) return shape_error("rmsnorm: bad shape");
  if (residual && !x_out) return shape_error("rmsnorm: residual needs x_out");
  if (T == 0) return 0;
  rmsnorm_kernel<<<T, NORM_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(x, residual, x_out, w, out, H, eps);
  return launch_status("rmsnorm");
}

int lbc_qkv_rope(const float *qkv, const float *bias, const float *cos_t, const float *sin_t, const int32_t *pos,
                 float *q_out, float *k_cache, float *v_cache, int B, int T, int H, int KV, int D, int S_max,
                 void *stream) {
  if (B <= 0 || T <= 0 || H <= 0 || KV <= 0 || H % KV || D <= 0 || D % 2 || S_max <= 0)
    return shape_error("qkv_rope: bad shape");
  qkv_rope_kernel<<<B * T, 128, 0, static_cast<cudaStream_t>(stream)>>>(qkv, bias, cos_t, sin_t, pos, q_out,
                                                                         k_cache, v_cache, T, H, KV, D, S_max);
  return launch_status("qkv_rope");
}

int lbc_attention(const float *q, const float *k_cache, const float *v_cache, const int32_t *pos, float *out,
                  int B, int T, int H, int KV, int D, int S_max, void *stream) {
  if (B <= 0 || T <= 0 || H <= 0 || KV <= 0 || H % KV || S_max <= 0) return shape_error("attention: bad shape");
  if (D != 32 && D != 64 && D != 128) return shape_error("attention: head_dim must be 32, 64 or 128");
  const size_t smem = ((size_t)S_max + ATT_THREADS) * sizeof(float);
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (smem + 64 > (size_t)optin) return shape_error("attention: KV cache longer than shared memory allows");
  const dim3 grid(B * T, H);
  const float scale = (float)(1.0 / std::sqrt((double)D));  // np.float32(1.0 / np.sqrt(D))
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define LBC_ATT(DPL)                                                                                     \
  {                                                                                                      \
    auto k = attention_kernel<DPL>;                                                                      \
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    k<<<grid, ATT_THREADS, smem, st>>>(q, k_cache, v_cache, pos, out, T, H, KV, S_max, scale);           \
  }
  if (D == 32) LBC_ATT(1) else if (D == 64) LBC_ATT(2) else LBC_ATT(4)
#undef LBC_ATT
  return launch_status("attention");
}

int lbc_silu_mul(const float *gu, float *out, int T, int I, void *stream) {
  if (T < 0 || I <= 0) return shape_error("silu_mul: bad shape");
  if (T == 0) return 0;
  const size_t total = (size_t)T * I;
  const int grid = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  silu_mul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(gu, out, I, total);
  return launch_status("silu_mul");
}

int lbc_advance_pos(int32_t *pos, int n, void *stream) {
  advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(pos, n);
  return launch_status("advance_pos");
}

}  // extern "C"
