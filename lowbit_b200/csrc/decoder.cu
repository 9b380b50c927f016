// Decoder-layer operators around the quantized GEMMs: the model-side path of
// the reference's numpy forward (src/lowbit/model.py:380-433) on the GPU.
//
//   rmsnorm      x <- x + residual (optional); out = x / sqrt(mean(x^2) + eps) * w
//                (src/lowbit/model.py:188-190 and the residual adds at :413, :421)
//   qkv_rope     bias add (the linear's y += b, :119-124), rotate-half RoPE on q and
//                k (:199-208), k and v appended to the KV cache (:343-345)
//   attention    causal grouped-query softmax attention over the cache (:336-361),
//                one CTA per (token, KV head) sharing the K/V loads of its query heads
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
#include <map>
#include <vector>
#include <mutex>
#include <utility>

#include "../../include/lowbit_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace lbc {
namespace {

constexpr int NORM_THREADS = 256;
constexpr int ATT_THREADS = 512;

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

// One CTA per (token, KV head): the G = H / KV query heads that share the KV
// head share its K and V loads (G <= ATT_MAX_G). Scores: thread t takes keys
// t, t + 512, ... and computes all G dot products from its own loads (q in
// shared memory, read as broadcasts). Softmax: warp w normalises heads w,
// w + 16, ... Output: thread (key group, element d) accumulates all G heads
// over keys j = group (mod groups), one load of v[j][d] serving every head,
// then the groups' partial sums are added in a fixed order.
//
// FUSE_ROPE (single-token steps, T == 1): the CTA first does lbc_qkv_rope's
// work for its heads -- bias, RoPE, q to shared memory, k and v of its KV head
// appended to the cache at pos -- so a decode step needs no separate launch.
// (With T > 1 other tokens' keys come from other CTAs, so prefill runs the
// two kernels separately.)
constexpr int ATT_MAX_G = 16;

template <int D, bool FUSE_ROPE>
__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const float *q, const float *bias,
                                                                const float *cos_t, const float *sin_t,
                                                                float *k_cache, float *v_cache,
                                                                const int32_t *pos_p, float *out, int T, int H,
                                                                int KV, int S_max, float scale) {
  extern __shared__ float4 smem4[];
  const int G = H / KV;
  constexpr int NG = ATT_THREADS / D;  // key groups in the output phase
  float *qs = reinterpret_cast<float *>(smem4);  // [G][D]
  float *part = qs + G * D;                       // [NG][G][D] output partials
  float *sc = part + NG * G * D;                  // [G][L] scores
  const int i = blockIdx.x, kvh = blockIdx.y, b = i / T, t = i % T;
  const int p0 = *pos_p;
  const int L = p0 + t + 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NWARP = ATT_THREADS / 32;
  float *kb = k_cache + ((size_t)b * KV + kvh) * S_max * D;
  float *vb = v_cache + ((size_t)b * KV + kvh) * S_max * D;
  if (FUSE_ROPE) {
    // q rows of this group's heads, then k and v of the KV head, as lbc_qkv_rope
    constexpr int half = D / 2;
    const int W = (H + 2 * KV) * D;
    const float *row = q + (size_t)i * W;
    const float *cs = cos_t + (size_t)(p0 + t) * half, *sn = sin_t + (size_t)(p0 + t) * half;
    for (int e = tid; e < (G + 1) * half; e += ATT_THREADS) {
      const int hh = e / half, d = e % half;
      const int head = hh < G ? kvh * G + hh : H + kvh;
      const int c1 = head * D + d, c2 = c1 + half;
      float x1 = row[c1], x2 = row[c2];
      if (bias) {
        x1 = __fadd_rn(x1, bias[c1]);
        x2 = __fadd_rn(x2, bias[c2]);
      }
      const float c = cs[d], sv = sn[d];
      const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sv));
      const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sv));
      if (hh < G) {
        qs[hh * D + d] = o1;
        qs[hh * D + d + half] = o2;
      } else {
        kb[(size_t)(p0 + t) * D + d] = o1;
        kb[(size_t)(p0 + t) * D + d + half] = o2;
      }
    }
    for (int d = tid; d < D; d += ATT_THREADS) {
      const int c = (H + KV + kvh) * D + d;
      float v = row[c];
      if (bias) v = __fadd_rn(v, bias[c]);
      vb[(size_t)(p0 + t) * D + d] = v;
    }
  } else {
    const float *qb = q + ((size_t)i * H + (size_t)kvh * G) * D;
    for (int e = tid; e < G * D; e += ATT_THREADS) qs[e] = qb[e];
  }
  __syncthreads();  // also orders this CTA's cache writes before its reads below
  for (int j = tid; j < L; j += ATT_THREADS) {
    // the key row in slices of 32 elements; each head's dot product runs
    // over d = 0..D-1 in order
    const float4 *kr = reinterpret_cast<const float4 *>(kb + (size_t)j * D);
    float s[ATT_MAX_G];
#pragma unroll
    for (int h = 0; h < ATT_MAX_G; ++h) s[h] = 0.f;
#pragma unroll
    for (int u0 = 0; u0 < D / 4; u0 += 8) {
      float4 kv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) kv[u] = kr[u0 + u];
#pragma unroll
      for (int h = 0; h < ATT_MAX_G; ++h) {
        if (h < G) {
          const float4 *qh = reinterpret_cast<const float4 *>(qs + h * D) + u0;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float4 a = qh[u];
            s[h] = __fmaf_rn(a.x, kv[u].x, s[h]);
            s[h] = __fmaf_rn(a.y, kv[u].y, s[h]);
            s[h] = __fmaf_rn(a.z, kv[u].z, s[h]);
            s[h] = __fmaf_rn(a.w, kv[u].w, s[h]);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < ATT_MAX_G; ++h)
      if (h < G) sc[h * L + j] = __fmul_rn(s[h], scale);
  }
  __syncthreads();
  for (int h = warp; h < G; h += NWARP) {
    float *row = sc + h * L;
    float mx = -INFINITY;
    for (int j = lane; j < L; j += 32) mx = fmaxf(mx, row[j]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < L; j += 32) {
      const float e = expf(__fsub_rn(row[j], mx));
      row[j] = e;
      sum = __fadd_rn(sum, e);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    for (int j = lane; j < L; j += 32) row[j] = __fdiv_rn(row[j], sum);
  }
  __syncthreads();
  const int d = tid % D, kg = tid / D;
  float acc[ATT_MAX_G];
#pragma unroll
  for (int h = 0; h < ATT_MAX_G; ++h) acc[h] = 0.f;
#pragma unroll 8
  for (int j = kg; j < L; j += NG) {
    const float v = vb[(size_t)j * D + d];
#pragma unroll
    for (int h = 0; h < ATT_MAX_G; ++h)
      if (h < G) acc[h] = __fmaf_rn(sc[h * L + j], v, acc[h]);
  }
#pragma unroll
  for (int h = 0; h < ATT_MAX_G; ++h)
    if (h < G) part[(kg * G + h) * D + d] = acc[h];
  __syncthreads();
  for (int e = tid; e < G * D; e += ATT_THREADS) {
    float o = 0.f;
    for (int g = 0; g < NG; ++g) o = __fadd_rn(o, part[g * G * D + e]);
    out[((size_t)i * H + (size_t)kvh * G) * D + e] = o;
  }
}

// Key-split attention for few (token, KV head) pairs: CTA (i, kvh, sp) takes
// keys [sp * ATT_SPLIT, min(L, (sp + 1) * ATT_SPLIT)) and writes, per query
// head, its maximum score, the sum of exp(score - max) and the unnormalised
// output sum_j exp(score_j - max) v_j; attention_combine_kernel merges the
// splits in order. With FUSE_ROPE the split that holds position pos + t also
// appends k and v there (no other split reads that key).
constexpr int ATT_SPLIT = 64;
constexpr int ATT_SPLIT_THREADS = 128;

template <int D, bool FUSE_ROPE>
__global__ void __launch_bounds__(ATT_SPLIT_THREADS) attention_split_kernel(
    const float *q, const float *bias, const float *cos_t, const float *sin_t, float *k_cache, float *v_cache,
    const int32_t *pos_p, float *ws, int T, int H, int KV, int S_max, int NS, float scale) {
  __shared__ __align__(16) float qs[ATT_MAX_G * D];
  __shared__ float sc[ATT_MAX_G][ATT_SPLIT];
  __shared__ float part[ATT_SPLIT_THREADS / D][ATT_MAX_G][D];
  const int G = H / KV;
  const int i = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z, b = i / T, t = i % T;
  const int p0 = *pos_p;
  const int L = p0 + t + 1;
  const int j0 = sp * ATT_SPLIT;
  if (j0 >= L) return;  // split past the current length: nothing to do
  const int nk = min(ATT_SPLIT, L - j0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NWARP = ATT_SPLIT_THREADS / 32;
  float *kb = k_cache + ((size_t)b * KV + kvh) * S_max * D;
  float *vb = v_cache + ((size_t)b * KV + kvh) * S_max * D;
  if (FUSE_ROPE) {
    constexpr int half = D / 2;
    const int W = (H + 2 * KV) * D;
    const float *row = q + (size_t)i * W;
    const int p = p0 + t;
    const bool mine = p >= j0 && p < j0 + ATT_SPLIT;  // this split appends k and v
    const float *cs = cos_t + (size_t)p * half, *sn = sin_t + (size_t)p * half;
    for (int e = tid; e < (G + 1) * half; e += ATT_SPLIT_THREADS) {
      const int hh = e / half, d = e % half;
      if (hh == G && !mine) continue;
      const int head = hh < G ? kvh * G + hh : H + kvh;
      const int c1 = head * D + d, c2 = c1 + half;
      float x1 = row[c1], x2 = row[c2];
      if (bias) {
        x1 = __fadd_rn(x1, bias[c1]);
        x2 = __fadd_rn(x2, bias[c2]);
      }
      const float c = cs[d], sv = sn[d];
      const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sv));
      const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sv));
      if (hh < G) {
        qs[hh * D + d] = o1;
        qs[hh * D + d + half] = o2;
      } else {
        kb[(size_t)p * D + d] = o1;
        kb[(size_t)p * D + d + half] = o2;
      }
    }
    if (mine) {
      for (int d = tid; d < D; d += ATT_SPLIT_THREADS) {
        const int c = (H + KV + kvh) * D + d;
        float v = row[c];
        if (bias) v = __fadd_rn(v, bias[c]);
        vb[(size_t)p * D + d] = v;
      }
    }
  } else {
    const float *qb = q + ((size_t)i * H + (size_t)kvh * G) * D;
    for (int e = tid; e < G * D; e += ATT_SPLIT_THREADS) qs[e] = qb[e];
  }
  __syncthreads();
  if (tid < nk) {
    const float4 *kr = reinterpret_cast<const float4 *>(kb + (size_t)(j0 + tid) * D);
    float s[ATT_MAX_G];
#pragma unroll
    for (int h = 0; h < ATT_MAX_G; ++h) s[h] = 0.f;
#pragma unroll
    for (int u0 = 0; u0 < D / 4; u0 += 8) {
      float4 kv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) kv[u] = kr[u0 + u];
#pragma unroll
      for (int h = 0; h < ATT_MAX_G; ++h) {
        if (h < G) {
          const float4 *qh = reinterpret_cast<const float4 *>(qs + h * D) + u0;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float4 a = qh[u];
            s[h] = __fmaf_rn(a.x, kv[u].x, s[h]);
            s[h] = __fmaf_rn(a.y, kv[u].y, s[h]);
            s[h] = __fmaf_rn(a.z, kv[u].z, s[h]);
            s[h] = __fmaf_rn(a.w, kv[u].w, s[h]);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < ATT_MAX_G; ++h)
      if (h < G) sc[h][tid] = __fmul_rn(s[h], scale);
  }
  __syncthreads();
  float *rec = ws + (((size_t)i * KV + kvh) * NS + sp) * (size_t)(G * (D + 2));  // [G][m, l, o[D]]
  for (int h = warp; h < G; h += NWARP) {
    float mx = -INFINITY;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sc[h][j]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < nk; j += 32) {
      const float e = expf(__fsub_rn(sc[h][j], mx));
      sc[h][j] = e;
      sum = __fadd_rn(sum, e);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      rec[h * (D + 2)] = mx;
      rec[h * (D + 2) + 1] = sum;
    }
  }
  __syncthreads();
  constexpr int NG = ATT_SPLIT_THREADS / D;
  const int d = tid % D, kg = tid / D;
  float acc[ATT_MAX_G];
#pragma unroll
  for (int h = 0; h < ATT_MAX_G; ++h) acc[h] = 0.f;
#pragma unroll 4
  for (int j = kg; j < nk; j += NG) {
    const float v = vb[(size_t)(j0 + j) * D + d];
#pragma unroll
    for (int h = 0; h < ATT_MAX_G; ++h)
      if (h < G) acc[h] = __fmaf_rn(sc[h][j], v, acc[h]);
  }
#pragma unroll
  for (int h = 0; h < ATT_MAX_G; ++h)
    if (h < G) part[kg][h][d] = acc[h];
  __syncthreads();
  for (int e = tid; e < G * D; e += ATT_SPLIT_THREADS) {
    const int h = e / D, dd = e % D;
    float o = 0.f;
    for (int g = 0; g < NG; ++g) o = __fadd_rn(o, part[g][h][dd]);
    rec[h * (D + 2) + 2 + dd] = o;
  }
}

// out = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M), M = max_s m_s, over the
// splits that hold keys (s * ATT_SPLIT < L), in split order
template <int D>
__global__ void __launch_bounds__(256) attention_combine_kernel(const float *ws, const int32_t *pos_p, float *out,
                                                                int T, int H, int KV, int NS) {
  const int G = H / KV;
  const int i = blockIdx.x, kvh = blockIdx.y, t = i % T;
  const int L = *pos_p + t + 1;
  const int ns = min(NS, (L + ATT_SPLIT - 1) / ATT_SPLIT);
  const float *base = ws + ((size_t)i * KV + kvh) * NS * (size_t)(G * (D + 2));
  const size_t stride = (size_t)G * (D + 2);
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int h = e / D, d = e % D;
    float mx = -INFINITY;
    for (int s = 0; s < ns; ++s) mx = fmaxf(mx, base[s * stride + h * (D + 2)]);
    float den = 0.f, num = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float *r = base + s * stride + h * (D + 2);
      const float w = expf(__fsub_rn(r[0], mx));
      den = __fmaf_rn(r[1], w, den);
      num = __fmaf_rn(r[2 + d], w, num);
    }
    out[((size_t)i * H + (size_t)kvh * G + h) * D + d] = __fdiv_rn(num, den);
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

}  // extern "C"

namespace lbc {
namespace {
// Scratch of the key-split path, one grow-only buffer per (device, stream),
// held until exit. A buffer once handed out is never freed (a CUDA graph of
// an earlier step may hold its address): a grown-out one is retired until the
// process exits, and growth at least doubles. It cannot grow inside a stream
// capture: a first call of each shape outside the capture sizes it.
float *att_workspace(size_t bytes, cudaStream_t st) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<void *, size_t>> cache;
  static std::vector<void *> retired;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  auto &slot = cache[{dev, st}];
  if (slot.first && slot.second >= bytes) return static_cast<float *>(slot.first);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
  const size_t nb = std::max(bytes, 2 * slot.second);
  void *p = nullptr;
  if (cudaMalloc(&p, nb) != cudaSuccess) return nullptr;
  if (slot.first) retired.push_back(slot.first);
  slot = {p, nb};
  return static_cast<float *>(p);
}

int attention_launch(const float *q, const float *bias, const float *cos_t, const float *sin_t, float *k_cache,
                     float *v_cache, const int32_t *pos, float *out, int B, int T, int H, int KV, int D, int S_max,
                     bool fuse, cudaStream_t st) {
  if (B <= 0 || T <= 0 || H <= 0 || KV <= 0 || H % KV || S_max <= 0) return shape_error("attention: bad shape");
  if (D != 32 && D != 64 && D != 128) return shape_error("attention: head_dim must be 32, 64 or 128");
  const int G = H / KV;
  if (G > ATT_MAX_G) return shape_error("attention: more than 16 query heads per KV head");
  int dev = 0, optin = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const dim3 grid(B * T, KV);
  const float scale = (float)(1.0 / std::sqrt((double)D));  // np.float32(1.0 / np.sqrt(D))
  // long caches with few (token, KV head) pairs: split the keys over more
  // CTAs (any cache length). Up to 1024 positions the single-pass kernel is
  // as fast on B200 (measured in a whole decode step) and needs no scratch.
  const int NS = (S_max + ATT_SPLIT - 1) / ATT_SPLIT;
  if (2 * B * T * KV <= sms && NS > 16) {
    const size_t bytes = (size_t)B * T * KV * NS * G * (D + 2) * sizeof(float);
    float *ws = att_workspace(bytes, st);
    if (!ws) return shape_error("attention: key-split scratch unavailable (allocation failed, or first use inside a stream capture)");
    const dim3 gs(B * T, KV, NS);
#define LBC_ATS(DD, F)                                                                                        \
  {                                                                                                           \
    attention_split_kernel<DD, F><<<gs, ATT_SPLIT_THREADS, 0, st>>>(q, bias, cos_t, sin_t, k_cache, v_cache, pos, \
                                                                  ws, T, H, KV, S_max, NS, scale);            \
    attention_combine_kernel<DD><<<grid, 256, 0, st>>>(ws, pos, out, T, H, KV, NS);                           \
  }
    if (fuse) {
      if (D == 32) LBC_ATS(32, true) else if (D == 64) LBC_ATS(64, true) else LBC_ATS(128, true)
    } else {
      if (D == 32) LBC_ATS(32, false) else if (D == 64) LBC_ATS(64, false) else LBC_ATS(128, false)
    }
#undef LBC_ATS
    return launch_status("attention (key split)");
  }
  const size_t smem = ((size_t)G * D * (1 + ATT_THREADS / D) + (size_t)G * S_max) * sizeof(float);
  if (smem > (size_t)optin) return shape_error("attention: KV cache longer than shared memory allows");
#define LBC_ATT(DD, F)                                                                                     \
  {                                                                                                        \
    auto k = attention_kernel<DD, F>;                                                                      \
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);   \
    k<<<grid, ATT_THREADS, smem, st>>>(q, bias, cos_t, sin_t, k_cache, v_cache, pos, out, T, H, KV, S_max,   \
                                       scale);                                                             \
  }
  if (fuse) {
    if (D == 32) LBC_ATT(32, true) else if (D == 64) LBC_ATT(64, true) else LBC_ATT(128, true)
  } else {
    if (D == 32) LBC_ATT(32, false) else if (D == 64) LBC_ATT(64, false) else LBC_ATT(128, false)
  }
#undef LBC_ATT
  return launch_status("attention");
}
}  // namespace
}  // namespace lbc

extern "C" {

int lbc_attention(const float *q, const float *k_cache, const float *v_cache, const int32_t *pos, float *out,
                  int B, int T, int H, int KV, int D, int S_max, void *stream) {
  return attention_launch(q, nullptr, nullptr, nullptr, const_cast<float *>(k_cache), const_cast<float *>(v_cache),
                          pos, out, B, T, H, KV, D, S_max, false, static_cast<cudaStream_t>(stream));
}

int lbc_rope_attention(const float *qkv, const float *bias, const float *cos_t, const float *sin_t,
                       const int32_t *pos, float *k_cache, float *v_cache, float *out, int B, int H, int KV, int D,
                       int S_max, void *stream) {
  if (D % 2) return shape_error("rope_attention: odd head_dim");
  return attention_launch(qkv, bias, cos_t, sin_t, k_cache, v_cache, pos, out, B, 1, H, KV, D, S_max, true,
                          static_cast<cudaStream_t>(stream));
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
