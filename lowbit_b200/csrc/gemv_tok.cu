// Few-token SIMT GEMM (W4A16 and MXFP4, 2 to 16 tokens): one weight row per
// lane, eight tokens per pass.
//
// The decode kernel (gemv_rows.cuh) keeps a thread's activations in registers,
// which caps it at two fp32 tokens; the tensor-core path has a fixed cost of
// 10-18 us. Between them, a CTA first copies the pass's eight activation rows
// into shared memory transposed, xs[k][8] (so the eight values of one K
// position are 32 contiguous bytes), then each lane owns R weight rows and
// walks a range of K steps (16 bytes = 32 codes per row per step): for every
// code it reads xs[k][0..8) as two 16-byte broadcasts (every lane of the warp
// reads the same address) and accumulates (q - z) * x into eight fp32 sums
// with packed fp32x2 FMAs. Exactness is the decode kernel's: (q - z) is
// exact in fp32 (2^23 magic number), products and sums are fp32, and the
// group scale (or MXFP4 block scale) multiplies the group's sum once, as the
// reference does (src/lowbit/csrc/kern_scalar.c:10-47). The warps of a CTA
// split the CTA's K steps; their partial sums meet in shared memory and are
// added in warp order. Passes of eight tokens are the grid's y dimension;
// when rows alone give too few CTAs, K is split into ranges (grid z) whose
// partial results a second kernel adds in range order (deterministic).

#include "gemv_rows.cuh"
#include "kernels.h"

namespace lbc {

namespace {

constexpr int TOK_MT = 8;          // tokens per pass
constexpr int TOK_MAX_WARPS = 16;

struct TokArgs {
  const float *x;        // [M, Kp]
  const uint8_t *qw;     // [N, Kp/2]
  const float *scales;   // int4: [N, Kp/128]
  const uint8_t *zeros;  // int4: [N, Kp/128] or nullptr (z = 8)
  const uint8_t *e8m0;   // MXFP4: [N, Kp/32]
  float *y;              // [M, N]
  float *part;           // K split: [ks][M, N] partial sums, else unused
  int M, N, Kp;
  int ks;                // K ranges (grid z), whole units each (tok_unit_steps)
};

// K steps (32 elements) per unit of a K range: an int4 group, an MXFP4 block
constexpr int tok_unit_steps(int fmt) { return fmt == FMT_MXFP4 ? 1 : 4; }

// (v, v) + negc for the fp32 v whose bits are (w & 15) | mag, mag = 2^23:
// with negc = -(2^23 + z) twice, the exact code value q - z in both halves
__device__ __forceinline__ uint64_t dup_sub(uint32_t w, uint32_t mag, uint64_t negc) {
  uint64_t r;
  asm("{\n\t.reg .b32 v;\n\t.reg .b64 p;\n\t"
      "lop3.b32 v, %1, 15, %2, 0xEA;\n\t"
      "mov.b64 p, {v, v};\n\t"
      "add.rn.f32x2 %0, p, %3;\n\t}"
      : "=l"(r)
      : "r"(w), "r"(mag), "l"(negc));
  return r;
}

// shared memory: xs [K range][8] floats, then the warps' partial sums [warps][32 R][8]
inline int tok_smem_bytes(int krange, int warps, int r) { return (krange * TOK_MT + warps * 32 * r * TOK_MT) * 4; }

template <int FMT, int R>
__global__ void __launch_bounds__(TOK_MAX_WARPS * 32) gemv_tok_kernel(const TokArgs a) {
  constexpr int MT = TOK_MT, P = MT / 2;
  extern __shared__ __align__(16) float xs[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
  const int m0 = blockIdx.y * MT;
  constexpr int SPU = tok_unit_steps(FMT);
  const int G = a.Kp >> 7, NB32 = a.Kp >> 5, RB = a.Kp >> 1, U = (a.Kp >> 5) / SPU;
  // this CTA's K range: units [u0, u1), steps [c0, c0 + nst), elements [kbeg, kbeg + krange)
  const int u0 = (int)((long long)blockIdx.z * U / a.ks), u1 = (int)((long long)(blockIdx.z + 1) * U / a.ks);
  const int c0 = SPU * u0, nst = SPU * (u1 - u0);
  const int kbeg = 32 * c0, krange = 32 * nst;
  const int s0 = c0 + (int)((long long)warp * nst / W), s1 = c0 + (int)((long long)(warp + 1) * nst / W);
  const uint64_t pol = policy_evict_first();
  const uint32_t MAG = opaque(0x4B000000u);
  float *red = xs + (size_t)krange * MT;

  const uint8_t *qrow[R];
  int row[R];
#pragma unroll
  for (int j = 0; j < R; ++j) {
    row[j] = blockIdx.x * 32 * R + 32 * j + lane;
    qrow[j] = a.qw + (size_t)min(row[j], a.N - 1) * RB;
  }
  // the first step's codes stream before the previous kernel (which may
  // produce X) has finished
  auto load_step = [&](int c, uint4 (&w)[R]) {
#pragma unroll
    for (int j = 0; j < R; ++j) w[j] = ldg_stream(qrow[j] + 16 * c, pol);
  };
  uint4 wn[R];
  if (s0 < s1) load_step(s0, wn);
  pdl_launch_dependents();
  pdl_wait_prior_grid();

  // xs[k - kbeg][t] = x[m0 + t][k] (0 past M): coalesced along k, 32-byte rows
  for (int kk = threadIdx.x; kk < krange; kk += blockDim.x) {
    const int k = kbeg + kk;
    float v[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) v[t] = (m0 + t < a.M) ? ld_act(a.x + (size_t)(m0 + t) * a.Kp + k) : 0.f;
    float4 *d = reinterpret_cast<float4 *>(xs + (size_t)kk * MT);
    d[0] = make_float4(v[0], v[1], v[2], v[3]);
    d[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();

  uint64_t yacc[R][P], acc[R][P];
#pragma unroll
  for (int j = 0; j < R; ++j)
#pragma unroll
    for (int p = 0; p < P; ++p) yacc[j][p] = acc[j][p] = 0ull;

  auto fold = [&](int j, float s) {
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const float lo = __fmaf_rn(lo_f(acc[j][p]), s, lo_f(yacc[j][p]));
      const float hi = __fmaf_rn(hi_f(acc[j][p]), s, hi_f(yacc[j][p]));
      yacc[j][p] = pack2(__float_as_uint(lo), __float_as_uint(hi));
      acc[j][p] = 0ull;
    }
  };

  for (int c = s0; c < s1; ++c) {
    uint4 w[R];
#pragma unroll
    for (int j = 0; j < R; ++j) w[j] = wn[j];
    if (c + 1 < s1) load_step(c + 1, wn);
    const int g = c >> 2;
    uint64_t negc[R];
    float scale[R];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int n = min(row[j], a.N - 1);
      if (FMT == FMT_MXFP4) {
        negc[j] = 0ull;
        scale[j] = e8m0_half_scale(__ldg(a.e8m0 + (size_t)n * NB32 + c));
      } else {
        const uint32_t z = a.zeros ? (uint32_t)__ldg(a.zeros + (size_t)n * G + g) : 8u;
        negc[j] = pack2(0xCB000000u | z, 0xCB000000u | z);  // -(2^23 + z)
        scale[j] = __ldg(a.scales + (size_t)n * G + g);
      }
    }
    // byte b of the step holds elements k0 + b (low nibble) and k0 + hstep + b
    // (high nibble): int4 groups pair j with 64 + j, MXFP4 blocks j with 16 + j
    const int k0 = (FMT == FMT_MXFP4) ? 32 * c : 128 * g + 16 * (c & 3);
    constexpr int hstep = (FMT == FMT_MXFP4) ? 16 : 64;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
#pragma unroll
      for (int hl = 0; hl < 2; ++hl) {
        const int k = k0 + b + hstep * hl;
        const float4 *xp = reinterpret_cast<const float4 *>(xs + (size_t)(k - kbeg) * MT);
        const float4 xa = xp[0], xb = xp[1];
        const uint64_t xv[P] = {pack2(__float_as_uint(xa.x), __float_as_uint(xa.y)),
                                pack2(__float_as_uint(xa.z), __float_as_uint(xa.w)),
                                pack2(__float_as_uint(xb.x), __float_as_uint(xb.y)),
                                pack2(__float_as_uint(xb.z), __float_as_uint(xb.w))};
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const uint32_t word = (b < 4) ? w[j].x : (b < 8) ? w[j].y : (b < 12) ? w[j].z : w[j].w;
          const uint32_t sh = word >> (8 * (b & 3) + 4 * hl);
          uint64_t v;
          if (FMT == FMT_MXFP4) {
            // E2M1 magnitude times 2 (0,1,2,3,4,6,8,12) with the sign, an
            // exact fp32; the block scale carries the factor 1/2
            const uint32_t code = sh & 15u;
            const uint32_t i3 = code & 7u;
            const uint32_t m2 = (i3 < 4u) ? i3 : ((0x0C080604u >> (8 * (i3 & 3u))) & 0xFFu);
            const float f = __fsub_rn(__uint_as_float(0x4B000000u | m2), 8388608.0f);
            const float sf = (code & 8u) ? -f : f;
            v = pack2(__float_as_uint(sf), __float_as_uint(sf));
          } else {
            v = dup_sub(sh, MAG, negc[j]);
          }
#pragma unroll
          for (int p = 0; p < P; ++p) acc[j][p] = ffma2(v, xv[p], acc[j][p]);
        }
      }
    }
    // a group (int4) or block (MXFP4) ends with this step, or the warp's range does
    if (FMT == FMT_MXFP4 || (c & 3) == 3 || c + 1 == s1) {
#pragma unroll
      for (int j = 0; j < R; ++j) fold(j, scale[j]);
    }
  }

  // partial sums of the warps meet in shared memory; warp order is fixed
  // partial sums of the warps meet in shared memory as red[warp][token][row]
  // (consecutive rows in consecutive words: conflict-free stores and sums);
  // warp order is fixed
  float *mine = red + (size_t)warp * MT * 32 * R;
#pragma unroll
  for (int j = 0; j < R; ++j)
#pragma unroll
    for (int p = 0; p < P; ++p) {
      mine[(2 * p) * 32 * R + 32 * j + lane] = lo_f(yacc[j][p]);
      mine[(2 * p + 1) * 32 * R + 32 * j + lane] = hi_f(yacc[j][p]);
    }
  __syncthreads();
  for (int o = threadIdx.x; o < 32 * R * MT; o += blockDim.x) {
    // o = t * 32R + row: consecutive threads store consecutive rows of a token
    const int t = o / (32 * R), rl = o % (32 * R);
    const int n = blockIdx.x * 32 * R + rl, m = m0 + t;
    float s = 0.f;
    for (int ww = 0; ww < W; ++ww) s += red[(size_t)ww * MT * 32 * R + o];
    if (n < a.N && m < a.M) {
      if (a.ks == 1)
        a.y[(size_t)m * a.N + n] = s;
      else
        a.part[((size_t)blockIdx.z * a.M + m) * a.N + n] = s;
    }
  }
}

// y = the K ranges' partial sums added in range order (deterministic)
__global__ void __launch_bounds__(256) tok_reduce_kernel(const float *part, float *y, int MN, int ks) {
  pdl_launch_dependents();
  pdl_wait_prior_grid();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= MN) return;
  float s = 0.f;
  for (int z = 0; z < ks; ++z) s += ld_act(part + (size_t)z * MN + i);
  y[i] = s;
}

template <int FMT, int R>
cudaError_t tok_launch(const TokArgs &a, int warps, cudaStream_t st) {
  const int U = (a.Kp >> 5) / tok_unit_steps(FMT);
  const int smem = tok_smem_bytes(32 * tok_unit_steps(FMT) * ((U + a.ks - 1) / a.ks), warps, R);
  auto k = gemv_tok_kernel<FMT, R>;
  static int enabled[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && enabled[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    enabled[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + 32 * R - 1) / (32 * R), (a.M + TOK_MT - 1) / TOK_MT, a.ks);
  cfg.blockDim = dim3(warps * 32, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, a);
  if (e != cudaSuccess || a.ks == 1) return e;
  const int MN = a.M * a.N;
  cfg.gridDim = dim3((MN + 255) / 256, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&cfg, tok_reduce_kernel, (const float *)a.part, a.y, MN, a.ks);
}

}  // namespace

int tok_max_kp(int smem_optin) {
  // xs for a K range plus the largest reduction buffer (16 warps, R = 2)
  return (smem_optin / 4 - TOK_MAX_WARPS * 64 * TOK_MT) / TOK_MT / 128 * 128;
}

cudaError_t tok_gemm(int fmt, const GemvArgs &g, int r, int warps, int ks, float *part, cudaStream_t st) {
  if (g.M < 1 || g.M > 16 || warps < 1 || warps > TOK_MAX_WARPS || (r != 1 && r != 2) || ks < 1 ||
      ks > (g.Kp >> 5) / tok_unit_steps(fmt) || (ks > 1 && !part))
    return cudaErrorInvalidValue;
  const TokArgs a{g.x, g.qw, g.scales, g.zeros, g.e8m0, g.y, part, g.M, g.N, g.Kp, ks};
  if (fmt == FMT_MXFP4) return r == 1 ? tok_launch<FMT_MXFP4, 1>(a, warps, st) : tok_launch<FMT_MXFP4, 2>(a, warps, st);
  return r == 1 ? tok_launch<FMT_W4A16, 1>(a, warps, st) : tok_launch<FMT_W4A16, 2>(a, warps, st);
}

}  // namespace lbc
