// W4A8 GEMM for 1-64 tokens (passes of up to 16, grid.y) on the tensor cores
// through mma.sync.m16n8k32 (s8 x s8 -> s32).
//
// The reference's W4A8 arithmetic (src/lowbit/csrc/kern_vnni.c:30-72,
// kern_scalar.c:49-59): y[m,n] = xs[m] * sum_g s[n,g] * (sum_{k in g} q*xq
// - z*sum_{k in g} xq), the group sums exact in int32. Here A = q - z as s8
// (|q - z| <= 15): the MMA's int32 accumulator of one 128-element group IS
// sum (q - z) * xq = sum q*xq - z*asum, exactly, so no zero-point term is
// needed afterwards; the group scale multiplies it into the row's fp32 sum
// in group order, the token scale at the store.
//
// Fragments: lane (g, t) (g = lane / 4, t = lane % 4) loads bytes
// [16t, 16t + 16) of rows g and g + 8 of a 16-row block in one group (the
// packed layout puts code j in the low nibble and code j + 64 in the high
// nibble of byte j), so word i of a row gives the s8 quads of elements
// 16t + 4i + [0, 4) (low nibbles) and 64 + 16t + 4i + [0, 4) (high): the A
// registers of k-step i for logical k = 4t + [0, 4) and 16 + 4t + [0, 4).
// The B fragment of token column c at k-step i is then the two 32-bit words
// of xq at those element positions, staged by each warp for its own groups
// in shared memory in fragment order (conflict-free 8-byte reads). Decoding
// a word into two s8 quads: (w & 0x0F0F0F0F) | 0x80808080 is 128 + q per
// byte, minus z per byte (no borrow: 128 + q - z >= 113), then xor 0x80
// gives q - z.
//
// Work: CTA c owns the 16-row blocks [c*B/P, (c+1)*B/P); its warps split
// every block's groups; each warp streams its (block, group) units' codes
// straight from HBM into registers DEPTH units ahead of the MMAs (16-byte
// loads, L1 no-allocate, L2 evict-first); per block the warps' fp32 partial
// sums are added in warp order through shared memory (deterministic).
#include <type_traits>

#include "gemv_dispatch.cuh"
#include "gemv_rows.cuh"

namespace lbc {

namespace {

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// two s8 quads (q - z) from one word of packed codes: low nibbles, high nibbles
__device__ __forceinline__ void s8_quads(uint32_t w, uint32_t zb, uint32_t &lo, uint32_t &hi) {
  lo = (((w & 0x0F0F0F0Fu) | 0x80808080u) - zb) ^ 0x80808080u;
  hi = ((((w >> 4) & 0x0F0F0F0Fu) | 0x80808080u) - zb) ^ 0x80808080u;
}

constexpr int I8_DEPTH = 4;  // units of codes in flight per warp ahead of the MMAs

}  // namespace

// Dynamic shared memory: B fragments [G][4 k-steps][NB][32 lanes] uint2, the
// warps' partial sums [NW][8 NB tokens][16 rows] fp32, token scales [8 NB].
__host__ __device__ inline int i8mma_smem_bytes(int nb, int nw, int Kp) {
  return (Kp / 128) * 4 * nb * 32 * 8 + nw * 16 * 8 * nb * 4 + 8 * nb * 4;
}

template <int NB, int NW>
__global__ void __launch_bounds__(NW * 32, 2) w4a8_mma_kernel(const GemvArgs a) {
  constexpr int TOK = 8 * NB;
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int G = a.Kp >> 7, RB = a.Kp >> 1;
  uint2 *bfrag = reinterpret_cast<uint2 *>(smem);
  float *part = reinterpret_cast<float *>(smem + (size_t)G * 4 * NB * 32 * 8);
  float *xs_s = part + NW * 16 * TOK;
  const int m0 = blockIdx.y * TOK;

  const int nrb = (a.N + 15) >> 4;
  const int rb0 = (int)((long long)blockIdx.x * nrb / gridDim.x);
  const int rb1 = (int)((long long)(blockIdx.x + 1) * nrb / gridDim.x);
  const int wg0 = warp * G / NW, wg1 = (warp + 1) * G / NW, ng = wg1 - wg0;
  const int nu = (rb1 - rb0) * ng;  // this warp's (block, group) units, block-major
  const bool has_z = a.zeros != nullptr;
  const uint64_t pol = policy_evict_first();

  // DEPTH units of codes in flight; a unit lives in slot u % DEPTH. Register
  // arrays are only indexed by constants (slot-templated code), so they stay
  // in registers. The issue position advances one unit at a time.
  uint4 wl[I8_DEPTH], wh[I8_DEPTH];
  float sl[I8_DEPTH], sh[I8_DEPTH];
  uint32_t zl[I8_DEPTH], zh[I8_DEPTH];
  int irb = rb0, ig = wg0;  // next unit to issue
  auto issue = [&](auto slot_c) {
    constexpr int S = decltype(slot_c)::value;
    const int r_lo = min(irb * 16 + gq, a.N - 1), r_hi = min(irb * 16 + gq + 8, a.N - 1);
    const size_t off = (size_t)ig * 64 + tq * 16;
    wl[S] = ldg_stream(a.qw + (size_t)r_lo * RB + off, pol);
    wh[S] = ldg_stream(a.qw + (size_t)r_hi * RB + off, pol);
    sl[S] = __ldg(a.scales + (size_t)r_lo * G + ig);
    sh[S] = __ldg(a.scales + (size_t)r_hi * G + ig);
    zl[S] = has_z ? (uint32_t)__ldg(a.zeros + (size_t)r_lo * G + ig) : 8u;
    zh[S] = has_z ? (uint32_t)__ldg(a.zeros + (size_t)r_hi * G + ig) : 8u;
    if (++ig == wg1) {
      ig = wg0;
      ++irb;
    }
  };

  // codes and metadata are static: the first units stream before the
  // previous kernel (which may produce the activations) has finished
  static_assert(I8_DEPTH == 4, "the prologue and the slot switch below issue four units");
  if (0 < nu) issue(std::integral_constant<int, 0>{});
  if (1 < nu) issue(std::integral_constant<int, 1>{});
  if (2 < nu) issue(std::integral_constant<int, 2>{});
  if (3 < nu) issue(std::integral_constant<int, 3>{});
  pdl_launch_dependents();
  pdl_wait_prior_grid();

  // B fragments of this pass's tokens for this warp's groups, in fragment
  // order (each warp reads only its own groups', so only a warp-level sync
  // stands between its staging and its MMAs). Item (g, n-block, lane) = the
  // two 16-byte runs of its token's codes at 16t and 64 + 16t in group g:
  // word j of each is the fragment of k-step j. All of a lane's loads are
  // issued before their stores (plain loads: the griddepcontrol.wait above
  // orders them after the producer kernel).
  static_assert(NB <= 2, "at most two n-blocks");
  constexpr int QMAX = 4 / NB;  // groups per warp staged per round
  for (int q0 = 0; q0 < ng; q0 += QMAX) {
    uint4 lo[QMAX][NB], hi[QMAX][NB];
#pragma unroll
    for (int q = 0; q < QMAX; ++q)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        lo[q][nb] = hi[q][nb] = make_uint4(0u, 0u, 0u, 0u);
        const int m = m0 + nb * 8 + gq;
        if (q0 + q < ng && m < a.M) {
          const int8_t *row = a.xq + (size_t)m * a.Kp + ((wg0 + q0 + q) << 7) + tq * 16;
          lo[q][nb] = *reinterpret_cast<const uint4 *>(row);
          hi[q][nb] = *reinterpret_cast<const uint4 *>(row + 64);
        }
      }
#pragma unroll
    for (int q = 0; q < QMAX; ++q)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        if (q0 + q < ng) {
          uint2 *dst = bfrag + ((size_t)(wg0 + q0 + q) * 4 * NB + nb) * 32 + lane;
          dst[0] = make_uint2(lo[q][nb].x, hi[q][nb].x);
          dst[NB * 32] = make_uint2(lo[q][nb].y, hi[q][nb].y);
          dst[2 * NB * 32] = make_uint2(lo[q][nb].z, hi[q][nb].z);
          dst[3 * NB * 32] = make_uint2(lo[q][nb].w, hi[q][nb].w);
        }
      }
  }
  for (int e = lane; e < TOK; e += 32)
    if (warp == 0) xs_s[e] = (m0 + e < a.M) ? ld_act(a.xs + m0 + e) : 0.f;
  __syncwarp();

  float y[NB][4];
  int u = 0;
  for (int rb = rb0; rb < rb1; ++rb) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) y[nb][e] = 0.f;
    for (int gi = 0; gi < ng; ++gi, ++u) {
      const int g = wg0 + gi;
      const uint2 *bf = bfrag + (size_t)g * 4 * NB * 32 + lane;
      auto unit = [&](auto slot_c) {
        constexpr int S = decltype(slot_c)::value;
        const uint4 w0 = wl[S], w1 = wh[S];
        const float s0 = sl[S], s1 = sh[S];
        const uint32_t zb0 = zl[S] * 0x01010101u, zb1 = zh[S] * 0x01010101u;
        if (u + I8_DEPTH < nu) issue(slot_c);
        const uint32_t wlo[4] = {w0.x, w0.y, w0.z, w0.w}, whi[4] = {w1.x, w1.y, w1.z, w1.w};
        int acc[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nb][e] = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t a0, a1, a2, a3;
          s8_quads(wlo[i], zb0, a0, a2);
          s8_quads(whi[i], zb1, a1, a3);
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            const uint2 b = bf[(i * NB + nb) * 32];
            mma_s8_16832(acc[nb], a0, a1, a2, a3, b.x, b.y);
          }
        }
        // the exact group sums, scaled into the rows' fp32 sums in group order
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          y[nb][0] = fmaf((float)acc[nb][0], s0, y[nb][0]);
          y[nb][1] = fmaf((float)acc[nb][1], s0, y[nb][1]);
          y[nb][2] = fmaf((float)acc[nb][2], s1, y[nb][2]);
          y[nb][3] = fmaf((float)acc[nb][3], s1, y[nb][3]);
        }
      };
      switch (u & (I8_DEPTH - 1)) {
        case 0: unit(std::integral_constant<int, 0>{}); break;
        case 1: unit(std::integral_constant<int, 1>{}); break;
        case 2: unit(std::integral_constant<int, 2>{}); break;
        default: unit(std::integral_constant<int, 3>{}); break;
      }
    }
    // the block's partial sums, token-major: [warp][token][row]; D fragment
    // (row gq, token 2tq + e) and (row gq + 8, token 2tq + e) of each n-block
    float *pw = part + warp * 16 * TOK;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int c = nb * 8 + 2 * tq;
      pw[c * 16 + gq] = y[nb][0];
      pw[(c + 1) * 16 + gq] = y[nb][1];
      pw[c * 16 + gq + 8] = y[nb][2];
      pw[(c + 1) * 16 + gq + 8] = y[nb][3];
    }
    __syncthreads();
    // sums over the warps in warp order (deterministic), token scale, store:
    // consecutive threads hold consecutive rows of one token (conflict-free
    // reads, 64-byte runs of Y)
    for (int e = tid; e < 16 * TOK; e += NW * 32) {
      const int r = e & 15, c = e >> 4;
      const int n = rb * 16 + r, m = m0 + c;
      float v = 0.f;
      for (int ww = 0; ww < NW; ++ww) v += part[ww * 16 * TOK + e];
      if (n < a.N && m < a.M) a.y[(size_t)m * a.N + n] = v * xs_s[c];
    }
    __syncthreads();
  }
}

namespace {

template <int NB, int NW>
cudaError_t i8mma_smem_attr(int smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  static int enabled[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && enabled[dev] >= smem) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(w4a8_mma_kernel<NB, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess && dev >= 0 && dev < 64) enabled[dev] = smem;
  return e;
}

template <int NB, int NW>
cudaError_t i8mma_launch_one(const GemvArgs &a, dim3 grid, cudaStream_t st) {
  const int smem = i8mma_smem_bytes(NB, NW, a.Kp);
  if (cudaError_t e = i8mma_smem_attr<NB, NW>(smem)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NW * 32, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, w4a8_mma_kernel<NB, NW>, a);
}

template <int NB, int NW>
int i8mma_occ_one(int smem) {
  int n = 0;
  if (i8mma_smem_attr<NB, NW>(smem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, w4a8_mma_kernel<NB, NW>, NW * 32, (size_t)smem) !=
          cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace

cudaError_t i8mma_launch(const GemvArgs &a, int nb, int nw, dim3 grid, cudaStream_t st) {
  if (nb == 1 && nw == 4) return i8mma_launch_one<1, 4>(a, grid, st);
  if (nb == 1 && nw == 8) return i8mma_launch_one<1, 8>(a, grid, st);
  if (nb == 2 && nw == 4) return i8mma_launch_one<2, 4>(a, grid, st);
  if (nb == 2 && nw == 8) return i8mma_launch_one<2, 8>(a, grid, st);
  return cudaErrorInvalidConfiguration;
}

int i8mma_smem(int nb, int nw, int Kp) { return i8mma_smem_bytes(nb, nw, Kp); }

int i8mma_occupancy(int nb, int nw, int smem) {
  if (nb == 1 && nw == 4) return i8mma_occ_one<1, 4>(smem);
  if (nb == 1 && nw == 8) return i8mma_occ_one<1, 8>(smem);
  if (nb == 2 && nw == 4) return i8mma_occ_one<2, 4>(smem);
  if (nb == 2 && nw == 8) return i8mma_occ_one<2, 8>(smem);
  return 0;
}

}  // namespace lbc
