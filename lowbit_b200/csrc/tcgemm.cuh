// Tensor-core fused dequantize + GEMM (tcgen05, sm_100a).
//
// Y[M,N] = X[M,K] . W[N,K]^T with the weights dequantized straight into
// tensor memory (TMEM) as the MMA's A operand and the activations as the B
// operand in shared memory:
//
//   * work unit = 128 weight rows (one MMA M) x 256 K elements (two 128-element
//     groups); units are numbered tile-major and each persistent CTA takes a
//     contiguous range of them (split-K across CTAs where a range crosses a
//     tile), flushing per-row partial sums into Y with red.global.add;
//   * warp roles (320 threads): 8 "row warps" -- thread = weight row = TMEM
//     lane, warp w handles lane quadrant w%4 and group w/4 of each unit --
//     read the packed codes from a 128-byte-swizzled TMA tile, decode them in
//     registers and tcgen05.st them into an A buffer; warp 8 streams weight
//     tiles (2-D TMA) and activation blocks (1-D bulk copies) into a
//     `stages`-deep ring; warp 9 allocates TMEM and issues the MMAs;
//   * per group of 128 K the MMA writes its own accumulator D_g (a ring of 4 in
//     TMEM); the row warps read it back and apply the group scale in fp32, so
//     the quantized values themselves are exact in the MMA's input format:
//       W4A16 : A = (q - z) in bf16 (exact), B = X split into three bf16
//               pieces x = b1 + b2 + b3 (exact to ~2^-25), D fp32;
//       W4A8  : A = q (u8), B = xq (s8), D int32 exact; the epilogue forms
//               D - z*asum[m,g] exactly as the reference does;
//       MXFP4 : A = e2m1(q) * 2^(e-127) in bf16 (exact), B = three bf16 pieces;
//   * the contraction order inside a unit is a fixed permutation of k chosen so
//     that decoding needs the fewest instructions; the prep kernel writes B in
//     the same permuted order (a permutation of k applied to both operands does
//     not change A . B^T).
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gemv.cuh"  // FMT_* ids, opaque(), prmt
#include "tc.cuh"

namespace lbc {

constexpr int TC_KB = 256;     // K elements per work unit
constexpr int TC_ROWS = 128;   // weight rows per tile (MMA M)
constexpr int TC_THREADS = 320;
constexpr int TC_WBYTES = 16384;  // 128 rows x 128 bytes of packed codes per unit
constexpr int TC_DCOL0 = 256;     // first TMEM column of the accumulator ring

struct TcArgs {
  const float *scales;   // [N, G] (int4)
  const uint8_t *zeros;  // [N, G] or nullptr
  const uint8_t *e8m0;   // [N, Kp/32] (MXFP4)
  const uint8_t *bglob;  // activation blocks: [chunks][nkb][b_block_bytes]
  const int32_t *asum;   // W4A8: [M, G]
  const float *xs;       // W4A8: [M]
  float *y;              // [M, N], zeroed by the prep kernel
  int M, N, Kp, G;
  int nkb;               // K blocks per row: ceil(Kp / 256)
  int ntiles;            // ceil(N / 128)
  int units;             // ntiles * nkb
  int stages;
  int b_block_bytes;     // bytes of one activation block
  int mt;                // tokens per chunk (rows of B per piece)
  int *status;
};

__host__ __device__ constexpr int tc_nmma(int mt, int npiece) {
  return ((mt * npiece + 15) / 16) * 16;
}

struct TcSmem {
  int w_off, b_off, bar_off, total;
};

__host__ __device__ inline TcSmem tc_smem_layout(int stages, int b_block_bytes) {
  TcSmem L;
  L.w_off = 0;  // 1024-aligned (128-byte swizzle atoms)
  L.b_off = stages * TC_WBYTES;
  L.bar_off = L.b_off + stages * ((b_block_bytes + 127) / 128 * 128);
  // full[S], empty[S], a_full[2], a_empty[2], d_full[4], d_empty[4], final, tmem slot
  L.total = L.bar_off + 8 * (2 * stages + 13) + 16 + 1024;  // + alignment slack
  return L;
}

// ------------------------------------------------------------------ PTX bits
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(c));
  return d;
}

// 16 bytes of row r, chunk c of a 128-byte-swizzled tile (TMA SWIZZLE_128B):
// the chunk sits at position c ^ (r % 8) of its 128-byte row.
__device__ __forceinline__ uint4 lds_swz(const uint8_t *tile, int r, int c) {
  return *reinterpret_cast<const uint4 *>(tile + r * 128 + ((c ^ (r & 7)) << 4));
}

// bf16 bits of 2^(e-128) (half the E8M0 scale), e=255 -> NaN
__device__ __forceinline__ uint32_t e8m0_half_bf16(uint32_t e) {
  if (e == 255u) return 0x7FC0u;
  if (e >= 2u) return (e - 1u) << 7;
  return 0x0020u << e;  // 2^-128 (e=0) or 2^-127 (e=1), subnormal
}

// ------------------------------------------------------------------ decoders
// Each decoder fills the TMEM columns of one (row, group) of a unit.
// W4A16 -> 64 columns of bf16 pairs (q - z); column cc*16 + i*4 + p of chunk
// cc, word i holds the pair selected by nibble shift 4p of that word.
__device__ __forceinline__ void deq_w4a16(const uint8_t *tile, int r, int h, uint32_t z,
                                          uint32_t (&av)[64], uint32_t MAG) {
  const uint32_t zz = (0x4300u | z) * 0x00010001u;  // bf16 pair (128+z, 128+z)
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const uint4 v = lds_swz(tile, r, 4 * h + cc);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t w = w4[i];
      av[cc * 16 + i * 4 + 0] = bf16x2_sub(lop_and_or(w, 0x000F000Fu, MAG), zz);
      av[cc * 16 + i * 4 + 1] = bf16x2_sub(lop_and_or(w >> 4, 0x000F000Fu, MAG), zz);
      av[cc * 16 + i * 4 + 2] = bf16x2_sub(lop_and_or(w >> 8, 0x000F000Fu, MAG), zz);
      av[cc * 16 + i * 4 + 3] = bf16x2_sub(lop_and_or(w >> 12, 0x000F000Fu, MAG), zz);
    }
  }
}

// W4A8 -> 32 columns of u8 codes; column cc*8 + i*2 + {0: low nibbles, 1: high}
__device__ __forceinline__ void deq_w4a8(const uint8_t *tile, int r, int h, uint32_t (&av)[64]) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const uint4 v = lds_swz(tile, r, 4 * h + cc);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      av[cc * 8 + i * 2 + 0] = w4[i] & 0x0F0F0F0Fu;
      av[cc * 8 + i * 2 + 1] = (w4[i] >> 4) & 0x0F0F0F0Fu;
    }
  }
}

// MXFP4 -> 64 columns of bf16 pairs e2m1(q) * 2^(e-127) (exact in bf16).
// Chunk cc of the group is block cc; column cc*16 + i*4 + half*2 + ab holds
// (low, high) elements of byte 2*half + ab of word i.
__device__ __forceinline__ void deq_mxfp4(const uint8_t *tile, int r, int h, const uint32_t (&e4)[4],
                                          uint32_t (&av)[64]) {
  const uint32_t TP0 = 0x13121110u, TP1 = 0x1C181614u;  // 16 + {0,1,2,3}, 16 + {4,6,8,12}
  const uint32_t TN0 = 0x0D0E0F10u, TN1 = 0x04080A0Cu;  // 16 - {0,1,2,3}, 16 - {4,6,8,12}
  const uint32_t HI = opaque(0x00000043u);
  const uint32_t B144 = 0x43104310u;  // bf16 pair (144, 144)
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const uint4 v = lds_swz(tile, r, 4 * h + cc);
    const uint32_t sc = e8m0_half_bf16(e4[cc]) * 0x00010001u;
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t w = w4[i];
      const uint32_t m = w & 0x77777777u;
      const uint32_t w4s = w << 4;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t sel = half ? (m >> 16) : m;
        const uint32_t pos = prmt(TP0, TP1, sel);
        const uint32_t neg = prmt(TN0, TN1, sel);
        const uint32_t msk = prmt(w4s, w, half ? 0xFBEAu : 0xD9C8u);
        const uint32_t val = (pos & ~msk) | (neg & msk);  // bytes 16 + 2*e2m1
        // bf16 pairs (144 + 2e) -> 2e -> 2e * 2^(E-128)
        const uint32_t pa = prmt(val, HI, 0x4140u);
        const uint32_t pb = prmt(val, HI, 0x4342u);
        av[cc * 16 + i * 4 + half * 2 + 0] = bf16x2_mul(bf16x2_sub(pa, B144), sc);
        av[cc * 16 + i * 4 + half * 2 + 1] = bf16x2_mul(bf16x2_sub(pb, B144), sc);
      }
    }
  }
}

// ------------------------------------------------------------------ kernel
template <int FMT, int MT, int NPIECE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tcgemm_kernel(const __grid_constant__ CUtensorMap wmap, const TcArgs a) {
  constexpr int NMMA = tc_nmma(MT, NPIECE);
  constexpr bool I8 = (FMT == FMT_W4A8);
  constexpr int GCOLS = I8 ? 32 : 64;   // TMEM columns per (row, group)
  constexpr int ACOLS = 2 * GCOLS;      // per unit (A buffer)
  constexpr int KSTEP = I8 ? 32 : 16;   // K per MMA instruction
  constexpr int NSTEP = 128 / KSTEP;    // MMAs per group
  static_assert(2 * ACOLS <= TC_DCOL0 && TC_DCOL0 + 4 * NMMA <= 512, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int S = a.stages;
  const TcSmem L = tc_smem_layout(S, a.b_block_bytes);
  const int BSTRIDE = (a.b_block_bytes + 127) / 128 * 128;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *full = bars, *empty = bars + S;
  uint64_t *a_full = bars + 2 * S, *a_empty = a_full + 2;
  uint64_t *d_full = a_empty + 2, *d_empty = d_full + 4, *fin = d_empty + 4;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chunk = blockIdx.y;
  const int u0 = (int)((long long)blockIdx.x * a.units / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * a.units / gridDim.x);
  const int nunits = u1 - u0;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 9);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&a_full[b], 8);
      mbar_init(&a_empty[b], 1);
    }
    for (int d = 0; d < 4; ++d) {
      mbar_init(&d_full[d], 1);
      mbar_init(&d_empty[d], 4);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tc::alloc(tmem_slot, 512);
    tc::relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t *bsrc = a.bglob + (size_t)chunk * a.nkb * a.b_block_bytes;
      const int pro = min(S, nunits);
      // weights are static: start them before the activation blocks exist
      for (int i = 0; i < pro; ++i) {
        const int u = u0 + i;
        mbar_expect_tx(&full[i], (uint32_t)(TC_WBYTES + a.b_block_bytes));
        tma_load_2d(smem + L.w_off + i * TC_WBYTES, &wmap, (u % a.nkb) * 128, (u / a.nkb) * TC_ROWS,
                    &full[i], pol);
      }
      pdl_wait_prior_grid();
      for (int i = 0; i < pro; ++i)
        bulk_g2s(smem + L.b_off + i * BSTRIDE, bsrc + (size_t)((u0 + i) % a.nkb) * a.b_block_bytes,
                 (uint32_t)a.b_block_bytes, &full[i], pol);
      for (int i = pro; i < nunits && !*abort_flag; ++i) {
        const int s = i % S;
        if (!mbar_wait(&empty[s], ((uint32_t)(i / S) & 1u) ^ 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        const int u = u0 + i;
        mbar_expect_tx(&full[s], (uint32_t)(TC_WBYTES + a.b_block_bytes));
        tma_load_2d(smem + L.w_off + s * TC_WBYTES, &wmap, (u % a.nkb) * 128, (u / a.nkb) * TC_ROWS,
                    &full[s], pol);
        bulk_g2s(smem + L.b_off + s * BSTRIDE, bsrc + (size_t)(u % a.nkb) * a.b_block_bytes,
                 (uint32_t)a.b_block_bytes, &full[s], pol);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = I8 ? tc::idesc_s8_s32(NMMA) : tc::idesc_bf16_f32(NMMA);
      // W4A8: A holds unsigned codes (a_fmt = 0), B signed activations
      const uint32_t idesc_i8u = idesc & ~(7u << 7);
      for (int i = 0; i < nunits && !*abort_flag; ++i) {
        const int s = i % S, ab = i & 1;
        if (!mbar_wait(&full[s], (uint32_t)(i / S) & 1u, a.status) ||
            !mbar_wait(&a_full[ab], (uint32_t)(i >> 1) & 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        tc::fence_after_sync();
        const uint32_t bbase = smem_u32(smem + L.b_off + s * BSTRIDE);
        // B row groups (8 rows) are 256/8*128 (bf16) or 256/16*128 (s8) bytes apart
        const uint32_t sbo = I8 ? 2048u : 4096u;
        for (int h = 0; h < 2; ++h) {
          const int v = 2 * i + h, d = v & 3;
          if (!mbar_wait(&d_empty[d], ((uint32_t)(v >> 2) & 1u) ^ 1u, a.status)) {
            *abort_flag = 1;
            break;
          }
          tc::fence_after_sync();
          const uint32_t dcol = tmem + TC_DCOL0 + d * NMMA;
#pragma unroll
          for (int j = 0; j < NSTEP; ++j) {
            const uint32_t acol = tmem + ab * ACOLS + h * GCOLS + j * 8;
            // K offset of this step inside the block: 128h + KSTEP*j elements,
            // i.e. (that / (16 bytes per core-matrix row)) core matrices of 128 B
            const uint32_t koff = I8 ? (uint32_t)(128 * h + 32 * j) / 16u : (uint32_t)(128 * h + 16 * j) / 8u;
            const uint64_t bd = tc::smem_desc(bbase + koff * 128u, 128u, sbo);
            if (I8)
              tc::mma_s8_ts(dcol, acol, bd, idesc_i8u, j > 0);
            else
              tc::mma_bf16_ts(dcol, acol, bd, idesc, j > 0);
          }
          tc::commit(&d_full[d]);
        }
        tc::commit(&a_empty[ab]);
        tc::commit(&empty[s]);
      }
      // every MMA has completed before TMEM is released
      tc::commit(fin);
      mbar_wait(fin, 0, a.status);
    }
  } else {
    // ------------------------------------------------------------ row warps
    const int q = warp & 3, h = warp >> 2;
    const int row = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const uint32_t MAG = opaque(0x43004300u);
    const int NB32 = a.Kp >> 5;
    float yacc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) yacc[t] = 0.f;
    bool waited_prior = false;

    // per-unit metadata of this thread's (row, group)
    struct Meta {
      float s;
      uint32_t z;
      uint32_t e4[4];
    };
    auto load_meta = [&](int u) {
      Meta m;
      m.s = 0.f;
      m.z = 8u;
      m.e4[0] = m.e4[1] = m.e4[2] = m.e4[3] = 0u;
      const int n = (u / a.nkb) * TC_ROWS + row;
      const int g = 2 * (u % a.nkb) + h;
      if (n < a.N) {
        if (FMT == FMT_MXFP4) {
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int blk = 4 * g + b;
            m.e4[b] = blk < NB32 ? (uint32_t)__ldg(a.e8m0 + (size_t)n * NB32 + blk) : 0u;
          }
          m.s = 1.f;
        } else if (g < a.G) {
          m.s = __ldg(a.scales + (size_t)n * a.G + g);
          if (a.zeros) m.z = __ldg(a.zeros + (size_t)n * a.G + g);
        }
      }
      return m;
    };

    auto flush = [&](int tile) {
      if (!waited_prior) {
        pdl_wait_prior_grid();  // Y was zeroed by the prep kernel
        waited_prior = true;
      }
      const int n = tile * TC_ROWS + row;
      if (n < a.N) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int m = chunk * MT + t;
          if (m < a.M) {
            float v = yacc[t];
            if (FMT == FMT_W4A8) v *= __ldg(a.xs + m);
            atomicAdd(a.y + (size_t)m * a.N + n, v);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) yacc[t] = 0.f;
    };

    Meta mcur = load_meta(u0), mprev;
    mprev = mcur;
    bool ok = true;
    for (int i = 0; i <= nunits; ++i) {
      Meta mnext = mcur;
      if (i + 1 < nunits) mnext = load_meta(u0 + i + 1);
      if (i < nunits) {
        // ---------------------------------------------- dequantize unit i
        const int s = i % S, ab = i & 1;
        if (ok) ok = !*abort_flag && mbar_wait(&full[s], (uint32_t)(i / S) & 1u, a.status);
        uint32_t av[64];
        const uint8_t *tile = smem + L.w_off + s * TC_WBYTES;
        if (FMT == FMT_W4A16)
          deq_w4a16(tile, row, h, mcur.z, av, MAG);
        else if (FMT == FMT_W4A8)
          deq_w4a8(tile, row, h, av);
        else
          deq_mxfp4(tile, row, h, mcur.e4, av);
        if (ok) ok = !*abort_flag && mbar_wait(&a_empty[ab], ((uint32_t)(i >> 1) & 1u) ^ 1u, a.status);
        tc::fence_after_sync();
        const uint32_t at = tmem + lane_base + ab * ACOLS + h * GCOLS;
        if (ok) {
          uint32_t part[16];
#pragma unroll
          for (int c = 0; c < GCOLS / 16; ++c) {
#pragma unroll
            for (int j = 0; j < 16; ++j) part[j] = av[16 * c + j];
            tc::st16(at + 16 * c, part);
          }
          tc::wait_st();
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[ab]);
          mbar_arrive(&empty[s]);
        }
      }
      if (i > 0) {
        // ---------------------------------------------- epilogue of unit i-1
        const int v = 2 * (i - 1) + h, d = v & 3;
        if (ok) ok = !*abort_flag && mbar_wait(&d_full[d], (uint32_t)(v >> 2) & 1u, a.status);
        tc::fence_after_sync();
        uint32_t dv[NMMA];
        if (ok) {
#pragma unroll
          for (int c = 0; c < NMMA / 16; ++c) {
            uint32_t part[16];
            tc::ld16(tmem + lane_base + TC_DCOL0 + d * NMMA + 16 * c, part);
#pragma unroll
            for (int j = 0; j < 16; ++j) dv[16 * c + j] = part[j];
          }
          tc::wait_ld();
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_empty[d]);
        if (ok) {
          const int up = u0 + i - 1;
          if (FMT == FMT_W4A8) {
            const int g = 2 * (up % a.nkb) + h;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              const int m = chunk * MT + t;
              const int as = (m < a.M && g < a.G) ? __ldg(a.asum + (size_t)m * a.G + g) : 0;
              const int acc = (int)dv[t] - (int)mprev.z * as;
              yacc[t] = fmaf((float)acc, mprev.s, yacc[t]);
            }
          } else {
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              float sum = 0.f;
#pragma unroll
              for (int p = 0; p < NPIECE; ++p) sum += __uint_as_float(dv[p * MT + t]);
              yacc[t] = fmaf(sum, mprev.s, yacc[t]);
            }
          }
          const bool last = (i == nunits) || ((u0 + i) / a.nkb != up / a.nkb);
          if (last) flush(up / a.nkb);
        }
      }
      mprev = mcur;
      mcur = mnext;
    }
    if (!waited_prior) pdl_wait_prior_grid();
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 9) {
    tc::fence_after_sync();
    tc::dealloc(tmem, 512);
  }
}

}  // namespace lbc
