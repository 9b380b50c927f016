// Tensor-core fused dequantize + GEMM (tcgen05, sm_100a).
//
// Y[M,N] = X[M,K] . W[N,K]^T with the weights dequantized straight into
// tensor memory (TMEM) as the MMA's A operand and the activations as the B
// operand in shared memory. One kernel per call, no preparation kernel:
//
//   * work unit = 128 weight rows (one MMA M) x 256 K elements (two 128-element
//     groups); units are numbered tile-major and each persistent CTA (one per
//     SM) takes a contiguous range of them (stream-K);
//   * warp roles (576 threads): 16 "row warps" -- thread = weight row = TMEM
//     lane; warp w handles lane quadrant w%4 and the 64-element K slice w/4
//     (group (w/4)/2, half (w/4)%2) of each unit -- decode the packed codes of
//     a 128-byte-swizzled TMA tile into registers and tcgen05.st them into an
//     A buffer. The first-half warps also read each group's accumulator back
//     and apply the group scale in fp32; for small token counts the
//     second-half warps write the unit's activation block (B) into shared
//     memory, otherwise B blocks prepared once per call are copied in by TMA.
//     Warp 16 streams the tiles (`stages`-deep ring); warp 17 owns TMEM and
//     issues the MMAs;
//   * per group of 128 K the MMA writes its own accumulator D_g (a ring of 4 in
//     TMEM), so the quantized values are exact in the MMA's input format:
//       W4A16 : A = (q - z) in bf16 (exact), B = X split into three bf16
//               pieces x = b1 + b2 + b3 (exact to ~2^-25), D fp32;
//       W4A8  : A = q (u8), B = xq (s8), D int32 exact; the epilogue forms
//               D - z*asum[m,g] exactly as the reference does;
//       MXFP4 : A = e2m1(q) * 2^(e-127) in bf16 (exact), B = three bf16 pieces;
//   * the contraction order inside a unit is a fixed permutation of k chosen so
//     that decoding needs the fewest instructions; B is written in the same
//     permuted order (a permutation of k applied to both operands does not
//     change A . B^T);
//   * a tile split between CTAs is finished without zeroing Y or atomics: a CTA
//     whose range starts inside a tile writes its partial rows to a workspace
//     slot and raises a per-call epoch flag; the CTA owning the tile's first
//     units (it reaches that tile last) adds the partials and stores Y.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "gemv.cuh"  // FMT_* ids, opaque(), prmt
#include "tc.cuh"

namespace lbc {

constexpr int TC_KB = 256;        // K elements per work unit
constexpr int TC_ROWS = 128;      // weight rows per tile (MMA M)
constexpr int TC_THREADS = 576;  // 16 row warps + producer warp + MMA warp
constexpr int TC_WBYTES = 16384;  // 128 rows x 128 bytes of packed codes per unit
constexpr int TC_DCOL0 = 256;     // first TMEM column of the accumulator ring

struct TcArgs {
  const float *x;        // fp formats: [M, Kp]
  const int8_t *xq;      // W4A8: [M, Kp]
  const float *scales;   // [N, G] (int4)
  const uint8_t *zeros;  // [N, G] or nullptr
  const uint8_t *e8m0;   // [N, Kp/32] (MXFP4)
  const int32_t *asum;   // W4A8: [M, G]
  const float *xs;       // W4A8: [M]
  float *y;              // [M, N]
  float *partial;        // fixup slots: [chunks][grid_x][128][mt]
  uint32_t *flags;       // fixup flags: [chunks][grid_x]
  const uint8_t *bglob;  // activation blocks [chunks][nkb][b_block_bytes] (TMA-fed B)
  uint32_t epoch;        // unique per call
  int M, N, Kp, G;
  int nkb;               // K blocks per row: ceil(Kp / 256)
  int ntiles;            // ceil(N / 128)
  int units;             // ntiles * nkb
  int stages;
  int b_block_bytes;     // bytes of one activation block in shared memory
  int *status;
};

__host__ __device__ constexpr int tc_nmma(int mt, int npiece) {
  return ((mt * npiece + 15) / 16) * 16;
}

struct TcSmem {
  int w_off, b_off, red_off, bar_off, total;
};

__host__ __device__ inline TcSmem tc_smem_layout(int stages, int b_block_bytes, int mt) {
  TcSmem L;
  L.w_off = 0;  // 1024-aligned (128-byte swizzle atoms)
  L.b_off = stages * TC_WBYTES;
  L.red_off = L.b_off + stages * ((b_block_bytes + 127) / 128 * 128);
  L.bar_off = L.red_off + TC_ROWS * mt * 4;
  // full[S], empty[S], a_full[2], a_empty[2], d_full[4], d_empty[4], fin, slot
  L.total = L.bar_off + 8 * (2 * stages + 13) + 32 + 1024;  // + alignment slack
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
__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ void st_release_u32(uint32_t *p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
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

// Element of a 128-element group that MMA position kk (0..127) contracts, for
// each format's decoder column order.
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

// ------------------------------------------------------------------ decoders
// Each decoder handles half a group (two 16-byte chunks, 64 elements) of one
// row: chunks c0 and c0+1 of the row's 128-byte tile row. Column indices are
// relative to the half group (the full group's order is chunk-major, so half
// hf of a group owns columns [hf*32, hf*32+32) for bf16 and [hf*16, +16) for u8).
// W4A16 -> 32 columns of bf16 pairs (q - z); column cc*16 + i*4 + p of chunk
// cc, word i holds the pair selected by nibble shift 4p of that word.
__device__ __forceinline__ void deq_w4a16(const uint8_t *tile, int r, int c0, uint32_t z,
                                          uint32_t (&av)[32], uint32_t MAG) {
  const uint32_t zz = (0x4300u | z) * 0x00010001u;  // bf16 pair (128+z, 128+z)
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint4 v = lds_swz(tile, r, c0 + cc);
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

// W4A8 -> 16 columns of u8 codes; column cc*8 + i*2 + {0: low nibbles, 1: high}
__device__ __forceinline__ void deq_w4a8(const uint8_t *tile, int r, int c0, uint32_t (&av)[32]) {
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint4 v = lds_swz(tile, r, c0 + cc);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      av[cc * 8 + i * 2 + 0] = w4[i] & 0x0F0F0F0Fu;
      av[cc * 8 + i * 2 + 1] = (w4[i] >> 4) & 0x0F0F0F0Fu;
    }
  }
}

// MXFP4 -> 32 columns of bf16 pairs e2m1(q) * 2^(e-127) (exact in bf16).
// Chunk cc is one block of 32; column cc*16 + i*4 + half*2 + ab holds the
// (low, high) elements of byte 2*half + ab of word i.
__device__ __forceinline__ void deq_mxfp4(const uint8_t *tile, int r, int c0, const uint32_t (&e2)[2],
                                          uint32_t (&av)[32]) {
  const uint32_t TP0 = 0x13121110u, TP1 = 0x1C181614u;  // 16 + {0,1,2,3}, 16 + {4,6,8,12}
  const uint32_t TN0 = 0x0D0E0F10u, TN1 = 0x04080A0Cu;  // 16 - {0,1,2,3}, 16 - {4,6,8,12}
  const uint32_t HI = opaque(0x00000043u);
  const uint32_t B144 = 0x43104310u;  // bf16 pair (144, 144)
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint4 v = lds_swz(tile, r, c0 + cc);
    const uint32_t sc = e8m0_half_bf16(e2[cc]) * 0x00010001u;
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
template <int FMT, int MT, int NPIECE, bool BTMA>
__global__ void __maxnreg__(96) tcgemm_kernel(const __grid_constant__ CUtensorMap wmap, const TcArgs a) {
  constexpr int NMMA = tc_nmma(MT, NPIECE);
  constexpr bool I8 = (FMT == FMT_W4A8);
  constexpr int GCOLS = I8 ? 32 : 64;   // TMEM columns per (row, group)
  constexpr int HCOLS = GCOLS / 2;      // per (row, half group)
  constexpr int ACOLS = 2 * GCOLS;      // per unit (A buffer)
  constexpr int KSTEP = I8 ? 32 : 16;   // K per MMA instruction
  constexpr int NSTEP = 128 / KSTEP;    // MMAs per group
  constexpr int SBO = I8 ? 2048 : 4096; // bytes between 8-row groups of B
  constexpr int NROWW = 16;             // row warps
  static_assert(2 * ACOLS <= TC_DCOL0 && TC_DCOL0 + 4 * NMMA <= 512, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int S = a.stages;
  const TcSmem L = tc_smem_layout(S, a.b_block_bytes, MT);
  const int BSTRIDE = (a.b_block_bytes + 127) / 128 * 128;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *full = bars, *empty = bars + S;
  uint64_t *a_full = bars + 2 * S, *a_empty = a_full + 2;
  uint64_t *d_full = a_empty + 2, *d_empty = d_full + 4, *fin = d_empty + 4;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float *red = reinterpret_cast<float *>(smem + L.red_off);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chunk = blockIdx.y;
  const int NCTA = gridDim.x;
  auto range_start = [&](int c) { return (int)((long long)c * a.units / NCTA); };
  const int u0 = range_start(blockIdx.x);
  const int u1 = range_start(blockIdx.x + 1);
  const int nunits = u1 - u0;
  const int bbytes_copy = a.b_block_bytes;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NROWW + 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&a_full[b], NROWW);
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
  if (warp == NROWW + 1) {
    tc::alloc(tmem_slot, 512);
    tc::relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == NROWW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t *bsrc = BTMA ? a.bglob + (size_t)chunk * a.nkb * a.b_block_bytes : nullptr;
      const uint32_t txb = (uint32_t)TC_WBYTES + (BTMA ? (uint32_t)bbytes_copy : 0u);
      const int pro = min(S, nunits);
      // weights are static: start streaming them before the previous kernel
      // (which may produce X or the activation blocks) has finished
      for (int i = 0; i < pro; ++i) {
        const int u = u0 + i;
        mbar_expect_tx(&full[i], txb);
        tma_load_2d(smem + L.w_off + i * TC_WBYTES, &wmap, (u % a.nkb) * 128, (u / a.nkb) * TC_ROWS,
                    &full[i], pol);
      }
      if (BTMA) {
        pdl_wait_prior_grid();
        for (int i = 0; i < pro; ++i)
          bulk_g2s(smem + L.b_off + i * BSTRIDE, bsrc + (size_t)((u0 + i) % a.nkb) * a.b_block_bytes,
                   (uint32_t)bbytes_copy, &full[i], pol);
      }
      for (int i = pro; i < nunits && !*abort_flag; ++i) {
        const int s = i % S;
        if (!mbar_wait(&empty[s], ((uint32_t)(i / S) & 1u) ^ 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        const int u = u0 + i;
        mbar_expect_tx(&full[s], txb);
        tma_load_2d(smem + L.w_off + s * TC_WBYTES, &wmap, (u % a.nkb) * 128, (u / a.nkb) * TC_ROWS,
                    &full[s], pol);
        if (BTMA)
          bulk_g2s(smem + L.b_off + s * BSTRIDE, bsrc + (size_t)(u % a.nkb) * a.b_block_bytes,
                   (uint32_t)bbytes_copy, &full[s], pol);
      }
    }
  } else if (warp == NROWW + 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc0 = I8 ? tc::idesc_s8_s32(NMMA) : tc::idesc_bf16_f32(NMMA);
      // W4A8: A holds unsigned codes (a_fmt = 0), B signed activations
      const uint32_t idesc = I8 ? (idesc0 & ~(7u << 7)) : idesc0;
      for (int i = 0; i < nunits && !*abort_flag; ++i) {
        const int s = i % S, ab = i & 1;
        if ((BTMA && !mbar_wait(&full[s], (uint32_t)(i / S) & 1u, a.status)) ||
            !mbar_wait(&a_full[ab], (uint32_t)(i >> 1) & 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        tc::fence_after_sync();
        const uint32_t bbase = smem_u32(smem + L.b_off + s * BSTRIDE);
        bool okd = true;
        for (int h = 0; h < 2 && okd; ++h) {
          const int v = 2 * i + h, d = v & 3;
          if (!mbar_wait(&d_empty[d], ((uint32_t)(v >> 2) & 1u) ^ 1u, a.status)) {
            *abort_flag = 1;
            okd = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t dcol = tmem + TC_DCOL0 + d * NMMA;
#pragma unroll
          for (int j = 0; j < NSTEP; ++j) {
            const uint32_t acol = tmem + ab * ACOLS + h * GCOLS + j * 8;
            // core matrices (16-byte rows) of K before this step, 128 B each
            const uint32_t koff = (uint32_t)(128 * h + KSTEP * j) / (I8 ? 16u : 8u);
            const uint64_t bd = tc::smem_desc(bbase + koff * 128u, 128u, (uint32_t)SBO);
            if (I8)
              tc::mma_s8_ts(dcol, acol, bd, idesc, j > 0);
            else
              tc::mma_bf16_ts(dcol, acol, bd, idesc, j > 0);
          }
          tc::commit(&d_full[d]);
        }
        if (!okd) break;
        tc::commit(&a_empty[ab]);
        tc::commit(&empty[s]);
      }
      // every MMA has completed before TMEM is released
      tc::commit(fin);
      mbar_wait(fin, 0, a.status);
    }
  } else {
    // ------------------------------------------------------------ row warps
    const int q = warp & 3, sl = warp >> 2;  // lane quadrant, K slice (0..3)
    const int g = sl >> 1, hf = sl & 1;      // group in the unit, half of the group
    const bool epi = (hf == 0);              // this warp reads the group's accumulator
    const int row = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const uint32_t MAG = opaque(0x43004300u);
    const int NB32 = a.Kp >> 5;
    float yacc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) yacc[t] = 0.f;

    if (!BTMA) {
      // B areas start zeroed: rows of absent tokens and padding stay zero
      for (int idx = tid; idx < S * BSTRIDE / 16; idx += NROWW * 32)
        reinterpret_cast<uint4 *>(smem + L.b_off)[idx] = make_uint4(0, 0, 0, 0);
      named_bar_sync(4, NROWW * 32);
    }
    // X (or xq, asum, the activation blocks) may come from the previous kernel
    pdl_wait_prior_grid();
    pdl_launch_dependents();

    struct Meta {
      float s;
      uint32_t z;
      uint32_t e2[2];
    };
    auto load_meta = [&](int u) {
      Meta m;
      m.s = 0.f;
      m.z = 8u;
      m.e2[0] = m.e2[1] = 0u;
      const int n = (u / a.nkb) * TC_ROWS + row;
      const int gi = 2 * (u % a.nkb) + g;  // global group index
      if (n < a.N) {
        if (FMT == FMT_MXFP4) {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const int blk = 4 * gi + 2 * hf + b;
            m.e2[b] = blk < NB32 ? (uint32_t)__ldg(a.e8m0 + (size_t)n * NB32 + blk) : 0u;
          }
          m.s = 1.f;
        } else if (gi < a.G) {
          if (epi) m.s = __ldg(a.scales + (size_t)n * a.G + gi);
          if (a.zeros) m.z = __ldg(a.zeros + (size_t)n * a.G + gi);
        }
      }
      return m;
    };
    auto prefetch_meta = [&](int u) {
      const int n = (u / a.nkb) * TC_ROWS + row;
      const int gi = 2 * (u % a.nkb) + g;
      if (n < a.N) {
        if (FMT == FMT_MXFP4) {
          if (4 * gi + 2 * hf < NB32) prefetch_l2(a.e8m0 + (size_t)n * NB32 + 4 * gi + 2 * hf);
        } else if (gi < a.G) {
          if (epi) prefetch_l2(a.scales + (size_t)n * a.G + gi);
          if (a.zeros) prefetch_l2(a.zeros + (size_t)n * a.G + gi);
        }
      }
    };

    // in-kernel B build (small token counts): the second-half warps own one
    // contraction position kk each
    const int kk = (warp >> 3) * 128 + (warp & 3) * 32 + lane;  // valid when !epi
    float xv[BTMA ? 1 : MT];
    int8_t qv[BTMA ? 1 : MT];
    auto load_x = [&](int u) {
      if (BTMA || epi) return;
      const int k = (u % a.nkb) * TC_KB + (kk >> 7) * 128 + tc_perm(FMT, kk & 127);
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int m = chunk * MT + t;
        const bool ok = m < a.M && k < a.Kp;
        if (I8)
          qv[t] = ok ? a.xq[(size_t)m * a.Kp + k] : (int8_t)0;
        else
          xv[t] = ok ? a.x[(size_t)m * a.Kp + k] : 0.f;
      }
    };
    auto build_b = [&](int s) {
      if (BTMA || epi) return;
      uint8_t *blk = smem + L.b_off + s * BSTRIDE;
      const int mlim = min(MT, a.M - chunk * MT);
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        if (t < mlim) {
          if (I8) {
            blk[(t >> 3) * SBO + (kk >> 4) * 128 + (t & 7) * 16 + (kk & 15)] = (uint8_t)qv[t];
          } else {
            // x = b1 + b2 + b3 exactly (each piece the bf16 rounding of the rest)
            float r = xv[t];
#pragma unroll
            for (int p = 0; p < NPIECE; ++p) {
              const uint16_t b = __bfloat16_as_ushort(__float2bfloat16_rn(r));
              r -= __uint_as_float((uint32_t)b << 16);
              const int n = p * MT + t;
              *reinterpret_cast<uint16_t *>(blk + (n >> 3) * SBO + (kk >> 3) * 128 + (n & 7) * 16 +
                                            (kk & 7) * 2) = b;
            }
          }
        }
      }
    };

    // ---- tile completion: the 8 accumulator warps call it at the same points
    const int tile_lo = u0 / a.nkb;
    const bool first_is_shared = (u0 % a.nkb) != 0;  // range starts inside a tile
    auto finish_tile = [&](int tile) {
      // combine the two groups of each row (warps 0-3: group 0, 8-11: group 1)
      if (g == 1) {
#pragma unroll
        for (int t = 0; t < MT; ++t) red[row * MT + t] = yacc[t];
      }
      named_bar_sync(2, 256);
      if (g == 0) {
#pragma unroll
        for (int t = 0; t < MT; ++t) yacc[t] += red[row * MT + t];
        const int n = tile * TC_ROWS + row;
        const int tend = (tile + 1) * a.nkb;
        const size_t slot = (size_t)chunk * NCTA + blockIdx.x;
        if (tile == tile_lo && first_is_shared) {
          // tail part of a tile begun by an earlier CTA: hand the partial over
          float *dst = a.partial + slot * (TC_ROWS * MT) + row * MT;
#pragma unroll
          for (int t = 0; t < MT; ++t) dst[t] = yacc[t];
          __threadfence();
          named_bar_sync(3, 128);
          if (row == 0) st_release_u32(a.flags + slot, a.epoch);
        } else {
          // this CTA holds the tile's first units: add later CTAs' parts
          for (int c = blockIdx.x + 1; c < NCTA && range_start(c) < tend; ++c) {
            if (row == 0) {
              const uint32_t *f = a.flags + (size_t)chunk * NCTA + c;
              bool seen = ld_acquire_u32(f) == a.epoch;
              const long long t0 = clock64();
              while (!seen) {
                seen = ld_acquire_u32(f) == a.epoch;
                if (!seen && clock64() - t0 > LBC_WAIT_CYCLES) {
                  set_status(a.status, LBC_ERR_TIMEOUT);
                  *abort_flag = 1;
                  break;
                }
              }
            }
            named_bar_sync(3, 128);
            const float *src = a.partial + ((size_t)chunk * NCTA + c) * (TC_ROWS * MT) + row * MT;
#pragma unroll
            for (int t = 0; t < MT; ++t) yacc[t] += __ldcg(src + t);
          }
          if (n < a.N) {
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              const int m = chunk * MT + t;
              if (m < a.M) {
                float v = yacc[t];
                if (FMT == FMT_W4A8) v *= __ldg(a.xs + m);
                a.y[(size_t)m * a.N + n] = v;
              }
            }
          }
        }
      }
      named_bar_sync(2, 256);
#pragma unroll
      for (int t = 0; t < MT; ++t) yacc[t] = 0.f;
    };

    Meta mcur = load_meta(u0), mprev = mcur;
    if (nunits > 0) load_x(u0);
    for (int p = 1; p <= 4 && p < nunits; ++p) prefetch_meta(u0 + p);
    bool ok = true;
    for (int i = 0; i <= nunits; ++i) {
      Meta mnext = mcur;
      if (i + 1 < nunits) mnext = load_meta(u0 + i + 1);
      if (i + 5 < nunits) prefetch_meta(u0 + i + 5);
      if (i < nunits) {
        // ---------------------------------------------- unit i: B and A
        const int s = i % S, ab = i & 1;
        if (ok) ok = !*abort_flag && mbar_wait(&full[s], (uint32_t)(i / S) & 1u, a.status);
        build_b(s);
        if (i + 1 < nunits) load_x(u0 + i + 1);
        uint32_t av[32];
        const uint8_t *tile = smem + L.w_off + s * TC_WBYTES;
        if (FMT == FMT_W4A16)
          deq_w4a16(tile, row, 4 * g + 2 * hf, mcur.z, av, MAG);
        else if (FMT == FMT_W4A8)
          deq_w4a8(tile, row, 4 * g + 2 * hf, av);
        else
          deq_mxfp4(tile, row, 4 * g + 2 * hf, mcur.e2, av);
        if (ok) ok = !*abort_flag && mbar_wait(&a_empty[ab], ((uint32_t)(i >> 1) & 1u) ^ 1u, a.status);
        tc::fence_after_sync();
        const uint32_t at = tmem + lane_base + ab * ACOLS + g * GCOLS + hf * HCOLS;
        if (ok) {
          uint32_t part[16];
#pragma unroll
          for (int c = 0; c < HCOLS / 16; ++c) {
#pragma unroll
            for (int j = 0; j < 16; ++j) part[j] = av[16 * c + j];
            tc::st16(at + 16 * c, part);
          }
          tc::wait_st();
        }
        tc::fence_before_sync();
        if (!BTMA) tc::fence_proxy_async_smem();  // B writes -> visible to the MMA
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[ab]);
          mbar_arrive(&empty[s]);
        }
      }
      if (epi && i > 0) {
        // ---------------------------------------------- epilogue of unit i-1
        const int v = 2 * (i - 1) + g, d = v & 3;
        if (ok) ok = !*abort_flag && mbar_wait(&d_full[d], (uint32_t)(v >> 2) & 1u, a.status);
        tc::fence_after_sync();
        // read the accumulator 16 columns at a time (column p*MT + t holds
        // piece p of token t) and sum the pieces in order
        float sum[MT];
        int32_t isum[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          sum[t] = 0.f;
          isum[t] = 0;
        }
        if (ok) {
#pragma unroll
          for (int c = 0; c < NMMA / 16; ++c) {
            uint32_t part[16];
            tc::ld16(tmem + lane_base + TC_DCOL0 + d * NMMA + 16 * c, part);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = 16 * c + j, p = col / MT, t = col % MT;
              if (p < NPIECE) {
                if (I8)
                  isum[t] = (int32_t)part[j];
                else
                  sum[t] += __uint_as_float(part[j]);
              }
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_empty[d]);
        const int up = u0 + i - 1;
        if (ok) {
          if (FMT == FMT_W4A8) {
            const int gi = 2 * (up % a.nkb) + g;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              const int m = chunk * MT + t;
              const int as = (m < a.M && gi < a.G) ? __ldg(a.asum + (size_t)m * a.G + gi) : 0;
              const int acc = isum[t] - (int)mprev.z * as;
              yacc[t] = fmaf((float)acc, mprev.s, yacc[t]);
            }
          } else {
#pragma unroll
            for (int t = 0; t < MT; ++t) yacc[t] = fmaf(sum[t], mprev.s, yacc[t]);
          }
        }
        const bool last = (i == nunits) || ((u0 + i) / a.nkb != up / a.nkb);
        if (last) finish_tile(up / a.nkb);
      }
      mprev = mcur;
      mcur = mnext;
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == NROWW + 1) {
    tc::fence_after_sync();
    tc::dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ B blocks
// Activation blocks for the TMA-fed variant: block (chunk, kb) is the B
// operand of every unit of K block kb for tokens [chunk*MT, chunk*MT+MT), in
// the permuted K order and canonical K-major layout the MMA reads, rows
// n = piece*MT + token, absent tokens / pieces / K positions zero. One CTA per
// block; each thread writes whole 16-byte rows (8 bf16 or 16 int8 values).
template <int FMT, int MT, int NPIECE>
__global__ void __launch_bounds__(256) tc_bblock_kernel(const float *__restrict__ x, const int8_t *__restrict__ xq,
                                                        uint8_t *__restrict__ out, int M, int Kp, int nkb,
                                                        int bbytes) {
  constexpr bool I8 = (FMT == FMT_W4A8);
  constexpr int SBO = I8 ? 2048 : 4096;
  constexpr int EPR = I8 ? 16 : 8;  // elements per 16-byte row
  const int kb = blockIdx.x, chunk = blockIdx.y;
  uint8_t *blk = out + ((size_t)chunk * nkb + kb) * bbytes;
  pdl_wait_prior_grid();
  pdl_launch_dependents();
  for (int idx = threadIdx.x; idx < bbytes / 16; idx += blockDim.x) {
    const int n8 = idx / (SBO / 16), rem = idx % (SBO / 16);
    const int n = n8 * 8 + (rem & 7);
    const int kk0 = (rem >> 3) * EPR;
    const int piece = n / MT, t = n % MT;
    const int m = chunk * MT + t;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (piece < NPIECE && m < M) {
#pragma unroll
      for (int e = 0; e < EPR; ++e) {
        const int kk = kk0 + e;
        const int k = kb * TC_KB + (kk >> 7) * 128 + tc_perm(FMT, kk & 127);
        if (k < Kp) {
          if (I8) {
            w[e >> 2] |= (uint32_t)(uint8_t)xq[(size_t)m * Kp + k] << (8 * (e & 3));
          } else {
            float r = x[(size_t)m * Kp + k];
            uint16_t b = 0;
#pragma unroll
            for (int p = 0; p < NPIECE; ++p) {
              b = __bfloat16_as_ushort(__float2bfloat16_rn(r));
              if (p == piece) break;
              r -= __uint_as_float((uint32_t)b << 16);
            }
            w[e >> 1] |= (uint32_t)b << (16 * (e & 1));
          }
        }
      }
    }
    reinterpret_cast<uint4 *>(blk)[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace lbc
