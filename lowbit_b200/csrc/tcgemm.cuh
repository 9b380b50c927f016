// Tensor-core fused dequantize + GEMM (tcgen05, sm_100a).
//
// Y[M,N] = X[M,K] . W[N,K]^T with the weights dequantized straight into
// tensor memory (TMEM) as the MMA's A operand and the activations as the B
// operand in shared memory:
//
//   * work unit = 128 weight rows (one MMA M) x 256 K elements (two 128-element
//     groups); units are numbered tile-major and each persistent CTA (one per
//     SM) takes a contiguous range of them (stream-K);
//   * warp roles (736 threads): 16 dequantising warps -- thread = weight row
//     = TMEM lane; warp w handles lane quadrant w%4 and the 64-element K slice
//     w/4 (group (w/4)/2, half (w/4)%2) of each unit -- decode the packed codes
//     of a 128-byte-swizzled TMA tile into registers and tcgen05.st them into
//     one of up to three A buffers; the activation blocks (B) are prepared
//     once per call by a small kernel and arrive by TMA with the weights
//     (the codes are read from the 128-byte swizzle: chunk c of row r sits at
//     position c ^ (r % 8) of its 128-byte row). Warp 16
//     streams the tiles (`stages`-deep ring), warps 17-18 issue the MMAs of
//     the unit's first and second group (warp 17 owns TMEM), warps 19-22 (one
//     per lane quadrant) read each group's accumulator back, apply the group
//     scale in fp32 and finish the tiles;
//   * unit indices advance incrementally (no integer division in the loops)
//     and each role loads the metadata of the next unit while working on the
//     current one;
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
//     units (it reaches that tile last) adds the partials, stores Y and clears
//     each flag it has seen, so a replay of a captured launch (same epoch)
//     finds every flag clear.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "gemv.cuh"  // FMT_* ids, opaque(), prmt
#include "tc.cuh"

namespace lbc {

constexpr int TC_KB = 256;        // K elements per work unit
constexpr int TC_ROWS = 128;      // weight rows per tile (MMA M)
constexpr int TC_THREADS = 736;   // 16 dequantising warps + producer + 2 MMA + 4 epilogue warps
constexpr int TC_WBYTES = 16384;  // 128 rows x 128 bytes of packed codes per unit

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
  int ksplit;            // prefill: K ranges per output tile (>= 1; > 1 adds into a zeroed Y)
  int *status;
  // prefill with the column-parallel all-gather fused into the store (ksplit
  // 1), else y_peers is nullptr: this rank's rows [row0, row0 + N) of every
  // output go to every rank's Y buffer of the call's parity
  float *const *y_peers;         // [2][world] Y buffers [M, ld_y] of every rank, by call parity
  uint32_t *const *flag_peers;   // [world] call counters of every rank: flag_peers[p][q] = calls of q seen by p
  uint32_t *ag_counter;          // this rank's CTA counter
  uint32_t *ag_epoch;            // this rank's call counter
  int rank, world, row0, ld_y;
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
  (void)mt;
  L.red_off = L.b_off + stages * ((b_block_bytes + 127) / 128 * 128);
  L.bar_off = L.red_off;
  // full[S], empty[S], a_full[3], a_empty[3], d_full[4], d_empty[4], fin, slot
  L.total = L.bar_off + 8 * (2 * stages + 15) + 32 + 1024;  // + alignment slack
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
// row, already loaded from the row's 128-byte tile row into registers. Column indices are
// relative to the half group (the full group's order is chunk-major, so half
// hf of a group owns columns [hf*32, hf*32+32) for bf16 and [hf*16, +16) for u8).
// W4A16 -> 32 columns of bf16 pairs (q - z); column cc*16 + i*4 + p of chunk
// cc, word i holds the pair selected by nibble shift 4p of that word.
__device__ __forceinline__ void deq_w4a16(const uint4 (&wv)[2], uint32_t z, uint32_t (&av)[32], uint32_t MAG) {
  const uint32_t zz = (0x4300u | z) * 0x00010001u;  // bf16 pair (128+z, 128+z)
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint4 v = wv[cc];
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
__device__ __forceinline__ void deq_w4a8(const uint4 (&wv)[2], uint32_t (&av)[32]) {
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint4 v = wv[cc];
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
__device__ __forceinline__ void deq_mxfp4(const uint4 (&wv)[2], const uint32_t (&e2)[2], uint32_t (&av)[32]) {
  const uint32_t TP0 = 0x13121110u, TP1 = 0x1C181614u;  // 16 + {0,1,2,3}, 16 + {4,6,8,12}
  const uint32_t TN0 = 0x0D0E0F10u, TN1 = 0x04080A0Cu;  // 16 - {0,1,2,3}, 16 - {4,6,8,12}
  const uint32_t HI = opaque(0x00000043u);
  const uint32_t B144 = 0x43104310u;  // bf16 pair (144, 144)
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const uint4 v = wv[cc];
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
// 23 warps: B200 splits an SM's 64K registers over 4 sub-partitions, so a
// sub-partition holding 6 of the warps allows 16384 / (6 * 32) -> 80 each.
// A buffers in TMEM: as many as fit next to the ring of 4 accumulators (<= 3)
__host__ __device__ constexpr int tc_nabuf(int fmt, int nmma) {
  return ((512 - 4 * nmma) / (fmt == FMT_W4A8 ? 64 : 128)) < 3 ? ((512 - 4 * nmma) / (fmt == FMT_W4A8 ? 64 : 128))
                                                               : 3;
}

template <int FMT, int MT, int NPIECE>
__global__ void __maxnreg__(80) tcgemm_kernel(const __grid_constant__ CUtensorMap wmap, const TcArgs a) {
  constexpr int NMMA = tc_nmma(MT, NPIECE);
  constexpr bool I8 = (FMT == FMT_W4A8);
  constexpr int GCOLS = I8 ? 32 : 64;   // TMEM columns per (row, group)
  constexpr int HCOLS = GCOLS / 2;      // per (row, half group)
  constexpr int ACOLS = 2 * GCOLS;      // per unit (A buffer)
  constexpr int NA = tc_nabuf(FMT, NMMA);
  constexpr int DCOL0 = NA * ACOLS;     // first column of the accumulator ring
  constexpr int KSTEP = I8 ? 32 : 16;   // K per MMA instruction
  constexpr int NSTEP = 128 / KSTEP;    // MMAs per group
  constexpr int SBO = I8 ? 2048 : 4096; // bytes between 8-row groups of B
  constexpr int NDQ = 16;               // dequantising warps
  constexpr int W_PROD = NDQ, W_MMA = NDQ + 1, W_EPI = NDQ + 3;
  constexpr int NPC = NPIECE * MT;      // accumulator columns in use
  static_assert(NA >= 2 && DCOL0 + 4 * NMMA <= 512, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int S = a.stages;
  const TcSmem L = tc_smem_layout(S, a.b_block_bytes, MT);
  const int BSTRIDE = (a.b_block_bytes + 127) / 128 * 128;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *full = bars, *empty = bars + S;
  uint64_t *a_full = bars + 2 * S, *a_empty = a_full + 3;
  uint64_t *d_full = a_empty + 3, *d_empty = d_full + 4, *fin = d_empty + 4;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chunk = blockIdx.y;
  const int NCTA = gridDim.x;
  auto range_start = [&](int c) { return (int)((long long)c * a.units / NCTA); };
  const int u0 = range_start(blockIdx.x);
  const int nunits = range_start(blockIdx.x + 1) - u0;
  const int tile0 = u0 / a.nkb, kb0 = u0 - tile0 * a.nkb;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NDQ + 2);
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&a_full[b], NDQ);
      mbar_init(&a_empty[b], 2);
    }
    for (int d = 0; d < 4; ++d) {
      mbar_init(&d_full[d], 1);
      mbar_init(&d_empty[d], 4);
    }
    mbar_init(fin, 2);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == W_MMA) {
    tc::alloc(tmem_slot, 512);
    tc::relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == W_PROD) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t *bsrc = a.bglob + (size_t)chunk * a.nkb * a.b_block_bytes;
      const uint32_t txb = (uint32_t)TC_WBYTES + (uint32_t)a.b_block_bytes;
      int tile = tile0, kb = kb0;
      const int pro = min(S, nunits);
      // weights are static: stream them before the previous kernel (which may
      // produce X or the activation blocks) has finished
      for (int i = 0; i < pro; ++i) {
        mbar_expect_tx(&full[i], txb);
        tma_load_2d(smem + L.w_off + i * TC_WBYTES, &wmap, kb * 128, tile * TC_ROWS, &full[i], pol);
        if (++kb == a.nkb) {
          kb = 0;
          ++tile;
        }
      }
      // the activation blocks come from the preparation kernel before this one
      pdl_wait_prior_grid();
      int kb2 = kb0;
      for (int i = 0; i < pro; ++i) {
        bulk_g2s(smem + L.b_off + i * BSTRIDE, bsrc + (size_t)kb2 * a.b_block_bytes, (uint32_t)a.b_block_bytes,
                 &full[i], pol);
        if (++kb2 == a.nkb) kb2 = 0;
      }
      // unit i uses stage i % S; its stage was last used by unit i - S, whose
      // release is phase i / S - 1 of empty[s]
      int s = pro % S;
      uint32_t ph = (uint32_t)(pro / S) & 1u;
      for (int i = pro; i < nunits; ++i) {
        if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&full[s], txb);
        tma_load_2d(smem + L.w_off + s * TC_WBYTES, &wmap, kb * 128, tile * TC_ROWS, &full[s], pol);
        bulk_g2s(smem + L.b_off + s * BSTRIDE, bsrc + (size_t)kb * a.b_block_bytes, (uint32_t)a.b_block_bytes,
                   &full[s], pol);
        if (++kb == a.nkb) {
          kb = 0;
          ++tile;
        }
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == W_MMA || warp == W_MMA + 1) {
    // ------------------------------------------------------------ MMA issuers
    // two issuing warps, one per group of the unit: an MMA instruction keeps
    // its issuing thread busy for tens of cycles, two issuers double the rate
    if (lane == 0) {
      const int h = warp - W_MMA;
      const uint32_t idesc0 = I8 ? tc::idesc_s8_s32(NMMA) : tc::idesc_bf16_f32(NMMA);
      // W4A8: A holds unsigned codes (a_fmt = 0), B signed activations
      const uint32_t idesc = I8 ? (idesc0 & ~(7u << 7)) : idesc0;
      // group h starts 128 K (16 core matrices bf16, 8 int8) into the block;
      // each MMA step advances 2 core matrices (16 bytes of descriptor address)
      const uint32_t hoff = (uint32_t)(128 * h) / (I8 ? 16u : 8u) * 128u;
      int s = 0, ab = 0;
      uint32_t ph = 0, aph = 0;
      for (int i = 0; i < nunits && !*abort_flag; ++i) {
        const int v = 2 * i + h, d = v & 3;
        if (!mbar_wait(&full[s], ph, a.status) || !mbar_wait(&a_full[ab], aph, a.status) ||
            !mbar_wait(&d_empty[d], ((uint32_t)(v >> 2) & 1u) ^ 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        tc::fence_after_sync();
        const uint64_t bd0 = tc::smem_desc(smem_u32(smem + L.b_off + s * BSTRIDE) + hoff, 128u, (uint32_t)SBO);
        const uint32_t dcol = tmem + DCOL0 + d * NMMA;
        const uint32_t acol0 = tmem + ab * ACOLS + h * GCOLS;
#pragma unroll
        for (int j = 0; j < NSTEP; ++j) {
          if (I8)
            tc::mma_s8_ts(dcol, acol0 + 8 * j, bd0 + 16u * j, idesc, j > 0);
          else
            tc::mma_bf16_ts(dcol, acol0 + 8 * j, bd0 + 16u * j, idesc, j > 0);
        }
        tc::commit(&d_full[d]);
        tc::commit(&a_empty[ab]);
        tc::commit(&empty[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
        if (++ab == NA) {
          ab = 0;
          aph ^= 1u;
        }
      }
      // every MMA has completed before TMEM is released
      tc::commit(fin);
      mbar_wait(fin, 0, a.status);
    }
  } else if (warp < NDQ) {
    // ------------------------------------------------------------ dequantisers
    const int q = warp & 3, sl = warp >> 2;  // lane quadrant, K slice (0..3)
    const int g = sl >> 1, hf = sl & 1;      // group in the unit, half of the group
    const int row = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const uint32_t MAG = opaque(0x43004300u);
    const int NB32 = a.Kp >> 5;
    // per-(row, group) decode metadata of a unit
    struct Meta {
      uint32_t z;
      uint32_t e2[2];
    };
    auto load_meta = [&](int tile, int kb) {
      Meta m;
      m.z = 8u;
      m.e2[0] = m.e2[1] = 0u;
      const int n = tile * TC_ROWS + row;
      const int gi = 2 * kb + g;
      if (n < a.N) {
        if (FMT == FMT_MXFP4) {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const int blk = 4 * gi + 2 * hf + b;
            m.e2[b] = blk < NB32 ? (uint32_t)__ldg(a.e8m0 + (size_t)n * NB32 + blk) : 0u;
          }
        } else if (FMT == FMT_W4A16 && a.zeros && gi < a.G) {
          m.z = __ldg(a.zeros + (size_t)n * a.G + gi);
        }
      }
      return m;
    };
    auto advance = [&](int &tile, int &kb) {
      if (++kb == a.nkb) {
        kb = 0;
        ++tile;
      }
    };
    // metadata through a 4-deep register queue: the loads for unit i + 4 are
    // issued while unit i is decoded, so HBM latency never stalls a unit
    int tq = tile0, kq = kb0;  // position of unit i + 4 once the queue is primed
    Meta mq[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mq[j] = load_meta(tq, kq);
      advance(tq, kq);
    }
    // the codes of unit i + 1 are read from shared memory while unit i is
    // decoded and stored; a warp releases a stage as soon as it has read it
    // (the stage is refilled only after the unit's MMAs, which need every
    // warp's A slice, have completed)
    const uint8_t *wbase = smem + L.w_off + row * 128;
    const int c0 = 4 * g + 2 * hf, sw = row & 7;
    auto lds_unit = [&](int s, uint4 (&w)[2]) {
      w[0] = *reinterpret_cast<const uint4 *>(wbase + s * TC_WBYTES + (((c0 + 0) ^ sw) << 4));
      w[1] = *reinterpret_cast<const uint4 *>(wbase + s * TC_WBYTES + (((c0 + 1) ^ sw) << 4));
    };
    int s = 0, ab = 0;
    uint32_t ph = 0, aph = 0;
    bool ok = true;
    uint4 wcur[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if (nunits > 0) {
      ok = mbar_wait(&full[0], 0, a.status);
      lds_unit(0, wcur);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[0]);
    }
    for (int i = 0; i < nunits; ++i) {
      const Meta mcur = mq[0];
#pragma unroll
      for (int j = 0; j < 3; ++j) mq[j] = mq[j + 1];
      if (i + 4 < nunits) mq[3] = load_meta(tq, kq);
      advance(tq, kq);
      uint32_t av[32];
      if (FMT == FMT_W4A16)
        deq_w4a16(wcur, mcur.z, av, MAG);
      else if (FMT == FMT_W4A8)
        deq_w4a8(wcur, av);
      else
        deq_mxfp4(wcur, mcur.e2, av);
      // next unit's codes
      int s1 = s + 1;
      uint32_t ph1 = ph;
      if (s1 == S) {
        s1 = 0;
        ph1 ^= 1u;
      }
      if (i + 1 < nunits) {
        if (ok) ok = !*abort_flag && mbar_wait(&full[s1], ph1, a.status);
        lds_unit(s1, wcur);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s1]);
      }
      if (ok) ok = !*abort_flag && mbar_wait(&a_empty[ab], aph ^ 1u, a.status);
      tc::fence_after_sync();
      if (ok) {
        const uint32_t at = tmem + lane_base + ab * ACOLS + g * GCOLS + hf * HCOLS;
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
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[ab]);
      s = s1;
      ph = ph1;
      if (++ab == NA) {
        ab = 0;
        aph ^= 1u;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    pdl_wait_prior_grid();  // Y, the partial slots and X's scale may be in use before
    float yacc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) yacc[t] = 0.f;
    float xsc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int m = chunk * MT + t;
      xsc[t] = (FMT == FMT_W4A8 && m < a.M) ? ld_act(a.xs + m) : 1.f;
    }
    // per-(row, group) scale (and zero point for W4A8) of the two groups of a unit
    struct EMeta {
      float s[2];
      uint32_t z[2];
    };
    auto load_emeta = [&](int tile, int kb) {
      EMeta m;
      const int n = tile * TC_ROWS + row;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gi = 2 * kb + h;
        const bool ok = n < a.N && gi < a.G;
        m.s[h] = (FMT == FMT_MXFP4) ? 1.f : (ok ? __ldg(a.scales + (size_t)n * a.G + gi) : 0.f);
        m.z[h] = (FMT == FMT_W4A8 && ok && a.zeros) ? (uint32_t)__ldg(a.zeros + (size_t)n * a.G + gi) : 8u;
      }
      return m;
    };
    const bool first_is_shared = kb0 != 0;  // range starts inside a tile
    auto finish_tile = [&](int tile) {
      const int n = tile * TC_ROWS + row;
      const int tend = (tile + 1) * a.nkb;
      const size_t slot = (size_t)chunk * NCTA + blockIdx.x;
      if (tile == tile0 && first_is_shared) {
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
            const long long t0 = clock64(), lim = wait_cycles(a.status);
            while (!seen) {
              __nanosleep(128);
              seen = ld_acquire_u32(f) == a.epoch;
              if (!seen && clock64() - t0 > lim) {
                set_status(a.status, LBC_ERR_TIMEOUT);
                *abort_flag = 1;
                break;
              }
            }
            // clear the flag once seen: a CUDA graph replays this launch with the
            // same epoch, and must find every flag clear until its own producer
            // CTA raises it (the next launch's producers write flags only after
            // griddepcontrol.wait, i.e. after this kernel has completed)
            if (seen) *const_cast<volatile uint32_t *>(f) = 0u;
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
            if (m < a.M) a.y[(size_t)m * a.N + n] = yacc[t] * xsc[t];
          }
        }
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) yacc[t] = 0.f;
    };

    // scales (and W4A8 zero points) through a 4-deep register queue
    int tq[5], kq[5];
    tq[0] = tile0;
    kq[0] = kb0;
#pragma unroll
    for (int j = 1; j < 5; ++j) {
      tq[j] = tq[j - 1];
      kq[j] = kq[j - 1] + 1;
      if (kq[j] == a.nkb) {
        kq[j] = 0;
        ++tq[j];
      }
    }
    EMeta mq[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) mq[j] = load_emeta(tq[j], kq[j]);
    bool ok = true;
    for (int i = 0; i < nunits; ++i) {
      const EMeta mcur = mq[0];
      const int tile = tq[0], kb = kq[0], ntile = tq[1];
#pragma unroll
      for (int j = 0; j < 3; ++j) mq[j] = mq[j + 1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tq[j] = tq[j + 1];
        kq[j] = kq[j + 1];
      }
      tq[4] = tq[3];
      kq[4] = kq[3] + 1;
      if (kq[4] == a.nkb) {
        kq[4] = 0;
        ++tq[4];
      }
      if (i + 4 < nunits) mq[3] = load_emeta(tq[3], kq[3]);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int v = 2 * i + h, d = v & 3;
        if (ok) ok = !*abort_flag && mbar_wait(&d_full[d], (uint32_t)(v >> 2) & 1u, a.status);
        tc::fence_after_sync();
        // column p*MT + t holds piece p of token t; sum the pieces in order
        float sum[MT];
        int32_t isum[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          sum[t] = 0.f;
          isum[t] = 0;
        }
        if (ok) {
#pragma unroll
          for (int c = 0; c < (NPC + 15) / 16; ++c) {
            uint32_t part[16];
            if (NPC - 16 * c <= 4) {
              uint32_t p4[4];
              tc::ld4(tmem + lane_base + DCOL0 + d * NMMA + 16 * c, p4);
#pragma unroll
              for (int j = 0; j < 4; ++j) part[j] = p4[j];
            } else if (NPC - 16 * c <= 8) {
              uint32_t p8[8];
              tc::ld8(tmem + lane_base + DCOL0 + d * NMMA + 16 * c, p8);
#pragma unroll
              for (int j = 0; j < 8; ++j) part[j] = p8[j];
            } else {
              tc::ld16(tmem + lane_base + DCOL0 + d * NMMA + 16 * c, part);
            }
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = 16 * c + j, p = col / MT, t = col % MT;
              if (col < NPC) {
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
        if (ok) {
          if (FMT == FMT_W4A8) {
            const int gi = 2 * kb + h;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              const int m = chunk * MT + t;
              const int as = (m < a.M && gi < a.G) ? ld_act(a.asum + (size_t)m * a.G + gi) : 0;
              yacc[t] = fmaf((float)(isum[t] - (int)mcur.z[h] * as), mcur.s[h], yacc[t]);
            }
          } else {
#pragma unroll
            for (int t = 0; t < MT; ++t) yacc[t] = fmaf(sum[t], mcur.s[h], yacc[t]);
          }
        }
      }
      if (i + 1 == nunits || ntile != tile) finish_tile(tile);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == W_MMA) {
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
template <int FMT, int MT, int NPIECE, int KBLK = TC_KB>
__global__ void __launch_bounds__(256) tc_bblock_kernel(const float *x, const int8_t *xq,
                                                        uint8_t *__restrict__ out, int M, int Kp, int nkb,
                                                        int bbytes) {
  constexpr bool I8 = (FMT == FMT_W4A8);
  constexpr int SBO = KBLK / (I8 ? 16 : 8) * 128;  // bytes between 8-row groups
  constexpr int EPR = I8 ? 16 : 8;                  // elements per 16-byte row
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
        const int k = kb * KBLK + (kk >> 7) * 128 + tc_perm(FMT, kk & 127);
        if (k < Kp) {
          if (I8) {
            w[e >> 2] |= (uint32_t)(uint8_t)ld_act(xq + (size_t)m * Kp + k) << (8 * (e & 3));
          } else {
            float r = ld_act(x + (size_t)m * Kp + k);
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
