// Decode-regime fused dequantize + GEMM on CUDA cores (any M; built for M <= 16).
//
// Arithmetic contract (the reference's scalar kernels, src/lowbit/csrc/
// kern_scalar.c:10-74):
//   W4A16 : y[m,n] = sum_g s[n,g] * sum_{k in g} (q[n,k] - z[n,g]) * x[m,k]     (fp32)
//   MXFP4 : y[m,n] = sum_b 2^(e[n,b]-127) * sum_{k in b} e2m1(q[n,k]) * x[m,k]    (fp32)
//   W4A8  : y[m,n] = xs[m] * sum_g s[n,g] * (sum_{k in g} q*xq - z*asum[m,g])  (int32 exact per
//           16-byte chunk, fp32 across chunks)
//
// Structure (persistent CTAs of 8 warps, 1-3 per SM):
//   * weight tiles (tile_rows rows x one K segment) stream HBM -> shared memory
//     as 1-D TMA bulk copies into a `stages`-deep ring guarded by full/empty
//     mbarriers; thread 0 issues the copies (no dedicated producer warp: B200
//     splits the register file over 4 SM sub-partitions, and a 9th warp would
//     cap every thread at 168 registers);
//   * consumer threads own fixed 16-byte chunks of K: the activations of
//     those chunks live in registers for the whole kernel, so shared memory
//     only carries weights (1 byte per 2 MACs per token);
//   * a "row team" of `tpr` threads covers one weight row; each thread keeps
//     partial sums for RT rows x MT tokens, reduced with a transposing warp
//     reduction and, for teams wider than a warp, one shared-memory step.
//
// Nibble decode without conversions: for a nibble at bit position p (0,4,8,12)
// of a 16-bit half word, (w & (0xF << p)) | 0x4B000000 is the fp32 value
// 2^23 + q*2^p; subtracting 2^23 + z*2^p gives (q - z)*2^p exactly. Four
// accumulators (one per p) are rescaled by 2^-p at the end of each chunk.
#pragma once

#include "common.cuh"

namespace lbc {

enum : int { FMT_W4A16 = 0, FMT_MXFP4 = 1, FMT_W4A8 = 2 };

// largest row team of the register-streamed decode kernel (gemv_rows.cuh);
// teams of one chunk per thread and one or two tokens may be up to
// ROWS_WIDE_WARPS warps (one CTA per SM at <= 128 registers), which covers
// rows of up to 16384 elements without the register-heavy multi-chunk tiles
constexpr int ROWS_MAX_WARPS = 8;
constexpr int ROWS_WIDE_WARPS = 16;

struct GemvArgs {
  const float *x;       // [M, Kp] fp32 (W4A16 / MXFP4)
  const int8_t *xq;     // [M, Kp] int8 (W4A8)
  const float *xs;      // [M]        (W4A8)
  const int32_t *asum;  // [M, Kp/128] (W4A8) per-group code sums
  const uint8_t *qw;    // [N, Kp/2]
  const float *scales;  // [N, Kp/128] (int4)
  const uint8_t *zeros; // [N, Kp/128] or nullptr (int4)
  const uint8_t *e8m0;  // [N, Kp/32]  (MXFP4)
  float *y;             // [M, N]
  int M, N, Kp;
  int seg_elems;        // K elements per split segment (multiple of 128)
  int nsplit;           // number of K segments
  int ctas_per_split;   // persistent CTAs working on one K segment
  int tile_rows;        // rows per pipeline tile (= RT * teams)
  int ntiles;           // ceil(N / tile_rows)
  int stages;           // pipeline depth
  int tpr;              // threads per row team (multiple of 32)
  int nt;               // consumer threads (multiple of tpr)
  int atomic_out;       // 1: accumulate into y with atomics (split-K)
  int meta_tma;         // 1: scales/zeros/e8m0 travel with the weights in each stage
  int *status;          // device status word (bounded-wait timeouts)
  // fused all-gather (column-parallel decode over NVLink peers), else unused:
  // y is then this rank's whole output [M, ld_y]
  uint64_t *const *land_peers;  // [world] landing buffers of every rank: [2 parities][2][ld_y]
                                // words (call tag << 32 | fp32 bits of the value)
  uint32_t *counter;            // this rank's CTA completion counter
  uint32_t *epoch;              // this rank's call counter (the words' tags carry it)
  int rank, world, row0, ld_y;  // this rank's first global row, Y row stride
  // fused activation prologue of the decode kernel (W4A16), else unused:
  const float *xres;  // [M, Kp] residual added to x before the norm, or nullptr
  float *xout;        // [M, Kp] x + xres, stored by the CTAs of column 0 (never aliases x)
  const float *lnw;   // [Kp] RMSNorm weight
  float eps;          // RMSNorm epsilon
};

// activation prologues of the decode kernel
constexpr int XM_PLAIN = 0;    // x as given
constexpr int XM_RMSNORM = 1;  // (x + xres) / sqrt(mean((x + xres)^2) + eps) * lnw
constexpr int XM_GLU = 2;      // silu(x[:, :Kp]) * x[:, Kp:] (x rows of 2 * Kp)
constexpr int XM_QUANT = 3;    // W4A8 from fp32 x: the per-token int8 quantizer inside the kernel
constexpr int QUANT_CLUSTER = 8;   // CTAs per cluster sharing one quantization (XM_QUANT)
constexpr int QUANT_MAX_KP = 8192; // XM_QUANT rows (the slices of one cluster fit in shared memory)

// Per-stage metadata region (scales + zero points, or E8M0 exponents) when it
// is staged by TMA: bytes per row of each part, rounded regions per stage.
struct GemvMeta {
  int sc_row;   // bytes of scales (int4: G*4) or e8m0 (MXFP4: Kp/32) per row
  int z_row;    // bytes of zero points per row (0 when absent / MXFP4)
  int sc_off;   // offset of the scale region inside a stage
  int z_off;    // offset of the zero-point region inside a stage
  int bytes;    // total stage bytes (weights + metadata)
};

__host__ __device__ inline int round16(int v) { return (v + 15) & ~15; }

__host__ __device__ inline GemvMeta gemv_meta(int fmt, int Kp, bool has_zeros, int tile_rows,
                                              int seg_bytes, bool meta_tma) {
  GemvMeta m;
  m.sc_row = (fmt == 1) ? (Kp >> 5) : (Kp >> 7) * 4;
  m.z_row = (fmt != 1 && has_zeros) ? (Kp >> 7) : 0;
  m.sc_off = tile_rows * seg_bytes;
  m.z_off = m.sc_off + (meta_tma ? round16(tile_rows * m.sc_row) : 0);
  m.bytes = m.z_off + (meta_tma ? round16(tile_rows * m.z_row) : 0);
  return m;
}

// shared-memory carve-up; identical on host and device
struct GemvSmem {
  int bar_off, red_off, abort_off, stage_off, stage_bytes, total;
};

__host__ __device__ inline GemvSmem gemv_smem_layout(int stages, int nt, int stage_bytes) {
  GemvSmem L;
  L.bar_off = 0;
  L.red_off = 16 * stages;  // full[S], empty[S] (8 B each)
  L.abort_off = L.red_off + 2 * (nt / 32) * 32 * 4;
  L.stage_off = (L.abort_off + 16 + 127) / 128 * 128;
  L.stage_bytes = (stage_bytes + 127) / 128 * 128;
  L.total = L.stage_off + stages * L.stage_bytes;
  return L;
}

// ---------------------------------------------------------------- PDL hooks
// Programmatic dependent launch: the next kernel in the stream may start once
// every CTA of this one has called launch_dependents; it must call
// wait_prior_grid before touching memory the previous kernel writes.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ------------------------------------------------------------------ reductions
// After the call, lane l holds in v[0] the warp-wide sum of value index
// l / (32 / V) (all lanes of that group hold it). V must be a power of two <= 32.
template <int V>
__device__ __forceinline__ float warp_reduce_multi(float (&v)[V], int lane) {
  constexpr int LOG2V = (V >= 32) ? 5 : (V >= 16) ? 4 : (V >= 8) ? 3 : (V >= 4) ? 2 : (V >= 2) ? 1 : 0;
#pragma unroll
  for (int st = 0; st < LOG2V; ++st) {
    const int s = 16 >> st;
    const int half = (V >> st) / 2;
    const bool up = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = up ? v[i] : v[i + half];
      const float keep = up ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
#pragma unroll
  for (int s = 16 >> LOG2V; s >= 1; s >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], s);
  return v[0];
}

// ------------------------------------------------------------------ decoders
// A register holding v that the compiler cannot constant-fold: LOP3 takes one
// immediate, so "(w & mask) | MAGIC" is a single instruction only when MAGIC
// lives in a register.
__device__ __forceinline__ uint32_t opaque(uint32_t v) {
  uint32_t r;
  asm volatile("mov.b32 %0, %1;" : "=r"(r) : "r"(v));
  return r;
}

// W4A16: one 16-byte chunk (32 codes of one group) against MT tokens.
// xr[t][j] = (x[lo + j], x[hi + j]) with lo/hi the element bases of the chunk.
// Two nibbles of w -> the fp32 pair (2^23 + q_a*2^pa, 2^23 + q_b*2^pb) with one
// lop3 each, written straight into the halves of a 64-bit register pair, then
// minus (2^23 + z*2^pa, 2^23 + z*2^pb) with one packed add: (q - z) * 2^p.
template <uint32_t MA, uint32_t MB>
__device__ __forceinline__ uint64_t nib2(uint32_t w, uint32_t mag, uint64_t negz) {
  uint64_t r;
  asm("{\n\t.reg .b32 lo, hi;\n\t.reg .b64 p;\n\t"
      "lop3.b32 lo, %1, %3, %2, 0xEA;\n\t"
      "lop3.b32 hi, %1, %4, %2, 0xEA;\n\t"
      "mov.b64 p, {lo, hi};\n\t"
      "add.rn.f32x2 %0, p, %5;\n\t}"
      : "=l"(r)
      : "r"(w), "r"(mag), "n"(MA), "n"(MB), "l"(negz));
  return r;
}

__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) {
  return (uint64_t)lo | ((uint64_t)hi << 32);
}

__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// W4A16: one 16-byte chunk (32 codes of one group) against MT tokens.
// xr[t][j] = (x[lo + j], x[hi + j]) as a packed fp32 pair, lo/hi the element
// bases of the chunk.
template <int MT>
__device__ __forceinline__ void dot_w4a16(const uint4 wv, uint32_t z, const uint64_t (*xr)[16],
                                          float (&dot)[MT], const uint32_t MAG) {
  const uint64_t nz01 = pack2(0xCB000000u | z, 0xCB000000u | (z << 4));
  const uint64_t nz23 = pack2(0xCB000000u | (z << 8), 0xCB000000u | (z << 12));
  uint64_t accA[MT], accB[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) accA[t] = accB[t] = 0ull;
  const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t w = w4[q];
    const uint32_t h = w >> 16;
    const uint64_t a = nib2<0x000Fu, 0x00F0u>(w, MAG, nz01);
    const uint64_t b = nib2<0x0F00u, 0xF000u>(w, MAG, nz23);
    const uint64_t c = nib2<0x000Fu, 0x00F0u>(h, MAG, nz01);
    const uint64_t d = nib2<0x0F00u, 0xF000u>(h, MAG, nz23);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      accA[t] = ffma2(a, xr[t][4 * q + 0], accA[t]);
      accB[t] = ffma2(b, xr[t][4 * q + 1], accB[t]);
      accA[t] = ffma2(c, xr[t][4 * q + 2], accA[t]);
      accB[t] = ffma2(d, xr[t][4 * q + 3], accB[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t)
    dot[t] = fmaf(hi_f(accB[t]), 1.0f / 4096.0f,
                  fmaf(lo_f(accB[t]), 1.0f / 256.0f, fmaf(hi_f(accA[t]), 1.0f / 16.0f, lo_f(accA[t]))));
}

// MXFP4: one 16-byte chunk = one block of 32 E2M1 codes. The result is
// 2 * sum e2m1(q) * x (the caller's block scale carries the factor 1/2).
// Codes are mapped through two 8-entry byte tables (prmt) to 16 + 2*e2m1(q),
// a value in [4, 28], then to fp32 with the 2^23 magic number.
// xr[t][off + j] = (x[lo + j], x[hi + j]) for token t.
template <int MT, int XN>
__device__ __forceinline__ void dot_mxfp4(const uint4 wv, const uint64_t (*xr)[XN], int off, float (&dot)[MT],
                                          const uint32_t MAGIC) {
  const uint32_t TP0 = 0x13121110u, TP1 = 0x1C181614u;  // 16 + {0,1,2,3}, 16 + {4,6,8,12}
  const uint32_t TN0 = 0x0D0E0F10u, TN1 = 0x04080A0Cu;  // 16 - {0,1,2,3}, 16 - {4,6,8,12}
  const uint64_t NB = pack2(0xCB000010u, 0xCB000010u);   // -(2^23 + 16) twice
  uint64_t accA[MT], accB[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) accA[t] = accB[t] = 0ull;
  const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t w = w4[q];
    const uint32_t m = w & 0x77777777u;
    const uint32_t w4s = w << 4;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t sel = half ? (m >> 16) : m;
      const uint32_t pos = prmt(TP0, TP1, sel);
      const uint32_t neg = prmt(TN0, TN1, sel);
      const uint32_t msk = prmt(w4s, w, half ? 0xFBEAu : 0xD9C8u);  // 0xFF where the code is negative
      const uint32_t val = (pos & ~msk) | (neg & msk);               // bytes: 16 + 2*e2m1
      uint64_t p0, p1;
      asm("{\n\t.reg .b32 a, b, c, d;\n\t.reg .b64 u, v;\n\t"
          "prmt.b32 a, %2, %3, 0x7540;\n\t"
          "prmt.b32 b, %2, %3, 0x7541;\n\t"
          "prmt.b32 c, %2, %3, 0x7542;\n\t"
          "prmt.b32 d, %2, %3, 0x7543;\n\t"
          "mov.b64 u, {a, b};\n\t"
          "mov.b64 v, {c, d};\n\t"
          "add.rn.f32x2 %0, u, %4;\n\t"
          "add.rn.f32x2 %1, v, %4;\n\t}"
          : "=l"(p0), "=l"(p1)
          : "r"(val), "r"(MAGIC), "l"(NB));
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        accA[t] = ffma2(p0, xr[t][off + 4 * q + 2 * half + 0], accA[t]);
        accB[t] = ffma2(p1, xr[t][off + 4 * q + 2 * half + 1], accB[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) dot[t] = (lo_f(accA[t]) + hi_f(accA[t])) + (lo_f(accB[t]) + hi_f(accB[t]));
}

// 2^(e-128) as fp32: half the E8M0 block scale (the MXFP4 decoder returns 2x).
// e == 255 is NaN, as in the OCP MX spec (src/lowbit/csrc/lowbit.h:84-88).
__device__ __forceinline__ float e8m0_half_scale(uint32_t e) {
  const uint32_t bits = (e == 255u) ? 0x7FC00000u : (e >= 2u ? (e - 1u) << 23 : (0x00200000u << e));
  return u2f(bits);
}

// ------------------------------------------------------------------ kernel
template <int FMT, int MT, int CH, int RT>
__global__ void __launch_bounds__(256, 1) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int V = RT * MT;
  static_assert(V <= 32 && (V & (V - 1)) == 0, "RT*MT must be a power of two <= 32");

  const int S = a.stages;
  const int ncw = a.nt >> 5;
  const int split = blockIdx.x / a.ctas_per_split;
  const int cta = blockIdx.x - split * a.ctas_per_split;
  const int k0 = split * a.seg_elems;
  const int k1 = min(a.Kp, k0 + a.seg_elems);
  const int Cs = (k1 - k0) >> 5;  // 16-byte chunks per row segment
  const int SB = Cs << 4;         // bytes per row segment
  const bool has_z = (FMT != FMT_MXFP4) && a.zeros != nullptr;
  const GemvMeta MM = gemv_meta(FMT, a.Kp, has_z, a.tile_rows, a.seg_elems / 2, a.meta_tma != 0);
  const GemvSmem L = gemv_smem_layout(S, a.nt, MM.bytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *empty = full + S;
  float *red = reinterpret_cast<float *>(smem + L.red_off);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.abort_off);
  uint8_t *stage_base = smem + L.stage_off;
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * MT;
  const int row_bytes = a.Kp >> 1;
  const int G = a.Kp >> 7;     // int4 groups per row
  const int NB32 = a.Kp >> 5;  // MXFP4 blocks per row

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ncw);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int my_tiles =
      (cta < a.ntiles) ? (a.ntiles - cta + a.ctas_per_split - 1) / a.ctas_per_split : 0;

  // whether tile i's metadata is staged by TMA (the tail tile may be unaligned)
  auto tile_meta = [&](int rows) -> bool {
    if (!a.meta_tma) return false;
    if (rows == a.tile_rows) return true;
    return ((rows * MM.sc_row) & 15) == 0 && ((rows * MM.z_row) & 15) == 0;
  };

  // Thread 0 doubles as the TMA producer: it fills the first `stages` tiles
  // up front, then refills the stage of tile i-1 with tile i-1+stages at the
  // top of iteration i, once every warp has released tile i-1. No warp is
  // dedicated to producing, so a CTA is exactly `nt` threads (8 warps) and
  // every warp may use up to 255 registers.
  const uint64_t pol = policy_evict_first();
  auto issue = [&](int i) {
    const int s = i % S;
    const int r0 = (cta + i * a.ctas_per_split) * a.tile_rows;
    const int rows = min(a.tile_rows, a.N - r0);
    uint8_t *dst = stage_base + s * L.stage_bytes;
    const uint8_t *src = a.qw + (size_t)r0 * row_bytes + (k0 >> 1);
    const bool tm = tile_meta(rows);
    const uint32_t mbytes = tm ? (uint32_t)(rows * (MM.sc_row + MM.z_row)) : 0u;
    mbar_expect_tx(&full[s], (uint32_t)(rows * SB) + mbytes);
    if (a.nsplit == 1) {
      bulk_g2s(dst, src, (uint32_t)(rows * SB), &full[s], pol);
    } else {
      for (int r = 0; r < rows; ++r)
        bulk_g2s(dst + r * SB, src + (size_t)r * row_bytes, (uint32_t)SB, &full[s], pol);
    }
    if (tm) {
      const uint8_t *msrc = (FMT == FMT_MXFP4) ? a.e8m0 : reinterpret_cast<const uint8_t *>(a.scales);
      bulk_g2s(dst + MM.sc_off, msrc + (size_t)r0 * MM.sc_row, (uint32_t)(rows * MM.sc_row), &full[s], pol);
      if (MM.z_row)
        bulk_g2s(dst + MM.z_off, a.zeros + (size_t)r0 * MM.z_row, (uint32_t)(rows * MM.z_row), &full[s], pol);
    }
  };
  // weights and their metadata are static: stream them before the previous
  // kernel in the stream (which may produce X) has finished
  if (tid == 0)
    for (int i = 0; i < min(S, my_tiles); ++i) issue(i);
  pdl_launch_dependents();

  const int lane = tid & 31, warp = tid >> 5;
  const int team = tid / a.tpr, tin = tid - team * a.tpr;
  const int RP = a.nt / a.tpr;

  // activations (written by the previous kernel, if any) of this thread's
  // chunks, resident in registers for the whole kernel
  pdl_wait_prior_grid();
  uint64_t xr[CH][MT][16];
  uint32_t xl[CH][MT][4], xh[CH][MT][4];
  int xsum[CH][MT];
  (void)xr; (void)xl; (void)xh; (void)xsum;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = tin + i * a.tpr;
    const int kc = (k0 >> 5) + c;  // global chunk index
    int lo, hi;
    if (FMT == FMT_MXFP4) {
      lo = kc << 5;
      hi = lo + 16;
    } else {
      lo = ((kc >> 2) << 7) + ((kc & 3) << 4);
      hi = lo + 64;
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int m = m0 + t;
      const bool ok = (c < Cs) && (m < a.M);
      if (FMT == FMT_W4A8) {
        uint4 vl = make_uint4(0, 0, 0, 0), vh = make_uint4(0, 0, 0, 0);
        if (ok) {
          vl = ld_act(reinterpret_cast<const uint4 *>(a.xq + (size_t)m * a.Kp + lo));
          vh = ld_act(reinterpret_cast<const uint4 *>(a.xq + (size_t)m * a.Kp + hi));
        }
        xl[i][t][0] = vl.x; xl[i][t][1] = vl.y; xl[i][t][2] = vl.z; xl[i][t][3] = vl.w;
        xh[i][t][0] = vh.x; xh[i][t][1] = vh.y; xh[i][t][2] = vh.z; xh[i][t][3] = vh.w;
        // z * asum[m,g] is subtracted once per group, in the group's first chunk,
        // exactly as the reference applies it (src/lowbit/csrc/kern_scalar.c:49-59)
        xsum[i][t] = (ok && (kc & 3) == 0) ? ld_act(a.asum + (size_t)m * G + (kc >> 2)) : 0;
      } else {
        const float4 *pl = reinterpret_cast<const float4 *>(a.x + (size_t)m * a.Kp + lo);
        const float4 *ph = reinterpret_cast<const float4 *>(a.x + (size_t)m * a.Kp + hi);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 l4 = make_float4(0.f, 0.f, 0.f, 0.f), h4 = l4;
          if (ok) {
            l4 = ld_act(pl + q);
            h4 = ld_act(ph + q);
          }
          xr[i][t][4 * q + 0] = pack2(__float_as_uint(l4.x), __float_as_uint(h4.x));
          xr[i][t][4 * q + 1] = pack2(__float_as_uint(l4.y), __float_as_uint(h4.y));
          xr[i][t][4 * q + 2] = pack2(__float_as_uint(l4.z), __float_as_uint(h4.z));
          xr[i][t][4 * q + 3] = pack2(__float_as_uint(l4.w), __float_as_uint(h4.w));
        }
      }
    }
  }

  // Per-thread chunk bookkeeping, fixed for the kernel. A chunk past the end
  // of the segment (c >= Cs) is clamped onto the last real chunk: its
  // activations are zero, so it adds exactly 0 and the inner loop needs no
  // bounds checks.
  int ch_off[CH], ch_g[CH], ch_kc[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = min(tin + i * a.tpr, Cs - 1);
    ch_off[i] = c << 4;
    ch_kc[i] = (k0 >> 5) + c;
    ch_g[i] = ch_kc[i] >> 2;
  }
  const uint32_t MAG = opaque(0x4B000000u);

  bool ok = true;
  int s = 0;
  uint32_t ph = 0;
  for (int it = 0; it < my_tiles; ++it) {
    // refill the stage released by tile it-1 with tile it-1+S
    if (tid == 0 && it >= 1 && it - 1 + S < my_tiles) {
      const int sp = (s == 0) ? S - 1 : s - 1;
      const uint32_t php = (s == 0) ? (ph ^ 1u) : ph;
      if (ok) ok = !(*abort_flag) && mbar_wait(&empty[sp], php, a.status);
      if (ok)
        issue(it - 1 + S);
      else
        *abort_flag = 1;
    }
    const int r0 = (cta + it * a.ctas_per_split) * a.tile_rows;
    const int rows = min(a.tile_rows, a.N - r0);
    const bool tm = tile_meta(rows);
    const uint8_t *st = stage_base + s * L.stage_bytes;

    // per-(row, chunk) scale and zero point: from the stage when TMA brought
    // them, else from global memory (fetched before waiting on the tile).
    // Rows past the end of a tail tile read clamped / stale values; their
    // results are never written.
    float sc[RT][CH];
    uint32_t zz[RT][CH];
    if (!tm) {
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        const int n = min(r0 + team + j * RP, a.N - 1);
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          if (FMT == FMT_MXFP4) {
            sc[j][i] = e8m0_half_scale(__ldg(a.e8m0 + (size_t)n * NB32 + ch_kc[i]));
          } else {
            sc[j][i] = __ldg(a.scales + (size_t)n * G + ch_g[i]);
            zz[j][i] = has_z ? (uint32_t)__ldg(a.zeros + (size_t)n * G + ch_g[i]) : 8u;
          }
        }
      }
    }

    if (ok) ok = !(*abort_flag) && mbar_wait(&full[s], ph, a.status);
    if (!ok) *abort_flag = 1;
    if (tm) {
#pragma unroll
      for (int j = 0; j < RT; ++j) {
        const int r = team + j * RP;
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          if (FMT == FMT_MXFP4) {
            sc[j][i] = e8m0_half_scale(st[MM.sc_off + r * NB32 + ch_kc[i]]);
          } else {
            sc[j][i] = reinterpret_cast<const float *>(st + MM.sc_off)[r * G + ch_g[i]];
            zz[j][i] = has_z ? (uint32_t)st[MM.z_off + r * G + ch_g[i]] : 8u;
          }
        }
      }
    }

    float part[RT][MT];
#pragma unroll
    for (int j = 0; j < RT; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) part[j][t] = 0.f;

#pragma unroll
    for (int j = 0; j < RT; ++j) {
      const uint8_t *rowp = st + (team + j * RP) * SB;
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const uint4 wv = lds128(rowp + ch_off[i]);
        if (FMT == FMT_W4A8) {
          int acc[MT];
#pragma unroll
          for (int t = 0; t < MT; ++t) acc[t] = 0;
          const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t lo = w4[q] & 0x0F0F0F0Fu;
            const uint32_t hi = (w4[q] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              acc[t] = dp4a_us(lo, xl[i][t][q], acc[t]);
              acc[t] = dp4a_us(hi, xh[i][t][q], acc[t]);
            }
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const int d = acc[t] - (int)zz[j][i] * xsum[i][t];
            part[j][t] = fmaf((float)d, sc[j][i], part[j][t]);
          }
        } else {
          float dot[MT];
          if (FMT == FMT_W4A16)
            dot_w4a16<MT>(wv, zz[j][i], xr[i], dot, MAG);
          else
            dot_mxfp4<MT, 16>(wv, xr[i], 0, dot, MAG);
#pragma unroll
          for (int t = 0; t < MT; ++t) part[j][t] = fmaf(dot[t], sc[j][i], part[j][t]);
        }
      }
    }
    // release the stage (every consumer warp arrives once per tile)
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    // reduce RT x MT partials over the row team
    float v[V];
#pragma unroll
    for (int j = 0; j < RT; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) v[j * MT + t] = part[j][t];
    const float tot = warp_reduce_multi<V>(v, lane);
    constexpr int PER = 32 / V;
    int out_idx = -1;
    float out_val = 0.f;
    if (a.tpr == 32) {
      if ((lane % PER) == 0) {
        out_idx = lane / PER;
        out_val = tot;
      }
    } else {
      float *rb = red + (it & 1) * ncw * 32;
      if ((lane % PER) == 0) rb[warp * 32 + lane / PER] = tot;
      named_bar_sync(1, a.nt);
      const int wpt = a.tpr >> 5;
      if (tin < V) {
        float acc = 0.f;
        for (int w = 0; w < wpt; ++w) acc += rb[(team * wpt + w) * 32 + tin];
        out_idx = tin;
        out_val = acc;
      }
    }
    if (ok && out_idx >= 0) {
      const int j = out_idx / MT, t = out_idx - (out_idx / MT) * MT;
      const int r = team + j * RP;
      const int m = m0 + t;
      if (r < rows && m < a.M) {
        float val = out_val;
        if (FMT == FMT_W4A8) val *= ld_act(a.xs + m);
        float *dst = a.y + (size_t)m * a.N + (r0 + r);
        if (a.atomic_out)
          atomicAdd(dst, val);
        else
          *dst = val;
      }
    }
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
  }
}

}  // namespace lbc
