// Warp-level tensor-core decode GEMV for one or two tokens (W4A16).
//
// Y[m, n] = sum_g s[n,g] * sum_{k in g} (q[n,k] - z[n,g]) * x[m,k], the
// reference's W4A16 arithmetic (src/lowbit/csrc/kern_avx512.c:28-74) to its
// 1e-5 * (|X| . |W|^T) bound, with the multiply-accumulate on the tensor cores
// through mma.sync.m16n8k16 (bf16 x bf16 -> fp32):
//
//   * A = 16 weight rows x 16 K as exact bf16 (q - z): one LOP3 turns a
//     nibble pair into the bf16 pair (128 + q_a, 128 + q_b) (the 2^7 magic
//     number), one packed bf16 subtraction of (128 + z, 128 + z) gives
//     (q - z) exactly (|q - z| <= 15);
//   * B = 16 K x 8 columns: column n = piece n % 3 of token n / 3, where
//     x = p1 + p2 + p3 with p1 = bf16(x), p2 = bf16(x - p1), p3 = bf16(x - p1
//     - p2) (each difference exact in fp32; the pieces carry 24 significant
//     bits of x, so every product (q - z) * p is exact in the fp32 accumulator);
//   * the 8 MMAs of one 128-element group accumulate into a fresh fragment,
//     which the group scale multiplies into the row's running sums in fp32
//     (as the reference applies s once per group); the three pieces are
//     added at the end.
//
// The contraction runs in a permuted K order inside each group, chosen so
// that a lane's 16 bytes of a row decode with the fewest instructions: lane
// (g, t) (g = lane / 4, t = lane % 4) reads bytes [16t, 16t + 16) of its rows
// g and g + 8 in every group; word i of those bytes yields four bf16 pairs
// (nibbles 0/2, 4/6 after >> 4, 8/10 after >> 8, 12/14 after >> 12 of each
// 16-bit half), which are the A fragments of MMAs 2i and 2i + 1. The B
// fragments hold x at the same K positions; they are built once per CTA in
// shared memory (X is read after griddepcontrol.wait: it may come from the
// previous kernel in the stream).
//
// Work split: CTA c owns the rows [c*N/P, (c+1)*N/P) (P = grid size), i.e.
// the same number of weight bytes +-1 row, in blocks of 16 rows (the last
// one possibly partial). A producer warp copies each stage -- one row block
// x one K segment -- into a shared-memory ring with one 1-D bulk copy per
// row (the TMA engine, no multicast), completion counted on the stage's
// mbarrier; the consumer warps split each stage's groups, copy their words
// to registers and release the slot before decoding. The CTA's scales and
// zero points are loaded into shared memory once, before griddepcontrol.wait.
// Each warp's per-block partial sums go to shared memory slots, which the CTA
// adds in warp order (deterministic).
#pragma once

#include <cuda_bf16.h>

#include "gemv_rows.cuh"

namespace lbc {

// bf16 bits of x rounded to nearest even (finite inputs)
__device__ __forceinline__ uint32_t bf16_bits_rn(float x) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf16_bits_to_f(uint32_t b) { return __uint_as_float(b << 16); }

// The three bf16 pieces of x (x = p1 + p2 + p3 to 24 significant bits). A
// non-finite x keeps its value in p1 (inf * (q - z) and NaN propagate as in
// the reference's fp32 products) and zero pieces after it.
__device__ __forceinline__ void split3_bf16(float x, uint32_t &p1, uint32_t &p2, uint32_t &p3) {
  if (!isfinite(x)) {
    p1 = __float_as_uint(x) >> 16 | ((__float_as_uint(x) & 0x7FFFFFu) ? 0x40u : 0u);
    p2 = p3 = 0u;
    return;
  }
  p1 = bf16_bits_rn(x);
  const float r1 = __fsub_rn(x, bf16_bits_to_f(p1));
  p2 = bf16_bits_rn(r1);
  const float r2 = __fsub_rn(r1, bf16_bits_to_f(p2));
  p3 = bf16_bits_rn(r2);
}

// (a & 0x000F000F) | mag: the nibbles at bits 0-3 and 16-19 of a as the bf16
// pair (128 + q_lo, 128 + q_hi) when mag holds the pair (128, 128)
__device__ __forceinline__ uint32_t nib_pair(uint32_t a, uint32_t mag) {
  uint32_t d;
  asm("lop3.b32 %0, %1, 0x000F000F, %2, 0xEA;" : "=r"(d) : "r"(a), "r"(mag));
  return d;
}

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// D = A . B + C, m16n8k16, bf16 inputs, fp32 accumulators
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds128_u32(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// Shared-memory layout of the MMA decode kernel, identical on host and device.
// A stage is one 16-row block x one K segment of GS groups; its rows sit
// SS bytes apart with SS = 64 (mod 128), so the 8 rows one 16-byte load
// instruction touches (4 lanes x 16 bytes each) fall on distinct bank halves.
struct MmvSmem {
  int nl;         // lanes holding B data: 4 per used column
  int gs;         // groups per K segment (units per warp per stage x warps)
  int nseg;       // K segments per row
  int ss;         // bytes between two rows of a stage
  int stage;      // bytes of one stage
  int ns;         // stages in the ring
  int chunk;      // row blocks whose partial sums are held before a reduction
  int part_bytes; // partial sums of one (row block, warp): 16 rows x 3 pieces x tokens
  int sc_stride;  // floats between two rows of the CTA's scales (G + 1: rows on distinct banks)
  int z_stride;   // bytes between two rows of the CTA's zero points (G + 4)
  int sc_off, z_off;  // the CTA's scales [rows][sc_stride] fp32 and zero points [rows][z_stride] u8
  int xf_off, part_off, ring_off, total;
};

__host__ __device__ inline MmvSmem mmv_smem_layout(int ntok, int nw, int jws, int ns, int G, int rows_max) {
  MmvSmem L;
  L.nl = 12 * ntok;
  L.gs = jws * nw;
  if (L.gs > G) L.gs = G;
  L.nseg = (G + L.gs - 1) / L.gs;
  L.ss = L.gs * 64 + (((L.gs * 64) & 127) == 0 ? 64 : 0);
  L.stage = (16 * L.ss + 127) / 128 * 128;
  L.ns = ns;
  const int nblk = (rows_max + 15) / 16;
  L.chunk = nblk < 4 ? (nblk > 0 ? nblk : 1) : 4;
  L.part_bytes = 16 * 3 * ntok * 4;
  L.sc_stride = G + 1;
  L.z_stride = G + 4;
  L.xf_off = 256;  // mbarriers and the abort flag first
  L.part_off = L.xf_off + G * 4 * L.nl * 16;
  L.sc_off = L.part_off + L.chunk * nw * L.part_bytes;
  L.z_off = L.sc_off + nblk * 16 * L.sc_stride * 4;
  L.ring_off = (L.z_off + nblk * 16 * L.z_stride + 127) / 128 * 128;
  L.total = L.ring_off + L.ns * L.stage;
  return L;
}

// NW consumer warps + one producer warp. Stage s = (row block s / nseg, K
// segment s % nseg) of the CTA's rows; consumer warp w decodes groups
// w, w + NW, ... (JWS of them) of every segment, so all warps share every
// stage and no reduction is needed inside a block's K walk; each warp's
// sums of a block are parked in shared memory and the CTA adds them in warp
// order (deterministic) every `chunk` blocks.
template <int NTOK, int NW, int JWS, bool HAS_Z>
__global__ void __launch_bounds__((NW + 1) * 32, NW <= 8 ? 2 : 1) gemv_mma_kernel(const GemvArgs a, int ns) {
  static_assert(NTOK == 1 || NTOK == 2, "one or two tokens (three pieces each in 8 MMA columns)");
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.Kp >> 7, RB = a.Kp >> 1;
  const int r0 = (int)((long long)blockIdx.x * a.N / gridDim.x);
  const int r1 = (int)((long long)(blockIdx.x + 1) * a.N / gridDim.x);
  const int nrows = r1 - r0;
  const int nblk = (nrows + 15) >> 4;
  const int rows_max = (a.N + gridDim.x - 1) / gridDim.x;
  const MmvSmem L = mmv_smem_layout(NTOK, NW, JWS, ns, G, rows_max);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + 8;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 192);
  const uint32_t xf_s = smem_u32(smem + L.xf_off);
  float *part = reinterpret_cast<float *>(smem + L.part_off);
  uint8_t *ring = smem + L.ring_off;
  const int nst = nblk * L.nseg;

  if (tid == 0) {
    for (int i = 0; i < L.ns; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == NW) {
    // ---------------- producer: per-row bulk copies of each stage (weights are
    // static, so no griddepcontrol.wait: the ring fills while the previous
    // kernel in the stream drains)
    const uint64_t pol = policy_evict_first();
    int issued = 0;
    int slot = 0, b = 0, seg = 0;
    uint32_t epar = 1;  // parity of the empty phase a refill waits for
    for (int st = 0; st < nst; ++st) {
      if (st >= L.ns) {
        bool ok = true;
        if (lane == 0) ok = !*abort_flag && mbar_wait(&empty[slot], epar, a.status);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          if (lane == 0) *abort_flag = 1;
          break;
        }
      }
      const int rb = r0 + 16 * b;
      const int nv = min(16, r1 - rb);
      const int gs = min(L.gs, G - seg * L.gs);
      if (lane == 0) mbar_expect_tx(&full[slot], (uint32_t)(nv * gs * 64));
      __syncwarp();
      if (lane < nv)
        bulk_g2s(ring + slot * L.stage + lane * L.ss, a.qw + (size_t)(rb + lane) * RB + seg * L.gs * 64,
                 (uint32_t)(gs * 64), &full[slot], pol);
      issued = st + 1;
      if (++slot == L.ns) {
        slot = 0;
        epar ^= 1u;
      }
      if (++seg == L.nseg) {
        seg = 0;
        ++b;
      }
    }
    // never leave a copy in flight into shared memory this CTA gives up:
    // wait (bounded) for the last stage issued into every slot
    if (lane == 0 && *abort_flag) {
      for (int st = max(0, issued - L.ns); st < issued; ++st)
        mbar_wait(&full[st % L.ns], (st / L.ns) & 1, a.status);
    }
    return;
  }

  // ---------------- consumers
  const int g = lane >> 2, t = lane & 3;
  // the CTA's scales and zero points into shared memory, padded so the 8 rows
  // one load instruction touches fall on distinct banks; they are static, so
  // this runs before griddepcontrol.wait, under the previous kernel's tail.
  // Rows of the last block past the CTA's rows repeat its last row.
  {
    float *ssm = reinterpret_cast<float *>(smem + L.sc_off);
    uint8_t *zsm = smem + L.z_off;
    const int nmeta = nblk * 16 * G;
    for (int i0 = 0; i0 < nmeta; i0 += 8 * NW * 32) {
      float sv[8];
      uint32_t zv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = i0 + q * NW * 32 + tid;
        const int rr = i / G, j = i - rr * G;
        const size_t gi = (size_t)min(r0 + rr, r1 - 1) * G + j;
        sv[q] = i < nmeta ? __ldg(a.scales + gi) : 0.f;
        zv[q] = (HAS_Z && i < nmeta) ? (uint32_t)__ldg(a.zeros + gi) : 8u;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = i0 + q * NW * 32 + tid;
        if (i < nmeta) {
          const int rr = i / G, j = i - rr * G;
          ssm[rr * L.sc_stride + j] = sv[q];
          zsm[rr * L.z_stride + j] = (uint8_t)zv[q];
        }
      }
    }
  }
  pdl_wait_prior_grid();

  // B fragments of every group, [j][word i][lane][4 regs]:
  // reg e of word i holds x at the group-local elements
  //   e=0: (16t+4i, 16t+4i+2)   e=1: (64+16t+4i, 64+16t+4i+2)
  //   e=2: (16t+4i+1, 16t+4i+3) e=3: (64+16t+4i+1, 64+16t+4i+3)
  // for lane 4n + t: piece n % 3 of token n / 3 (low half = first element).
  // A float4 of x at group-local elements 4f'..4f'+3 (f' < 16: t = f'/4,
  // i = f'%4; f' >= 16 the same 64 elements higher) gives the pairs
  // (x0, x2) -> e = 0|1 and (x1, x3) -> e = 2|3 of every piece. All of a
  // thread's X loads are issued before any is used (one memory latency).
  {
    constexpr int NT = NW * 32;
    constexpr int PER = 4;  // float4s per thread per pass
    const int nf = a.Kp >> 2;  // float4s per token
    uint32_t *xf = reinterpret_cast<uint32_t *>(smem + L.xf_off);
    for (int tok = 0; tok < a.M && tok < NTOK; ++tok) {
      const float4 *xs = reinterpret_cast<const float4 *>(a.x + (size_t)tok * a.Kp);
      for (int f0 = 0; f0 < nf; f0 += PER * NT) {
        float4 xv[PER];
#pragma unroll
        for (int q = 0; q < PER; ++q) {
          const int f = f0 + q * NT + tid;
          xv[q] = f < nf ? ld_act(xs + f) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < PER; ++q) {
          const int f = f0 + q * NT + tid;
          if (f < nf) {
            const int j = f >> 5, fl = f & 31;  // group, float4 within the group
            const int hi = fl >> 4, tt = (fl >> 2) & 3, i = fl & 3;
            uint32_t p0[3], p1[3], p2[3], p3[3];
            split3_bf16(xv[q].x, p0[0], p0[1], p0[2]);
            split3_bf16(xv[q].y, p1[0], p1[1], p1[2]);
            split3_bf16(xv[q].z, p2[0], p2[1], p2[2]);
            split3_bf16(xv[q].w, p3[0], p3[1], p3[2]);
            uint32_t *dst = xf + (size_t)(j * 4 + i) * L.nl * 4;
#pragma unroll
            for (int p = 0; p < 3; ++p) {
              const int ln = 4 * (3 * tok + p) + tt;
              dst[ln * 4 + hi] = p0[p] | (p2[p] << 16);
              dst[ln * 4 + 2 + hi] = p1[p] | (p3[p] << 16);
            }
          }
        }
      }
    }
  }
  named_bar_sync(1, NW * 32);

  const uint32_t MAG = opaque(0x43004300u);  // bf16 pair (128, 128)
  const uint32_t ZP8 = opaque(0x43084308u);  // bf16 pair (136, 136): z = 8
  constexpr int NL = 12 * NTOK;              // lanes whose B columns are used
  // lanes past NL read lane t's fragments: their MMA columns are never used
  const uint32_t xf_lane = xf_s + (uint32_t)((lane < NL ? lane : t) * 16);
  const uint32_t ring_lane = smem_u32(ring) + (uint32_t)(g * L.ss + t * 16);
  const uint32_t row8 = (uint32_t)(8 * L.ss);

  const uint32_t sc_lane = smem_u32(smem + L.sc_off) + (uint32_t)(g * L.sc_stride * 4);
  const uint32_t z_lane = smem_u32(smem + L.z_off) + (uint32_t)(g * L.z_stride);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int chunk0 = 0;
  bool ok = true;

  auto reduce_chunk = [&](int b_end) {
    // y[tok, rows of blocks chunk0 .. b_end-1]: pieces, then warps in order
    named_bar_sync(2, NW * 32);
    const int row0 = 16 * chunk0, rowsn = min(16 * b_end, nrows) - row0;
    for (int it = tid; it < rowsn * NTOK; it += NW * 32) {
      const int tok = it / rowsn, rr = it - tok * rowsn;
      if (tok >= a.M) continue;
      const int bc = rr >> 4, row = rr & 15;
      float v[3] = {0.f, 0.f, 0.f};
      for (int w = 0; w < NW; ++w) {
        const float *pp = part + ((size_t)(bc * NW + w) * 16 + row) * (3 * NTOK) + 3 * tok;
#pragma unroll
        for (int p = 0; p < 3; ++p) v[p] += pp[p];
      }
      a.y[(size_t)tok * a.N + r0 + row0 + rr] = (v[0] + v[1]) + v[2];
    }
    named_bar_sync(2, NW * 32);
  };

  // one stage: wait for its bytes, decode the warp's JWS groups from it,
  // release it; `cur` holds its metadata, `nxt` receives the next stage's
  auto do_stage = [&](int slot, uint32_t par, int b, int seg) {
    if (ok) {
      ok = !*abort_flag && mbar_wait(&full[slot], par, a.status);
      if (!ok) *abort_flag = 1;
    }
    const int gs = min(L.gs, G - seg * L.gs);
    const uint32_t xb = xf_lane + (uint32_t)((seg * L.gs + warp) * 4 * NL * 16);
    const uint32_t wb_ = ring_lane + (uint32_t)(slot * L.stage + warp * 64);
    // The warp first copies its units' weight words out of the stage and
    // releases it (the producer refills the slot while the warp decodes), then
    // decodes and multiplies from registers.
    uint4 wva[JWS], wvb[JWS];
    const bool full_seg = gs == JWS * NW;  // every warp has all JWS groups
#pragma unroll
    for (int jj = 0; jj < JWS; ++jj) {
      if (ok && (full_seg || warp + jj * NW < gs)) {
        wva[jj] = lds128_u32(wb_ + jj * NW * 64);
        wvb[jj] = lds128_u32(wb_ + row8 + jj * NW * 64);
      } else {
        wva[jj] = wvb[jj] = make_uint4(0, 0, 0, 0);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    // one unit: group warp + jj*NW of the segment, rows g and g + 8
    auto unit = [&](int jj) {
      uint4 bfr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) bfr[i] = lds128_u32(xb + (uint32_t)((jj * NW * 4 + i) * NL * 16));
      const uint32_t jg = (uint32_t)(seg * L.gs + warp + jj * NW);  // group within the row
      const float s_a = lds_f32(sc_lane + (uint32_t)((16 * b * L.sc_stride + jg) * 4));
      const float s_b = lds_f32(sc_lane + (uint32_t)(((16 * b + 8) * L.sc_stride + jg) * 4));
      const uint32_t zpa = HAS_Z ? (0x4300u | lds_u8(z_lane + (uint32_t)(16 * b * L.z_stride) + jg)) * 0x00010001u : ZP8;
      const uint32_t zpb =
          HAS_Z ? (0x4300u | lds_u8(z_lane + (uint32_t)((16 * b + 8) * L.z_stride) + jg)) * 0x00010001u : ZP8;
      const uint32_t wa[4] = {wva[jj].x, wva[jj].y, wva[jj].z, wva[jj].w};
      const uint32_t wb[4] = {wvb[jj].x, wvb[jj].y, wvb[jj].z, wvb[jj].w};
      // two accumulator chains (words 0, 2 and 1, 3) halve the MMA dependency chain
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t a00 = bf2_sub(nib_pair(wa[i], MAG), zpa);
        const uint32_t a01 = bf2_sub(nib_pair(wa[i] >> 4, MAG), zpa);
        const uint32_t a02 = bf2_sub(nib_pair(wa[i] >> 8, MAG), zpa);
        const uint32_t a03 = bf2_sub(nib_pair(wa[i] >> 12, MAG), zpa);
        const uint32_t a10 = bf2_sub(nib_pair(wb[i], MAG), zpb);
        const uint32_t a11 = bf2_sub(nib_pair(wb[i] >> 4, MAG), zpb);
        const uint32_t a12 = bf2_sub(nib_pair(wb[i] >> 8, MAG), zpb);
        const uint32_t a13 = bf2_sub(nib_pair(wb[i] >> 12, MAG), zpb);
        mma_bf16_16816(c[i & 1], a00, a10, a01, a11, bfr[i].x, bfr[i].y);
        mma_bf16_16816(c[i & 1], a02, a12, a03, a13, bfr[i].z, bfr[i].w);
      }
      acc[0] = fmaf(s_a, c[0][0] + c[1][0], acc[0]);
      acc[1] = fmaf(s_a, c[0][1] + c[1][1], acc[1]);
      acc[2] = fmaf(s_b, c[0][2] + c[1][2], acc[2]);
      acc[3] = fmaf(s_b, c[0][3] + c[1][3], acc[3]);
    };
    if (ok) {
      if (full_seg) {
        // straight-line code, so the units' decodes and MMA chains interleave
#pragma unroll
        for (int jj = 0; jj < JWS; ++jj) unit(jj);
      } else {
#pragma unroll
        for (int jj = 0; jj < JWS; ++jj)
          if (warp + jj * NW < gs) unit(jj);
      }
    }
    if (seg == L.nseg - 1) {  // the block's K walk is complete: park its sums
      constexpr int NC = 3 * NTOK;  // used columns: piece p of token tk is column 3 tk + p
      float *pp = part + ((size_t)((b - chunk0) * NW + warp) * 16) * NC;
      if (2 * t < NC) {
        pp[g * NC + 2 * t] = acc[0];
        pp[(g + 8) * NC + 2 * t] = acc[2];
      }
      if (2 * t + 1 < NC) {
        pp[g * NC + 2 * t + 1] = acc[1];
        pp[(g + 8) * NC + 2 * t + 1] = acc[3];
      }
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      if (b + 1 - chunk0 == L.chunk && b + 1 < nblk) {
        reduce_chunk(b + 1);
        chunk0 = b + 1;
      }
    }
  };

  // stage cursor (slot, phase parity, block, K segment) advanced without divisions
  int slot = 0, b = 0, seg = 0;
  uint32_t par = 0;
  auto next = [&](int &sl, uint32_t &pr, int &bb, int &sg) {
    if (++sl == L.ns) {
      sl = 0;
      pr ^= 1u;
    }
    if (++sg == L.nseg) {
      sg = 0;
      ++bb;
    }
  };
  for (int st = 0; st < nst; ++st) {
    do_stage(slot, par, b, seg);
    next(slot, par, b, seg);
  }
  reduce_chunk(nblk);
}

}  // namespace lbc
