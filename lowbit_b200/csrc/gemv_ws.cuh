// Warp-specialised decode GEMV for one or two tokens (int4 formats).
//
// One CTA = NW consumer warps + 1 producer warp. Thread t of the consumers
// owns CA adjacent 16-byte chunks of every weight row (chunks CA*t ..
// CA*t+CA-1, all inside one 128-element group when CA <= 4), so its
// activations stay in registers for the whole kernel and one zero point,
// one scale and one rescale serve CA*32 elements of a row. The CTA walks a
// contiguous range of rows in blocks of R rows; the producer streams block
// after block -- R whole rows of codes plus their scales and zero points,
// contiguous in HBM -- into an S-deep shared-memory ring with 1-D bulk
// copies (no multicast), so the bytes in flight cost no registers. Consumers
// read their chunks of each row from shared memory (consecutive threads,
// consecutive 16-byte chunks: conflict-free), reduce the R x MT partial dot
// products with a transposing warp reduction and one named barrier per
// block, and release the stage.
//
// Arithmetic per chunk is the SIMT kernel's (gemv.cuh): exact (q - z) * 2^p
// through the 2^23 magic number and packed fp32x2 FMAs (W4A16), dp4a with
// -z * asum once per group (W4A8) -- the reference's arithmetic
// (src/lowbit/csrc/kern_scalar.c:22-59) to the same rounding bound.
#pragma once

#include "gemv.cuh"

namespace lbc {

constexpr int WS_MAX_WARPS = 8;  // consumer warps per CTA

struct WsSmem {
  int stage_bytes, codes_bytes, sc_off, z_off, bar_off, red_off, total;
};

// Stage layout: R rows of codes (R * Kp/2 bytes), then R rows of scales
// (R * G * 4), then R rows of zero points (R * G), each part 16-byte aligned.
__host__ __device__ inline WsSmem ws_smem_layout(int Kp, int R, int S, int nw, int v, bool has_z) {
  WsSmem L;
  const int G = Kp >> 7;
  L.codes_bytes = R * (Kp >> 1);
  L.sc_off = L.codes_bytes;
  L.z_off = L.sc_off + ((R * G * 4 + 15) & ~15);
  L.stage_bytes = ((L.z_off + (has_z ? ((R * G + 15) & ~15) : 0)) + 127) & ~127;
  L.bar_off = S * L.stage_bytes;
  L.red_off = L.bar_off + 16 * S + 16;
  L.total = L.red_off + 2 * nw * v * 4;
  return L;
}

template <int FMT, int MT, int CA, int R>
__global__ void __launch_bounds__((WS_MAX_WARPS + 1) * 32) gemv_ws_kernel(const GemvArgs a) {
  static_assert(FMT != FMT_MXFP4, "int4 formats only");
  constexpr int V = R * MT;
  static_assert(V <= 32 && (V & (V - 1)) == 0, "R*MT must be a power of two <= 32");
  extern __shared__ __align__(128) uint8_t smem[];

  const int NW = (blockDim.x >> 5) - 1;  // consumer warps
  const int NC = NW * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = a.stages;
  const int G = a.Kp >> 7, Cs = a.Kp >> 5, RB = a.Kp >> 1;
  const bool has_z = a.zeros != nullptr;
  const WsSmem L = ws_smem_layout(a.Kp, R, S, NW, V, has_z);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *empty = full + S;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.bar_off + 16 * S);
  float *red = reinterpret_cast<float *>(smem + L.red_off);

  const int m0 = blockIdx.y * MT;
  const int r_begin = (int)((long long)blockIdx.x * a.N / gridDim.x);
  const int r_end = (int)((long long)(blockIdx.x + 1) * a.N / gridDim.x);
  const int nrows = r_end - r_begin;
  const int nblk = (nrows + R - 1) / R;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      auto issue = [&](int b) {
        const int s = b % S;
        const int r0 = r_begin + b * R;
        const int rows = min(R, r_end - r0);
        uint8_t *st = smem + s * L.stage_bytes;
        const uint32_t cb = (uint32_t)(rows * RB), sb = (uint32_t)(rows * G * 4), zb = (uint32_t)(rows * G);
        mbar_expect_tx(&full[s], cb + sb + (has_z ? zb : 0u));
        bulk_g2s(st, a.qw + (size_t)r0 * RB, cb, &full[s], pol);
        bulk_g2s(st + L.sc_off, reinterpret_cast<const uint8_t *>(a.scales) + (size_t)r0 * G * 4, sb, &full[s], pol);
        if (has_z) bulk_g2s(st + L.z_off, a.zeros + (size_t)r0 * G, zb, &full[s], pol);
      };
      // weights are static: stream them before the previous kernel finishes
      const int pro = min(S, nblk);
      for (int b = 0; b < pro; ++b) issue(b);
      for (int b = pro; b < nblk; ++b) {
        const int s = b % S;
        if (*abort_flag || !mbar_wait(&empty[s], ((uint32_t)(b / S) & 1u) ^ 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        issue(b);
      }
    }
    pdl_launch_dependents();
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_launch_dependents();
  pdl_wait_prior_grid();  // X (or xq / asum) may come from the previous kernel

  // chunks CA*tid .. CA*tid + CA - 1; past the row end: zero activations
  const int c0 = min(CA * tid, Cs - CA);
  const bool active = CA * tid < Cs;
  const int g0 = c0 >> 2;  // the chunks' group (CA <= 4, chunks never straddle)
  uint64_t xr[CA][MT][16];
  uint32_t xl[CA][MT][4], xh[CA][MT][4];
  int xsum[MT];
  (void)xr;
  (void)xl;
  (void)xh;
  (void)xsum;
#pragma unroll
  for (int i = 0; i < CA; ++i) {
    const int c = c0 + i;
    const int lo = ((c >> 2) << 7) + ((c & 3) << 4), hi = lo + 64;
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int m = m0 + t;
      const bool ok = active && (m < a.M);
      if (FMT == FMT_W4A8) {
        uint4 vl = make_uint4(0, 0, 0, 0), vh = make_uint4(0, 0, 0, 0);
        if (ok) {
          vl = __ldg(reinterpret_cast<const uint4 *>(a.xq + (size_t)m * a.Kp + lo));
          vh = __ldg(reinterpret_cast<const uint4 *>(a.xq + (size_t)m * a.Kp + hi));
        }
        xl[i][t][0] = vl.x; xl[i][t][1] = vl.y; xl[i][t][2] = vl.z; xl[i][t][3] = vl.w;
        xh[i][t][0] = vh.x; xh[i][t][1] = vh.y; xh[i][t][2] = vh.z; xh[i][t][3] = vh.w;
      } else {
        const float4 *pl = reinterpret_cast<const float4 *>(a.x + (size_t)m * a.Kp + lo);
        const float4 *ph = reinterpret_cast<const float4 *>(a.x + (size_t)m * a.Kp + hi);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 l4 = make_float4(0.f, 0.f, 0.f, 0.f), h4 = l4;
          if (ok) {
            l4 = __ldg(pl + q);
            h4 = __ldg(ph + q);
          }
          xr[i][t][4 * q + 0] = pack2(__float_as_uint(l4.x), __float_as_uint(h4.x));
          xr[i][t][4 * q + 1] = pack2(__float_as_uint(l4.y), __float_as_uint(h4.y));
          xr[i][t][4 * q + 2] = pack2(__float_as_uint(l4.z), __float_as_uint(h4.z));
          xr[i][t][4 * q + 3] = pack2(__float_as_uint(l4.w), __float_as_uint(h4.w));
        }
      }
    }
  }
  if (FMT == FMT_W4A8) {
    // z * asum[m,g] is subtracted once per group, by the thread holding the
    // group's first chunk, as the reference applies it (kern_scalar.c:49-59)
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int m = m0 + t;
      xsum[t] = (active && m < a.M && (c0 & 3) == 0) ? __ldg(a.asum + (size_t)m * G + g0) : 0;
    }
  }
  float xsc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) xsc[t] = (FMT == FMT_W4A8 && m0 + t < a.M) ? __ldg(a.xs + m0 + t) : 1.f;
  const uint32_t MAG = opaque(0x4B000000u);

  bool ok = true;
  for (int b = 0; b < nblk; ++b) {
    const int s = b % S;
    const int rows = min(R, nrows - b * R);
    if (ok) ok = !*abort_flag && mbar_wait(&full[s], (uint32_t)(b / S) & 1u, a.status);
    if (!ok) *abort_flag = 1;
    const uint8_t *st = smem + s * L.stage_bytes;
    const float *ssc = reinterpret_cast<const float *>(st + L.sc_off);
    const uint8_t *sz = st + L.z_off;

    float part[R][MT];
    // full blocks take a branch-free path (rows interleave freely); the
    // last, partial block guards every row
    auto row_dot = [&](int r) {
        const float sc = ssc[r * G + g0];
        const uint32_t z = has_z ? (uint32_t)sz[r * G + g0] : 8u;
        const uint8_t *rowp = st + r * RB + (c0 << 4);
        if (FMT == FMT_W4A8) {
          int acc[MT];
#pragma unroll
          for (int t = 0; t < MT; ++t) acc[t] = 0;
#pragma unroll
          for (int i = 0; i < CA; ++i) {
            const uint4 wv = lds128(rowp + 16 * i);
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
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) part[r][t] = (float)(acc[t] - (int)z * xsum[t]) * sc;
        } else {
          // -(2^23 + z * 2^p) for the four nibble positions
          const uint64_t nz01 = pack2(0xCB000000u | z, 0xCB000000u | (z << 4));
          const uint64_t nz23 = pack2(0xCB000000u | (z << 8), 0xCB000000u | (z << 12));
          uint64_t accA[MT], accB[MT];
#pragma unroll
          for (int t = 0; t < MT; ++t) accA[t] = accB[t] = 0ull;
#pragma unroll
          for (int i = 0; i < CA; ++i) {
            const uint4 wv = lds128(rowp + 16 * i);
            const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t w = w4[q];
              const uint32_t h = w >> 16;
              const uint64_t pa = nib2<0x000Fu, 0x00F0u>(w, MAG, nz01);
              const uint64_t pb = nib2<0x0F00u, 0xF000u>(w, MAG, nz23);
              const uint64_t pc = nib2<0x000Fu, 0x00F0u>(h, MAG, nz01);
              const uint64_t pd = nib2<0x0F00u, 0xF000u>(h, MAG, nz23);
#pragma unroll
              for (int t = 0; t < MT; ++t) {
                accA[t] = ffma2(pa, xr[i][t][4 * q + 0], accA[t]);
                accB[t] = ffma2(pb, xr[i][t][4 * q + 1], accB[t]);
                accA[t] = ffma2(pc, xr[i][t][4 * q + 2], accA[t]);
                accB[t] = ffma2(pd, xr[i][t][4 * q + 3], accB[t]);
              }
            }
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const float d = fmaf(hi_f(accB[t]), 1.0f / 4096.0f,
                                 fmaf(lo_f(accB[t]), 1.0f / 256.0f, fmaf(hi_f(accA[t]), 1.0f / 16.0f, lo_f(accA[t]))));
            part[r][t] = d * sc;
          }
        }
    };
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < MT; ++t) part[r][t] = 0.f;
    if (rows == R) {
#pragma unroll
      for (int r = 0; r < R; ++r) row_dot(r);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < rows) row_dot(r);
    }
    // the stage's shared memory is no longer read: hand it back
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    float v[V];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < MT; ++t) v[r * MT + t] = part[r][t];
    const float tot = warp_reduce_multi<V>(v, lane);
    constexpr int PER = 32 / V;
    float *rb = red + (b & 1) * NW * V;
    if ((lane % PER) == 0) rb[warp * V + lane / PER] = tot;
    named_bar_sync(1, NC);
    if (tid < V) {
      float sum = 0.f;
      for (int w = 0; w < NW; ++w) sum += rb[w * V + tid];
      const int r = tid / MT, t = tid % MT;
      const int m = m0 + t;
      if (ok && r < rows && m < a.M)
        a.y[(size_t)m * a.N + r_begin + b * R + r] = (FMT == FMT_W4A8) ? sum * xsc[t] : sum;
    }
  }
}

}  // namespace lbc
