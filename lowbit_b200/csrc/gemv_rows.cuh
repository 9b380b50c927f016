// Register-streamed decode GEMV for one or two tokens per pass.
//
// One CTA = one row team of NW warps (NW * 32 * CH >= Kp / 32, NW <= 8):
// thread t owns the 16-byte chunks c = t + i*NW*32 (i < CH) of every weight
// row, so its activations stay in registers for the whole kernel. The CTA
// walks a contiguous range of whole blocks of R rows (block counts differ by
// at most one across the grid): each thread loads its chunks of the R rows
// straight from HBM into registers (ld.global.nc, no L1 allocation, L2
// evict-first), the loads of block b+1 in flight while block b is decoded --
// no shared-memory staging, no mbarriers and no producer thread between HBM
// and the FMA pipes. The R x MT partial dot products are reduced over the
// team with a transposing warp reduction and one named barrier per block.
//
// Arithmetic per chunk is the SIMT kernel's (gemv.cuh): exact (q - z) * 2^p
// through the 2^23 magic number and packed fp32x2 FMAs (W4A16), byte tables
// for E2M1 (MXFP4), dp4a with -z * asum once per group (W4A8) -- the
// reference's arithmetic (src/lowbit/csrc/kern_scalar.c:22-59) to the same
// rounding bound.
#pragma once

#include "gemv.cuh"

namespace lbc {

// 16 bytes of streamed weights: read-only path, no L1 allocation, L2 evict-first
__device__ __forceinline__ uint4 ldg_stream(const void *p, uint64_t pol) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ float4 zero4() { return make_float4(0.f, 0.f, 0.f, 0.f); }
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
__device__ __forceinline__ float sumsq4(float4 v, float s) {
  s = __fmaf_rn(v.x, v.x, s);
  s = __fmaf_rn(v.y, v.y, s);
  s = __fmaf_rn(v.z, v.z, s);
  return __fmaf_rn(v.w, v.w, s);
}
// silu(g) * u, rounded as the standalone SiLU-multiply kernel rounds it
__device__ __forceinline__ float glu1(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}
__device__ __forceinline__ float4 glu4(float4 g, float4 u) {
  return make_float4(glu1(g.x, u.x), glu1(g.y, u.y), glu1(g.z, u.z), glu1(g.w, u.w));
}

// 8-byte words that carry their own call tag: a single-copy-atomic store is
// seen by a peer either whole or not at all, so no fence orders data and flag
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// GATHER: column-parallel decode with the all-gather fused in. The call's
// epoch is the device counter + 1 (read after griddepcontrol.wait, so a
// launch that starts early under PDL sees the previous call's update). Each
// output value goes to this rank's own Y rows and, as one 8-byte word
// (epoch << 32 | fp32 bits), into every peer's landing buffer (peer pointers
// over NVLink) at the epoch's parity; the stores leave as the rows finish,
// overlapping the rest of the GEMV. Then every CTA polls its share of the
// global rows in its own landing buffer (bounded) until each word carries
// this epoch and copies the values into Y. The word is its own flag: no
// fence, arrival counter or last-CTA copy sits between the GEMV and the
// exchange. Every CTA of the grid is resident at once (the host sizes the
// grid by occupancy), so a CTA's wait on a peer's row never blocks the CTA
// that produces it. The CTA completing the grid advances the call counter.
// When the kernel completes, Y is whole on this GPU; no epoch is baked into
// the launch, so a CUDA graph of these calls replays correctly.
template <int FMT, int MT, int CH, int R, int NW, bool GATHER = false, int XM = XM_PLAIN>
__global__ void __launch_bounds__(NW * 32) gemv_rows_kernel(const GemvArgs a) {
  static_assert(XM == XM_PLAIN || FMT == FMT_W4A16, "fused prologues are W4A16 only");
  constexpr int V = R * MT;
  static_assert(V <= 32 && (V & (V - 1)) == 0, "R*MT must be a power of two <= 32");
  static_assert(NW >= 1 && (NW <= ROWS_MAX_WARPS || (NW <= ROWS_WIDE_WARPS && CH == 1 && MT <= 2)),
                "1..ROWS_MAX_WARPS warps per row team (ROWS_WIDE_WARPS with one chunk and token pair)");
  constexpr int NT = NW * 32;
  __shared__ float red[2][NW][V];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.y * MT;
  const int G = a.Kp >> 7, NB32 = a.Kp >> 5, Cs = a.Kp >> 5, RB = a.Kp >> 1;
  // whole blocks of R rows per CTA (block counts differ by at most one across
  // the grid); only the matrix's last block can be partial
  const int ntile = (a.N + R - 1) / R;
  const int t_begin = (int)((long long)blockIdx.x * ntile / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * ntile / gridDim.x);
  const int r_begin = t_begin * R;
  const int nrows = min(a.N, t_end * R) - r_begin;
  const int nblk = t_end - t_begin;
  const bool has_z = (FMT != FMT_MXFP4) && a.zeros != nullptr;

  // chunk bookkeeping; a chunk past the row end is clamped onto the last real
  // chunk and meets zero activations, so it adds exactly 0
  int ch_c[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) ch_c[i] = min(tid + i * NT, Cs - 1);

  // per-row base pointers of this CTA's first row; row rr adds rr * stride
  const uint8_t *qbase = a.qw + (size_t)r_begin * RB;
  const float *sbase = (FMT != FMT_MXFP4) ? a.scales + (size_t)r_begin * G : nullptr;
  const uint8_t *zbase = has_z ? a.zeros + (size_t)r_begin * G : nullptr;
  const uint8_t *ebase = (FMT == FMT_MXFP4) ? a.e8m0 + (size_t)r_begin * NB32 : nullptr;

  const uint64_t pol = policy_evict_first();
  uint4 w[2][R][CH];
  float sc[2][R][CH];
  uint32_t zz[2][R][CH];
  (void)zz;
  auto load_row = [&](int b, int j, int buf) {
    const int rr = b * R + j;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      w[buf][j][i] = ldg_stream(qbase + (size_t)rr * RB + (ch_c[i] << 4), pol);
      if (FMT == FMT_MXFP4) {
        sc[buf][j][i] = e8m0_half_scale(__ldg(ebase + (size_t)rr * NB32 + ch_c[i]));
      } else {
        sc[buf][j][i] = __ldg(sbase + (size_t)rr * G + (ch_c[i] >> 2));
        zz[buf][j][i] = has_z ? (uint32_t)__ldg(zbase + (size_t)rr * G + (ch_c[i] >> 2)) : 8u;
      }
    }
  };
  auto load = [&](int b, int buf) {
    if (b * R + R <= nrows) {
#pragma unroll
      for (int j = 0; j < R; ++j) load_row(b, j, buf);
    } else {
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (b * R + j < nrows) load_row(b, j, buf);
    }
  };

  // landing buffers of every rank (static across calls), from shared memory
  __shared__ uint64_t *land[GATHER ? LBC_GATHER_MAX_WORLD : 1];
  if (GATHER && tid < a.world) land[tid] = a.land_peers[tid];
  (void)land;

  // weights are static: the first block streams before the previous kernel
  // (which may produce X) has finished
  if (nblk > 0) load(0, 0);
  if (GATHER) __syncthreads();  // land[] is read by other threads
  pdl_launch_dependents();
  pdl_wait_prior_grid();

  // RMSNorm prologue: the team's threads hold the whole row of x between them
  // (CH * NT chunks cover Kp), so the sum of squares of x + residual comes
  // from the registers the loads below fill; the factor is applied after a
  // team-wide reduction
  float ss[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) ss[t] = 0.f;
  (void)ss;
  uint64_t xr[CH][MT][16];
  uint32_t xl[CH][MT][4], xh[CH][MT][4];
  int xsum[CH][MT];
  (void)xr;
  (void)xl;
  (void)xh;
  (void)xsum;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int c = tid + i * NT;
    int lo, hi;
    if (FMT == FMT_MXFP4) {
      lo = c << 5;
      hi = lo + 16;
    } else {
      lo = ((c >> 2) << 7) + ((c & 3) << 4);
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
        // z * asum[m,g] is subtracted once per group, in its first chunk, as
        // the reference applies it (src/lowbit/csrc/kern_scalar.c:49-59)
        xsum[i][t] = (ok && (c & 3) == 0) ? ld_act(a.asum + (size_t)m * G + (c >> 2)) : 0;
      } else {
        const size_t xrow = (size_t)m * a.Kp * (XM == XM_GLU ? 2 : 1);
        const float4 *pl = reinterpret_cast<const float4 *>(a.x + xrow + lo);
        const float4 *ph = reinterpret_cast<const float4 *>(a.x + xrow + hi);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 l4 = make_float4(0.f, 0.f, 0.f, 0.f), h4 = l4;
          if (ok) {
            l4 = ld_act(pl + q);
            h4 = ld_act(ph + q);
            if (XM == XM_RMSNORM) {
              if (a.xres) {
                l4 = add4(l4, ld_act(reinterpret_cast<const float4 *>(a.xres + xrow + lo) + q));
                h4 = add4(h4, ld_act(reinterpret_cast<const float4 *>(a.xres + xrow + hi) + q));
                if (a.xout && blockIdx.x == 0) {
                  reinterpret_cast<float4 *>(a.xout + xrow + lo)[q] = l4;
                  reinterpret_cast<float4 *>(a.xout + xrow + hi)[q] = h4;
                }
              }
              ss[t] = sumsq4(h4, sumsq4(l4, ss[t]));
            } else if (XM == XM_GLU) {
              l4 = glu4(l4, ld_act(pl + q + a.Kp / 4));
              h4 = glu4(h4, ld_act(ph + q + a.Kp / 4));
            }
          }
          xr[i][t][4 * q + 0] = pack2(__float_as_uint(l4.x), __float_as_uint(h4.x));
          xr[i][t][4 * q + 1] = pack2(__float_as_uint(l4.y), __float_as_uint(h4.y));
          xr[i][t][4 * q + 2] = pack2(__float_as_uint(l4.z), __float_as_uint(h4.z));
          xr[i][t][4 * q + 3] = pack2(__float_as_uint(l4.w), __float_as_uint(h4.w));
        }
      }
    }
  }
  if (XM == XM_RMSNORM) {
    __shared__ float nred[NW][MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], o);
      if (lane == 0) nred[warp][t] = ss[t];
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      float tot = 0.f;
      for (int ww = 0; ww < NW; ++ww) tot += nred[ww][t];
      const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.Kp), a.eps)));
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = tid + i * NT;
        const int lo = ((c >> 2) << 7) + ((c & 3) << 4), hi = lo + 64;
        const bool ok = c < Cs;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 wl = zero4(), wh = zero4();
          if (ok) {
            wl = __ldg(reinterpret_cast<const float4 *>(a.lnw + lo) + q);
            wh = __ldg(reinterpret_cast<const float4 *>(a.lnw + hi) + q);
          }
          const float wlv[4] = {wl.x, wl.y, wl.z, wl.w}, whv[4] = {wh.x, wh.y, wh.z, wh.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint64_t v = xr[i][t][4 * q + e];
            xr[i][t][4 * q + e] = pack2(__float_as_uint(__fmul_rn(__fmul_rn(lo_f(v), r), wlv[e])),
                                        __float_as_uint(__fmul_rn(__fmul_rn(hi_f(v), r), whv[e])));
          }
        }
      }
    }
  }
  float xsc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) xsc[t] = (FMT == FMT_W4A8 && m0 + t < a.M) ? ld_act(a.xs + m0 + t) : 1.f;
  const uint32_t MAG = opaque(0x4B000000u);
  uint32_t epoch = 0;
  size_t land_off = 0;  // the epoch parity's half of every landing buffer
  if (GATHER) {
    epoch = *reinterpret_cast<volatile const uint32_t *>(a.epoch) + 1u;
    land_off = (size_t)(epoch & 1u) * 2 * a.ld_y;
  }
  (void)land_off;

  auto compute = [&](int b, int buf) {
    float part[R][MT];
#pragma unroll
    for (int j = 0; j < R; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) part[j][t] = 0.f;
#pragma unroll
    for (int j = 0; j < R; ++j) {
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const uint4 wv = w[buf][j][i];
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
            const int d = acc[t] - (int)zz[buf][j][i] * xsum[i][t];
            part[j][t] = fmaf((float)d, sc[buf][j][i], part[j][t]);
          }
        } else {
          float dot[MT];
          if (FMT == FMT_W4A16)
            dot_w4a16<MT>(wv, zz[buf][j][i], xr[i], dot, MAG);
          else
            dot_mxfp4<MT, 16>(wv, xr[i], 0, dot, MAG);
#pragma unroll
          for (int t = 0; t < MT; ++t) part[j][t] = fmaf(dot[t], sc[buf][j][i], part[j][t]);
        }
      }
    }
    float v[V];
#pragma unroll
    for (int j = 0; j < R; ++j)
#pragma unroll
      for (int t = 0; t < MT; ++t) v[j * MT + t] = part[j][t];
    const float tot = warp_reduce_multi<V>(v, lane);
    constexpr int PER = 32 / V;
    int idx = -1;
    float val = 0.f;
    if (NW == 1) {
      if ((lane % PER) == 0) {
        idx = lane / PER;
        val = tot;
      }
    } else {
      if ((lane % PER) == 0) red[b & 1][warp][lane / PER] = tot;
      named_bar_sync(1, NT);
      if (tid < V) {
        float s = 0.f;
        for (int ww = 0; ww < NW; ++ww) s += red[b & 1][ww][tid];
        idx = tid;
        val = s;
      }
    }
    if (idx >= 0) {
      const int j = idx / MT, t = idx % MT;
      const int rr = b * R + j, m = m0 + t;
      if (rr < nrows && m < a.M) {
        const float out = (FMT == FMT_W4A8) ? val * xsc[t] : val;
        if (GATHER) {
          const size_t at = (size_t)m * a.ld_y + a.row0 + r_begin + rr;
          a.y[at] = out;
          const uint64_t word = ((uint64_t)epoch << 32) | __float_as_uint(out);
          for (int p = 0; p < a.world; ++p)
            if (p != a.rank) st_relaxed_sys_u64(land[p] + land_off + at, word);
        } else {
          a.y[(size_t)m * a.N + r_begin + rr] = out;
        }
      }
    }
  };

  for (int b = 0; b < nblk; b += 2) {
    if (b + 1 < nblk) load(b + 1, 1);
    compute(b, 0);
    if (b + 1 < nblk) {
      if (b + 2 < nblk) load(b + 2, 0);
      compute(b + 1, 1);
    }
  }

  if (GATHER) {
    // this CTA's share of the global rows (any split works: every CTA is
    // resident); this rank's own rows are already in Y
    const int g0 = (int)((long long)blockIdx.x * a.ld_y / gridDim.x);
    const int g1 = (int)((long long)(blockIdx.x + 1) * a.ld_y / gridDim.x);
    const int span = g1 - g0;
    const uint64_t *mine = land[a.rank] + land_off;
    const long long t0 = clock64(), lim = wait_cycles(a.status);
    bool gave_up = false;
    for (int e = tid; e < a.M * span && !gave_up; e += NT) {
      const int m = e / span, row = g0 + e % span;
      if (row >= a.row0 && row < a.row0 + a.N) continue;
      const size_t at = (size_t)m * a.ld_y + row;
      uint64_t v = ld_relaxed_sys_u64(mine + at);
      while ((uint32_t)(v >> 32) != epoch) {
        if (clock64() - t0 > lim) {
          set_status(a.status, LBC_ERR_TIMEOUT);
          gave_up = true;
          break;
        }
        v = ld_relaxed_sys_u64(mine + at);
      }
      if (!gave_up) a.y[at] = __uint_as_float((uint32_t)v);
    }
    __syncthreads();
    if (tid == 0) {
      // every CTA read the epoch before counting itself (acq_rel atomic)
      if (atom_add_acq_rel_gpu(a.counter, 1u) + 1u == gridDim.x * gridDim.y) {
        atomicExch(a.counter, 0u);  // ready for the next call
        *a.epoch = epoch;
      }
    }
  }
}

}  // namespace lbc
