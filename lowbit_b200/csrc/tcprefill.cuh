// Tensor-core prefill GEMM (tcgen05, sm_100a) for many tokens.
//
// Y[M,N] = X[M,K] . W[N,K]^T, W4A16, MXFP4 and W4A8. An output tile is 128 weight
// rows (the MMA's M) x 128 tokens (its N); a persistent CTA walks its tiles
// and, per tile, the 256-K units of the row, two 128-element groups each:
//
//   * the tokens' activations are cast to bf16 once per call (one piece: the
//     prefill tolerance is 4e-3 * (|X| . |W|^T)) by the activation-block
//     kernel of the decode path, in the same permuted, canonical layout, and
//     arrive by TMA with the weights;
//   * W4A16: A = (q - z) in bf16 -- exact -- and the group scale is applied in
//     fp32 to each group's accumulator, so the only rounding is that of X
//     (|error| <= 2^-8 * (|X| . |W|^T)); MXFP4: A = e2m1(q) * 2^(e-127), exact
//     in bf16, scale 1;
//   * W4A8 (kind::i8): A = q - z as s8 (|q - z| <= 15), B = the per-token int8
//     activations, so each group's int32 accumulator is exactly the
//     reference's sum(q * a) - z * sum(a); the epilogue converts it exactly
//     (|acc| < 2^22) and applies the group scale in fp32, the token scale xs
//     at the store -- no tolerance beyond the reference's own;
//   * TMEM (512 columns): the unit's two A groups [0, 128) and a ring of
//     three per-group accumulators D [128, 512). The MMAs of the next groups
//     run while the epilogue warps fold D_g * s_g into their running sums,
//     held in registers: eight epilogue warps, two per lane quadrant, each
//     owning 64 of the tile's 128 token columns. After the tile's last group
//     they store Y to HBM (lanes are consecutive weight rows, so each store
//     instruction writes 128 contiguous bytes of a token's row);
//   * warps: 4 dequantising warps (one per lane quadrant, both groups of a
//     unit), a producer, two MMA issuers (one per group) and 8 epilogue warps;
//     15 warps leave 128 registers per thread on B200's four sub-partitions;
//     where
//     several warps wait for the same event, one polls the mbarrier and the
//     others wait on a named barrier, blocked in hardware;
//   * column parallelism (a.y_peers): each rank owns rows [row0, row0 + N) of
//     an ld_y-row weight; the epilogue stores every finished tile into every
//     rank's Y over NVLink (peer pointers) while later tiles are still being
//     computed, so the all-gather overlaps the GEMM; a per-call counter per
//     rank tells each GPU when all rows have arrived.
#pragma once

#include "tcgemm.cuh"

namespace lbc {

constexpr int PF_TOK = 128;     // tokens per tile (MMA N)
constexpr int PF_THREADS = 480;  // 4 dequantising + producer + 2 MMA + 8 epilogue warps

// SPLIT: the split-K instantiation (a.ksplit > 1); without it the K range of
// an item is the whole row and the position bookkeeping folds away. GATHER:
// the column-parallel instantiation (a.y_peers, never split).
template <int FMT, bool SPLIT, bool GATHER = false>
__global__ void __maxnreg__(128) tcprefill_kernel(const __grid_constant__ CUtensorMap wmap, const TcArgs a) {
  constexpr bool I8 = (FMT == FMT_W4A8);
  constexpr int NMMA = PF_TOK;
  constexpr int GCOLS = I8 ? 32 : 64, HCOLS = GCOLS / 2;  // TMEM columns per (row, group) / half group
  constexpr int DCOL0 = 128, NDR = 3;                      // accumulator ring
  constexpr int NSTEP = I8 ? 4 : 8;                        // K=32 (i8) or K=16 (bf16) MMAs per group
  constexpr int EPR = I8 ? 16 : 8;                         // B elements per 16-byte core-matrix row
  constexpr int SBO = TC_KB / EPR * 128;                   // bytes between 8-row groups of B
  constexpr int NDQ = 4;
  constexpr int W_PROD = NDQ, W_MMA = NDQ + 1, W_EPI = NDQ + 3, NEPI = 8;
  constexpr int ECOLS = NMMA / 2;        // token columns per epilogue thread

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int S = a.stages;
  const TcSmem L = tc_smem_layout(S, a.b_block_bytes, PF_TOK);
  const int BSTRIDE = (a.b_block_bytes + 127) / 128 * 128;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *full = bars, *empty = bars + S;
  uint64_t *a_full = bars + 2 * S, *a_empty = a_full + 2;
  uint64_t *d_full = a_empty + 2, *d_empty = d_full + NDR, *fin = d_empty + NDR;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nch = (a.M + PF_TOK - 1) / PF_TOK;  // token chunks
  const int ntile = a.ntiles * nch;             // output tiles
  // work items: tile t split into KS contiguous K ranges (split-K when the
  // tiles alone cannot fill the GPU): each split stores its partial tile to a
  // workspace slot and tc_split_reduce_kernel adds the slots in split order
  // (deterministic; no CTA waits on another)
  const int KS = SPLIT ? a.ksplit : 1;
  const int nitem = ntile * KS;

  // position of a unit: tile t (n tile t / nch, token chunk t % nch), K block
  // kb, the end of its item's K range, the item's split index
  struct Pos {
    int t, kb, khi, sp;
  };
  auto start = [&](int w) {
    const int sp = w % KS;
    return Pos{w / KS, sp * a.nkb / KS, (sp + 1) * a.nkb / KS, sp};
  };
  auto advance = [&](Pos &p) {
    if constexpr (SPLIT) {
      if (++p.kb == p.khi) p = start(p.t * KS + p.sp + gridDim.x);
    } else {
      if (++p.kb == a.nkb) {
        p.kb = 0;
        p.t += gridDim.x;
      }
    }
  };
  int nunits = 0;
  for (int w = blockIdx.x; w < nitem; w += gridDim.x) {
    const Pos p = start(w);
    nunits += p.khi - p.kb;
  }

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NDQ + 2);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&a_full[g], NDQ);
      mbar_init(&a_empty[g], 1);
    }
    for (int d = 0; d < NDR; ++d) {
      mbar_init(&d_full[d], 1);
      mbar_init(&d_empty[d], NEPI);
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
      const uint32_t txb = (uint32_t)TC_WBYTES + (uint32_t)a.b_block_bytes;
      const int pro = min(S, nunits);
      Pos p = start(blockIdx.x);
      // weights are static: stream them before the previous kernel finishes
      for (int i = 0; i < pro; ++i) {
        mbar_expect_tx(&full[i], txb);
        tma_load_2d(smem + L.w_off + i * TC_WBYTES, &wmap, p.kb * 128, (p.t / nch) * TC_ROWS, &full[i], pol);
        advance(p);
      }
      // the activation blocks come from the preparation kernel before this one
      pdl_wait_prior_grid();
      Pos pb = start(blockIdx.x);
      for (int i = 0; i < pro; ++i) {
        bulk_g2s(smem + L.b_off + i * BSTRIDE, a.bglob + ((size_t)(pb.t % nch) * a.nkb + pb.kb) * a.b_block_bytes,
                 (uint32_t)a.b_block_bytes, &full[i], pol);
        advance(pb);
      }
      int s = pro % S;
      uint32_t ph = (uint32_t)(pro / S) & 1u;
      for (int i = pro; i < nunits; ++i) {
        if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&full[s], txb);
        tma_load_2d(smem + L.w_off + s * TC_WBYTES, &wmap, p.kb * 128, (p.t / nch) * TC_ROWS, &full[s], pol);
        bulk_g2s(smem + L.b_off + s * BSTRIDE, a.bglob + ((size_t)(p.t % nch) * a.nkb + p.kb) * a.b_block_bytes,
                 (uint32_t)a.b_block_bytes, &full[s], pol);
        advance(p);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == W_MMA || warp == W_MMA + 1) {
    // ------------------------------------------------------------ MMA issuers (one per group)
    if (lane == 0) {
      const int h = warp - W_MMA;
      const uint32_t idesc = I8 ? tc::idesc_s8_s32(NMMA) : tc::idesc_bf16_f32(NMMA);
      const uint32_t hoff = (uint32_t)(128 * h) / (uint32_t)EPR * 128u;
      int s = 0, d = h, dr = 0;  // group sequence v = 2i + h: slot v % 3, round v / 3
      uint32_t ph = 0;
      for (int i = 0; i < nunits && !*abort_flag; ++i) {
        if (!mbar_wait(&full[s], ph, a.status) || !mbar_wait(&a_full[h], (uint32_t)i & 1u, a.status) ||
            !mbar_wait(&d_empty[d], ((uint32_t)dr & 1u) ^ 1u, a.status)) {
          *abort_flag = 1;
          break;
        }
        tc::fence_after_sync();
        const uint64_t bd0 = tc::smem_desc(smem_u32(smem + L.b_off + s * BSTRIDE) + hoff, 128u, (uint32_t)SBO);
        const uint32_t dcol = tmem + DCOL0 + d * NMMA;
        const uint32_t acol0 = tmem + h * GCOLS;
#pragma unroll
        for (int j = 0; j < NSTEP; ++j) {
          if (I8)
            tc::mma_s8_ts(dcol, acol0 + 8 * j, bd0 + 16u * j, idesc, j > 0);
          else
            tc::mma_bf16_ts(dcol, acol0 + 8 * j, bd0 + 16u * j, idesc, j > 0);
        }
        tc::commit(&d_full[d]);
        tc::commit(&a_empty[h]);
        tc::commit(&empty[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
        d += 2;  // v advances by 2
        if (d >= NDR) {
          d -= NDR;
          ++dr;
        }
      }
      tc::commit(fin);
      mbar_wait(fin, 0, a.status);
    }
  } else if (warp < NDQ) {
    // ------------------------------------------------------------ dequantisers
    // one warp per lane quadrant: thread = weight row, both groups of the unit
    const int q = warp;
    const int row = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const uint32_t MAG = opaque(0x43004300u);
    const int NB32 = a.Kp >> 5;
    struct Meta {
      uint32_t z[2];
      uint32_t e2[8];
    };
    auto load_meta = [&](Pos p) {
      Meta m;
#pragma unroll
      for (int g = 0; g < 2; ++g) m.z[g] = 8u;
#pragma unroll
      for (int b = 0; b < 8; ++b) m.e2[b] = 0u;
      const int n = (p.t / nch) * TC_ROWS + row;
      if (p.t < ntile && n < a.N) {
        if (FMT == FMT_MXFP4) {
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            const int blk = 8 * p.kb + b;
            m.e2[b] = blk < NB32 ? (uint32_t)__ldg(a.e8m0 + (size_t)n * NB32 + blk) : 0u;
          }
        } else if (a.zeros) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int gi = 2 * p.kb + g;
            if (gi < a.G) m.z[g] = __ldg(a.zeros + (size_t)n * a.G + gi);
          }
        }
      }
      return m;
    };
    // metadata through a 2-deep register queue (loads for unit i + 2)
    Pos pq = start(blockIdx.x);
    Meta mq[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      mq[j] = load_meta(pq);
      advance(pq);
    }
    // warp 0 polls; the other three wait on a named barrier
    auto group_wait = [&](uint64_t *bar, uint32_t parity) {
      if (q == 0 && !*abort_flag && !mbar_wait(bar, parity, a.status)) *abort_flag = 1;
      named_bar_sync(1, NDQ * 32);
      return !*abort_flag;
    };
    const uint8_t *wbase = smem + L.w_off + row * 128;
    const int sw = row & 7;
    auto lds_unit = [&](int s, uint4 (&w)[8]) {
#pragma unroll
      for (int c = 0; c < 8; ++c) w[c] = *reinterpret_cast<const uint4 *>(wbase + s * TC_WBYTES + ((c ^ sw) << 4));
    };
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    uint4 wcur[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) wcur[c] = make_uint4(0, 0, 0, 0);
    if (nunits > 0) {
      ok = group_wait(&full[0], 0);
      lds_unit(0, wcur);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[0]);
    }
    for (int i = 0; i < nunits; ++i) {
      const Meta mcur = mq[0];
      mq[0] = mq[1];
      if (i + 2 < nunits) mq[1] = load_meta(pq);
      advance(pq);
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        // group g's A buffer is free once the previous unit's MMAs on it are done
        ok = group_wait(&a_empty[g], ((uint32_t)i & 1u) ^ 1u) && ok;
        tc::fence_after_sync();
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t av[32];
          const uint4 wh[2] = {wcur[4 * g + 2 * hf], wcur[4 * g + 2 * hf + 1]};
          if (FMT == FMT_W4A16) {
            deq_w4a16(wh, mcur.z[g], av, MAG);
          } else if (FMT == FMT_W4A8) {
            // u8 codes, then q - z as s8 bytes: q + (128 - z) stays below 256 in
            // every byte (no carry between bytes), and flipping bit 7 maps it
            // to the two's complement of q - z
            deq_w4a8(wh, av);
            const uint32_t zc = (128u - mcur.z[g]) * 0x01010101u;
#pragma unroll
            for (int c = 0; c < 16; ++c) av[c] = (av[c] + zc) ^ 0x80808080u;
          } else {
            const uint32_t e2[2] = {mcur.e2[4 * g + 2 * hf], mcur.e2[4 * g + 2 * hf + 1]};
            deq_mxfp4(wh, e2, av);
          }
          if (ok) {
            const uint32_t at = tmem + lane_base + g * GCOLS + hf * HCOLS;
            uint32_t part[16];
#pragma unroll
            for (int c = 0; c < HCOLS / 16; ++c) {
#pragma unroll
              for (int j = 0; j < 16; ++j) part[j] = av[16 * c + j];
              tc::st16(at + 16 * c, part);
            }
          }
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[g]);
      }
      // next unit's codes
      int s1 = s + 1;
      uint32_t ph1 = ph;
      if (s1 == S) {
        s1 = 0;
        ph1 ^= 1u;
      }
      if (i + 1 < nunits) {
        ok = group_wait(&full[s1], ph1) && ok;
        lds_unit(s1, wcur);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s1]);
      }
      s = s1;
      ph = ph1;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3, ch = (warp - W_EPI) >> 2;  // lane quadrant, column half
    const int row = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    pdl_wait_prior_grid();  // Y may still be read by the previous kernel
    // fused all-gather: this call's parity of every rank's Y buffers
    float *const *ydst = nullptr;
    if (GATHER) {
      const uint32_t ep = *reinterpret_cast<volatile const uint32_t *>(a.ag_epoch) + 1u;
      ydst = a.y_peers + (ep & 1u) * a.world;
    }
    auto load_scales = [&](Pos p, float (&sc)[2]) {
      const int n = (p.t / nch) * TC_ROWS + row;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gi = 2 * p.kb + h;
        sc[h] = (FMT == FMT_MXFP4) ? 1.f
                                   : ((p.t < ntile && n < a.N && gi < a.G) ? __ldg(a.scales + (size_t)n * a.G + gi) : 0.f);
      }
    };
    Pos pq = start(blockIdx.x);
    float sq[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      load_scales(pq, sq[j]);
      advance(pq);
    }
    Pos pc = start(blockIdx.x);
    float yacc[ECOLS];
#pragma unroll
    for (int j = 0; j < ECOLS; ++j) yacc[j] = 0.f;
    bool ok = true;
    int d = 0, dr = 0;
    for (int i = 0; i < nunits; ++i) {
      // scales through a 2-deep register queue (loads for unit i + 2)
      const float s0 = sq[0][0], s1 = sq[0][1];
      sq[0][0] = sq[1][0];
      sq[0][1] = sq[1][1];
      if (i + 2 < nunits) load_scales(pq, sq[1]);
      advance(pq);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float sc = h ? s1 : s0;
        if (warp == W_EPI && !*abort_flag && !mbar_wait(&d_full[d], (uint32_t)dr & 1u, a.status)) *abort_flag = 1;
        named_bar_sync(3, NEPI * 32);
        ok = ok && !*abort_flag;
        tc::fence_after_sync();
        if (ok) {
#pragma unroll
          for (int c = 0; c < ECOLS / 8; ++c) {
            uint32_t dv[8];
            tc::ld8(tmem + lane_base + DCOL0 + d * NMMA + ch * ECOLS + 8 * c, dv);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              // int32 accumulator to fp32 exactly: |acc| < 2^22, so 1.5 * 2^23 + acc
              // is an fp32 with acc in its low mantissa bits
              const float dvf = I8 ? __fsub_rn(__int_as_float((int)dv[j] + 0x4B400000), 12582912.0f)
                                   : __uint_as_float(dv[j]);
              yacc[8 * c + j] = fmaf(dvf, sc, yacc[8 * c + j]);
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_empty[d]);
        if (++d == NDR) {
          d = 0;
          ++dr;
        }
      }
      if (pc.kb == (SPLIT ? pc.khi : a.nkb) - 1) {
        // tile done: store this thread's 64 token columns of weight row n
        const int n = (pc.t / nch) * TC_ROWS + row;
        const int m0 = (pc.t % nch) * PF_TOK + ch * ECOLS;
        const int mlim = a.M - m0;
        if constexpr (SPLIT) {
          // partial tile [token][row]: for each token the warp's 32 rows are
          // 128 contiguous bytes
          float *slot = a.partial + ((size_t)(pc.t * KS + pc.sp) * PF_TOK + ch * ECOLS) * TC_ROWS + row;
          if (ok) {
#pragma unroll
            for (int j = 0; j < ECOLS; ++j) slot[(size_t)j * TC_ROWS] = yacc[j];
          }
        } else if (GATHER) {
          // fused all-gather: the tile's values go to every rank's Y at
          // global row row0 + n (own buffer first, then the peers in rank
          // order from the next one, so the ranks' stores spread over the
          // links); each store instruction is 128 contiguous bytes
          if (ok && n < a.N) {
            if (I8) {
#pragma unroll
              for (int j = 0; j < ECOLS; ++j)
                if (j < mlim) yacc[j] *= ld_act(a.xs + m0 + j);
            }
            for (int i = 0; i < a.world; ++i) {
              const int pr = (a.rank + i < a.world) ? a.rank + i : a.rank + i - a.world;
              float *yp = ydst[pr] + (size_t)m0 * a.ld_y + a.row0 + n;
#pragma unroll
              for (int j = 0; j < ECOLS; ++j) {
                if (j < mlim) *yp = yacc[j];
                yp += a.ld_y;
              }
            }
          }
        } else if (ok && n < a.N) {
          float *yp = a.y + (size_t)m0 * a.N + n;
#pragma unroll
          for (int j = 0; j < ECOLS; ++j) {
            if (j < mlim) *yp = I8 ? yacc[j] * ld_act(a.xs + m0 + j) : yacc[j];
            yp += a.N;
          }
        }
#pragma unroll
        for (int j = 0; j < ECOLS; ++j) yacc[j] = 0.f;
      }
      advance(pc);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == W_MMA) {
    tc::fence_after_sync();
    tc::dealloc(tmem, 512);
  }
  // fused all-gather: every thread's stores precede the barrier above; one
  // system-scope fence orders them before this CTA counts itself. The CTA
  // completing this rank's grid adds one call to every rank's counter for
  // this rank, waits (bounded) until every rank has counted this call in
  // this rank's counters, and advances the call counter. Counters only grow,
  // so a rank already at a later call has also passed this one.
  if (GATHER && tid == 0) {
    const uint32_t ep = *reinterpret_cast<volatile const uint32_t *>(a.ag_epoch) + 1u;
    fence_acq_rel_sys();
    if (atom_add_acq_rel_gpu(a.ag_counter, 1u) + 1u == gridDim.x) {
      atomicExch(a.ag_counter, 0u);  // ready for the next call
      fence_acq_rel_sys();
      for (int p = 0; p < a.world; ++p) red_add_relaxed_sys_u32(a.flag_peers[p] + a.rank, 1u);
      const uint32_t *mine = a.flag_peers[a.rank];
      const long long t0 = clock64(), lim = wait_cycles(a.status);
      bool gave_up = false;
      for (int p = 0; p < a.world && !gave_up; ++p) {
        while ((int32_t)(ld_acquire_sys_u32(mine + p) - ep) < 0) {
          if (clock64() - t0 > lim) {
            set_status(a.status, LBC_ERR_TIMEOUT);
            gave_up = true;
            break;
          }
          __nanosleep(64);
        }
      }
      *a.ag_epoch = ep;
    }
  }
}

// Split-K finish: Y[m, n] = sum over the KS splits, in split order, of the
// partial tiles [item][token][row] (times the token scale for W4A8). One CTA
// per (tile, token), one thread per weight row: reads and writes coalesced.
__global__ void __launch_bounds__(TC_ROWS) tc_split_reduce_kernel(const float *partial, const float *xs,
                                                                   float *y, int M,
                                                                   int N, int nch, int ks) {
  const int t = blockIdx.x, tok = blockIdx.y, r = threadIdx.x;
  const int m = (t % nch) * PF_TOK + tok, n = (t / nch) * TC_ROWS + r;
  pdl_wait_prior_grid();
  pdl_launch_dependents();
  if (m >= M || n >= N) return;
  const float *p = partial + ((size_t)t * ks * PF_TOK + tok) * TC_ROWS + r;
  float v = 0.f;
  for (int sp = 0; sp < ks; ++sp) v += ld_act(p + (size_t)sp * PF_TOK * TC_ROWS);
  y[(size_t)m * N + n] = xs ? v * ld_act(xs + m) : v;
}

}  // namespace lbc
