// extern "C" entry points of liblowbit_b200.so (declared in include/lowbit_b200.h)
// and the launch planner that turns (format, M, N, Kp, params) into a kernel
// configuration. The reference's equivalents are the public functions of
// src/lowbit/csrc/dispatch.c:205-305 and its tiling driver run() (:148-203).
#include <algorithm>
#include <array>
#include <map>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "../../include/lowbit_b200.h"
#include "gemv_dispatch.cuh"
#include "kernels.h"

namespace lbc {
// device status block (see common.cuh): int status, pad, int64 wait limit in
// clock cycles (0 = default); one per device, address passed to kernels
__device__ __align__(16) long long g_status_block[2] = {0, 0};
}

namespace {

thread_local char g_err[512] = "";

int fail_cuda(const char *what, cudaError_t e) {
  snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
  return LBC_ERR_CUDA;
}

int fail(int code, const char *msg) {
  snprintf(g_err, sizeof g_err, "%s", msg);
  return code;
}

struct DevInfo {
  int ok = 0, sms = 0, smem_optin = 0, smem_sm = 0;
  int *status = nullptr;
};

DevInfo dev_info() {
  static DevInfo cache[64];
  static bool init[64] = {false};
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return DevInfo{};
  if (!init[d]) {
    DevInfo di;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d);
    cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d);
    cudaDeviceGetAttribute(&di.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d);
    cudaDeviceGetAttribute(&di.smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, d);
    di.ok = (major == 10 && minor == 0);
    if (di.ok && cudaGetSymbolAddress(reinterpret_cast<void **>(&di.status), lbc::g_status_block) != cudaSuccess) {
      cudaGetLastError();
      di.status = nullptr;
    }
    cache[d] = di;
    init[d] = true;
  }
  return cache[d];
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int round_up(int a, int b) { return ceil_div(a, b) * b; }

int check_shape(int M, int Kp, int N, int block) {
  if (M <= 0 || N <= 0 || Kp <= 0 || Kp % block) return fail(LBC_ERR_SHAPE, "bad shape");
  return 0;
}

// ------------------------------------------------------------------ planner
struct GemvPlan {
  int mt = 1, ch = 1, rt = 4, tpr = 32, nt = 256, tile_rows = 4, stages = 4;
  int nsplit = 1, seg = 0, ctas_per_split = 1, ntiles = 1, passes = 1, meta_tma = 0;
  int threads = 256, smem = 0;
};

bool combo_ok(int fmt, int mt, int ch, int rt) {
  if (rt != 1 && rt != 4) return false;
  if (fmt == lbc::FMT_W4A8) {
    if (ch == 1) return mt == 1 || mt == 2 || mt == 4 || mt == 8;
    if (ch == 2) return mt == 1 || mt == 2 || mt == 4;
    if (ch == 4) return mt == 1 || mt == 2;
    return false;
  }
  if (ch == 1) return mt == 1 || mt == 2 || mt == 4;
  if (ch == 2) return mt == 1 || mt == 2;
  if (ch == 4) return mt == 1;
  return false;
}

int occupancy(int fmt, int mt, int ch, int rt, int threads, int smem);

// Chooses the SIMT kernel configuration. Parameters follow lbc_params
// (include/lowbit_b200.h); zero fields take the defaults below.
int plan_gemv(int fmt, int M, int N, int Kp, const lbc_params *p, GemvPlan &P, bool meta_ptrs_aligned,
              bool has_zeros) {
  const DevInfo di = dev_info();
  const int kgran = (fmt == lbc::FMT_MXFP4) ? 32 : 128;
  const int MAXSEG = 1024 * 32;  // 256 threads x 4 chunks x 32 elements
  const bool user_kb = p && p->kb > 0;

  auto pick_threads = [&](int seg, int &tpr, int &ch) {
    const int Cs = seg / 32;
    ch = 1;
    if (Cs <= 32) tpr = 32;
    else if (Cs <= 64) tpr = 64;
    else if (Cs <= 128) tpr = 128;
    else if (Cs <= 256) tpr = 256;
    else { tpr = 256; ch = Cs <= 512 ? 2 : 4; }
  };
  auto pick_mt = [&](int ch) {
    int cap = (fmt == lbc::FMT_W4A8) ? (ch == 1 ? 8 : ch == 2 ? 4 : 2) : (ch == 1 ? 4 : ch == 2 ? 2 : 1);
    int mt = 1;
    while (mt < M && mt < cap) mt <<= 1;
    return mt;
  };

  int seg = Kp;
  if (user_kb) seg = std::min(Kp, round_up(p->kb, 128));
  if (seg > MAXSEG) seg = MAXSEG;
  int tpr, ch;
  pick_threads(seg, tpr, ch);
  int mt = (p && p->mr > 0) ? p->mr : pick_mt(ch);
  int rt = (p && p->nr > 0) ? (p->nr >= 4 ? 4 : 1) : (mt <= 2 ? 4 : 1);
  const int nt = 256;  // consumer threads = CTA size (tpr <= 256)
  int tile_rows = rt * (nt / tpr);
  int passes = ceil_div(M, mt);

  // split K when the row tiles alone cannot fill the GPU
  if (!user_kb && seg == Kp && Kp >= 1024) {
    const int work = ceil_div(N, tile_rows) * passes;
    if (2 * work <= di.sms) {
      int ns = std::min(std::min(ceil_div(di.sms, work), Kp / 512), 16);
      if (ns > 1) {
        seg = round_up(ceil_div(Kp, ns), 128);
        pick_threads(seg, tpr, ch);
        mt = (p && p->mr > 0) ? p->mr : pick_mt(ch);
        rt = (p && p->nr > 0) ? (p->nr >= 4 ? 4 : 1) : (mt <= 2 ? 4 : 1);
        tile_rows = rt * (nt / tpr);
        passes = ceil_div(M, mt);
      }
    }
  }
  if (seg % kgran) return fail(LBC_ERR_PARAMS, "split-K length must be a multiple of 128");
  if (!combo_ok(fmt, mt, ch, rt)) return fail(LBC_ERR_PARAMS, "tile (mr, nr) not compiled");

  P.mt = mt; P.ch = ch; P.rt = rt; P.tpr = tpr; P.nt = nt; P.tile_rows = tile_rows;
  P.seg = seg; P.nsplit = ceil_div(Kp, seg); P.passes = passes;
  P.ntiles = ceil_div(N, tile_rows);
  P.threads = nt;

  // scales / zero points / e8m0 ride in the stage when every tile's slice of
  // them is a 16-byte aligned contiguous block (whole-K segments only)
  {
    const lbc::GemvMeta mm = lbc::gemv_meta(fmt, Kp, has_zeros, tile_rows, seg / 2, true);
    P.meta_tma = (P.nsplit == 1) && meta_ptrs_aligned && ((tile_rows * mm.sc_row) % 16 == 0) &&
                 ((tile_rows * mm.z_row) % 16 == 0);
  }
  const int stage_bytes = lbc::gemv_meta(fmt, Kp, has_zeros, tile_rows, seg / 2, P.meta_tma).bytes;
  int stages = (p && p->order > 0) ? p->order : std::min(16, std::max(2, ceil_div(65536, stage_bytes)));
  if (stages > 32) stages = 32;
  while (stages > 2 && lbc::gemv_smem_layout(stages, nt, stage_bytes).total > di.smem_optin) --stages;
  const int smem = lbc::gemv_smem_layout(stages, nt, stage_bytes).total;
  if (smem > di.smem_optin) return fail(LBC_ERR_PARAMS, "tile does not fit in shared memory");
  P.stages = stages;
  P.smem = smem;

  int cps = (p && p->nb > 0) ? p->nb : 2;
  const int occ = occupancy(fmt, mt, ch, rt, P.threads, smem);
  if (occ <= 0) {
    snprintf(g_err, sizeof g_err,
             "kernel configuration cannot be resident on an SM (fmt=%d mt=%d ch=%d rt=%d threads=%d "
             "smem=%d: %s %s)", fmt, mt, ch, rt, P.threads, smem,
             occ < 0 ? cudaGetErrorString((cudaError_t)(-occ)) : "occupancy 0", lbc::occ_note());
    return LBC_ERR_PARAMS;
  }
  cps = std::min(cps, occ);
  P.ctas_per_split = std::min(P.ntiles, std::max(1, di.sms * cps / P.nsplit));
  return 0;
}

int occupancy_uncached(int fmt, int mt, int ch, int rt, int threads, int smem) {
  switch (fmt) {
    case lbc::FMT_W4A16: return lbc::gemv_occupancy<lbc::FMT_W4A16>(mt, ch, rt, threads, smem);
    case lbc::FMT_MXFP4: return lbc::gemv_occupancy<lbc::FMT_MXFP4>(mt, ch, rt, threads, smem);
    default: return lbc::gemv_occupancy<lbc::FMT_W4A8>(mt, ch, rt, threads, smem);
  }
}

// occupancy results are cached per (device, kernel, block, smem): the planner
// runs on every call and must not issue CUDA queries during graph capture
int occupancy(int fmt, int mt, int ch, int rt, int threads, int smem) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int d = 0;
  cudaGetDevice(&d);
  const uint64_t key = ((uint64_t)(d & 63) << 58) | ((uint64_t)(fmt & 3) << 56) |
                       ((uint64_t)(mt & 15) << 52) | ((uint64_t)(ch & 7) << 49) |
                       ((uint64_t)(rt & 7) << 46) | ((uint64_t)(threads & 2047) << 32) |
                       (uint64_t)(uint32_t)smem;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int v = occupancy_uncached(fmt, mt, ch, rt, threads, smem);
  std::lock_guard<std::mutex> g(mu);
  cache[key] = v;
  return v;
}

bool meta_aligned(int fmt, const lbc::GemvArgs &a) {
  if (fmt == lbc::FMT_MXFP4) return al16(a.e8m0);
  return al16(a.scales) && (a.zeros == nullptr || al16(a.zeros));
}

// ------------------------------------------------------------------ decode plan
// The register-streamed kernel (gemv_rows.cuh) serves one or two tokens of
// the int4 formats when no staged-kernel tiling was requested (mr, nr, kb,
// order unset; nb = CTAs per SM is honoured).
struct RowsPlan {
  int mt = 1, ch = 1, r = 4, threads = 128, grid = 1, cps = 4, passes = 1;
};

bool rows_eligible(int fmt, int M, int Kp, const lbc_params *p) {
  if (p && (p->mr > 0 || p->nr > 0 || p->kb > 0 || p->order > 0)) return false;
  const int Cs = Kp / 32;
  // W4A8 with 3-16 tokens: 4 or 8 tokens per pass (int8 activations in
  // registers), one chunk per thread, so rows up to 8 warps x 32 chunks
  if (M > 2) return fmt == lbc::FMT_W4A8 && M <= 16 && Cs <= lbc::ROWS_MAX_WARPS * 32;
  // MXFP4's table decode is ALU-heavier: with two tokens its staged kernel is
  // as fast or faster (measured), with one the decode kernel wins
  if (fmt == lbc::FMT_MXFP4 && M > 1) return false;
  return Cs <= lbc::ROWS_MAX_WARPS * 32 * (M == 1 ? 4 : 2);
}

int rows_occupancy_cached(int fmt, int mt, int ch, int r, int threads) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int d = 0;
  cudaGetDevice(&d);
  const uint64_t key = ((uint64_t)(d & 63) << 40) | ((uint64_t)(fmt & 3) << 32) | ((uint64_t)(mt & 15) << 24) |
                       ((uint64_t)(ch & 15) << 16) | ((uint64_t)(r & 255) << 8) | (uint64_t)(threads >> 5);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int v = lbc::rows_occupancy(fmt, mt, ch, r, threads);
  std::lock_guard<std::mutex> g(mu);
  cache[key] = v;
  return v;
}

int plan_rows(int fmt, int M, int N, int Kp, const lbc_params *p, RowsPlan &P) {
  const DevInfo di = dev_info();
  const int Cs = Kp / 32;
  // one chunk per thread while a team of up to 8 warps (16 for one or two
  // tokens, except one W4A8 token, whose lighter two-chunk tile measured
  // faster) covers the row; longer rows take 2 or 4 chunks per thread with
  // the fewest warps that still cover the row (threads past the row's end
  // would decode a clamped chunk against zero activations: wasted issue)
  const bool wide = M == 2 || (M == 1 && fmt != lbc::FMT_W4A8);
  int ch = 1, nw = ceil_div(Cs, 32);
  if (nw > (wide ? lbc::ROWS_WIDE_WARPS : lbc::ROWS_MAX_WARPS)) {
    ch = ceil_div(Cs, lbc::ROWS_MAX_WARPS * 32);
    if (ch == 3) ch = 4;
    nw = std::min(lbc::ROWS_MAX_WARPS, ceil_div(Cs, 32 * ch));
  }
  P.mt = M <= 2 ? M : (M <= 4 ? 4 : 8);
  P.passes = ceil_div(M, P.mt);
  P.ch = ch;
  P.r = (M == 1) ? (ch == 4 ? 2 : 4) : (P.mt == 4 ? 4 : 2);
  P.threads = nw * 32;
  if (!lbc::rows_combo(P.mt, P.ch, P.r)) return fail(LBC_ERR_PARAMS, "decode tile not compiled");
  const int occ = rows_occupancy_cached(fmt, P.mt, P.ch, P.r, P.threads);
  if (occ <= 0) return fail(LBC_ERR_PARAMS, "decode kernel cannot be resident on an SM");
  // about 16 resident warps per SM by default: small-K rows (one-warp teams)
  // need many CTAs per SM to keep enough loads in flight; W4A8 with one or
  // two tokens (two chunks per thread, fewer registers) runs 8 (the tuner
  // measured 1.10-1.40x over 4 on the BASELINE shapes)
  const int cps_def = (fmt == lbc::FMT_W4A8 && M <= 2) ? 8 : std::max(4, 16 / nw);
  P.cps = std::min((p && p->nb > 0) ? p->nb : cps_def, occ);
  // the kernel hands out whole blocks of r rows
  P.grid = std::max(1, std::min(ceil_div(N, P.r), di.sms * P.cps));
  return 0;
}

int run_rows(int fmt, lbc::GemvArgs a, const lbc_params *p, cudaStream_t st) {
  RowsPlan P;
  if (int rc = plan_rows(fmt, a.M, a.N, a.Kp, p, P)) return rc;
  a.status = dev_info().status;
  cudaError_t e = lbc::rows_launch(fmt, a, P.mt, P.ch, P.r, dim3(P.grid, P.passes, 1), P.threads, st);
  if (e != cudaSuccess) return fail_cuda("decode gemv launch", e);
  return LBC_PATH_SIMT;
}

int run_gemv(int fmt, lbc::GemvArgs a, const lbc_params *p, cudaStream_t st) {
  if (rows_eligible(fmt, a.M, a.Kp, p)) return run_rows(fmt, a, p, st);
  GemvPlan P;
  int rc = plan_gemv(fmt, a.M, a.N, a.Kp, p, P, meta_aligned(fmt, a), a.zeros != nullptr);
  if (rc) return rc;
  a.seg_elems = P.seg;
  a.nsplit = P.nsplit;
  a.ctas_per_split = P.ctas_per_split;
  a.tile_rows = P.tile_rows;
  a.ntiles = P.ntiles;
  a.stages = P.stages;
  a.tpr = P.tpr;
  a.nt = P.nt;
  a.atomic_out = P.nsplit > 1;
  a.meta_tma = P.meta_tma;
  a.status = dev_info().status;
  if (a.atomic_out) {
    cudaError_t e = cudaMemsetAsync(a.y, 0, sizeof(float) * (size_t)a.M * a.N, st);
    if (e != cudaSuccess) return fail_cuda("cudaMemsetAsync(y)", e);
  }
  const dim3 grid(P.nsplit * P.ctas_per_split, P.passes);
  cudaError_t e;
  switch (fmt) {
    case lbc::FMT_W4A16: e = lbc::gemv_launch<lbc::FMT_W4A16>(a, P.mt, P.ch, P.rt, grid, P.threads, P.smem, st); break;
    case lbc::FMT_MXFP4: e = lbc::gemv_launch<lbc::FMT_MXFP4>(a, P.mt, P.ch, P.rt, grid, P.threads, P.smem, st); break;
    default: e = lbc::gemv_launch<lbc::FMT_W4A8>(a, P.mt, P.ch, P.rt, grid, P.threads, P.smem, st); break;
  }
  if (e != cudaSuccess) return fail_cuda("gemv launch", e);
  return LBC_PATH_SIMT;
}

int device_gate() {
  const DevInfo di = dev_info();
  if (!di.ok) return fail(LBC_ERR_DEVICE, "current device is not an sm_100 GPU");
  return 0;
}

size_t w4a8_ws_layout(int M, int Kp, size_t *off_xs, size_t *off_asum, size_t *off_tc = nullptr) {
  const size_t xq_bytes = ((size_t)M * Kp + 255) / 256 * 256;
  const size_t xs_bytes = ((size_t)M * 4 + 255) / 256 * 256;
  const size_t as_bytes = ((size_t)M * (Kp / 128) * 4 + 255) / 256 * 256;
  const size_t tc_bytes = (lbc::tc_scratch_bytes(lbc::FMT_W4A8, M, Kp, std::max(1, dev_info().sms)) + 255) / 256 * 256;
  if (off_xs) *off_xs = xq_bytes;
  if (off_asum) *off_asum = xq_bytes + xs_bytes;
  if (off_tc) *off_tc = xq_bytes + xs_bytes + as_bytes;
  return xq_bytes + xs_bytes + as_bytes + tc_bytes;
}

// automatic kernel choice: no path requested, or one of the reference's CPU
// ISA ids (2 = avx512; 3 is this library's mma path)
bool path_auto(const lbc_params *p) {
  return !p || p->isa == LBC_PATH_AUTO || (p->isa >= 2 && p->isa != LBC_PATH_MMA);
}

// ------------------------------------------------------------------ tensor-core decode (mma.sync)
// W4A16 with one or two tokens on the warp-level tensor-core kernel
// (gemv_mma.cuh). Params on this path: nb = CTAs per SM (default 1), nr =
// consumer warps per CTA (default 8), kb = K elements per ring stage (a
// multiple of 128 x warps; default 4 groups per warp for one token, 2 for
// two), order = ring stages (default 2 for one token; for two, as many as
// fit beside the activation fragments in half an SM's shared memory, at
// most 8). Measured on the 11008 x 4096 headline shape (CUDA graph of
// rotating weight copies): one token 9.36 us at (8 warps, 4 groups, 2
// stages), 10.6-12.3 us at other tilings, against 9.6 us for the
// register-streamed SIMT kernel; two tokens 13.45 us against 14.35 us.
struct MmaPlan {
  int ntok = 1, nw = 8, jws = 2, ns = 4, grid = 1, smem = 0;
};

constexpr int MMA_MAX_STAGES = 8;

int plan_mma(int fmt, int M, int N, int Kp, const lbc_params *p, MmaPlan &P) {
  if (fmt != lbc::FMT_W4A16 || M > 2) return fail(LBC_ERR_PARAMS, "mma decode path: W4A16 with 1 or 2 tokens");
  const DevInfo di = dev_info();
  P.ntok = M;
  P.nw = (p && p->nr > 0) ? p->nr : 8;
  P.jws = (p && p->kb > 0) ? std::max(1, p->kb / (128 * P.nw)) : (M == 1 ? 4 : 2);
  const int cps = (p && p->nb > 0) ? p->nb : 1;
  P.grid = std::max(1, std::min(di.sms * cps, ceil_div(N, 16)));
  if (!lbc::mma_combo(P.ntok, P.nw, P.jws)) return fail(LBC_ERR_PARAMS, "mma decode tile not compiled");
  const int budget = di.smem_sm / 2 - 1024;
  if (p && p->order > 0) {
    P.ns = std::min(p->order, MMA_MAX_STAGES);
  } else if (M == 1) {
    P.ns = 2;
  } else {
    P.ns = MMA_MAX_STAGES;
    while (P.ns > 2 && lbc::mma_smem_bytes(P.ntok, P.nw, P.jws, P.ns, Kp, N, P.grid) > budget) --P.ns;
  }
  P.smem = lbc::mma_smem_bytes(P.ntok, P.nw, P.jws, P.ns, Kp, N, P.grid);
  if (P.smem > di.smem_optin) return fail(LBC_ERR_PARAMS, "mma decode: stages and activations do not fit in shared memory");
  return 0;
}

// Requested explicitly (params.isa = LBC_PATH_MMA), or by the tuner. The
// automatic choice keeps the register-streamed SIMT kernel for one and two
// tokens: it is as fast or faster at one token, and the fused decode
// prologues (RMSNorm, SiLU.up) of the model run on it, whose results must
// equal the separate kernels' bit for bit.
bool want_mma(const lbc_params *p, int fmt, int M, int N, int Kp) {
  (void)fmt;
  (void)M;
  (void)N;
  (void)Kp;
  return p && p->isa == LBC_PATH_MMA;
}

// W4A8 on mma.sync.m16n8k32 s8 (gemv_i8mma.cu): 8 or 16 tokens per pass
// (n-blocks of 8; up to 64 tokens in passes), nr = warps per CTA (4 or 8;
// default 8), nb = CTAs per SM (default: up to 4, as many as fit)
struct I8Plan {
  int nb = 1, nw = 8, passes = 1, grid = 1, smem = 0, cps = 1;
};

int plan_i8mma(int M, int N, int Kp, const lbc_params *p, I8Plan &P) {
  const DevInfo di = dev_info();
  if (M > 64) return fail(LBC_ERR_PARAMS, "w4a8 mma path: at most 64 tokens");
  P.nb = M <= 8 ? 1 : 2;
  P.passes = ceil_div(M, 8 * P.nb);
  P.nw = (p && p->nr > 0) ? p->nr : 8;
  if (P.nw != 4 && P.nw != 8) return fail(LBC_ERR_PARAMS, "w4a8 mma path: 4 or 8 warps per CTA (nr)");
  P.smem = lbc::i8mma_smem(P.nb, P.nw, Kp);
  if (P.smem > di.smem_optin) return fail(LBC_ERR_PARAMS, "w4a8 mma path: the activations do not fit in shared memory");
  const int occ = lbc::i8mma_occupancy(P.nb, P.nw, P.smem);
  if (occ <= 0) return fail(LBC_ERR_PARAMS, "w4a8 mma path: kernel cannot be resident on an SM");
  P.cps = std::min((p && p->nb > 0) ? p->nb : 4, occ);
  P.grid = std::max(1, std::min(ceil_div(N, 16), di.sms * P.cps));
  return 0;
}

// The int8 MMA kernel serves W4A8 on request (isa = LBC_PATH_MMA, up to 64
// tokens) and, automatically with default tiling, 8-63 tokens, and 3-7
// tokens whose rows are too long for the decode kernel. Measured on the
// BASELINE shapes: 1.2-2x over the decode / staged kernels at 8-16 tokens,
// 2-3.5x over the staged / tcgen05 exact kernels at 17-63 (passes of 16
// tokens re-read weights that are still in L2). The decode kernel stays
// faster at 1-4 tokens on rows it takes, the prefill kernel from 64 tokens.
bool want_i8mma(const lbc_params *p, int M, int N, int Kp) {
  (void)N;
  if (p && p->isa == LBC_PATH_MMA) return true;
  if (!path_auto(p) || (p && (p->mr > 0 || p->nr > 0 || p->kb > 0 || p->order > 0))) return false;
  if (M < 3 || M > 63 || lbc::i8mma_smem(M <= 8 ? 1 : 2, 8, Kp) > dev_info().smem_optin) return false;
  return M >= 8 || !rows_eligible(lbc::FMT_W4A8, M, Kp, p);
}

int run_i8mma(lbc::GemvArgs a, const lbc_params *p, cudaStream_t st) {
  I8Plan P;
  if (int rc = plan_i8mma(a.M, a.N, a.Kp, p, P)) return rc;
  a.status = dev_info().status;
  cudaError_t e = lbc::i8mma_launch(a, P.nb, P.nw, dim3(P.grid, P.passes, 1), st);
  if (e != cudaSuccess) return fail_cuda("w4a8 mma gemm launch", e);
  return LBC_PATH_MMA;
}

int run_mma(int fmt, lbc::GemvArgs a, const lbc_params *p, cudaStream_t st) {
  MmaPlan P;
  if (int rc = plan_mma(fmt, a.M, a.N, a.Kp, p, P)) return rc;
  a.status = dev_info().status;
  cudaError_t e = lbc::mma_launch(a, P.ntok, P.nw, P.jws, P.ns, P.grid, st);
  if (e != cudaSuccess) return fail_cuda("mma decode gemv launch", e);
  return LBC_PATH_MMA;
}

// ------------------------------------------------------------------ few-token path
// Partial sums of the few-token kernel's K ranges: one grow-only buffer per
// (device, stream), so a decode loop issues no allocation. A buffer once
// handed out is never freed (a CUDA graph captured around an earlier call may
// hold its address): a grown-out one is retired until the process exits, and
// growth at least doubles. While the stream is being captured a growth is a
// stream-ordered allocation freed after the launches.
struct TokScratch {
  float *p;
  bool owned;
};
TokScratch tok_scratch(size_t bytes, cudaStream_t st) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, std::pair<void *, size_t>> cache;
  static std::vector<void *> retired;
  int d = 0;
  cudaGetDevice(&d);
  const uint64_t key = ((uint64_t)(d & 63) << 58) ^ (uint64_t)(uintptr_t)st;
  std::lock_guard<std::mutex> g(mu);
  auto &slot = cache[key];
  if (slot.first && slot.second >= bytes) return {static_cast<float *>(slot.first), false};
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  void *p = nullptr;
  if (cs != cudaStreamCaptureStatusNone) {
    if (cudaMallocAsync(&p, bytes, st) != cudaSuccess) {
      cudaGetLastError();
      return {nullptr, false};
    }
    return {static_cast<float *>(p), true};
  }
  const size_t nb = std::max(bytes, 2 * slot.second);
  if (cudaMalloc(&p, nb) != cudaSuccess) {
    cudaGetLastError();
    return {nullptr, false};
  }
  if (slot.first) retired.push_back(slot.first);
  slot = {p, nb};
  return {static_cast<float *>(p), false};
}

struct TokPlan {
  int r, warps, ks;
};

// rows per lane (2 once that still gives a CTA per SM); K ranges only for
// rows of 2048+ elements (the second kernel that adds the ranges costs more
// than it saves on short rows): about two CTAs per SM, two units per range
// at least, each range's activations within shared memory; warps per CTA
// (two K steps each at least)
TokPlan tok_plan(int fmt, int M, int N, int Kp) {
  const DevInfo di = dev_info();
  const int spu = fmt == lbc::FMT_MXFP4 ? 1 : 4;  // K steps per unit (group / block)
  const int U = Kp / 32 / spu;
  TokPlan P;
  P.r = ceil_div(N, 64) >= di.sms ? 2 : 1;
  const int ctas = ceil_div(N, 32 * P.r) * ceil_div(M, 8);
  int ks = Kp >= 2048 ? std::max(1, std::min(U / 2, 2 * di.sms / ctas)) : 1;
  const int maxkp = lbc::tok_max_kp(di.smem_optin);
  while (ks < U && 32 * spu * ceil_div(U, ks) > maxkp) ++ks;
  P.ks = ks;
  P.warps = std::max(1, std::min(16, spu * ceil_div(U, ks) / 2));
  return P;
}

// The few-token kernel serves W4A16 with 8-16 tokens and MXFP4 with 4-16 on
// automatic paths for matrices of up to LBC_TOK_MAX_WEIGHTS weights, where it
// beats both the staged SIMT kernel and the tensor-core path's fixed cost
// (measured: e.g. 896x896 at 16 tokens 14.4 -> 5.4 us, 896x4864 29 -> 13 us)
constexpr double LBC_TOK_MAX_WEIGHTS = 5e6;
bool want_tok(const lbc_params *p, int fmt, int M, int N, int Kp) {
  if (fmt == lbc::FMT_W4A8) return false;
  if (!path_auto(p)) return false;
  if (p && (p->mr > 0 || p->nr > 0 || p->kb > 0 || p->order > 0 || p->nb > 0)) return false;
  if (M > 16 || M < (fmt == lbc::FMT_MXFP4 ? 4 : 8)) return false;
  return (double)N * Kp <= LBC_TOK_MAX_WEIGHTS;
}

int run_tok(int fmt, const lbc::GemvArgs &a, cudaStream_t st) {
  const TokPlan P = tok_plan(fmt, a.M, a.N, a.Kp);
  TokScratch sc{nullptr, false};
  if (P.ks > 1) {
    sc = tok_scratch(sizeof(float) * (size_t)P.ks * a.M * a.N, st);
    if (!sc.p) return fail(LBC_ERR_ALLOC, "few-token GEMM partial-sum buffer allocation failed");
  }
  cudaError_t e = lbc::tok_gemm(fmt, a, P.r, P.warps, P.ks, sc.p, st);
  if (sc.owned) cudaFreeAsync(sc.p, st);
  if (e != cudaSuccess) return fail_cuda("few-token GEMM launch", e);
  return LBC_PATH_SIMT;
}

// Kernel path: explicit requests are honoured; automatic selection sends one
// or two tokens to the register-streamed decode kernel and three or more to
// the tensor-core kernel (W4A8 from 32 tokens, or 12 on large matrices: below
// that its int32 dp4a SIMT kernel is faster), except small matrices below 32
// tokens: the tensor-core
// path's fixed cost (activation-block kernel, TMEM and pipeline set-up, about
// 10-18 us on B200) exceeds the SIMT kernels' time there (measured: N*Kp below
// 10M weights up to 4 tokens, below 6M up to 31).
bool want_tc(const lbc_params *p, int fmt, int M, int N, int Kp) {
  if (p && p->isa == LBC_PATH_TCGEN05) return true;
  if (!path_auto(p)) return false;
  if (p && (p->mr > 0 || p->nr > 0 || p->kb > 0 || p->order > 0 || p->nb > 0)) return false;
  // W4A8: the dp4a SIMT kernels up to 31 tokens (the decode kernel takes up
  // to 16 tokens on rows of up to 8192), except large matrices (32M+
  // weights) from 17 tokens, or from 12 when the rows are longer than the
  // decode kernel takes, where the tensor cores win (measured)
  if (fmt == lbc::FMT_W4A8) {
    if (M >= 32) return true;
    const bool big = (double)N * Kp >= 32e6;
    return big && (M > 16 || (M >= 12 && Kp > lbc::ROWS_MAX_WARPS * 32 * 32));
  }
  if (M < 3) return false;
  const double w = (double)N * Kp;
  if (M < 32 && w < (M <= 4 ? 10e6 : 6e6)) return false;
  return true;
}

// prefill kernel (128-token tiles) from 64 tokens unless tokens per pass (mr)
// are given, which keeps the exact kernel: W4A16 / MXFP4 with bf16
// activations (4e-3 tolerance, the north-star prefill contract), W4A8 with
// int8 activations and exact int32 group sums (no extra tolerance)
bool want_prefill(const lbc_params *p, int fmt, int M) {
  (void)fmt;
  return M >= 64 && !(p && p->mr > 0);
}

int run_tc(lbc::TcCall c, cudaStream_t st) {
  const DevInfo di = dev_info();
  c.status = di.status;
  c.sms = di.sms;
  c.smem_optin = di.smem_optin;
  char msg[256] = "";
  const int rc = lbc::tc_gemm(c, st, msg, sizeof msg);
  if (rc < 0) return fail(rc, msg);
  return rc;
}

}  // namespace

void lbc::set_last_error(const char *msg) { snprintf(g_err, sizeof g_err, "%s", msg); }

// ====================================================================== C ABI
extern "C" {

int lbc_version(void) { return 1; }

int lbc_device_ok(void) { return dev_info().ok; }

int lbc_sm_count(void) { return dev_info().sms; }

const char *lbc_last_error(void) { return g_err; }

int lbc_device_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lbc::g_status_block, sizeof(int)) != cudaSuccess) return LBC_ERR_CUDA;
  if (reset && v) {
    const int z = 0;
    cudaMemcpyToSymbol(lbc::g_status_block, &z, sizeof(int));
  }
  return v;
}

int lbc_set_wait_cycles(long long cycles) {
  const long long v = cycles > 0 ? cycles : 0;
  cudaError_t e = cudaMemcpyToSymbol(lbc::g_status_block, &v, sizeof v, sizeof(long long));
  return e == cudaSuccess ? 0 : fail_cuda("cudaMemcpyToSymbol(wait limit)", e);
}

long long lbc_wait_cycles(void) {
  long long v = 0;
  if (cudaMemcpyFromSymbol(&v, lbc::g_status_block, sizeof v, sizeof(long long)) != cudaSuccess) return LBC_ERR_CUDA;
  return v > 0 ? v : 4000000000LL;
}

int lbc_tc_selftest(int kind, int32_t *out, void *stream) {
  if ((kind != 0 && kind != 1) || !out) return fail(LBC_ERR_SHAPE, "kind must be 0 or 1, out non-NULL");
  if (int rc = device_gate()) return rc;
  cudaError_t e = lbc::launch_tc_selftest(kind, out, dev_info().status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda("tc_selftest launch", e);
  return 0;
}

int lbc_describe_plan(int kind, int M, int N, int Kp, const lbc_params *p, char *buf, int buflen) {
  if (kind < 0 || kind > 2) return fail(LBC_ERR_SHAPE, "kind must be 0 (w4a16), 1 (mxfp4) or 2 (w4a8)");
  if (int rc = check_shape(M, Kp, N, kind == 1 ? LBC_MXBLOCK : LBC_GROUP)) return rc;
  if (int rc = device_gate()) return rc;
  const int fmt = kind == 0 ? lbc::FMT_W4A16 : kind == 1 ? lbc::FMT_MXFP4 : lbc::FMT_W4A8;
  if (fmt == lbc::FMT_W4A8 && want_i8mma(p, M, N, Kp)) {
    I8Plan P;
    if (int rc = plan_i8mma(M, N, Kp, p, P)) return rc;
    if (buf && buflen > 0)
      snprintf(buf, (size_t)buflen,
               "{\"path\": \"mma\", \"kernel\": \"i8mma\", \"nblocks\": %d, \"warps\": %d, \"passes\": %d, "
               "\"grid\": %d, \"ctas_per_sm\": %d, \"smem\": %d}", P.nb, P.nw, P.passes, P.grid, P.cps, P.smem);
    return LBC_PATH_MMA;
  }
  if (want_mma(p, fmt, M, N, Kp)) {
    MmaPlan P;
    if (int rc = plan_mma(fmt, M, N, Kp, p, P)) return rc;
    if (buf && buflen > 0)
      snprintf(buf, (size_t)buflen,
               "{\"path\": \"mma\", \"kernel\": \"mma\", \"tokens\": %d, \"warps\": %d, \"units_per_stage\": %d, "
               "\"stages\": %d, \"grid\": %d, \"smem\": %d}", P.ntok, P.nw, P.jws, P.ns, P.grid, P.smem);
    return LBC_PATH_MMA;
  }
  if (want_tok(p, fmt, M, N, Kp)) {
    const TokPlan P = tok_plan(fmt, M, N, Kp);
    if (buf && buflen > 0)
      snprintf(buf, (size_t)buflen,
               "{\"path\": \"simt\", \"kernel\": \"tok\", \"passes\": %d, \"r\": %d, \"warps\": %d, \"ksplit\": %d}",
               ceil_div(M, 8), P.r, P.warps, P.ks);
    return LBC_PATH_SIMT;
  }
  if (want_tc(p, fmt, M, N, Kp)) {
    if (buf && buflen > 0)
      snprintf(buf, (size_t)buflen, "{\"path\": \"tcgen05\", \"kernel\": \"%s\"}",
               want_prefill(p, fmt, M) ? "prefill" : "tcgemm");
    return LBC_PATH_TCGEN05;
  }
  if (rows_eligible(fmt, M, Kp, p)) {
    RowsPlan R;
    if (int rc = plan_rows(fmt, M, N, Kp, p, R)) return rc;
    if (buf && buflen > 0)
      snprintf(buf, (size_t)buflen,
               "{\"path\": \"simt\", \"kernel\": \"rows\", \"mt\": %d, \"ch\": %d, \"r\": %d, "
               "\"threads\": %d, \"grid\": %d, \"passes\": %d, \"ctas_per_sm\": %d}",
               R.mt, R.ch, R.r, R.threads, R.grid, R.passes, R.cps);
    return LBC_PATH_SIMT;
  }
  GemvPlan P;
  const int rc = plan_gemv(fmt, M, N, Kp, p, P, true, kind != 1);
  if (rc) return rc;
  if (buf && buflen > 0)
    snprintf(buf, (size_t)buflen,
             "{\"path\": \"simt\", \"kernel\": \"staged\", \"mt\": %d, \"ch\": %d, \"rt\": %d, \"tpr\": %d, \"nt\": %d, "
             "\"tile_rows\": %d, \"stages\": %d, \"nsplit\": %d, \"seg\": %d, \"ctas_per_split\": %d, "
             "\"ntiles\": %d, \"passes\": %d, \"threads\": %d, \"smem\": %d, \"meta_tma\": %d}",
             P.mt, P.ch, P.rt, P.tpr, P.nt, P.tile_rows, P.stages, P.nsplit, P.seg, P.ctas_per_split,
             P.ntiles, P.passes, P.threads, P.smem, P.meta_tma);
  return LBC_PATH_SIMT;
}

int lbc_gemm_w4a16(const float *x, int M, int Kp, const uint8_t *qw, const float *scales,
                   const uint8_t *zeros, int N, float *y, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  if (!x || !qw || !scales || !y || !al16(x) || !al16(qw))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer (x, qw need 16-byte alignment)");
  if (int rc = device_gate()) return rc;
  if (want_mma(p, lbc::FMT_W4A16, M, N, Kp)) {
    lbc::GemvArgs a{};
    a.x = x; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
    a.M = M; a.N = N; a.Kp = Kp;
    return run_mma(lbc::FMT_W4A16, a, p, static_cast<cudaStream_t>(stream));
  }
  if (want_tok(p, lbc::FMT_W4A16, M, N, Kp)) {
    lbc::GemvArgs a{};
    a.x = x; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
    a.M = M; a.N = N; a.Kp = Kp;
    return run_tok(lbc::FMT_W4A16, a, static_cast<cudaStream_t>(stream));
  }
  if (want_tc(p, lbc::FMT_W4A16, M, N, Kp)) {
    lbc::TcCall c{};
    c.fmt = lbc::FMT_W4A16; c.x = x; c.qw = qw; c.scales = scales; c.zeros = zeros; c.y = y;
    c.M = M; c.N = N; c.Kp = Kp;
    c.prefill = want_prefill(p, c.fmt, M);
    return run_tc(c, static_cast<cudaStream_t>(stream));
  }
  lbc::GemvArgs a{};
  a.x = x; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
  a.M = M; a.N = N; a.Kp = Kp;
  return run_gemv(lbc::FMT_W4A16, a, p, static_cast<cudaStream_t>(stream));
}

// W4A16 decode with a fused activation prologue (rows kernel only: M <= 2,
// default tiling); LBC_ERR_PARAMS tells the caller to run the two-kernel path
static int run_fused_w4a16(lbc::GemvArgs a, int xm, const lbc_params *p, cudaStream_t st) {
  if (!rows_eligible(lbc::FMT_W4A16, a.M, a.Kp, p) || (p && (p->isa == LBC_PATH_TCGEN05 || p->nb > 0)))
    return fail(LBC_ERR_PARAMS, "fused decode prologue: M <= 2 with default tiling only");
  RowsPlan P;
  if (int rc = plan_rows(lbc::FMT_W4A16, a.M, a.N, a.Kp, p, P)) return rc;
  a.status = dev_info().status;
  cudaError_t e = lbc::rows_fused_launch(a, xm, P.mt, P.ch, P.r, dim3(P.grid, 1, 1), P.threads, st);
  if (e != cudaSuccess) return fail_cuda("fused decode gemv launch", e);
  return LBC_PATH_SIMT;
}

int lbc_gemm_w4a16_rmsnorm(const float *x, const float *residual, float *x_out, const float *norm_w, float eps,
                           int M, int Kp, const uint8_t *qw, const float *scales, const uint8_t *zeros, int N,
                           float *y, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  if (!x || !norm_w || !qw || !scales || !y || !al16(x) || !al16(qw) || !al16(norm_w) ||
      (residual && (!al16(residual) || !x_out)) || (x_out && (x_out == x || x_out == residual)))
    return fail(LBC_ERR_SHAPE, "NULL, misaligned or aliasing pointer (x_out must be a separate buffer)");
  if (int rc = device_gate()) return rc;
  lbc::GemvArgs a{};
  a.x = x; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
  a.M = M; a.N = N; a.Kp = Kp;
  a.xres = residual; a.xout = residual ? x_out : nullptr; a.lnw = norm_w; a.eps = eps;
  return run_fused_w4a16(a, lbc::XM_RMSNORM, p, static_cast<cudaStream_t>(stream));
}

int lbc_gemm_w4a16_glu(const float *gu, int M, int Kp, const uint8_t *qw, const float *scales,
                       const uint8_t *zeros, int N, float *y, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  if (!gu || !qw || !scales || !y || !al16(gu) || !al16(qw))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer");
  if (int rc = device_gate()) return rc;
  lbc::GemvArgs a{};
  a.x = gu; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
  a.M = M; a.N = N; a.Kp = Kp;
  return run_fused_w4a16(a, lbc::XM_GLU, p, static_cast<cudaStream_t>(stream));
}

int lbc_gemm_mxfp4(const float *x, int M, int Kp, const uint8_t *qw, const uint8_t *e8m0, int N,
                   float *y, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_MXBLOCK)) return rc;
  if (p && p->isa == LBC_PATH_MMA) return fail(LBC_ERR_PARAMS, "mma path: W4A16 and W4A8 only");
  if (!x || !qw || !e8m0 || !y || !al16(x) || !al16(qw))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer (x, qw need 16-byte alignment)");
  if (int rc = device_gate()) return rc;
  if (want_tok(p, lbc::FMT_MXFP4, M, N, Kp)) {
    lbc::GemvArgs a{};
    a.x = x; a.qw = qw; a.e8m0 = e8m0; a.y = y;
    a.M = M; a.N = N; a.Kp = Kp;
    return run_tok(lbc::FMT_MXFP4, a, static_cast<cudaStream_t>(stream));
  }
  if (want_tc(p, lbc::FMT_MXFP4, M, N, Kp)) {
    lbc::TcCall c{};
    c.fmt = lbc::FMT_MXFP4; c.x = x; c.qw = qw; c.e8m0 = e8m0; c.y = y;
    c.M = M; c.N = N; c.Kp = Kp;
    c.prefill = want_prefill(p, c.fmt, M);
    return run_tc(c, static_cast<cudaStream_t>(stream));
  }
  lbc::GemvArgs a{};
  a.x = x; a.qw = qw; a.e8m0 = e8m0; a.y = y;
  a.M = M; a.N = N; a.Kp = Kp;
  return run_gemv(lbc::FMT_MXFP4, a, p, static_cast<cudaStream_t>(stream));
}

int lbc_quant_act_int8(const float *x, int M, int Kp, int8_t *xq, float *xs, int32_t *asum,
                       void *stream) {
  if (int rc = check_shape(M, Kp, 1, LBC_GROUP)) return rc;
  if (!x || !xq || !xs || !asum || !al16(x) || (reinterpret_cast<uintptr_t>(xq) & 3u))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer");
  if (int rc = device_gate()) return rc;
  cudaError_t e = lbc::launch_quant_act_int8(x, M, Kp, xq, xs, asum, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda("quant_act_int8 launch", e);
  return 0;
}

int lbc_gemm_w4a8_q(const int8_t *xq, const float *xs, const int32_t *asum, int M, int Kp,
                    const uint8_t *qw, const float *scales, const uint8_t *zeros, int N, float *y,
                    const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  if (!xq || !xs || !asum || !qw || !scales || !y || !al16(xq) || !al16(qw))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer (xq, qw need 16-byte alignment)");
  if (int rc = device_gate()) return rc;
  if (want_i8mma(p, M, N, Kp)) {
    lbc::GemvArgs a{};
    a.xq = xq; a.xs = xs; a.asum = asum; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
    a.M = M; a.N = N; a.Kp = Kp;
    return run_i8mma(a, p, static_cast<cudaStream_t>(stream));
  }
  if (want_tc(p, lbc::FMT_W4A8, M, N, Kp)) {
    lbc::TcCall c{};
    c.fmt = lbc::FMT_W4A8; c.xq = xq; c.xs = xs; c.asum = asum; c.qw = qw; c.scales = scales;
    c.zeros = zeros; c.y = y; c.M = M; c.N = N; c.Kp = Kp;
    c.prefill = want_prefill(p, c.fmt, M);
    return run_tc(c, static_cast<cudaStream_t>(stream));
  }
  lbc::GemvArgs a{};
  a.xq = xq; a.xs = xs; a.asum = asum; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
  a.M = M; a.N = N; a.Kp = Kp;
  return run_gemv(lbc::FMT_W4A8, a, p, static_cast<cudaStream_t>(stream));
}

size_t lbc_gemm_w4a8_workspace_size(int M, int Kp) {
  if (M <= 0 || Kp <= 0) return 0;
  return w4a8_ws_layout(M, Kp, nullptr, nullptr);
}

int lbc_gemm_w4a8(const float *x, int M, int Kp, const uint8_t *qw, const float *scales,
                  const uint8_t *zeros, int N, float *y, const lbc_params *p, void *workspace,
                  void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  if (p && p->isa == LBC_PATH_MMA && M > 64) return fail(LBC_ERR_PARAMS, "w4a8 mma path: at most 64 tokens");
  if (!x || !qw || !scales || !y || !al16(x) || !al16(qw))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer (x, qw need 16-byte alignment)");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(LBC_ERR_SHAPE, "workspace must be 256-byte aligned");
  if (int rc = device_gate()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  size_t off_xs, off_as, off_tc;
  const size_t bytes = w4a8_ws_layout(M, Kp, &off_xs, &off_as, &off_tc);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  bool owned = false;
  if (!ws) {
    void *tmp = nullptr;
    if (cudaMallocAsync(&tmp, bytes, st) != cudaSuccess) {
      cudaGetLastError();
      return fail(LBC_ERR_ALLOC, "cudaMallocAsync(workspace) failed");
    }
    ws = static_cast<uint8_t *>(tmp);
    owned = true;
  }
  int8_t *xq = reinterpret_cast<int8_t *>(ws);
  float *xs = reinterpret_cast<float *>(ws + off_xs);
  int32_t *asum = reinterpret_cast<int32_t *>(ws + off_as);
  int rc = 0;
  cudaError_t e = lbc::launch_quant_act_int8(x, M, Kp, xq, xs, asum, st);
  if (e != cudaSuccess) rc = fail_cuda("quant_act_int8 launch", e);
  if (rc == 0 && want_i8mma(p, M, N, Kp)) {
    lbc::GemvArgs a{};
    a.xq = xq; a.xs = xs; a.asum = asum; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
    a.M = M; a.N = N; a.Kp = Kp;
    rc = run_i8mma(a, p, st);
  } else if (rc == 0 && want_tc(p, lbc::FMT_W4A8, M, N, Kp)) {
    lbc::TcCall c{};
    c.fmt = lbc::FMT_W4A8; c.xq = xq; c.xs = xs; c.asum = asum; c.qw = qw; c.scales = scales;
    c.zeros = zeros; c.y = y; c.M = M; c.N = N; c.Kp = Kp;
    c.prefill = want_prefill(p, c.fmt, M);
    c.scratch = ws + off_tc;
    c.scratch_bytes = bytes - off_tc;
    rc = run_tc(c, st);
  } else if (rc == 0) {
    lbc::GemvArgs a{};
    a.xq = xq; a.xs = xs; a.asum = asum; a.qw = qw; a.scales = scales; a.zeros = zeros; a.y = y;
    a.M = M; a.N = N; a.Kp = Kp;
    rc = run_gemv(lbc::FMT_W4A8, a, p, st);
  }
  if (owned) cudaFreeAsync(ws, st);
  return rc;
}

int lbc_w4a8_group_acc(const int8_t *xq, const int32_t *asum, int M, int Kp, const uint8_t *qw,
                       const uint8_t *zeros, int N, int32_t *out, int isa, void *stream) {
  (void)isa;
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  if (!xq || !asum || !qw || !out || !al16(xq) || !al16(qw))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer (xq, qw need 16-byte alignment)");
  if (int rc = device_gate()) return rc;
  cudaError_t e = lbc::launch_w4a8_group_acc(xq, asum, M, Kp, qw, zeros, N, out,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda("w4a8_group_acc launch", e);
  return 0;
}

// ------------------------------------------------------------------ multi-GPU
int lbc_device_alloc(size_t bytes, void **dev_ptr) {
  if (!dev_ptr || bytes == 0) return fail(LBC_ERR_SHAPE, "bytes must be > 0 and dev_ptr non-NULL");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LBC_ERR_ALLOC, "cudaMalloc failed");
  }
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail_cuda("cudaMemset", e);
  }
  *dev_ptr = p;
  return 0;
}

int lbc_device_free(void *dev_ptr) {
  cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? 0 : fail_cuda("cudaFree", e);
}

int lbc_ipc_get_handle(const void *dev_ptr, void *handle) {
  if (!dev_ptr || !handle) return fail(LBC_ERR_SHAPE, "NULL pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr));
  if (e != cudaSuccess) return fail_cuda("cudaIpcGetMemHandle", e);
  static_assert(sizeof(h) == LBC_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof h);
  return 0;
}

int lbc_ipc_open_handle(const void *handle, void **dev_ptr) {
  if (!handle || !dev_ptr) return fail(LBC_ERR_SHAPE, "NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail_cuda("cudaIpcOpenMemHandle", e);
  return 0;
}

int lbc_ipc_close_handle(void *dev_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? 0 : fail_cuda("cudaIpcCloseMemHandle", e);
}

int lbc_gemm_w4a16_allgather(const float *x, int M, int Kp, const uint8_t *qw, const float *scales,
                             const uint8_t *zeros, int N_local, int row0, int N_total, float *y,
                             uint64_t *const *land_peers, uint32_t *counter, uint32_t *epoch, int rank,
                             int world, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N_local, LBC_GROUP)) return rc;
  if (!x || !qw || !scales || !y || !land_peers || !counter || !epoch || !al16(x) || !al16(qw))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer");
  if (world < 1 || world > LBC_GATHER_MAX_WORLD || rank < 0 || rank >= world || row0 < 0 ||
      row0 + N_local > N_total)
    return fail(LBC_ERR_SHAPE, "rank / world / row range out of bounds");
  if (!rows_eligible(lbc::FMT_W4A16, M, Kp, p))
    return fail(LBC_ERR_PARAMS, "the fused all-gather decode serves one or two tokens with default tiling");
  if (int rc = device_gate()) return rc;
  RowsPlan P;
  if (int rc = plan_rows(lbc::FMT_W4A16, M, N_local, Kp, p, P)) return rc;
  // a CTA waits for peers' rows that other ranks' CTAs produce: every CTA of
  // the grid must be resident at once
  const int occ = lbc::rows_gather_occupancy(P.mt, P.ch, P.r, P.threads);
  if (occ <= 0) return fail(LBC_ERR_PARAMS, "decode tile has no fused all-gather variant");
  P.grid = std::min(P.grid, dev_info().sms * std::min(P.cps, occ));
  lbc::GemvArgs a{};
  a.x = x; a.qw = qw; a.scales = scales; a.zeros = zeros;
  a.M = M; a.N = N_local; a.Kp = Kp; a.y = y;
  a.status = dev_info().status;
  a.land_peers = land_peers; a.counter = counter;
  a.epoch = epoch; a.rank = rank; a.world = world; a.row0 = row0; a.ld_y = N_total;
  cudaError_t e = lbc::rows_gather_launch(a, P.mt, P.ch, P.r, dim3(P.grid, 1, 1), P.threads,
                                          static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidConfiguration) return fail(LBC_ERR_PARAMS, "decode tile has no fused all-gather variant");
  if (e != cudaSuccess) return fail_cuda("fused all-gather decode launch", e);
  return LBC_PATH_SIMT;
}

int lbc_gemm_allgather(int kind, const float *x, int M, int Kp, const uint8_t *qw, const float *scales,
                       const uint8_t *zeros, const uint8_t *e8m0, int N_local, int row0, int N_total,
                       float *const *y_peers, uint32_t *const *flag_peers, uint32_t *counter, uint32_t *epoch,
                       int rank, int world, const lbc_params *p, void *stream) {
  const int fmt = kind == 0 ? lbc::FMT_W4A16 : kind == 1 ? lbc::FMT_MXFP4 : kind == 2 ? lbc::FMT_W4A8 : -1;
  if (fmt < 0) return fail(LBC_ERR_SHAPE, "kind must be 0 (w4a16), 1 (mxfp4) or 2 (w4a8)");
  if (int rc = check_shape(M, Kp, N_local, fmt == lbc::FMT_MXFP4 ? LBC_MXBLOCK : LBC_GROUP)) return rc;
  if (!x || !qw || !y_peers || !flag_peers || !counter || !epoch || !al16(x) || !al16(qw) ||
      (fmt == lbc::FMT_MXFP4 ? !e8m0 : !scales))
    return fail(LBC_ERR_SHAPE, "NULL or misaligned pointer");
  if (world < 1 || rank < 0 || rank >= world || row0 < 0 || row0 + N_local > N_total)
    return fail(LBC_ERR_SHAPE, "rank / world / row range out of bounds");
  if (!want_prefill(p, fmt, M) || (p && p->isa >= 0 && p->isa != LBC_PATH_TCGEN05))
    return fail(LBC_ERR_PARAMS, "the fused all-gather GEMM runs the prefill kernel: 64+ tokens, default tiling "
                                "(one or two tokens: lbc_gemm_w4a16_allgather)");
  if (int rc = device_gate()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  lbc::TcCall c{};
  c.fmt = fmt; c.x = x; c.qw = qw; c.scales = scales; c.zeros = zeros; c.e8m0 = e8m0;
  c.M = M; c.N = N_local; c.Kp = Kp; c.prefill = 1;
  c.y_peers = y_peers; c.flag_peers = flag_peers; c.counter = counter; c.epoch = epoch;
  c.rank = rank; c.world = world; c.row0 = row0; c.ld_y = N_total;
  if (fmt != lbc::FMT_W4A8) return run_tc(c, st);
  // W4A8: the per-token int8 activations first, in a stream-ordered workspace
  size_t off_xs, off_as, off_tc;
  const size_t bytes = w4a8_ws_layout(M, Kp, &off_xs, &off_as, &off_tc);
  void *tmp = nullptr;
  if (cudaMallocAsync(&tmp, bytes, st) != cudaSuccess) {
    cudaGetLastError();
    return fail(LBC_ERR_ALLOC, "cudaMallocAsync(workspace) failed");
  }
  uint8_t *ws = static_cast<uint8_t *>(tmp);
  int8_t *xq = reinterpret_cast<int8_t *>(ws);
  float *xs = reinterpret_cast<float *>(ws + off_xs);
  int32_t *asum = reinterpret_cast<int32_t *>(ws + off_as);
  int rc = 0;
  cudaError_t e = lbc::launch_quant_act_int8(x, M, Kp, xq, xs, asum, st);
  if (e != cudaSuccess) rc = fail_cuda("quant_act_int8 launch", e);
  if (rc == 0) {
    c.x = nullptr; c.xq = xq; c.xs = xs; c.asum = asum;
    c.scratch = ws + off_tc;
    c.scratch_bytes = bytes - off_tc;
    rc = run_tc(c, st);
  }
  cudaFreeAsync(ws, st);
  return rc;
}

}  // extern "C"

// ------------------------------------------------------------------ host buffers

namespace {

// What a host-buffer call's captured work depends on besides the staging
// addresses: format, shape, weight pointers and params.
using HostKey = std::array<uint64_t, 8>;

HostKey host_key(int fmt, int M, int N, int Kp, const void *w0, const void *w1, const void *w2,
                 const lbc_params *p) {
  HostKey k{};
  k[0] = ((uint64_t)(uint32_t)fmt << 32) | (uint32_t)M;
  k[1] = ((uint64_t)(uint32_t)N << 32) | (uint32_t)Kp;
  k[2] = (uint64_t)(uintptr_t)w0;
  k[3] = (uint64_t)(uintptr_t)w1;
  k[4] = (uint64_t)(uintptr_t)w2;
  if (p) {
    k[5] = 1 | ((uint64_t)(uint32_t)p->isa << 32);
    k[6] = ((uint64_t)(uint32_t)p->mr << 32) | (uint32_t)p->nr;
    k[7] = ((uint64_t)(uint32_t)p->nb << 48) ^ ((uint64_t)(uint32_t)p->kb << 16) ^ (uint32_t)p->order ^
           ((uint64_t)(uint32_t)p->nthreads << 40);
  }
  return k;
}

constexpr size_t HOST_GRAPHS_MAX = 64;

// Per (device, stream) state of the host-buffer entry points: device staging
// (X, Y, W4A8 workspace), pinned and mapped host bounce buffers for X and Y,
// a private capture stream, and one instantiated CUDA graph per HostKey
// holding [bounce -> X copy, the GEMM's launches, Y -> bounce copy]. The mutex is held
// for a whole call, which ends with the stream drained, so the next call on
// that stream can reuse every buffer.
struct Stage {
  std::mutex mu;
  void *dev = nullptr;
  size_t dev_bytes = 0;
  void *hx = nullptr, *hy = nullptr;  // pinned, mapped: hx_d / hy_d are their device addresses
  float *hx_d = nullptr, *hy_d = nullptr;
  size_t hx_bytes = 0, hy_bytes = 0;
  cudaStream_t cap = nullptr;
  std::map<HostKey, std::pair<cudaGraphExec_t, int>> graphs;

  void drop_graphs() {
    for (auto &kv : graphs)
      if (kv.second.first) cudaGraphExecDestroy(kv.second.first);
    graphs.clear();
  }
};

Stage *stage_of(cudaStream_t st) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, std::unique_ptr<Stage>> map;
  int d = 0;
  cudaGetDevice(&d);
  const uint64_t key = ((uint64_t)(d & 63) << 58) ^ (uint64_t)(uintptr_t)st;
  std::lock_guard<std::mutex> g(mu);
  std::unique_ptr<Stage> &s = map[key];
  if (!s) s.reset(new Stage);
  return s.get();
}

inline size_t al256(size_t b) { return (b + 255) / 256 * 256; }

// grow one staging buffer (device or pinned host) to at least `need` bytes
int grow(Stage &s, void **buf, size_t *bytes, size_t need, bool host) {
  if (*bytes >= need) return 0;
  s.drop_graphs();  // captured graphs hold the old addresses
  s.hx_d = s.hy_d = nullptr;
  if (*buf) host ? cudaFreeHost(*buf) : cudaFree(*buf);
  *buf = nullptr;
  *bytes = 0;
  const size_t nb = std::max(need, (size_t)1 << 16);
  const cudaError_t e =
      host ? cudaHostAlloc(buf, nb, cudaHostAllocPortable | cudaHostAllocMapped) : cudaMalloc(buf, nb);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *buf = nullptr;
    return fail(LBC_ERR_ALLOC, host ? "cudaHostAlloc(host-call bounce buffer) failed"
                                    : "cudaMalloc(host-call staging) failed");
  }
  *bytes = nb;
  return 0;
}

// Copies and launches of one call, enqueued on `st`: X from the mapped
// bounce buffer into device staging, the GEMM (launch(xd, yd, ws, st) enqueues
// the device-pointer entry point), Y back into the mapped bounce buffer. The
// copies are kernels (SM loads and stores of mapped host memory), which beat
// copy-engine transfers at these sizes and overlap the GEMM's weight stream.
template <class Launch>
int enqueue_host(Stage &s, float *xd, float *yd, void *ws, size_t xb, size_t yb, cudaStream_t st,
                 Launch &launch) {
  const int sms = dev_info().sms;
  cudaError_t e = lbc::launch_copy_f32(s.hx_d, xd, xb / sizeof(float), sms, st);
  if (e != cudaSuccess) return fail_cuda("stage-in copy launch", e);
  const int rc = launch(xd, yd, ws, st);
  if (rc < 0) return rc;
  e = lbc::launch_copy_f32(yd, s.hy_d, yb / sizeof(float), sms, st);
  if (e != cudaSuccess) return fail_cuda("stage-out copy launch", e);
  return rc;
}

// X is copied into the pinned bounce buffer, the call's graph (captured on
// the first call with this key, after one uncaptured run on the private
// stream that also serves that call) runs on `stream`, and Y is copied out
// of the bounce buffer once the stream has drained.
template <class Launch>
int run_host(const HostKey &key, const float *x_host, int M, int Kp, int N, float *y_host, size_t ws_bytes,
             void *stream, Launch launch) {
  if (!x_host || !y_host) return fail(LBC_ERR_SHAPE, "NULL host pointer");
  if (int rc = device_gate()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(st, &cs);
  if (e != cudaSuccess) return fail_cuda("cudaStreamIsCapturing", e);
  if (cs != cudaStreamCaptureStatusNone)
    return fail(LBC_ERR_PARAMS, "host-buffer entry points synchronise their stream and cannot be captured");
  const size_t xb = (size_t)M * Kp * sizeof(float), yb = (size_t)M * N * sizeof(float);
  Stage &s = *stage_of(st);
  std::lock_guard<std::mutex> g(s.mu);
  if (!s.cap && (e = cudaStreamCreateWithFlags(&s.cap, cudaStreamNonBlocking)) != cudaSuccess) {
    s.cap = nullptr;
    return fail_cuda("cudaStreamCreateWithFlags", e);
  }
  if (int rc = grow(s, &s.dev, &s.dev_bytes, al256(xb) + al256(yb) + al256(ws_bytes), false)) return rc;
  if (int rc = grow(s, &s.hx, &s.hx_bytes, xb, true)) return rc;
  if (int rc = grow(s, &s.hy, &s.hy_bytes, yb, true)) return rc;
  if (!s.hx_d || !s.hy_d) {
    if ((e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&s.hx_d), s.hx, 0)) != cudaSuccess ||
        (e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&s.hy_d), s.hy, 0)) != cudaSuccess) {
      s.hx_d = s.hy_d = nullptr;
      return fail_cuda("cudaHostGetDevicePointer", e);
    }
  }
  uint8_t *base = static_cast<uint8_t *>(s.dev);
  float *xd = reinterpret_cast<float *>(base);
  float *yd = reinterpret_cast<float *>(base + al256(xb));
  void *ws = ws_bytes ? base + al256(xb) + al256(yb) : nullptr;
  memcpy(s.hx, x_host, xb);

  auto it = s.graphs.find(key);
  int rc;
  if (it != s.graphs.end() && it->second.first) {
    e = cudaGraphLaunch(it->second.first, st);
    if (e != cudaSuccess) return fail_cuda("cudaGraphLaunch", e);
    rc = it->second.second;
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda("cudaStreamSynchronize", e);
  } else if (it != s.graphs.end()) {
    // this key's work could not be captured: run it on `stream` directly
    rc = enqueue_host(s, xd, yd, ws, xb, yb, st, launch);
    e = cudaStreamSynchronize(st);
    if (rc < 0) return rc;
    if (e != cudaSuccess) return fail_cuda("cudaStreamSynchronize", e);
  } else {
    // first call with this key: drain `stream` (the call is ordered after its
    // earlier work), run on the private stream, then capture the same work
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda("cudaStreamSynchronize", e);
    rc = enqueue_host(s, xd, yd, ws, xb, yb, s.cap, launch);
    e = cudaStreamSynchronize(s.cap);
    if (rc < 0) return rc;
    if (e != cudaSuccess) return fail_cuda("cudaStreamSynchronize", e);
    if (s.graphs.size() >= HOST_GRAPHS_MAX) s.drop_graphs();
    // a failed capture is not a failed call: the key runs uncaptured from now
    // on, and lbc_last_error says why
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    e = cudaStreamBeginCapture(s.cap, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      const int crc = enqueue_host(s, xd, yd, ws, xb, yb, s.cap, launch);
      e = cudaStreamEndCapture(s.cap, &graph);
      if (crc < 0) {
        char msg[400];
        snprintf(msg, sizeof msg, "host-call graph capture failed: %s", g_err);
        fail(crc, msg);
      } else if (e != cudaSuccess || !graph) {
        fail_cuda("host-call graph capture: cudaStreamEndCapture", e);
      } else if ((e = cudaGraphInstantiate(&exec, graph, 0)) != cudaSuccess) {
        fail_cuda("host-call graph capture: cudaGraphInstantiate", e);
        exec = nullptr;
      }
      if (graph) cudaGraphDestroy(graph);
    } else {
      fail_cuda("host-call graph capture: cudaStreamBeginCapture", e);
    }
    cudaGetLastError();
    s.graphs[key] = {exec, rc};
  }
  memcpy(y_host, s.hy, yb);
  return rc;
}

}  // namespace

// lbc_gemm_*_host: X and Y in host memory, as the reference's own entry points
// take them (src/lowbit/csrc/dispatch.c:205-305), weights already on the
// device. One call copies X in, runs the GEMM, copies Y out and returns after
// the stream has drained.
extern "C" {

int lbc_gemm_w4a16_host(const float *x, int M, int Kp, const uint8_t *qw, const float *scales,
                        const uint8_t *zeros, int N, float *y, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  const HostKey key = host_key(lbc::FMT_W4A16, M, N, Kp, qw, scales, zeros, p);
  return run_host(key, x, M, Kp, N, y, 0, stream, [&](const float *xd, float *yd, void *, cudaStream_t st) {
    return lbc_gemm_w4a16(xd, M, Kp, qw, scales, zeros, N, yd, p, st);
  });
}

int lbc_gemm_mxfp4_host(const float *x, int M, int Kp, const uint8_t *qw, const uint8_t *e8m0, int N,
                        float *y, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_MXBLOCK)) return rc;
  const HostKey key = host_key(lbc::FMT_MXFP4, M, N, Kp, qw, e8m0, nullptr, p);
  return run_host(key, x, M, Kp, N, y, 0, stream, [&](const float *xd, float *yd, void *, cudaStream_t st) {
    return lbc_gemm_mxfp4(xd, M, Kp, qw, e8m0, N, yd, p, st);
  });
}

int lbc_gemm_w4a8_host(const float *x, int M, int Kp, const uint8_t *qw, const float *scales,
                       const uint8_t *zeros, int N, float *y, const lbc_params *p, void *stream) {
  if (int rc = check_shape(M, Kp, N, LBC_GROUP)) return rc;
  const HostKey key = host_key(lbc::FMT_W4A8, M, N, Kp, qw, scales, zeros, p);
  return run_host(key, x, M, Kp, N, y, w4a8_ws_layout(M, Kp, nullptr, nullptr), stream,
                  [&](const float *xd, float *yd, void *ws, cudaStream_t st) {
                    return lbc_gemm_w4a8(xd, M, Kp, qw, scales, zeros, N, yd, p, ws, st);
                  });
}

}  // extern "C"
