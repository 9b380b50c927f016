#include <algorithm>
// Tensor-core GEMM: instantiations, planning and launch (see tcgemm.cuh).
#include <atomic>
#include <chrono>
#include <cstdio>
#include <map>
#include <vector>
#include <mutex>
#include <utility>

#include "kernels.h"
#include "tcgemm_host.cuh"

namespace lbc {

namespace {

int tc_mt(int M) { return M == 1 ? 1 : M == 2 ? 2 : M <= 4 ? 4 : (M <= 8 ? 8 : 16); }
int tc_npiece(int fmt) { return fmt == FMT_W4A8 ? 1 : 3; }
int tc_bblock(int fmt, int mt) { return tc_nmma(mt, tc_npiece(fmt)) * 256 * (fmt == FMT_W4A8 ? 1 : 2); }

// B blocks come from a preparation kernel and arrive by TMA with the weights.
bool tc_btma(int) { return true; }

size_t round256(size_t b) { return (b + 255) / 256 * 256; }

// scratch: partial rows [chunks][ctas][128][mt] floats, flags [chunks][ctas],
// then (TMA-fed B) activation blocks [chunks][nkb][bblock]
size_t scratch_bytes(int fmt, int M, int Kp, int ctas) {
  const int mt = tc_mt(M);
  const size_t chunks = (size_t)((M + mt - 1) / mt);
  const size_t part = round256(chunks * ctas * TC_ROWS * mt * sizeof(float));
  const size_t flags = round256(chunks * ctas * sizeof(uint32_t));
  const size_t nkb = (size_t)((Kp + TC_KB - 1) / TC_KB);
  const size_t bglob = tc_btma(mt) ? round256(chunks * nkb * tc_bblock(fmt, mt)) : 0;
  // 64+ tokens may take the prefill kernel instead: its activation blocks
  // (activation blocks, plus split-K partial tiles: at most one 128 x 128
  // fp32 tile per SM)
  const size_t pf = M >= 64 ? round256((size_t)((M + PF_TOK - 1) / PF_TOK) * nkb * tc_nmma(PF_TOK, 1) * 256 *
                                       (fmt == FMT_W4A8 ? 1 : 2)) +
                                  round256((size_t)ctas * TC_ROWS * PF_TOK * sizeof(float))
                            : 0;
  return std::max(part + flags + bglob, pf);
}

// A value no earlier call in this process used: partial-tile flags carry it.
uint32_t next_epoch() {
  static std::atomic<uint32_t> ctr{(uint32_t)(std::chrono::steady_clock::now().time_since_epoch().count() &
                                              0x3FFFFFFF) | 1u};
  uint32_t e;
  do {
    e = ctr.fetch_add(1);
  } while (e == 0u);
  return e;
}

// Fixup scratch for calls without a workspace: one grow-only, zero-initialised
// buffer per (device, stream), so back-to-back GEMMs on a stream issue no
// allocation between them. A buffer once handed out is never freed: a CUDA
// graph captured around an earlier call (the host-buffer entry points' cached
// graphs, or a caller's own) holds its address, so a grown-out buffer is
// retired, not released, and lives until the process exits; growth at least
// doubles, so few are retired. During stream capture a growth falls back to
// a stream-ordered allocation freed after the launches.
void *cached_scratch(size_t need, cudaStream_t st, bool *owned) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<void *, size_t>> cache;
  static std::vector<void *> retired;
  *owned = false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  auto &slot = cache[{dev, st}];
  if (slot.first && slot.second >= need) return slot.first;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  if (cs != cudaStreamCaptureStatusNone) {
    void *p = nullptr;
    if (cudaMallocAsync(&p, need, st) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    *owned = true;
    return p;
  }
  const size_t bytes = std::max(need, 2 * slot.second);
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  cudaMemsetAsync(p, 0, bytes, st);
  if (slot.first) retired.push_back(slot.first);
  slot = {p, bytes};
  return p;
}

template <int FMT, int NP>
cudaError_t dispatch_mt(int mt, const CUtensorMap &map, const TcArgs &a, int chunks, int grid_x, int smem,
                        cudaStream_t st) {
  switch (mt) {
    case 1: return tc_launch_one<FMT, 1, NP>(map, a, chunks, grid_x, smem, st);
    case 2: return tc_launch_one<FMT, 2, NP>(map, a, chunks, grid_x, smem, st);
    case 4: return tc_launch_one<FMT, 4, NP>(map, a, chunks, grid_x, smem, st);
    case 8: return tc_launch_one<FMT, 8, NP>(map, a, chunks, grid_x, smem, st);
    default: return tc_launch_one<FMT, 16, NP>(map, a, chunks, grid_x, smem, st);
  }
}

}  // namespace

size_t tc_scratch_bytes(int fmt, int M, int Kp, int ctas) { return scratch_bytes(fmt, M, Kp, ctas); }

namespace {

// Prefill: activation blocks [token chunks][K blocks][128 rows x 256 K bf16 or
// int8]
// in the scratch, then the prefill kernel over (128-row, 128-token) tiles.
int tc_prefill(const TcCall &c, cudaStream_t st, char *err, size_t errlen) {
  const int fmt = c.fmt;
  TcArgs a{};
  a.x = c.x;
  a.xq = c.xq;
  a.xs = c.xs;
  a.scales = c.scales;
  a.zeros = c.zeros;
  a.e8m0 = c.e8m0;
  a.y = c.y;
  a.M = c.M;
  a.N = c.N;
  a.Kp = c.Kp;
  a.G = c.Kp / 128;
  a.nkb = (c.Kp + 255) / 256;
  a.ntiles = (c.N + TC_ROWS - 1) / TC_ROWS;
  const int nch = (c.M + PF_TOK - 1) / PF_TOK;
  a.units = a.ntiles * nch;
  a.b_block_bytes = tc_nmma(PF_TOK, 1) * 256 * (fmt == FMT_W4A8 ? 1 : 2);
  a.status = c.status;
  int stages = 4;
  while (stages > 2 && tc_smem_layout(stages, a.b_block_bytes, PF_TOK).total > c.smem_optin) --stages;
  a.stages = stages;
  const int smem = tc_smem_layout(stages, a.b_block_bytes, PF_TOK).total;
  if (smem > c.smem_optin) {
    snprintf(err, errlen, "prefill tile does not fit in shared memory");
    return LBC_ERR_PARAMS;
  }
  // split K when the output tiles cannot fill the GPU (few weight-row tiles
  // at 64-512 tokens): every split keeps at least one 256-K unit
  // (at most one item per SM, so no CTA runs two)
  a.ksplit = 1;
  if (2 * a.units <= c.sms && !c.y_peers) a.ksplit = std::min(a.nkb, c.sms / a.units);
  a.y_peers = c.y_peers;  // fused all-gather (never split: the store is the exchange)
  a.flag_peers = c.flag_peers;
  a.ag_counter = c.counter;
  a.ag_epoch = c.epoch;
  a.rank = c.rank;
  a.world = c.world;
  a.row0 = c.row0;
  a.ld_y = c.ld_y;
  const int items = a.units * a.ksplit;
  const int grid_x = items < c.sms ? items : c.sms;
  CUtensorMap map;
  if (make_weight_map(&map, c.qw, c.N, c.Kp) != cudaSuccess) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed for the weight tensor");
    return LBC_ERR_CUDA;
  }
  // scratch: activation blocks, then (split-K) one partial tile per work item
  // [items][128 tokens][128 rows] fp32
  const size_t bglob_bytes = round256((size_t)nch * a.nkb * a.b_block_bytes);
  const size_t part_bytes = a.ksplit > 1 ? round256((size_t)items * TC_ROWS * PF_TOK * sizeof(float)) : 0;
  const size_t need = bglob_bytes + part_bytes;
  bool owned = false;
  uint8_t *scr = static_cast<uint8_t *>(c.scratch);  // a caller's workspace, when large enough
  if (!scr || c.scratch_bytes < need) scr = static_cast<uint8_t *>(cached_scratch(need, st, &owned));
  if (!scr) {
    snprintf(err, errlen, "allocation of %zu bytes of GEMM scratch failed", need);
    return LBC_ERR_ALLOC;
  }
  a.bglob = scr;
  if (a.ksplit > 1) a.partial = reinterpret_cast<float *>(scr + bglob_bytes);
  cudaError_t e = fmt == FMT_W4A16  ? tc_prefill_launch<FMT_W4A16>(map, a, nch, grid_x, smem, st)
                   : fmt == FMT_W4A8 ? tc_prefill_launch<FMT_W4A8>(map, a, nch, grid_x, smem, st)
                                     : tc_prefill_launch<FMT_MXFP4>(map, a, nch, grid_x, smem, st);
  if (owned) cudaFreeAsync(scr, st);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "tensor-core prefill launch: %s%s", cudaGetErrorString(e), tc_launch_note());
    return LBC_ERR_CUDA;
  }
  return LBC_PATH_TCGEN05;
}

}  // namespace

int tc_gemm(const TcCall &c, cudaStream_t st, char *err, size_t errlen) {
  if (c.prefill) return tc_prefill(c, st, err, errlen);
  const int fmt = c.fmt;
  const int mt = tc_mt(c.M);
  const int chunks = (c.M + mt - 1) / mt;
  const int bbytes = tc_bblock(fmt, mt);
  TcArgs a{};
  a.x = c.x;
  a.xq = c.xq;
  a.scales = c.scales;
  a.zeros = c.zeros;
  a.e8m0 = c.e8m0;
  a.asum = c.asum;
  a.xs = c.xs;
  a.y = c.y;
  a.M = c.M;
  a.N = c.N;
  a.Kp = c.Kp;
  a.G = c.Kp / 128;
  a.nkb = (c.Kp + 255) / 256;
  a.ntiles = (c.N + TC_ROWS - 1) / TC_ROWS;
  a.units = a.nkb * a.ntiles;
  a.b_block_bytes = bbytes;
  a.status = c.status;
  a.epoch = next_epoch();
  int stages = 8;
  while (stages > 2 && tc_smem_layout(stages, bbytes, mt).total > c.smem_optin) --stages;
  a.stages = stages;
  const int smem = tc_smem_layout(stages, bbytes, mt).total;
  if (smem > c.smem_optin) {
    snprintf(err, errlen, "tensor-core tile does not fit in shared memory");
    return LBC_ERR_PARAMS;
  }
  const int grid_x = a.units < c.sms ? a.units : c.sms;
  CUtensorMap map;
  cudaError_t e = make_weight_map(&map, c.qw, c.N, c.Kp);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed for the weight tensor");
    return LBC_ERR_CUDA;
  }
  const size_t need = scratch_bytes(fmt, c.M, c.Kp, grid_x);
  uint8_t *scr = static_cast<uint8_t *>(c.scratch);
  bool owned = false;
  if (!scr || c.scratch_bytes < need) {
    scr = static_cast<uint8_t *>(cached_scratch(need, st, &owned));
    if (!scr) {
      snprintf(err, errlen, "allocation of %zu bytes of GEMM scratch failed", need);
      return LBC_ERR_ALLOC;
    }
  }
  const size_t part_bytes = round256((size_t)chunks * grid_x * TC_ROWS * mt * sizeof(float));
  const size_t flag_bytes = round256((size_t)chunks * grid_x * sizeof(uint32_t));
  a.partial = reinterpret_cast<float *>(scr);
  a.flags = reinterpret_cast<uint32_t *>(scr + part_bytes);
  a.bglob = tc_btma(mt) ? scr + part_bytes + flag_bytes : nullptr;
  if (fmt == FMT_W4A16)
    e = dispatch_mt<FMT_W4A16, 3>(mt, map, a, chunks, grid_x, smem, st);
  else if (fmt == FMT_MXFP4)
    e = dispatch_mt<FMT_MXFP4, 3>(mt, map, a, chunks, grid_x, smem, st);
  else
    e = dispatch_mt<FMT_W4A8, 1>(mt, map, a, chunks, grid_x, smem, st);
  if (owned) cudaFreeAsync(scr, st);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "tensor-core GEMM launch: %s%s", cudaGetErrorString(e), tc_launch_note());
    return LBC_ERR_CUDA;
  }
  return LBC_PATH_TCGEN05;
}

}  // namespace lbc
