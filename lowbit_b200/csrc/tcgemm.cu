// Tensor-core GEMM: instantiations, planning and launch (see tcgemm.cuh).
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include "kernels.h"
#include "tcgemm_host.cuh"

namespace lbc {

namespace {

int tc_mt(int M) { return M <= 4 ? 4 : (M <= 8 ? 8 : 16); }
int tc_npiece(int fmt) { return fmt == FMT_W4A8 ? 1 : 3; }
int tc_bblock(int fmt, int mt) { return tc_nmma(mt, tc_npiece(fmt)) * 256 * (fmt == FMT_W4A8 ? 1 : 2); }

template <int FMT, int NP>
cudaError_t dispatch_mt(int mt, const CUtensorMap &map, const TcArgs &a, int chunks, int grid_x, int smem,
                        cudaStream_t st) {
  switch (mt) {
    case 4: return tc_launch_one<FMT, 4, NP>(map, a, chunks, grid_x, smem, st);
    case 8: return tc_launch_one<FMT, 8, NP>(map, a, chunks, grid_x, smem, st);
    default: return tc_launch_one<FMT, 16, NP>(map, a, chunks, grid_x, smem, st);
  }
}

// Activation-block scratch for calls without a workspace: one grow-only buffer
// per (device, stream), so back-to-back GEMMs on a stream issue no allocation
// between them (an allocation would break their programmatic overlap). The
// buffers live until the process exits. During stream capture a growth falls
// back to a stream-ordered allocation for that call.
void *cached_scratch(size_t need, cudaStream_t st, bool *owned) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<void *, size_t>> cache;
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
  if (slot.first) {
    cudaStreamSynchronize(st);
    cudaFree(slot.first);
    slot = {nullptr, 0};
  }
  void *p = nullptr;
  if (cudaMalloc(&p, need) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  slot = {p, need};
  return p;
}

}  // namespace

size_t tc_bglob_bytes(int fmt, int M, int Kp) {
  const int mt = tc_mt(M);
  const size_t chunks = (size_t)((M + mt - 1) / mt);
  const size_t nkb = (size_t)((Kp + 255) / 256);
  return chunks * nkb * (size_t)tc_bblock(fmt, mt);
}

int tc_gemm(const TcCall &c, cudaStream_t st, char *err, size_t errlen) {
  const int fmt = c.fmt;
  const int mt = tc_mt(c.M);
  const int np = tc_npiece(fmt);
  const int nmma = tc_nmma(mt, np);
  const int chunks = (c.M + mt - 1) / mt;
  const int bbytes = tc_bblock(fmt, mt);
  TcArgs a{};
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
  a.mt = mt;
  a.status = c.status;
  const int per_stage = TC_WBYTES + (bbytes + 127) / 128 * 128;
  int stages = 6;
  while (stages > 2 && tc_smem_layout(stages, bbytes).total > c.smem_optin) --stages;
  a.stages = stages;
  const int smem = tc_smem_layout(stages, bbytes).total;
  (void)per_stage;
  if (smem > c.smem_optin) {
    snprintf(err, errlen, "tensor-core tile does not fit in shared memory");
    return LBC_ERR_PARAMS;
  }
  CUtensorMap map;
  cudaError_t e = make_weight_map(&map, c.qw, c.N, c.Kp);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed for the weight tensor");
    return LBC_ERR_CUDA;
  }
  const size_t need = tc_bglob_bytes(fmt, c.M, c.Kp);
  uint8_t *bglob = static_cast<uint8_t *>(c.bscratch);
  bool owned = false;
  if (!bglob || c.bscratch_bytes < need) {
    bglob = static_cast<uint8_t *>(cached_scratch(need, st, &owned));
    if (!bglob) {
      snprintf(err, errlen, "allocation of %zu bytes of activation blocks failed", need);
      return LBC_ERR_ALLOC;
    }
  }
  a.bglob = bglob;
  const dim3 pgrid(a.nkb, chunks, 1);
  if (fmt == FMT_W4A16)
    e = launch_pdl(tc_prep_kernel<FMT_W4A16>, pgrid, dim3(256), 0, st, c.x, (const int8_t *)nullptr, c.M, c.Kp,
                   a.nkb, mt, nmma, np, bglob, bbytes, c.y, c.N);
  else if (fmt == FMT_MXFP4)
    e = launch_pdl(tc_prep_kernel<FMT_MXFP4>, pgrid, dim3(256), 0, st, c.x, (const int8_t *)nullptr, c.M, c.Kp,
                   a.nkb, mt, nmma, np, bglob, bbytes, c.y, c.N);
  else
    e = launch_pdl(tc_prep_kernel<FMT_W4A8>, pgrid, dim3(256), 0, st, (const float *)nullptr, c.xq, c.M, c.Kp,
                   a.nkb, mt, nmma, np, bglob, bbytes, c.y, c.N);
  if (e == cudaSuccess) {
    const int grid_x = a.units < c.sms ? a.units : c.sms;
    if (fmt == FMT_W4A16)
      e = dispatch_mt<FMT_W4A16, 3>(mt, map, a, chunks, grid_x, smem, st);
    else if (fmt == FMT_MXFP4)
      e = dispatch_mt<FMT_MXFP4, 3>(mt, map, a, chunks, grid_x, smem, st);
    else
      e = dispatch_mt<FMT_W4A8, 1>(mt, map, a, chunks, grid_x, smem, st);
  }
  if (owned) cudaFreeAsync(bglob, st);
  if (e != cudaSuccess) {
    snprintf(err, errlen, "tensor-core GEMM launch: %s", cudaGetErrorString(e));
    return LBC_ERR_CUDA;
  }
  return LBC_PATH_TCGEN05;
}

}  // namespace lbc
