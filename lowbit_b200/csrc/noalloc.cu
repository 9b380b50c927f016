// lbc_gemm_w4a8_noalloc: the W4A8 GEMM for callers that cannot allocate
// device memory.
//
// lbc_gemm_w4a8 needs scratch for the quantized activations (int8 codes,
// per-token scales, per-group code sums). It either takes a caller-provided
// workspace or allocates one with cudaMallocAsync. Some callers can do
// neither: a component that is handed only input and output pointers by its
// host framework has no workspace to pass and no allocator it may call, and a
// serving loop with a latency budget may not be allowed to enter the CUDA
// allocator on its hot path. This entry point serves them by keeping the
// scratch in a fixed device array that is part of this library.
//
// Properties a caller must know:
//   * the array is LBC_NOALLOC_SCRATCH_BYTES (4 MiB) per GPU, in global memory
//     of every device that loads this library, held until the process exits;
//   * a call needs lbc_gemm_w4a8_workspace_size(M, Kp) bytes of it; larger
//     problems are rejected with LBC_ERR_SHAPE and nothing is launched;
//   * on the first call on a device (with that device current) the library
//     looks up the array's device address with cudaGetSymbolAddress and caches
//     it; make that first call before any stream capture begins;
//   * every call on a device shares the one array: calls whose GPU work can
//     overlap (different streams without ordering between them) race on it
//     and must not be issued; calls on one stream are ordered and safe;
//   * the array keeps the previous call's contents; nothing needs clearing,
//     because the activation quantizer writes every byte the GEMM then reads;
//   * no cudaMalloc, cudaMallocAsync, cudaFree or other allocating call is
//     made on this path.
#include <cstdio>
#include <mutex>

#include "../../include/lowbit_b200.h"
#include "kernels.h"

namespace {

// the scratch: xq [M, Kp] i8, xs [M] f32, asum [M, Kp/128] i32, laid out by
// lbc_gemm_w4a8 inside one 256-byte-aligned workspace
static __device__ __align__(256) unsigned char g_noalloc_scratch[LBC_NOALLOC_SCRATCH_BYTES];

struct ScratchSlot {
  bool ready = false;
  void *ptr = nullptr;
};

// Device address of g_noalloc_scratch for the current device, looked up once
// per device. Host code must not use the array's name as a device pointer:
// on the host it only names a placeholder.
cudaError_t scratch_address(void **out) {
  static std::mutex mu;
  static ScratchSlot slots[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!slots[dev].ready) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    slots[dev].ptr = p;
    slots[dev].ready = true;
  }
  *out = slots[dev].ptr;
  return cudaSuccess;
}

}  // namespace

extern "C" int lbc_gemm_w4a8_noalloc(const float *x, int M, int Kp, const uint8_t *qw,
                                     const float *scales, const uint8_t *zeros, int N, float *y,
                                     const lbc_params *p, void *stream) {
  if (M <= 0 || N <= 0 || Kp <= 0 || Kp % LBC_GROUP) {
    lbc::set_last_error("lbc_gemm_w4a8_noalloc: bad shape (M, N, Kp must be positive, Kp a multiple of 128)");
    return LBC_ERR_SHAPE;
  }
  const size_t need = lbc_gemm_w4a8_workspace_size(M, Kp);
  if (need > (size_t)LBC_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof msg,
             "lbc_gemm_w4a8_noalloc: M=%d, Kp=%d needs %zu bytes of scratch, more than the "
             "%d-byte static buffer; use lbc_gemm_w4a8 with a workspace",
             M, Kp, need, LBC_NOALLOC_SCRATCH_BYTES);
    lbc::set_last_error(msg);
    return LBC_ERR_SHAPE;
  }
  void *scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) {
    cudaGetLastError();
    char msg[256];
    snprintf(msg, sizeof msg, "lbc_gemm_w4a8_noalloc: cudaGetSymbolAddress failed: %s",
             cudaGetErrorString(e));
    lbc::set_last_error(msg);
    return LBC_ERR_CUDA;
  }
  // the regular entry point with the static array as its workspace: it then
  // allocates nothing
  return lbc_gemm_w4a8(x, M, Kp, qw, scales, zeros, N, y, p, scratch, stream);
}
