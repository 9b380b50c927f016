// Internal launcher declarations (not part of the public C ABI).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace lbc {

cudaError_t launch_quant_act_int8(const float *x, int M, int Kp, int8_t *xq, float *xs,
                                  int32_t *asum, cudaStream_t st);

cudaError_t launch_w4a8_group_acc(const int8_t *xq, const int32_t *asum, int M, int Kp,
                                  const uint8_t *qw, const uint8_t *zeros, int N, int32_t *out,
                                  cudaStream_t st);

cudaError_t launch_tc_selftest(int kind, int32_t *out, int *status, cudaStream_t st);

struct GemvArgs;  // gemv.cuh

// few-token SIMT GEMM (gemv_tok.cu), W4A16 / MXFP4, 1 <= M <= 16, Kp <=
// tok_max_kp(opt-in shared memory per block) for ks == 1: `r` (1 or 2) rows
// per lane, `warps` (<= 16) warps per CTA, K split into `ks` ranges whose
// partial sums go to `part` (ks * M * N floats) and are added by a second
// kernel
int tok_max_kp(int smem_optin);
cudaError_t tok_gemm(int fmt, const GemvArgs &g, int r, int warps, int ks, float *part, cudaStream_t st);

// dst[0:n] = src[0:n] (floats, 16-byte aligned) by SM loads/stores, with
// programmatic stream serialisation; either side may be mapped pinned host
// memory (hostcopy.cu)
cudaError_t launch_copy_f32(const float *src, float *dst, size_t n, int sms, cudaStream_t st);

// one tensor-core GEMM call (tcgemm.cu)
struct TcCall {
  int fmt;                 // FMT_W4A16 / FMT_MXFP4 / FMT_W4A8 (gemv.cuh ids: 0 / 1 / 2)
  const float *x;          // fp formats: [M, Kp]
  const int8_t *xq;        // W4A8: [M, Kp]
  const float *xs;         // W4A8: [M]
  const int32_t *asum;     // W4A8: [M, Kp/128]
  const uint8_t *qw;
  const float *scales;
  const uint8_t *zeros;
  const uint8_t *e8m0;
  float *y;
  int M, N, Kp;
  void *scratch;           // fixup scratch (tc_scratch_bytes), or nullptr
  size_t scratch_bytes;
  int *status;
  int sms, smem_optin;
  int prefill;             // 1: 128-token prefill kernel (bf16 W4A16 / MXFP4: 4e-3 tolerance; W4A8 exact), 0: exact kernel
  // prefill only: the all-gather fused into the store (TcArgs), else nullptr
  float *const *y_peers;
  uint32_t *const *flag_peers;
  uint32_t *counter, *epoch;
  int rank, world, row0, ld_y;
};
// scratch for format `fmt` (FMT_* id), M tokens, Kp columns when the grid
// has `ctas` CTAs (at most the SM count)
size_t tc_scratch_bytes(int fmt, int M, int Kp, int ctas);
// returns LBC_PATH_TCGEN05 or a negative LBC_ERR_* with a message in err
int tc_gemm(const TcCall &c, cudaStream_t st, char *err, size_t errlen);

// records `msg` as the text lbc_last_error() returns on this thread
void set_last_error(const char *msg);

}  // namespace lbc
