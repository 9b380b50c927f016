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

// records `msg` as the text lbc_last_error() returns on this thread
void set_last_error(const char *msg);

}  // namespace lbc
