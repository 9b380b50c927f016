// Device helpers shared by the lowbit_b200 kernels (sm_100a only).
//
// Everything that waits on the GPU (mbarrier phases, flags) is bounded: a
// wait gives up after the wait limit (LBC_WAIT_CYCLES clock cycles unless the
// host set another with lbc_set_wait_cycles), records LBC_ERR_TIMEOUT in the
// device status word and lets the caller return, so a logic error surfaces as
// an error code instead of a hung GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/lowbit_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "lowbit_b200 kernels target sm_100a only"
#endif

namespace lbc {

// Default limit of a bounded wait: ~2 s at 2 GHz, far above any legitimate
// wait inside one GEMM launch.
constexpr long long LBC_WAIT_CYCLES = 4000000000LL;

// Device status block, passed to kernels by the address of its first word:
// word 0 = status (0 = ok; written only on a bounded-wait timeout), words 2-3 =
// the wait limit in clock cycles (<= 0: the default), set by the host with
// lbc_set_wait_cycles. nullptr disables reporting and uses the default limit.
__device__ __forceinline__ void set_status(int *status, int code) {
  if (status) atomicExch(status, code);
}
__device__ __forceinline__ long long wait_cycles(const int *status) {
  if (!status) return LBC_WAIT_CYCLES;
  const long long v = *reinterpret_cast<const volatile long long *>(status + 2);
  return v > 0 ? v : LBC_WAIT_CYCLES;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// ---------------------------------------------------------------- activation loads
// Kernels launched with programmatic dependent launch start while the kernel
// before them in the stream (which produces their activations) is still
// running, and read those activations only after griddepcontrol.wait. Such
// data must not be read with ld.global.nc (__ldg): a non-coherent load
// declares the data constant for the kernel's whole lifetime, so the compiler
// may issue it before the wait and see the previous call's values. These
// loads are coherent and volatile: never moved above the wait.
__device__ __forceinline__ float ld_act(const float *p) {
  float v;
  asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ int ld_act(const int *p) {
  int v;
  asm volatile("ld.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_act(const float4 *p) {
  float4 v;
  asm volatile("ld.global.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_act(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ int8_t ld_act(const int8_t *p) {
  int16_t v;
  asm volatile("ld.global.s8 %0, [%1];" : "=h"(v) : "l"(p));
  return (int8_t)v;
}

// ---------------------------------------------------------------- cross-CTA / cross-GPU
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_add_relaxed_sys_u32(uint32_t *p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------- thread-block clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every thread of every CTA of the cluster (convergent call sites only)
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}
// the shared::cluster address of `p` (this CTA's shared memory) in CTA `rank`
__device__ __forceinline__ uint32_t dsmem_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ int ld_dsmem_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_dsmem_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// make mbarrier initialisation visible to the async (TMA) proxy
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// One potentially blocking test of the phase: a waiting thread is suspended
// (issuing nothing) until the phase completes or about 1 ms has passed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false (and sets
// the device status) if the phase did not complete within the wait limit.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64(), lim = wait_cycles(status);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > lim) {
      set_status(status, LBC_ERR_TIMEOUT);
      return false;
    }
  }
}

// ---------------------------------------------------------------- bulk copies
// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar`.
// No multicast: the destination is this CTA's own shared memory.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 policy for data read exactly once (streamed weights).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// named barrier among `nthreads` threads (multiple of 32)
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// plain shared-memory load: ordered after the "memory"-clobbering mbarrier wait
__device__ __forceinline__ uint4 lds128(const void *p) { return *reinterpret_cast<const uint4 *>(p); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// unsigned bytes of a times signed bytes of b, summed into c (exact int32)
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

}  // namespace lbc
