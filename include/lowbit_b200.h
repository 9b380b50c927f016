/*
 * lowbit_b200 — C ABI of the B200 (sm_100a) fused dequantize + GEMM kernels.
 *
 * Every GEMM computes  Y[M,N] = X[M,Kp] . W[N,Kp]^T  (nn.Linear convention,
 * one weight row per output feature), exactly like lowbit's CPU library
 * (src/lowbit/csrc/lowbit.h:1-20).  The packed weight layouts are the
 * reference's, byte for byte, so weights quantized by lowbit are consumed
 * unchanged:
 *
 *   int4, group 128 : row n holds Kp/2 bytes; group g = bytes [64g, 64g+64).
 *                     Byte j of a group holds element 128g+j in its low nibble
 *                     and element 128g+64+j in its high nibble.  Codes are
 *                     unsigned 0..15; value = (q - z) * s with
 *                     z = zeros[n,g] (8 when zeros == NULL), s = scales[n,g].
 *   MXFP4, block 32 : block b = bytes [16b, 16b+16); byte j holds element
 *                     32b+j (low nibble) and 32b+16+j (high nibble) as OCP
 *                     E2M1 codes; value = e2m1(q) * 2^(e8m0[n,b] - 127),
 *                     e8m0 == 255 decodes to NaN.
 *
 * Conventions shared by every entry point below:
 *   - all data pointers are DEVICE pointers (cudaMalloc / torch CUDA memory)
 *     on the current device; X is fp32 [M,Kp] zero-padded to Kp, Y is fp32
 *     [M,N] and is OVERWRITTEN (the reference memsets Y then accumulates,
 *     src/lowbit/csrc/dispatch.c:168);
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); calls are
 *     stream-ordered and return before the GPU work finishes;
 *   - return value >= 0 is the kernel path that ran (LBC_PATH_*); negative
 *     values are the reference's error codes (src/lowbit/csrc/dispatch.c:
 *     160,205-208,270-286) plus CUDA-specific ones.
 */
#ifndef LOWBIT_B200_H
#define LOWBIT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LBC_GROUP 128  /* int4 group size (elements)   — lowbit.h:31 */
#define LBC_MXBLOCK 32 /* MXFP4 block size (elements)  — lowbit.h:32 */

/* kernel paths (returned by the GEMM entry points, requested via params.isa) */
#define LBC_PATH_AUTO (-1)
#define LBC_PATH_SIMT 0    /* CUDA-core fp32 FMA (int32 dp4a for W4A8) */
#define LBC_PATH_TCGEN05 1 /* tcgen05 tensor-core prefill path */
#define LBC_PATH_MMA 3     /* warp-level tensor-core (mma.sync) decode, W4A16 1-2 tokens;
                              2 is the reference's avx512 id and means auto */

/* error codes: -1..-3 keep the reference's meaning */
#define LBC_ERR_SHAPE (-1)  /* M,N,Kp <= 0, Kp % block, NULL pointer */
#define LBC_ERR_PARAMS (-2) /* tile parameters not supported ("tile not compiled") */
#define LBC_ERR_ALLOC (-3)  /* device scratch allocation failed */
#define LBC_ERR_CUDA (-5)   /* a CUDA call or launch failed (see lbc_last_error) */
#define LBC_ERR_DEVICE (-6) /* current device is not sm_100 */
#define LBC_ERR_TIMEOUT (-7) /* a bounded device-side wait gave up */

/*
 * Tuning parameters.  Same memory layout as the reference's lb_params
 * (src/lowbit/csrc/lowbit.h:37-45) so a caller's struct passes unchanged;
 * the fields are reinterpreted for the GPU.  Zero or negative = default.
 *   isa      : kernel path, LBC_PATH_* (-1 auto; reference ISA ids >= 2 = auto)
 *   mr       : tokens per pass of the SIMT kernels (1,2,4,8)
 *   nr       : weight rows per pipeline tile of the SIMT kernels (1..32)
 *   nb       : resident CTAs per SM for the SIMT kernels
 *   kb       : split-K length in elements (multiple of 128), 0 = whole K
 *   order    : TMA pipeline stages
 *   nthreads : ignored (CPU thread count; meaningless on the GPU)
 */
typedef struct {
    int isa;
    int mr;
    int nr;
    int nb;
    int kb;
    int order;
    int nthreads;
} lbc_params;

/* ---- library / device queries (replace lb_version / lb_cpu_isa / ...,
 *      src/lowbit/csrc/lowbit.h:95-102) ---- */
int lbc_version(void);
/* 1 if the current device is sm_100 and this build has kernels for it */
int lbc_device_ok(void);
/* number of SMs of the current device (0 on error) */
int lbc_sm_count(void);
/* last CUDA error text recorded by this library (thread-local, never NULL) */
const char *lbc_last_error(void);
/* device status word of the current device: 0, or LBC_ERR_TIMEOUT after a
 * bounded device-side wait gave up; reset != 0 clears it. Synchronous. */
int lbc_device_status(int reset);
/* Limit of every bounded device-side wait (mbarrier phases, the tensor-core
 * kernel's split-tile flags, the fused all-gather's arrivals) on the current
 * device, in SM clock cycles, for kernels launched afterwards; <= 0 restores
 * the default (4e9 cycles, about 2 s). A wait that runs out records
 * LBC_ERR_TIMEOUT in lbc_device_status and its kernel returns. Synchronous.
 * Returns 0 or LBC_ERR_CUDA. No reference counterpart (the reference has no
 * device-side waits). */
int lbc_set_wait_cycles(long long cycles);
/* the current device's wait limit in clock cycles (the default when unset) */
long long lbc_wait_cycles(void);

/* Kernel configuration the planner picks for a GEMM of `kind` (0 w4a16,
 * 1 mxfp4, 2 w4a8) as a JSON object in buf; returns the path or an error.
 * Introspection for tuning; no reference counterpart (the reference's
 * tiling driver, src/lowbit/csrc/dispatch.c:148-203, exposes none). */
int lbc_describe_plan(int kind, int M, int N, int Kp, const lbc_params *p, char *buf,
                      int buflen);

/* Device self-test of the tensor-core building blocks (TMEM allocation, MMA
 * with A in tensor memory and B in shared memory, accumulator readback):
 * writes D[128,16] = A.B^T for fixed small-integer A, B into out (int32,
 * 2048 entries, device memory); kind 0 = bf16 x bf16 -> f32 (K=32),
 * 1 = s8 x s8 -> s32 (K=64). Diagnostic; no reference counterpart. */
int lbc_tc_selftest(int kind, int32_t *out, void *stream);

/* ---- GEMMs ---- */

/* W4A16: replaces lb_gemm_w4a16 (src/lowbit/csrc/lowbit.h:104-106,
 * src/lowbit/csrc/dispatch.c:210-218). zeros may be NULL (symmetric, z=8). */
int lbc_gemm_w4a16(const float *x, int M, int Kp, const uint8_t *qw,
                   const float *scales, const uint8_t *zeros, int N, float *y,
                   const lbc_params *p, void *stream);

/* MXFP4: replaces lb_gemm_mxfp4 (src/lowbit/csrc/lowbit.h:107-108,
 * src/lowbit/csrc/dispatch.c:220-229). Kp % 32 == 0. */
int lbc_gemm_mxfp4(const float *x, int M, int Kp, const uint8_t *qw,
                   const uint8_t *e8m0, int N, float *y, const lbc_params *p,
                   void *stream);

/* W4A8 with fp32 X: per-token int8 quantization runs inside the call, as in
 * lb_gemm_w4a8 (src/lowbit/csrc/lowbit.h:109-112, dispatch.c:270-286).
 * `workspace` is caller-owned device scratch of at least
 * lbc_gemm_w4a8_workspace_size(M, Kp) bytes (256-byte aligned); when NULL the
 * call allocates and frees it stream-ordered (cudaMallocAsync), which mirrors
 * the reference's internal scratch allocation. */
size_t lbc_gemm_w4a8_workspace_size(int M, int Kp);
int lbc_gemm_w4a8(const float *x, int M, int Kp, const uint8_t *qw,
                  const float *scales, const uint8_t *zeros, int N, float *y,
                  const lbc_params *p, void *workspace, void *stream);

/* W4A8 with fp32 X for callers that cannot allocate device memory: no
 * counterpart in the reference. Identical results to lbc_gemm_w4a8, but the
 * activation scratch lives in a fixed LBC_NOALLOC_SCRATCH_BYTES array inside
 * this library (one per GPU, held until exit) instead of a caller workspace or
 * an allocation, so nothing is allocated on this path. It serves components
 * that receive only input/output pointers and have no allocator or workspace
 * to draw from, and latency-bound loops that must not enter the allocator.
 * Problems needing more than the array (lbc_gemm_w4a8_workspace_size(M, Kp) >
 * LBC_NOALLOC_SCRATCH_BYTES) return LBC_ERR_SHAPE without launching. The first
 * call on a device looks up the array's address (cudaGetSymbolAddress) with
 * that device current; make it before any stream capture. All calls on a
 * device share the array: calls whose GPU work may overlap race on it. */
#define LBC_NOALLOC_SCRATCH_BYTES (4 << 20)
int lbc_gemm_w4a8_noalloc(const float *x, int M, int Kp, const uint8_t *qw,
                          const float *scales, const uint8_t *zeros, int N, float *y,
                          const lbc_params *p, void *stream);

/* Host-buffer variants: x (M x Kp fp32) and y (M x N fp32) are HOST memory,
 * as in the reference's own entry points lb_gemm_w4a16 / lb_gemm_mxfp4 /
 * lb_gemm_w4a8 (src/lowbit/csrc/lowbit.h:104-112), while qw, scales, zeros
 * and e8m0 are device memory (weights are uploaded once). Each call copies x
 * to library-owned device staging (one per device and stream, grown on
 * demand), runs the device entry point above on `stream`, copies y back and
 * returns after the stream has drained, so y is ready on return. Pinned host
 * buffers (cudaHostAlloc / cudaHostRegister) copy fastest; pageable ones
 * work. Calls on one stream are serialised by the library. Not capturable
 * (LBC_ERR_PARAMS while `stream` is capturing). */
int lbc_gemm_w4a16_host(const float *x, int M, int Kp, const uint8_t *qw,
                        const float *scales, const uint8_t *zeros, int N, float *y,
                        const lbc_params *p, void *stream);
int lbc_gemm_mxfp4_host(const float *x, int M, int Kp, const uint8_t *qw,
                        const uint8_t *e8m0, int N, float *y, const lbc_params *p,
                        void *stream);
int lbc_gemm_w4a8_host(const float *x, int M, int Kp, const uint8_t *qw,
                       const float *scales, const uint8_t *zeros, int N, float *y,
                       const lbc_params *p, void *stream);

/* W4A8 on pre-quantized activations: replaces lb_gemm_w4a8_q
 * (src/lowbit/csrc/lowbit.h:113-116, dispatch.c:259-268). */
int lbc_gemm_w4a8_q(const int8_t *xq, const float *xs, const int32_t *asum,
                    int M, int Kp, const uint8_t *qw, const float *scales,
                    const uint8_t *zeros, int N, float *y, const lbc_params *p,
                    void *stream);

/* Per-token symmetric int8 quantization, bit-identical to lb_quant_act_int8
 * (src/lowbit/csrc/lowbit.h:117-119, dispatch.c:231-257): sc = amax/127
 * (1 when amax == 0), q = clamp(rne(x/sc), -127, 127), asum[m,g] = sum of
 * the group's codes. Returns 0 or a negative error. */
int lbc_quant_act_int8(const float *x, int M, int Kp, int8_t *xq, float *xs,
                       int32_t *asum, void *stream);

/* Exact int32 group accumulators out[m,n,g] = sum_{k in g} (q-z)*xq[m,k]
 * (debug/test), replaces lb_w4a8_group_acc (src/lowbit/csrc/lowbit.h:
 * 120-123, dispatch.c:288-305). `isa` is accepted and ignored. */
int lbc_w4a8_group_acc(const int8_t *xq, const int32_t *asum, int M, int Kp,
                       const uint8_t *qw, const uint8_t *zeros, int N,
                       int32_t *out, int isa, void *stream);

/* ---- multi-GPU (column-parallel) decode: no reference counterpart; this is
 * the north star's "N-sharded W with an all-gather of Y" made one kernel.
 *
 * Device buffers another process on the node can map (CUDA IPC): allocate
 * with lbc_device_alloc (zero-filled, an IPC-exportable base allocation),
 * export a handle, open the peers' handles. */
#define LBC_IPC_HANDLE_BYTES 64
int lbc_device_alloc(size_t bytes, void **dev_ptr);
int lbc_device_free(void *dev_ptr);
int lbc_ipc_get_handle(const void *dev_ptr, void *handle);
int lbc_ipc_open_handle(const void *handle, void **dev_ptr);
int lbc_ipc_close_handle(void *dev_ptr);

/* W4A16 decode (M <= 2) of this rank's weight rows [row0, row0 + N_local) of
 * an N_total-row matrix, with the all-gather fused in: when the stream's work
 * completes, y (this rank's [M, N_total] fp32 output, device memory) holds
 * every rank's rows. The call's epoch is *epoch + 1 (`epoch`: this rank's
 * zero-initialised device counter). Each output value is written to this
 * rank's rows of y and, as one 8-byte word (epoch << 32 | the value's fp32
 * bits), into the landing buffer of every other rank at
 * [epoch % 2][m][row0 + n]; land_peers is a DEVICE array of `world` pointers
 * (this rank's own included, peers' opened over IPC) to zero-initialised
 * landing buffers of LBC_GATHER_LAND_BYTES(N_total) bytes. The kernel then
 * waits (bounded: LBC_ERR_TIMEOUT in lbc_device_status) until the other
 * ranks' rows in its own landing buffer carry the epoch, copies them into y
 * and stores the epoch in *epoch. The ranks' row ranges must tile
 * [0, N_total). Nothing is baked into the launch, so CUDA graphs of these
 * calls replay correctly. `counter` is this rank's zero-initialised CTA
 * counter (one uint32). world <= LBC_GATHER_MAX_WORLD. Returns LBC_PATH_SIMT
 * or a negative error (LBC_ERR_PARAMS for M > 2 or explicit tiling params). */
#define LBC_GATHER_MAX_WORLD 8
#define LBC_GATHER_LAND_BYTES(n_total) ((size_t)(n_total) * 2 * 2 * 8)
int lbc_gemm_w4a16_allgather(const float *x, int M, int Kp, const uint8_t *qw,
                             const float *scales, const uint8_t *zeros, int N_local,
                             int row0, int N_total, float *y, uint64_t *const *land_peers,
                             uint32_t *counter, uint32_t *epoch, int rank, int world,
                             const lbc_params *p, void *stream);

/* Many-token GEMM (M >= 64: the tcgen05 prefill kernel; kind 0 w4a16, 1
 * mxfp4, 2 w4a8, arguments as lbc_gemm_w4a16 / _mxfp4 / _w4a8) of this
 * rank's weight rows [row0, row0 + N_local) of an N_total-row matrix, with
 * the all-gather fused into the GEMM's store: every finished output tile is
 * written to every rank's Y buffer y_peers[(epoch % 2) * world + p] (a DEVICE
 * array of 2 * world pointers to [M, N_total] fp32 buffers, two per rank by
 * call parity, peers' opened over IPC) at row0 + n, over NVLink while later
 * tiles are computed. The call's epoch is *epoch + 1; when this rank's CTAs
 * are done, its last CTA adds one to flag_peers[p][rank] for every p
 * (zero-initialised uint32 call counters, [world] per rank), waits (bounded:
 * LBC_ERR_TIMEOUT in lbc_device_status) until flag_peers[rank][q] has
 * reached the epoch for every q and stores the epoch in *epoch. When the
 * stream's work completes, Y of the call's parity is whole on this GPU;
 * CUDA graphs of these calls replay correctly. `counter` is this rank's
 * zero-initialised CTA counter. Returns LBC_PATH_TCGEN05 or a negative
 * error (LBC_ERR_PARAMS below 64 tokens or with explicit tiling). */
int lbc_gemm_allgather(int kind, const float *x, int M, int Kp, const uint8_t *qw,
                       const float *scales, const uint8_t *zeros, const uint8_t *e8m0,
                       int N_local, int row0, int N_total, float *const *y_peers,
                       uint32_t *const *flag_peers, uint32_t *counter, uint32_t *epoch,
                       int rank, int world, const lbc_params *p, void *stream);

/* ---- on-device weight quantizers: bit-identical to the reference's numpy
 * quantizers (src/lowbit/formats.py:90-142 and :175-212), writing the packed
 * layouts above from a row-major fp32 W [N, K] in device memory (Kp = K
 * rounded up to 128, resp. 32; padding gets the code that decodes to 0).
 * mode: 0 absmax (symmetric), 1 asym (zeros required), 2 signed-max. */
#define LBC_QUANT_ABSMAX 0
#define LBC_QUANT_ASYM 1
#define LBC_QUANT_SIGNED_MAX 2
int lbc_quantize_int4(const float *w, int N, int K, int mode, uint8_t *qw, float *scales,
                      uint8_t *zeros, void *stream);
int lbc_quantize_mxfp4(const float *w, int N, int K, uint8_t *qw, uint8_t *e8m0, void *stream);

/* ---- decoder-layer operators around the GEMMs (the model-side callers of
 * the reference, src/lowbit/model.py:380-433, on the GPU). fp32 activations,
 * row-major; `pos` is a DEVICE int32 holding the number of tokens already in
 * the KV cache, read by the kernels (CUDA graphs of a decode step replay at
 * every position). B sequences of T tokens each share one position; token
 * row i is (sequence i / T, step i % T). KV caches of one layer are
 * [B, KV, S_max, D]. All return 0 or a negative LBC_ERR_*. */

/* out = x' / sqrt(mean(x'^2) + eps) * w per row of H, x' = x + residual when
 * residual is non-NULL (then also stored to x_out, which may alias x)
 * (src/lowbit/model.py:188-190 with the residual adds of :413 and :421). */
int lbc_rmsnorm(const float *x, const float *residual, float *x_out, const float *w,
                float *out, int T, int H, float eps, void *stream);
/* qkv [B*T, (H + 2*KV)*D] (+ bias [(H + 2*KV)*D] when non-NULL): rotate-half
 * RoPE at position pos + t (cos/sin tables [positions, D/2]) on the q and k
 * heads; q to q_out [B*T, H, D], k and v into the caches at pos + t
 * (src/lowbit/model.py:199-208, :343-345, :403-406). */
int lbc_qkv_rope(const float *qkv, const float *bias, const float *cos_t, const float *sin_t,
                 const int32_t *pos, float *q_out, float *k_cache, float *v_cache, int B, int T,
                 int H, int KV, int D, int S_max, void *stream);
/* causal grouped-query attention: query (i, h) attends to keys 0..pos + i % T
 * of KV head h / (H / KV); out [B*T, H*D] (src/lowbit/model.py:336-361).
 * D is 32, 64 or 128; at most 16 query heads per KV head. For caches longer
 * than 1024 positions, when the (token, KV head) pairs fill at most half the
 * SMs, keys are split in blocks of 64 over more CTAs and merged by a second
 * kernel (scratch: one grow-only buffer per device and stream, which cannot
 * first grow inside a stream capture); otherwise the scores of one token's
 * head group, G * S_max fp32, must fit in shared memory (227 KB). */
int lbc_attention(const float *q, const float *k_cache, const float *v_cache, const int32_t *pos,
                  float *out, int B, int T, int H, int KV, int D, int S_max, void *stream);
/* W4A16 decode GEMMs with the operator before them fused into the kernel's
 * activation load (M <= 2 and default params only; otherwise LBC_ERR_PARAMS
 * and nothing runs, so the caller uses the separate kernels):
 *   _rmsnorm: y = lbc_rmsnorm(x, residual, x_out, norm_w, eps) . W^T, with
 *             x + residual stored to x_out (a buffer distinct from x and
 *             residual) when residual is non-NULL; K = Kp.
 *   _glu:     y = (silu(gu[:, :Kp]) * gu[:, Kp:]) . W^T, gu rows of 2*Kp
 *             (lbc_silu_mul then the GEMM).
 * Results equal the two-kernel path up to the order of the norm's sum of
 * squares. Returns LBC_PATH_SIMT or a negative LBC_ERR_*. */
int lbc_gemm_w4a16_rmsnorm(const float *x, const float *residual, float *x_out, const float *norm_w,
                           float eps, int M, int Kp, const uint8_t *qw, const float *scales,
                           const uint8_t *zeros, int N, float *y, const lbc_params *p, void *stream);
int lbc_gemm_w4a16_glu(const float *gu, int M, int Kp, const uint8_t *qw, const float *scales,
                       const uint8_t *zeros, int N, float *y, const lbc_params *p, void *stream);
/* One-token steps (T == 1): lbc_qkv_rope and lbc_attention in one launch --
 * each (sequence, KV head) CTA ropes its query heads and appends its k and v
 * at pos before attending. qkv [B, (H + 2*KV)*D], out [B, H*D]. */
int lbc_rope_attention(const float *qkv, const float *bias, const float *cos_t, const float *sin_t,
                       const int32_t *pos, float *k_cache, float *v_cache, float *out, int B, int H,
                       int KV, int D, int S_max, void *stream);
/* out [T, I] = silu(gu[:, :I]) * gu[:, I:] (src/lowbit/model.py:211-212, :417). */
int lbc_silu_mul(const float *gu, float *out, int T, int I, void *stream);
/* *pos += n on the device, in stream order (end of a captured decode step). */
int lbc_advance_pos(int32_t *pos, int n, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LOWBIT_B200_H */
