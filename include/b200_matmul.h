/*
 * b200_matmul.h -- C-ABI of the B200 (sm_100a) GEMM backend.
 *
 * Drop-in replacement for the CUDA library of chudinovAI/matrix-multiplication
 * (src/matmul.cu, loaded through ctypes by src/gpumat.py).  The five reference
 * exports keep their names, signatures, ABI version (3) and error convention:
 * 0 = success, 1 = failure with "operation: detail" written to the caller-owned
 * buffer `error` of `error_size` bytes.  All matrices are row-major and owned by
 * the caller: A is m x k, B is k x n (input dtype), C is m x n FP32.  Base
 * pointers need only element alignment (4 bytes for FP32/TF32, 2 bytes for
 * FP16/BF16); any m, k, n >= 1 that fit in an int are accepted.
 *
 * Implementation ids (the reference's ids 0-6 name kernels this library does
 * not contain and are rejected with an error):
 *   7  "tcgen05"  TF32 (1), FP16 (2), BF16 (3): tcgen05.mma with TMEM accumulators
 *   8  "ffma"     FP32 pedantic (0): register-blocked FFMA, no TF32 anywhere (TMA-staged
 *                 operands when they are 16-byte aligned)
 * Precision ids follow src/precision.py:8-10: 0 fp32, 1 tf32, 2 fp16, 3 bf16.
 */
#ifndef B200_MATMUL_H
#define B200_MATMUL_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_MATMUL_ABI_VERSION 3
#define B200_IMPL_TCGEN05 7
#define B200_IMPL_FFMA 8

/* Replaces matmul_abi_version (src/matmul.cu:213-216); returns 3, the value
 * src/gpumat.py:31-44 checks. */
int matmul_abi_version(void);

/* Replaces matmul_kernel_info (src/matmul.cu:218-272): writes a JSON object with
 * the reference's keys (implementation, precision, tile_m, tile_n, tile_k,
 * threads, warp_tile_m, warp_tile_n, microtile_m, microtile_n, buffering,
 * load_method, tensor_cores) plus this library's own geometry keys.  Needs no
 * GPU. */
int matmul_kernel_info(int implementation, int precision, char *json, size_t json_size,
                       char *error, size_t error_size);

/* Replaces matmul_create (src/matmul.cu:274-328): one context per device.  All
 * per-device setup happens here (kernel attributes, the tensor-map encoder, a
 * stream-ordered scratch pool); never call it during stream capture.  Returns
 * NULL on failure and consumes the sticky CUDA error of a failed cudaSetDevice
 * (src/matmul.cu:280-283). */
void *matmul_create(int device, char *error, size_t error_size);

/* Replaces matmul_destroy (src/matmul.cu:330-347). */
int matmul_destroy(void *context, char *error, size_t error_size);

/* Replaces matmul_launch (src/matmul.cu:349-479): C = A * B on `stream`
 * (a cudaStream_t), asynchronous, CUDA-graph capturable.  TF32 inputs are
 * rounded to nearest-even before the tensor-core product, by the TMA loads of
 * TFLOAT32 tensor maps; operands TMA cannot address (base not 16-byte aligned,
 * or a row pitch that is not a multiple of 16 bytes) are repacked into
 * stream-ordered scratch first.
 * TF32 problems with m*k*n <= 2^25 run on the FFMA kernel with each K tile of
 * the operands rounded to TF32 (nearest even) in shared memory: the same exact
 * products, accumulated in FP32, without the tensor-core start-up. */
int matmul_launch(void *context, int implementation, int precision,
                  const void *a, const void *b, float *c, int m, int k, int n,
                  void *stream, char *error, size_t error_size);

/* No counterpart in the reference (its end_to_end mode converts with torch's
 * `.to(dtype)` after the host-to-device copy, src/benchmark_backends.py:295-307).
 * Converts `count` FP32 values at `src` on `stream` into the input format of
 * `precision` at `dst`: BF16/FP16 by round-to-nearest-even, TF32 as FP32 words
 * rounded to 10 fraction bits (ties to even), FP32 as a copy. */
int matmul_convert(void *context, int precision, const float *src, void *dst, size_t count,
                   void *stream, char *error, size_t error_size);

/* No counterpart in the reference.  Waits for the device, then reports (and
 * with `clear` != 0 resets) the library's device status word: 0 when every
 * kernel finished normally, otherwise bit flags set by a kernel whose bounded
 * mbarrier wait ran out (1 = operand load, 2 = tensor-core issue,
 * 4 = epilogue, 8 = teardown drain). */
int matmul_device_status(void *context, int clear, unsigned int *status,
                         char *error, size_t error_size);

/* No counterpart in the reference: the GPU form of its FP64 check
 * (GemmReference.verify, src/precision.py:99-161).  For every output of C
 * (m x n, FP32) computes the FP64 product of the precision-rounded inputs
 * (TF32: round to nearest even) and the ratio |C - ref| / (5e-4 + 5e-4 |ref| +
 * gamma_K |A||B|), gamma_K from u = 2^-23 and, for TF32, the magnitude envelope
 * of the legal input models; writes the largest ratio to result[0] (<= 1 passes,
 * +inf for a non-finite output) and the largest |C - ref| to result[1].
 * Synchronises `stream`; calls that overlap on the GPU share one result slot. */
int matmul_check_fp64(void *context, int precision, const void *a, const void *b, const float *c,
                      int m, int k, int n, void *stream, double *result,
                      char *error, size_t error_size);

/* No counterpart in the reference (the nearest is matmul_kernel_info, which
 * describes a kernel, not a launch).  Writes, as a JSON object, the launch that
 * matmul_launch would make for an m x k x n problem on this context's device:
 * "kernel" (tc2_pair with a 256 x 256 or 256 x 512 tile, tc_single,
 * tc_skinny, ffma_async, or ffma_tf32_rne for small TF32 problems), "tile_m",
 * "tile_n", "splits" (K slices summed in a fixed order) and, where they apply,
 * "cluster", "threads", "grid" and "vector_loads_if_aligned" (FFMA: 16-byte
 * copies when the base pointers are 16-byte aligned too).  Needs no stream and
 * launches nothing. */
int matmul_plan(void *context, int implementation, int precision, int m, int k, int n, char *json,
                size_t json_size, char *error, size_t error_size);

/* No counterpart in the reference.  Limits the tensor-core launches of this
 * context to `sms` SMs (0 = the whole device): persistent grids, CTA pairs and
 * split-K clusters are sized for the limit and the launch plan assumes it.  For
 * running a GEMM next to communication kernels that need SMs of their own (the
 * row-sharded multi-GPU GEMM overlaps its NCCL exchanges this way).  FP32 FFMA
 * grids are not limited.  Takes effect for later launches; not synchronised with
 * launches from other threads on the same context. */
int matmul_set_sm_limit(void *context, int sms, char *error, size_t error_size);

/* No counterpart in the reference (whose kernels have no waits that can run
 * out; its error convention is src/matmul.cu:36-47, launch errors :475-478).
 * Sets the limit, in nanoseconds of GPU time, of the tensor-core kernels'
 * progress waits (a stage to land, an accumulator to fill or to be read) for
 * later launches of this context; 0 restores the default of 2 s, larger values
 * are rejected.  Waits for copies and MMAs already issued keep 2 s.  When a
 * progress wait runs out the kernel sets bits of the device status word (see
 * matmul_device_status), writes NaN over every output element it did not
 * finish, releases its tensor memory and returns, so that the context stays
 * usable and an FP64 check of C fails.  For watchdog tests and for callers that
 * want a kernel to give up sooner.  The FFMA kernel's TMA-staged 128 x 128 tile
 * (16-byte aligned operands) bounds its stage waits the same way; its cp.async
 * forms have no waits. */
int matmul_set_wait_limit(void *context, unsigned long long nanoseconds, char *error, size_t error_size);

/* No counterpart in the reference (which runs on one GPU).  Copies `bytes` (a
 * multiple of 16) from `src` on this context's device into each of the `peers`
 * (at most 7) device addresses `peer_dst[0..peers-1]` -- the same block in other
 * GPUs' buffers mapped into this process (peer-enabled allocations, e.g. symmetric
 * memory) -- with 16-byte loads of this GPU's memory and 16-byte stores over
 * NVLink, on `ctas` CTAs (0 = 16) of `stream`, asynchronously.  The C exchange of
 * the row-sharded multi-GPU GEMM: each finished row block of C goes to every
 * peer while the next block's GEMM runs on the remaining SMs.  All pointers must
 * be 16-byte aligned.  Completion on the peers is the caller's to order (a
 * collective after this launch on every rank). */
int matmul_peer_push(void *context, const void *src, void *const *peer_dst, int peers, size_t bytes, int ctas,
                     void *stream, char *error, size_t error_size);

/* No counterpart in the reference.  Same arguments, result and error convention
 * as matmul_launch, for implementation 7 (tcgen05) only, but it never allocates:
 * for callers that must not call cudaMalloc or a stream-ordered allocator --
 * typically a process whose framework has already reserved nearly all device
 * memory in its own pool, where one more allocation at launch time would fail
 * or force that pool to give memory back.  The repacked copies of unaligned
 * operands that matmul_launch places in pool memory go instead into one fixed 32 MiB
 * array compiled into the library (every GPU that loads the library holds it
 * until the process exits).  A problem whose copies need more than 32 MiB is
 * rejected with "matmul_launch_noalloc: this problem needs N bytes of scratch,
 * more than the fixed ...".  The rule is the one matmul_launch applies, whatever
 * kernel the launch plan then picks (split K included): an operand whose base
 * address is not 16-byte aligned, or whose row pitch (e*k bytes for A, e*n for
 * B, e = 4 for TF32 and 2 for FP16/BF16) is not a multiple of 16, is repacked
 * into m*k' (A) or k*n' (B) elements with k', n' rounded up to 16/e; each copy is
 * rounded up to 256 bytes.  Aligned operands, and TF32 problems with
 * m*k*n <= 2^25 (FFMA kernel), need no scratch.  The first call through a
 * context looks up the array's device address with that context's device
 * current and keeps it in the context; make that first call before any stream
 * capture (a context does not survive a device reset; create a new one after
 * it).  All calls share the one array and every call rewrites the part it uses,
 * so calls that overlap on the GPU (other streams, or other threads) race:
 * order them on one stream. */
int matmul_launch_noalloc(void *context, int implementation, int precision,
                          const void *a, const void *b, float *c, int m, int k, int n,
                          void *stream, char *error, size_t error_size);

#ifdef __cplusplus
}
#endif

#endif /* B200_MATMUL_H */
