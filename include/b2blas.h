/*
 * b2blas.h -- C ABI of the B200 (sm_100a) Level-3 / Level-2 BLAS library that
 * replaces cublas-rs's cuda-oxide kernels and PTX loading.
 *
 * Conventions (all taken from the reference's Handle API):
 *   - Matrices are row-major and contiguous: A[m x k], B[k x n], C[m x n]
 *     (crates/cublas-core/src/config.rs:1-9; indexing sgemm.rs:94-101).
 *   - C <- alpha * A * B + beta * C.  When beta == 0, C is not read (so NaN or
 *     uninitialised C does not propagate), which is the cuBLAS rule; for
 *     finite C this gives the same values as the reference, whose kernels
 *     compute alpha*sum + beta*c unconditionally (sgemm.rs:121-127).
 *   - m == 0 || n == 0 || k == 0 (or batch == 0) returns B2B_OK with no launch
 *     and C untouched (sgemm.rs:379-381, batched.rs:123-125).
 *   - Device-buffer calls ("xxx") are asynchronous on the handle's stream;
 *     host-slice calls ("xxx_simple") copy in, launch, copy out and block
 *     (sgemm.rs:460-482).  Host-slice calls take slice lengths in elements
 *     and return B2B_ERR_DIMENSION where the reference panics on a length
 *     mismatch (sgemm.rs:469-471, batched.rs:171-173, gemv.rs:279-282).
 *   - Sizes and strides are 64-bit (the reference casts them to u32,
 *     batched.rs:142-152).
 *   - Every function returns a b2b_status; b2b_last_error() gives the message
 *     of the last failure on the calling thread.
 *   - Device-buffer calls can be captured in a CUDA graph once one eager call
 *     of the same shapes has sized the handle's workspace; host-slice calls
 *     and the value-returning reductions synchronise and cannot.
 */
#ifndef B2BLAS_H
#define B2BLAS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2B_API __attribute__((visibility("default")))

/* Status codes.  Maps onto cublas_core::CublasError
 * (crates/cublas-core/src/error.rs:7-24): CUDA -> Driver, DIMENSION ->
 * DimensionMismatch, INVALID_ARG -> InvalidArgument; DEVICE_TIMEOUT is a
 * bounded device-side wait that gave up (reported through Driver). */
typedef enum {
    B2B_OK = 0,
    B2B_ERR_CUDA = 1,
    B2B_ERR_DIMENSION = 2,
    B2B_ERR_INVALID_ARG = 3,
    B2B_ERR_DEVICE_TIMEOUT = 4,
    B2B_ERR_NOT_SUPPORTED = 5,
    B2B_ERR_ALLOC = 6
} b2b_status;

/* cublas_core::Transpose (crates/cublas-core/src/config.rs:20-23). */
typedef enum { B2B_OP_N = 0, B2B_OP_T = 1 } b2b_transpose;

/* Kernel choice.  The reference exposes one method per kernel variant
 * (Handle::sgemm_naive / _tiled / _vectorized / _double_buf,
 * crates/cublas-rs/src/lib.rs:439-524; sgemv / sgemv_tiled, lib.rs:230-309).
 * On B200 each of those names runs the same tuned kernel; the values are kept
 * so the facade can forward the variant it was called as.  B2B_ALGO_3XTF32
 * is the opt-in split-precision tensor-core SGEMM (no reference
 * counterpart; the reference's tensor-core slot is a todo!, hgemm.rs:189-193). */
typedef enum {
    B2B_ALGO_DEFAULT = 0,
    B2B_ALGO_NAIVE = 1,
    B2B_ALGO_TILED = 2,
    B2B_ALGO_VECTORIZED = 3,
    B2B_ALGO_DOUBLE_BUF = 4,
    B2B_ALGO_3XTF32 = 5
} b2b_algo;

typedef struct b2b_handle b2b_handle;

/* ------------------------------------------------------------ lifecycle */

/* Handle::new / Handle::with_device (crates/cublas-rs/src/lib.rs:53-68):
 * binds the device, creates the handle's stream and its device status word.
 * Replaces Modules::load x3 (crates/cublas-l3/src/lib.rs:51-61 and the L1/L2
 * equivalents): kernels are linked into this library, no PTX is read from
 * the working directory. */
B2B_API int b2b_create(int device, b2b_handle **out);
B2B_API int b2b_destroy(b2b_handle *h);
/* Handle::stream (lib.rs:72-74).  Returns the cudaStream_t as void*. */
B2B_API int b2b_get_stream(b2b_handle *h, void **stream);
/* Run subsequent calls on a caller-owned cudaStream_t.  NULL selects the
 * handle's own stream again; the legacy default stream is selected with
 * cudaStreamLegacy ((void *)0x1).  No reference counterpart; the cuBLAS
 * equivalent is cublasSetStream.  Used to share a stream with torch / NCCL.
 * Switching streams makes the new stream wait (an event) for the work already
 * queued on the previous one, because every call reuses the handle's
 * workspace and reduction counter.  Handles are not thread-safe: use one per
 * thread. */
B2B_API int b2b_set_stream(b2b_handle *h, void *stream);
/* Handle::synchronize (lib.rs:79-82): blocks on the stream, then reports a
 * device-side bounded-wait timeout, if one was recorded, as
 * B2B_ERR_DEVICE_TIMEOUT (and clears it). */
B2B_API int b2b_synchronize(b2b_handle *h);
/* Device ordinal, SM count and clock, for the facade and the bench. */
B2B_API int b2b_device_info(b2b_handle *h, int *device, int *sm_count, int *sm_clock_khz);
B2B_API const char *b2b_status_string(int status);
B2B_API const char *b2b_last_error(void);
/* Library version, (major << 16) | (minor << 8) | patch. */
B2B_API int b2b_version(void);

/* ---------------------------------------------- device memory (DeviceBuf)
 * Stand-ins for cuda_core::DeviceBuffer<T> (re-exported as DeviceBuf,
 * lib.rs:34): zeroed(stream, n), from_host(stream, &[T]), to_host_vec(stream)
 * and Handle::upload / Handle::download (lib.rs:88-97).  Copies are ordered
 * on the handle's stream; the d2h copy blocks until the data has arrived. */
B2B_API int b2b_malloc(b2b_handle *h, size_t bytes, void **dptr);
B2B_API int b2b_free(b2b_handle *h, void *dptr);
B2B_API int b2b_memcpy_h2d(b2b_handle *h, void *dst, const void *src, size_t bytes);
B2B_API int b2b_memcpy_d2h(b2b_handle *h, void *dst, const void *src, size_t bytes);
B2B_API int b2b_memcpy_d2d(b2b_handle *h, void *dst, const void *src, size_t bytes);
B2B_API int b2b_memset(b2b_handle *h, void *dptr, int value, size_t bytes);
/* Page-locked host memory, so host-slice calls can overlap copy and compute. */
B2B_API int b2b_host_alloc(size_t bytes, void **hptr);
B2B_API int b2b_host_free(void *hptr);

/* ------------------------------------------------------ Level 3: SGEMM */

/* Handle::sgemm_{naive,tiled,vectorized,double_buf}(config, a, b, c)
 * (crates/cublas-rs/src/lib.rs:439-505) -> cublas_l3::sgemm_*_dev
 * (crates/cublas-l3/src/sgemm.rs:370-394, 432-453, 491-515, 553-574).
 * Device pointers. */
B2B_API int b2b_sgemm(b2b_handle *h, int algo, size_t m, size_t n, size_t k, float alpha, const float *A,
                      const float *B, float beta, float *C);
/* Handle::sgemm_*_simple (lib.rs:450-524) -> cublas_l3::sgemm_* host-slice
 * launchers (sgemm.rs:401-424, 460-482, 522-545, 582-603).  Host pointers
 * with slice lengths in elements; C is read (when beta != 0) and written. */
B2B_API int b2b_sgemm_simple(b2b_handle *h, int algo, size_t m, size_t n, size_t k, float alpha, const float *A,
                             size_t a_len, const float *B, size_t b_len, float beta, float *C, size_t c_len);

/* SGEMM with the bias broadcast and ReLU folded into the epilogue:
 * C <- act(alpha*A*B + beta*C + bias[j]) for every row, act = max(0, .) when
 * relu != 0; bias is a device vector of n floats or NULL.  Replaces the
 * mlp example's sgemm + saxpy-of-a-pre-broadcast-bias pair
 * (examples/mlp/src/main.rs:130-144, bias materialised at :52) and its
 * pending ReLU step (:146); no counterpart in the reference library. */
B2B_API int b2b_sgemm_bias(b2b_handle *h, int algo, size_t m, size_t n, size_t k, float alpha, const float *A,
                           const float *B, float beta, float *C, const float *bias, int relu);

/* Split-K of the FP32 FFMA SGEMM; no counterpart in the reference (its
 * kernels have no K split).  A GEMM whose output tiles fill the GPU badly
 * (under one wave of 128 x 256 tiles, or just past a whole number of waves)
 * is computed as S independent k ranges whose raw sums are added in range
 * order by a second kernel; the result is deterministic, but its bits depend
 * on S.  b2b_sgemm_splits returns the S that b2b_sgemm / b2b_sgemm_bias
 * (default algo, 16-byte aligned operands) choose for an m x n x k call;
 * b2b_set_sgemm_splits fixes S for the handle's later calls: 0 = choose per
 * call (the default), 1 = never split, S in 2..16 = always S where the
 * TMA-fed kernel takes the call (S partial sums of m x n floats live in the
 * handle's workspace).  A caller that computes one GEMM as several row or
 * column pieces gets the whole GEMM's bits by fixing the whole GEMM's S for
 * the pieces (the host-slice calls do this themselves). */
B2B_API int b2b_sgemm_splits(b2b_handle *h, size_t m, size_t n, size_t k, int *splits);
B2B_API int b2b_set_sgemm_splits(b2b_handle *h, int splits);

/* ------------------------------------------------------ Level 3: DGEMM */

/* Handle::dgemm_* (lib.rs:527-612) -> crates/cublas-l3/src/dgemm.rs:342-569.
 * Grids that fill the GPU badly are split along K as for SGEMM (partial sums
 * in handle workspace, added in a fixed order): the result is deterministic,
 * and its bits depend on the split, which the host-slice call keeps equal to
 * the device call's (B2B_DGEMM_KSPLIT forces one). */
B2B_API int b2b_dgemm(b2b_handle *h, int algo, size_t m, size_t n, size_t k, double alpha, const double *A,
                      const double *B, double beta, double *C);
B2B_API int b2b_dgemm_simple(b2b_handle *h, int algo, size_t m, size_t n, size_t k, double alpha,
                             const double *A, size_t a_len, const double *B, size_t b_len, double beta, double *C,
                             size_t c_len);

/* ------------------------------------------------------ Level 3: HGEMM */

/* Handle::hgemm_half / hgemm_tensor_core (lib.rs:616-635) ->
 * cublas_l3::hgemm_half (crates/cublas-l3/src/hgemm.rs:135-187); the
 * tensor-core slot (hgemm.rs:189-193) is this function's tcgen05 path.
 * f16 bit patterns (uint16_t, as hgemm.rs:151-156 reinterprets half::f16),
 * f32 accumulate, f16 output rounded to nearest even; alpha/beta are f32
 * (hgemm.rs:175,178).  Device pointers. */
B2B_API int b2b_hgemm(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                      const uint16_t *B, float beta, uint16_t *C);
/* Host-slice flavour (the only one the reference has). */
B2B_API int b2b_hgemm_simple(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                             size_t a_len, const uint16_t *B, size_t b_len, float beta, uint16_t *C,
                             size_t c_len);

/* ----------------------------------------- Level 3: batched SGEMM family */

/* Handle::strided_batched_sgemm (lib.rs:660-683) ->
 * cublas_l3::strided_batched_sgemm_dev (crates/cublas-l3/src/batched.rs:112-155).
 * Batch b uses A + b*stride_a, B + b*stride_b, C + b*stride_c (elements).
 * No 65535 batch limit. */
B2B_API int b2b_sgemm_strided_batched(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                                      size_t stride_a, const float *B, size_t stride_b, float beta, float *C,
                                      size_t stride_c, size_t batch);
/* Handle::strided_batched_sgemm_simple (lib.rs:686-709) -> batched.rs:162-200.
 * The reference asserts len >= batch*stride (batched.rs:171-173). */
B2B_API int b2b_sgemm_strided_batched_simple(b2b_handle *h, size_t m, size_t n, size_t k, float alpha,
                                             const float *A, size_t a_len, size_t stride_a, const float *B,
                                             size_t b_len, size_t stride_b, float beta, float *C, size_t c_len,
                                             size_t stride_c, size_t batch);
/* Handle::batched_sgemm (lib.rs:639-656) -> batched.rs:211-261: per-batch
 * host slices, each of exact length m*k / k*n / m*n (asserts :236-238);
 * concatenated into one strided batch. */
B2B_API int b2b_sgemm_batched_simple(b2b_handle *h, size_t m, size_t n, size_t k, float alpha,
                                     const float *const *A, const size_t *a_lens, const float *const *B,
                                     const size_t *b_lens, float beta, float *const *C, const size_t *c_lens,
                                     size_t batch);

/* -------------------------------------------------------- Level 2: SGEMV */

/* Handle::sgemv / sgemv_tiled (lib.rs:230-283) -> cublas_l2::sgemv_dev /
 * sgemv_tiled_dev (crates/cublas-l2/src/gemv.rs:233-259, 307-337).
 * y <- alpha*op(A)*x + beta*y, A m x n row-major; op(A) = A (N: x has n,
 * y has m) or A^T (T: x has m, y has n) (gemv.rs:1-5).  Device pointers. */
B2B_API int b2b_sgemv(b2b_handle *h, int algo, int trans, size_t m, size_t n, float alpha, const float *A,
                      const float *x, float beta, float *y);
/* Handle::sgemv_simple / sgemv_tiled_simple (lib.rs:244-309) -> gemv.rs:266-305,
 * 344-376 (A length must equal m*n; x, y at least their op lengths). */
B2B_API int b2b_sgemv_simple(b2b_handle *h, int algo, int trans, size_t m, size_t n, float alpha, const float *A,
                             size_t a_len, const float *x, size_t x_len, float beta, float *y, size_t y_len);

/* SGEMV that allocates no device memory.  No counterpart in the reference.
 * Some callers cannot call cudaMalloc or cudaFree: a process whose device
 * memory is already reserved by another allocator (a framework's caching
 * pool), a service with a fixed memory budget set at start-up, or a loop
 * that must not stall on the device-wide synchronisation cudaFree implies.
 * b2b_sgemv's transposed path keeps its split-row partial sums in handle
 * workspace, which it grows with cudaMallocAsync; this variant keeps them in
 * a fixed 1 MiB device array built into the library (held by every GPU that
 * loads it until the process exits).  Same arguments and results as b2b_sgemv.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture.  The address is cached per device and
 *     context: after cudaDeviceReset the next call looks it up again (so
 *     make one call before capturing in the new context too).
 *   - All calls, across handles and streams, share the one array, which
 *     keeps the last call's contents; nothing in it needs clearing (every
 *     partial is written before it is read), but calls that may overlap on
 *     the GPU race on it and must be serialised by the caller.
 *   - A shape whose partial sums do not fit the array is rejected with
 *     B2B_ERR_INVALID_ARG, before any launch, and a message naming the
 *     sizes (on a 148-SM GPU every shape fits; a handle created with
 *     B2B_NOALLOC_SCRATCH_FLOATS=<n> in the environment uses n as a lower
 *     limit). */
B2B_API int b2b_sgemv_noalloc(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const float *A,
                              const float *x, float beta, float *y);

/* ------------------------------------------------ Level 2: DGEMV, HGEMV */

/* Handle::dgemv (lib.rs:312-324) -> cublas_l2::dgemv_dev
 * (crates/cublas-l2/src/gemv.rs:446-471): y <- alpha*op(A)*x + beta*y in
 * f64, A m x n row-major, op as in b2b_sgemv.  Device pointers. */
B2B_API int b2b_dgemv(b2b_handle *h, int trans, size_t m, size_t n, double alpha, const double *A,
                      const double *x, double beta, double *y);
/* Handle::dgemv_simple (lib.rs:327-339) -> gemv.rs:478-509 (A length must
 * equal m*n; x, y at least their op lengths). */
B2B_API int b2b_dgemv_simple(b2b_handle *h, int trans, size_t m, size_t n, double alpha, const double *A,
                             size_t a_len, const double *x, size_t x_len, double beta, double *y, size_t y_len);
/* Device-pointer HGEMV.  The reference has the host-slice flavour only
 * (lib.rs:341-343); this one is its kernel step.  f16 bit patterns, f32
 * accumulate, f16 result rounded to nearest even; alpha/beta as f32. */
B2B_API int b2b_hgemv(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const uint16_t *A,
                      const uint16_t *x, float beta, uint16_t *y);
/* Handle::hgemv (lib.rs:344-366) -> cublas_l2::hgemv (gemv.rs:619-673):
 * host slices of f16 bit patterns; alpha/beta are the f32 values the
 * reference passes its kernels (alpha.to_f32(), gemv.rs:651-652). */
B2B_API int b2b_hgemv_simple(b2b_handle *h, int trans, size_t m, size_t n, float alpha, const uint16_t *A,
                             size_t a_len, const uint16_t *x, size_t x_len, float beta, uint16_t *y,
                             size_t y_len);

/* -------------------------------------------------------- Level 1: SAXPY */

/* Handle::saxpy (lib.rs:110-118) -> crates/cublas-l1/src/saxpy.rs:25-40:
 * y <- alpha*x + y over n elements.  Device pointers. */
B2B_API int b2b_saxpy(b2b_handle *h, size_t n, float alpha, const float *x, float *y);
/* Handle::saxpy_simple (lib.rs:121-129) -> saxpy.rs:45-66 (x, y at least n). */
B2B_API int b2b_saxpy_simple(b2b_handle *h, size_t n, float alpha, const float *x, size_t x_len, float *y,
                             size_t y_len);

/* ------------------------------------------------- Level 1: reductions
 * One multi-block launch each, f64 accumulation, deterministic order (the
 * reference runs one 32-thread block, crates/cublas-l1/src/dot.rs:21-53).
 * The device-buffer flavours take device x/y, write the result to a host
 * pointer and block until it is there, as the reference's *_dev functions
 * return a host value (dot.rs:59-78).  n == 0 gives 0.  The host flavours
 * check x_len/y_len >= n and copy only the first n elements (dot.rs:81-96). */
typedef enum b2b_reduce_op {
    B2B_REDUCE_DOT = 0,   /* sum x[i]*y[i]                     (f32 result) */
    B2B_REDUCE_NRM2 = 1,  /* sqrt(sum x[i]^2)                  (f32 result) */
    B2B_REDUCE_ASUM = 2,  /* sum |x[i]|                        (f32 result) */
    B2B_REDUCE_IAMAX = 3  /* smallest 0-based i of max |x[i]|  (uint64 result) */
} b2b_reduce_op;

/* Handle::sdot / sdot_simple (lib.rs:157-165) -> dot.rs:59-96. */
B2B_API int b2b_sdot(b2b_handle *h, size_t n, const float *x, const float *y, float *result);
B2B_API int b2b_sdot_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, const float *y, size_t y_len,
                            float *result);
/* Handle::snrm2 / snrm2_simple (lib.rs:167-175) -> nrm2.rs:54-87.  The sum
 * of squares is kept in f64, so no finite input overflows it. */
B2B_API int b2b_snrm2(b2b_handle *h, size_t n, const float *x, float *result);
B2B_API int b2b_snrm2_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, float *result);
/* Handle::sasum / sasum_simple (lib.rs:177-185) -> asum.rs:53-86. */
B2B_API int b2b_sasum(b2b_handle *h, size_t n, const float *x, float *result);
B2B_API int b2b_sasum_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, float *result);
/* Handle::isamax / isamax_simple (lib.rs:187-195) -> iamax.rs:67-100.
 * Ties give the smallest index; NaN elements never win; all-NaN gives 0. */
B2B_API int b2b_isamax(b2b_handle *h, size_t n, const float *x, size_t *result);
B2B_API int b2b_isamax_simple(b2b_handle *h, size_t n, const float *x, size_t x_len, size_t *result);
/* Stream-ordered reduction whose result stays on the device: d_result is a
 * float (DOT, NRM2, ASUM) or a uint64_t (IAMAX) in device memory, written
 * when the launch completes; the call returns without waiting.  No reference
 * counterpart.  y is read by DOT only.  Reductions on one handle share a
 * counter and partial-sum workspace, so they must not run concurrently on
 * different streams through the same handle. */
B2B_API int b2b_sreduce_async(b2b_handle *h, int op, size_t n, const float *x, const float *y, void *d_result);

/* ------------------------------------------------------------ GpuTimer
 * benches/src/timer.rs:6-19 (GpuTimer::start / stop, todo! stubs in the
 * reference): start records a CUDA event on the handle's current stream;
 * stop records a second one, waits for it, writes the elapsed milliseconds
 * and frees the timer (stop consumes it, as `stop(self)` does). */
typedef struct b2b_gpu_timer b2b_gpu_timer;
B2B_API int b2b_gpu_timer_start(b2b_handle *h, b2b_gpu_timer **timer);
B2B_API int b2b_gpu_timer_stop(b2b_gpu_timer *timer, double *ms);

/* --------------------------------------------- multi-GPU column sharding
 * No reference counterpart (the reference is single-device,
 * crates/cublas-rs/src/lib.rs:57-68).  A large GEMM is split by column
 * blocks of B and C across G ranks with A replicated; when the caller asks
 * for a gathered C, the ranks all-gather their m x n_g panels (NCCL, through
 * the caller's process group) into a panel-major buffer, and this call lays
 * it out row-major.  panels holds G panels back to back, panel g being
 * m x widths[g] row-major; C is m x n with n = sum(widths).  elem_bytes is
 * 2, 4 or 8.  Device pointers, asynchronous. */
B2B_API int b2b_panels_to_rowmajor(b2b_handle *h, size_t elem_bytes, size_t m, size_t g, const size_t *widths,
                                   const void *panels, void *C);

/* ------------------------------------- multi-GPU: GEMM + all-gather, fused
 * No reference counterpart.  Rank g of a column-sharded GEMM computes its
 * m x n panel alpha*A*B_g + beta*C_g and writes it into every rank's full
 * row-major C (m x ldc, columns [col_off, col_off + n)): dst[d] is rank d's
 * C as a device pointer valid in this process (its own allocation, or a
 * peer's opened with b2b_ipc_open_handle); dst[self_index] is this rank's and
 * also holds the input panel when beta != 0.  1 <= ndst <= 8.  HGEMM with
 * beta == 0 on CTA-pair shapes stores each output box to every destination
 * from the kernel's epilogue (the transfer overlaps the MMAs, no separate
 * all-gather or re-layout); the other cases compute the panel, then copy it
 * to each destination.  Asynchronous on the handle's stream; C is complete
 * on every rank only after all ranks' calls have finished, so order readers
 * behind a barrier or collective, as for an all-gather. */
B2B_API int b2b_hgemm_gather(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                             const uint16_t *B, float beta, size_t ldc, size_t col_off, uint16_t *const *dst,
                             int ndst, int self_index);
B2B_API int b2b_sgemm_gather(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const float *A,
                             const float *B, float beta, size_t ldc, size_t col_off, float *const *dst, int ndst,
                             int self_index);
B2B_API int b2b_dgemm_gather(b2b_handle *h, size_t m, size_t n, size_t k, double alpha, const double *A,
                             const double *B, double beta, size_t ldc, size_t col_off, double *const *dst, int ndst,
                             int self_index);

/* The HGEMM gather through an NVLink multicast object instead of per-peer
 * pointers: mc is the multicast address bound to every rank's full C (same
 * size and layout on each), own this rank's buffer.  Each output store goes
 * once through NVSwitch, which writes it to every member, so a panel crosses
 * NVLink once instead of once per peer.  beta is 0; shapes the CTA-pair
 * kernel cannot take return B2B_ERR_NOT_SUPPORTED (use b2b_hgemm_gather).
 * Same ordering rule as above. */
B2B_API int b2b_hgemm_gather_multicast(b2b_handle *h, size_t m, size_t n, size_t k, float alpha, const uint16_t *A,
                                       const uint16_t *B, size_t ldc, size_t col_off, uint16_t *mc, uint16_t *own);

/* CUDA IPC for the destinations above: a 64-byte handle for a b2b_malloc
 * allocation (pass its base pointer), opened in another process on the same
 * node to get a device pointer to it; close it before the owner frees it. */
#define B2B_IPC_HANDLE_BYTES 64
B2B_API int b2b_ipc_get_handle(b2b_handle *h, void *dptr, void *handle);
B2B_API int b2b_ipc_open_handle(b2b_handle *h, const void *handle, void **dptr);
B2B_API int b2b_ipc_close_handle(b2b_handle *h, void *dptr);

/* ------------------------------------------------------------ self-test
 * No reference counterpart.  Launches one CTA whose mbarrier wait can never
 * complete; the bounded wait gives up after limit_ns (0 < limit <= 5 s),
 * records the timeout in the handle's device status word and exits
 * normally.  The next b2b_synchronize returns B2B_ERR_DEVICE_TIMEOUT and the
 * handle stays usable.  This is how the timeout path of the tensor-core
 * kernels' waits is tested without hanging or faulting a GPU. */
B2B_API int b2b_selftest_bounded_wait(b2b_handle *h, uint64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* B2BLAS_H */
