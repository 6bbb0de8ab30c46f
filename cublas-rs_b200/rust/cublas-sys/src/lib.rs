//! Raw FFI declarations of libb2blas, the B200 (sm_100a) library behind
//! cublas-rs's `Handle` (crates/cublas-rs/src/lib.rs:42-710): one `extern "C"`
//! declaration per entry point of `include/b2blas.h`, in header order, with
//! the status, transpose, algorithm and reduction constants.
//!
//! `cublas-core` (or `cublas-rs`) depends on this crate and maps the status
//! codes onto `CublasError` (crates/cublas-core/src/error.rs:7-24); the
//! `Handle` methods call these functions instead of launching the PTX that
//! `Modules::load` (crates/cublas-l3/src/lib.rs:51-61) read from the working
//! directory.  build.rs builds and links the library.
#![allow(non_camel_case_types)]
#![no_std]

use core::ffi::{c_char, c_int, c_void};

#[repr(C)] pub struct b2b_handle { _p: [u8; 0] }
#[repr(C)] pub struct b2b_gpu_timer { _p: [u8; 0] }

pub const B2B_OK: c_int = 0;
pub const B2B_ERR_CUDA: c_int = 1;
pub const B2B_ERR_DIMENSION: c_int = 2;
pub const B2B_ERR_INVALID_ARG: c_int = 3;
pub const B2B_ERR_DEVICE_TIMEOUT: c_int = 4;
pub const B2B_ERR_NOT_SUPPORTED: c_int = 5;
pub const B2B_ERR_ALLOC: c_int = 6;
pub const B2B_OP_N: c_int = 0;
pub const B2B_OP_T: c_int = 1;
pub const B2B_ALGO_DEFAULT: c_int = 0;
pub const B2B_ALGO_NAIVE: c_int = 1;
pub const B2B_ALGO_TILED: c_int = 2;
pub const B2B_ALGO_VECTORIZED: c_int = 3;
pub const B2B_ALGO_DOUBLE_BUF: c_int = 4;
pub const B2B_ALGO_3XTF32: c_int = 5;
pub const B2B_REDUCE_DOT: c_int = 0;
pub const B2B_REDUCE_NRM2: c_int = 1;
pub const B2B_REDUCE_ASUM: c_int = 2;
pub const B2B_REDUCE_IAMAX: c_int = 3;
pub const B2B_IPC_HANDLE_BYTES: usize = 64;

extern "C" {
    pub fn b2b_create(device: c_int, out: *mut *mut b2b_handle) -> c_int;
    pub fn b2b_destroy(h: *mut b2b_handle) -> c_int;
    pub fn b2b_get_stream(h: *mut b2b_handle, stream: *mut *mut c_void) -> c_int;
    pub fn b2b_set_stream(h: *mut b2b_handle, stream: *mut c_void) -> c_int;
    pub fn b2b_synchronize(h: *mut b2b_handle) -> c_int;
    pub fn b2b_device_info(h: *mut b2b_handle, device: *mut c_int, sm_count: *mut c_int,
                           sm_clock_khz: *mut c_int) -> c_int;
    pub fn b2b_status_string(status: c_int) -> *const c_char;
    pub fn b2b_last_error() -> *const c_char;
    pub fn b2b_version() -> c_int;
    pub fn b2b_malloc(h: *mut b2b_handle, bytes: usize, dptr: *mut *mut c_void) -> c_int;
    pub fn b2b_free(h: *mut b2b_handle, dptr: *mut c_void) -> c_int;
    pub fn b2b_memcpy_h2d(h: *mut b2b_handle, dst: *mut c_void, src: *const c_void, bytes: usize) -> c_int;
    pub fn b2b_memcpy_d2h(h: *mut b2b_handle, dst: *mut c_void, src: *const c_void, bytes: usize) -> c_int;
    pub fn b2b_memcpy_d2d(h: *mut b2b_handle, dst: *mut c_void, src: *const c_void, bytes: usize) -> c_int;
    pub fn b2b_memset(h: *mut b2b_handle, dptr: *mut c_void, value: c_int, bytes: usize) -> c_int;
    pub fn b2b_host_alloc(bytes: usize, hptr: *mut *mut c_void) -> c_int;
    pub fn b2b_host_free(hptr: *mut c_void) -> c_int;
    pub fn b2b_sgemm(h: *mut b2b_handle, algo: c_int, m: usize, n: usize, k: usize, alpha: f32,
                     a: *const f32, b: *const f32, beta: f32, c: *mut f32) -> c_int;
    pub fn b2b_sgemm_simple(h: *mut b2b_handle, algo: c_int, m: usize, n: usize, k: usize, alpha: f32,
                            a: *const f32, a_len: usize, b: *const f32, b_len: usize, beta: f32, c: *mut f32,
                            c_len: usize) -> c_int;
    pub fn b2b_sgemm_bias(h: *mut b2b_handle, algo: c_int, m: usize, n: usize, k: usize, alpha: f32,
                          a: *const f32, b: *const f32, beta: f32, c: *mut f32, bias: *const f32,
                          relu: c_int) -> c_int;
    pub fn b2b_sgemm_splits(h: *mut b2b_handle, m: usize, n: usize, k: usize, splits: *mut c_int) -> c_int;
    pub fn b2b_set_sgemm_splits(h: *mut b2b_handle, splits: c_int) -> c_int;
    pub fn b2b_dgemm(h: *mut b2b_handle, algo: c_int, m: usize, n: usize, k: usize, alpha: f64,
                     a: *const f64, b: *const f64, beta: f64, c: *mut f64) -> c_int;
    pub fn b2b_dgemm_simple(h: *mut b2b_handle, algo: c_int, m: usize, n: usize, k: usize, alpha: f64,
                            a: *const f64, a_len: usize, b: *const f64, b_len: usize, beta: f64, c: *mut f64,
                            c_len: usize) -> c_int;
    pub fn b2b_hgemm(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32, a: *const u16,
                     b: *const u16, beta: f32, c: *mut u16) -> c_int;
    pub fn b2b_hgemm_simple(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32, a: *const u16,
                            a_len: usize, b: *const u16, b_len: usize, beta: f32, c: *mut u16,
                            c_len: usize) -> c_int;
    pub fn b2b_sgemm_strided_batched(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32,
                                     a: *const f32, stride_a: usize, b: *const f32, stride_b: usize,
                                     beta: f32, c: *mut f32, stride_c: usize, batch: usize) -> c_int;
    pub fn b2b_sgemm_strided_batched_simple(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32,
                                            a: *const f32, a_len: usize, stride_a: usize, b: *const f32,
                                            b_len: usize, stride_b: usize, beta: f32, c: *mut f32,
                                            c_len: usize, stride_c: usize, batch: usize) -> c_int;
    pub fn b2b_sgemm_batched_simple(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32,
                                    a: *const *const f32, a_lens: *const usize, b: *const *const f32,
                                    b_lens: *const usize, beta: f32, c: *const *mut f32,
                                    c_lens: *const usize, batch: usize) -> c_int;
    pub fn b2b_sgemv(h: *mut b2b_handle, algo: c_int, trans: c_int, m: usize, n: usize, alpha: f32,
                     a: *const f32, x: *const f32, beta: f32, y: *mut f32) -> c_int;
    pub fn b2b_sgemv_simple(h: *mut b2b_handle, algo: c_int, trans: c_int, m: usize, n: usize, alpha: f32,
                            a: *const f32, a_len: usize, x: *const f32, x_len: usize, beta: f32, y: *mut f32,
                            y_len: usize) -> c_int;
    pub fn b2b_sgemv_noalloc(h: *mut b2b_handle, trans: c_int, m: usize, n: usize, alpha: f32, a: *const f32,
                             x: *const f32, beta: f32, y: *mut f32) -> c_int;
    pub fn b2b_dgemv(h: *mut b2b_handle, trans: c_int, m: usize, n: usize, alpha: f64, a: *const f64,
                     x: *const f64, beta: f64, y: *mut f64) -> c_int;
    pub fn b2b_dgemv_simple(h: *mut b2b_handle, trans: c_int, m: usize, n: usize, alpha: f64, a: *const f64,
                            a_len: usize, x: *const f64, x_len: usize, beta: f64, y: *mut f64,
                            y_len: usize) -> c_int;
    pub fn b2b_hgemv(h: *mut b2b_handle, trans: c_int, m: usize, n: usize, alpha: f32, a: *const u16,
                     x: *const u16, beta: f32, y: *mut u16) -> c_int;
    pub fn b2b_hgemv_simple(h: *mut b2b_handle, trans: c_int, m: usize, n: usize, alpha: f32, a: *const u16,
                            a_len: usize, x: *const u16, x_len: usize, beta: f32, y: *mut u16,
                            y_len: usize) -> c_int;
    pub fn b2b_saxpy(h: *mut b2b_handle, n: usize, alpha: f32, x: *const f32, y: *mut f32) -> c_int;
    pub fn b2b_saxpy_simple(h: *mut b2b_handle, n: usize, alpha: f32, x: *const f32, x_len: usize,
                            y: *mut f32, y_len: usize) -> c_int;
    pub fn b2b_sdot(h: *mut b2b_handle, n: usize, x: *const f32, y: *const f32, result: *mut f32) -> c_int;
    pub fn b2b_sdot_simple(h: *mut b2b_handle, n: usize, x: *const f32, x_len: usize, y: *const f32,
                           y_len: usize, result: *mut f32) -> c_int;
    pub fn b2b_snrm2(h: *mut b2b_handle, n: usize, x: *const f32, result: *mut f32) -> c_int;
    pub fn b2b_snrm2_simple(h: *mut b2b_handle, n: usize, x: *const f32, x_len: usize,
                            result: *mut f32) -> c_int;
    pub fn b2b_sasum(h: *mut b2b_handle, n: usize, x: *const f32, result: *mut f32) -> c_int;
    pub fn b2b_sasum_simple(h: *mut b2b_handle, n: usize, x: *const f32, x_len: usize,
                            result: *mut f32) -> c_int;
    pub fn b2b_isamax(h: *mut b2b_handle, n: usize, x: *const f32, result: *mut usize) -> c_int;
    pub fn b2b_isamax_simple(h: *mut b2b_handle, n: usize, x: *const f32, x_len: usize,
                             result: *mut usize) -> c_int;
    pub fn b2b_sreduce_async(h: *mut b2b_handle, op: c_int, n: usize, x: *const f32, y: *const f32,
                             d_result: *mut c_void) -> c_int;
    pub fn b2b_gpu_timer_start(h: *mut b2b_handle, timer: *mut *mut b2b_gpu_timer) -> c_int;
    pub fn b2b_gpu_timer_stop(timer: *mut b2b_gpu_timer, ms: *mut f64) -> c_int;
    pub fn b2b_panels_to_rowmajor(h: *mut b2b_handle, elem_bytes: usize, m: usize, g: usize,
                                  widths: *const usize, panels: *const c_void, c: *mut c_void) -> c_int;
    pub fn b2b_hgemm_gather(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32, a: *const u16,
                            b: *const u16, beta: f32, ldc: usize, col_off: usize, dst: *const *mut u16,
                            ndst: c_int, self_index: c_int) -> c_int;
    pub fn b2b_sgemm_gather(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32, a: *const f32,
                            b: *const f32, beta: f32, ldc: usize, col_off: usize, dst: *const *mut f32,
                            ndst: c_int, self_index: c_int) -> c_int;
    pub fn b2b_dgemm_gather(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f64, a: *const f64,
                            b: *const f64, beta: f64, ldc: usize, col_off: usize, dst: *const *mut f64,
                            ndst: c_int, self_index: c_int) -> c_int;
    pub fn b2b_hgemm_gather_multicast(h: *mut b2b_handle, m: usize, n: usize, k: usize, alpha: f32,
                                      a: *const u16, b: *const u16, ldc: usize, col_off: usize, mc: *mut u16,
                                      own: *mut u16) -> c_int;
    pub fn b2b_ipc_get_handle(h: *mut b2b_handle, dptr: *mut c_void, handle: *mut c_void) -> c_int;
    pub fn b2b_ipc_open_handle(h: *mut b2b_handle, handle: *const c_void, dptr: *mut *mut c_void) -> c_int;
    pub fn b2b_ipc_close_handle(h: *mut b2b_handle, dptr: *mut c_void) -> c_int;
    pub fn b2b_selftest_bounded_wait(h: *mut b2b_handle, limit_ns: u64) -> c_int;
}
