"""Loads libb2blas.so (built in-tree next to this file) and declares the C ABI
of include/b2blas.h for ctypes.

There is no fallback: if the library is missing, importing b2blas fails with
an error that says how to build it.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb2blas.so")

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i = ctypes.c_int
_f = ctypes.c_float
_d = ctypes.c_double
_szp = ctypes.POINTER(ctypes.c_size_t)
_fp = ctypes.POINTER(ctypes.c_float)
_vpp = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); every entry point declared in include/b2blas.h.
SIGNATURES = {
    "b2b_version": (_i, []),
    "b2b_last_error": (ctypes.c_char_p, []),
    "b2b_status_string": (ctypes.c_char_p, [_i]),
    "b2b_create": (_i, [_i, _vpp]),
    "b2b_destroy": (_i, [_vp]),
    "b2b_get_stream": (_i, [_vp, _vpp]),
    "b2b_set_stream": (_i, [_vp, _vp]),
    "b2b_synchronize": (_i, [_vp]),
    "b2b_device_info": (_i, [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "b2b_malloc": (_i, [_vp, _sz, _vpp]),
    "b2b_free": (_i, [_vp, _vp]),
    "b2b_memcpy_h2d": (_i, [_vp, _vp, _vp, _sz]),
    "b2b_memcpy_d2h": (_i, [_vp, _vp, _vp, _sz]),
    "b2b_memcpy_d2d": (_i, [_vp, _vp, _vp, _sz]),
    "b2b_memset": (_i, [_vp, _vp, _i, _sz]),
    "b2b_host_alloc": (_i, [_sz, _vpp]),
    "b2b_host_free": (_i, [_vp]),
    "b2b_sgemm": (_i, [_vp, _i, _sz, _sz, _sz, _f, _vp, _vp, _f, _vp]),
    "b2b_sgemm_simple": (_i, [_vp, _i, _sz, _sz, _sz, _f, _vp, _sz, _vp, _sz, _f, _vp, _sz]),
    "b2b_sgemm_bias": (_i, [_vp, _i, _sz, _sz, _sz, _f, _vp, _vp, _f, _vp, _vp, _i]),
    "b2b_sgemm_splits": (_i, [_vp, _sz, _sz, _sz, ctypes.POINTER(_i)]),
    "b2b_set_sgemm_splits": (_i, [_vp, _i]),
    "b2b_dgemm": (_i, [_vp, _i, _sz, _sz, _sz, _d, _vp, _vp, _d, _vp]),
    "b2b_dgemm_simple": (_i, [_vp, _i, _sz, _sz, _sz, _d, _vp, _sz, _vp, _sz, _d, _vp, _sz]),
    "b2b_hgemm": (_i, [_vp, _sz, _sz, _sz, _f, _vp, _vp, _f, _vp]),
    "b2b_hgemm_simple": (_i, [_vp, _sz, _sz, _sz, _f, _vp, _sz, _vp, _sz, _f, _vp, _sz]),
    "b2b_sgemm_strided_batched": (_i, [_vp, _sz, _sz, _sz, _f, _vp, _sz, _vp, _sz, _f, _vp, _sz, _sz]),
    "b2b_sgemm_strided_batched_simple": (
        _i, [_vp, _sz, _sz, _sz, _f, _vp, _sz, _sz, _vp, _sz, _sz, _f, _vp, _sz, _sz, _sz]),
    "b2b_sgemm_batched_simple": (_i, [_vp, _sz, _sz, _sz, _f, _vpp, _szp, _vpp, _szp, _f, _vpp, _szp, _sz]),
    "b2b_sgemv": (_i, [_vp, _i, _i, _sz, _sz, _f, _vp, _vp, _f, _vp]),
    "b2b_sgemv_simple": (_i, [_vp, _i, _i, _sz, _sz, _f, _vp, _sz, _vp, _sz, _f, _vp, _sz]),
    "b2b_sgemv_noalloc": (_i, [_vp, _i, _sz, _sz, _f, _vp, _vp, _f, _vp]),
    "b2b_dgemv": (_i, [_vp, _i, _sz, _sz, _d, _vp, _vp, _d, _vp]),
    "b2b_dgemv_simple": (_i, [_vp, _i, _sz, _sz, _d, _vp, _sz, _vp, _sz, _d, _vp, _sz]),
    "b2b_hgemv": (_i, [_vp, _i, _sz, _sz, _f, _vp, _vp, _f, _vp]),
    "b2b_hgemv_simple": (_i, [_vp, _i, _sz, _sz, _f, _vp, _sz, _vp, _sz, _f, _vp, _sz]),
    "b2b_sdot": (_i, [_vp, _sz, _vp, _vp, _fp]),
    "b2b_sdot_simple": (_i, [_vp, _sz, _vp, _sz, _vp, _sz, _fp]),
    "b2b_snrm2": (_i, [_vp, _sz, _vp, _fp]),
    "b2b_snrm2_simple": (_i, [_vp, _sz, _vp, _sz, _fp]),
    "b2b_sasum": (_i, [_vp, _sz, _vp, _fp]),
    "b2b_sasum_simple": (_i, [_vp, _sz, _vp, _sz, _fp]),
    "b2b_isamax": (_i, [_vp, _sz, _vp, _szp]),
    "b2b_isamax_simple": (_i, [_vp, _sz, _vp, _sz, _szp]),
    "b2b_sreduce_async": (_i, [_vp, _i, _sz, _vp, _vp, _vp]),
    "b2b_saxpy": (_i, [_vp, _sz, _f, _vp, _vp]),
    "b2b_saxpy_simple": (_i, [_vp, _sz, _f, _vp, _sz, _vp, _sz]),
    "b2b_gpu_timer_start": (_i, [_vp, _vpp]),
    "b2b_gpu_timer_stop": (_i, [_vp, ctypes.POINTER(ctypes.c_double)]),
    "b2b_hgemm_gather": (_i, [_vp, _sz, _sz, _sz, _f, _vp, _vp, _f, _sz, _sz, _vpp, _i, _i]),
    "b2b_sgemm_gather": (_i, [_vp, _sz, _sz, _sz, _f, _vp, _vp, _f, _sz, _sz, _vpp, _i, _i]),
    "b2b_dgemm_gather": (_i, [_vp, _sz, _sz, _sz, _d, _vp, _vp, _d, _sz, _sz, _vpp, _i, _i]),
    "b2b_hgemm_gather_multicast": (_i, [_vp, _sz, _sz, _sz, _f, _vp, _vp, _sz, _sz, _vp, _vp]),
    "b2b_ipc_get_handle": (_i, [_vp, _vp, _vp]),
    "b2b_ipc_open_handle": (_i, [_vp, _vp, _vpp]),
    "b2b_ipc_close_handle": (_i, [_vp, _vp]),
    "b2b_panels_to_rowmajor": (_i, [_vp, _sz, _sz, _sz, _szp, _vp, _vp]),
    "b2b_selftest_bounded_wait": (_i, [_vp, ctypes.c_uint64]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Returns the loaded library, loading it on first use."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C cublas-rs_b200` "
            "(or __graft_entry__.build()); b2blas has no CPU fallback")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
