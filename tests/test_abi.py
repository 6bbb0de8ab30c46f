"""The C-ABI library loads and exports exactly what include/b2blas.h declares;
argument checks that need no GPU (CPU only, no compute calls)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _header_functions():
    src = open(os.path.join(ROOT, "include", "b2blas.h")).read()
    return sorted(set(re.findall(r"B2B_API\s+[\w\s\*]+?\b(b2b_\w+)\s*\(", src)))


def test_header_parses():
    names = _header_functions()
    assert "b2b_hgemm" in names and "b2b_sgemm_strided_batched" in names and len(names) >= 25


def test_library_exports_every_declared_symbol():
    import b2blas
    from b2blas import _lib

    lib = b2blas.load_library()
    names = _header_functions()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # The ctypes declarations cover exactly the header.
    assert sorted(_lib.SIGNATURES) == names


def test_rust_binding_covers_the_header():
    # The cublas-sys crate declares every entry point once, in header order,
    # and the header's constants with the same values.
    src = open(os.path.join(ROOT, "cublas-rs_b200", "rust", "cublas-sys", "src", "lib.rs")).read()
    declared = re.findall(r"pub fn (b2b_\w+)\(", src)
    hdr = open(os.path.join(ROOT, "include", "b2blas.h")).read()
    in_order = re.findall(r"B2B_API\s+[\w\s\*]+?\b(b2b_\w+)\s*\(", hdr)
    assert declared == in_order
    consts = dict(re.findall(r"pub const (B2B_\w+): \w+ = (\d+);", src))
    for name, value in re.findall(r"\b(B2B_\w+)\s*=\s*(\d+)", hdr):
        assert consts.get(name) == value, name
    assert consts.get("B2B_IPC_HANDLE_BYTES") == "64"


def test_library_exports_nothing_else():
    # Only b2b_* symbols are visible (the .so is built with hidden visibility).
    import subprocess

    from b2blas import _lib

    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    syms = [l.split()[-1] for l in out.splitlines() if l.strip() and l.split()[1] in ("T", "t")]
    ours = [s for s in syms if s.startswith("b2b_")]
    assert sorted(ours) == _header_functions()


def test_status_strings_and_version():
    import b2blas

    lib = b2blas.load_library()
    assert lib.b2b_status_string(0) == b"ok"
    assert lib.b2b_status_string(2) == b"dimension mismatch"
    assert b2blas.version() == 0x000100


def test_null_handle_is_invalid_argument():
    import b2blas

    lib = b2blas.load_library()
    rc = lib.b2b_sgemm(None, 0, 4, 4, 4, 1.0, None, None, 0.0, None)
    assert rc == 3
    assert b"NULL handle" in lib.b2b_last_error()
    assert lib.b2b_hgemm_simple(None, 1, 1, 1, 1.0, None, 1, None, 1, 0.0, None, 1) == 3
    assert lib.b2b_synchronize(None) == 3
    assert lib.b2b_destroy(None) == 0


def test_create_without_gpu_reports_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import b2blas

    with pytest.raises(b2blas.CublasError) as ei:
        b2blas.Handle(0)
    assert ei.value.kind == "Driver"


def test_host_slice_type_checks():
    import numpy as np

    import b2blas

    with pytest.raises(TypeError):
        b2blas._host(np.zeros(4, np.float64), np.float32)
    a = b2blas._host(np.zeros(4, np.float16), np.uint16)
    assert a.dtype == np.uint16
