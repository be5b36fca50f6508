"""The C-ABI library loads and exports every symbol include/larql_cuda.h declares (CPU only)."""
import ctypes as C
import os
import subprocess

import pytest

import larql_cuda as L


def test_header_declares_the_trait_mirrors():
    names = L.header_functions()
    for required in ["larql_cuda_create", "larql_cuda_destroy", "larql_cuda_register_weight",
                     "larql_cuda_q4k_matvec", "larql_cuda_matvec", "larql_cuda_matvec_dev",
                     "larql_cuda_last_error", "larql_cuda_has_q4", "larql_cuda_name"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    missing = [n for n in L.header_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_exports_nothing_undeclared():
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln and "larql_cuda_" in ln}
    assert exported == set(L.header_functions())


def test_status_strings_and_version():
    lib = L.lib()
    assert lib.larql_cuda_version() >= 100
    assert lib.larql_cuda_status_string(0) == b"ok"
    assert lib.larql_cuda_status_string(L.ERR_UNSUPPORTED) == b"unsupported"


def test_errors_are_status_codes_not_aborts():
    """Null arguments come back as LARQL_ERR_INVALID_ARG with a message (no GPU needed)."""
    lib = L.lib()
    assert lib.larql_cuda_create(0, None) == L.ERR_INVALID_ARG
    assert "null" in L.last_error()
    assert lib.larql_cuda_sync(None) == L.ERR_INVALID_ARG
    assert lib.larql_cuda_matvec(None, 1, None, 1, None) == L.ERR_INVALID_ARG
    assert lib.larql_cuda_decode_set_persistent(None, 1) == L.ERR_INVALID_ARG


def test_library_links_no_oracle():
    out = subprocess.run(["ldd", L.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in out and "q4dot" not in out
